// The model quantizer on the GPU: the reference's tools/quantize.cpp (nexterabert-quantize), which
// re-encodes the 2-D weights of an F32 / F16 GGUF in one of ggml's block formats.
//
// File side (host): the same presets, the same per-tensor type rule (quantize.cpp:75-98,
// :172-182: 2-D ".weight" matrices of at least 32 x 32 other than classifier.weight, the "_M"
// presets' extra bits for the residual-stream writers, --tensor-type overrides, the fallback of
// K-quants for rows that are not a multiple of 256) and the same output metadata
// (general.file_type, general.quantization_version).  The GGUF is copied key by key; tensors
// that keep their type are copied byte for byte.
//
// Block side (device): one thread per block.
//   Q8_0 Q4_0 Q4_1 Q5_0 Q5_1  ggml's reference quantizers, in the operation order gguf-py 0.19
//                             restates them (gguf/quants.py), so blocks are bit-identical to it
//   Q2_K Q3_K Q4_K Q5_K Q6_K  a direct fit per sub-block (affine for Q2_K / Q4_K / Q5_K,
//                             symmetric for Q3_K / Q6_K) with 6-bit (4-bit for Q2_K) sub-block
//                             scales under an fp16 super-block scale, written in the published
//                             block layouts; ggml's own K-quant search (an iterative refinement of
//                             each sub-block's scale and minimum) is not in this environment, so
//                             these blocks are valid encodings that ggml and this library decode,
//                             not byte copies of ggml's
//   F16                       round to nearest even
// All scalar arithmetic is written with explicit round-to-nearest intrinsics (the library is
// built with -fmad=false as well).
#include "gguf.hpp"
#include "nexterabert.h"
#include "nextera_kernels.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace nxk {
namespace quant {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q2_K = 10,
             T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// fp32 -> fp16 bits, round to nearest even (cvt.rn.f16.f32), widened to 32 bits, and back (exact).
// The bits are kept in 32-bit registers and leave by one 16-bit store (every fp16 field of a block
// sits at an even offset, and blocks are an even number of bytes).
__device__ __forceinline__ uint32_t f16_bits(float v) {
    uint32_t b;
    asm("{\n\t.reg .b16 h;\n\tcvt.rn.f16.f32 h, %1;\n\tcvt.u32.u16 %0, h;\n\t}" : "=r"(b) : "f"(v));
    return b;
}
__device__ __forceinline__ float f16_value(uint32_t b) {
    float v;
    asm("{\n\t.reg .b16 h;\n\tcvt.u16.u32 h, %1;\n\tcvt.f32.f16 %0, h;\n\t}" : "=f"(v) : "r"(b));
    return v;
}
__device__ __forceinline__ void put_f16(uint8_t * p, float v) {
    *reinterpret_cast<unsigned short *>(p) = (unsigned short) f16_bits(v);
}
__device__ __forceinline__ float f16r(float v) { return f16_value(f16_bits(v)); }
__device__ __forceinline__ float safe_inv(float d) { return d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d); }

// index of the first value of largest magnitude (numpy argmax of |x|: first on ties)
__device__ __forceinline__ float signed_absmax(const float * x, int n) {
    float best = x[0], ba = fabsf(x[0]);
    for (int i = 1; i < n; ++i) {
        const float a = fabsf(x[i]);
        if (a > ba) { ba = a; best = x[i]; }
    }
    return best;
}

// ---- legacy 32-value blocks (gguf/quants.py Q8_0 / Q4_0 / Q4_1 / Q5_0 / Q5_1 quantize_blocks)
__device__ void q8_0(const float * x, uint8_t * o) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float d = __fdiv_rn(amax, 127.0f), id = safe_inv(d);
    put_f16(o, d);
    for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t) (int8_t) roundf(__fmul_rn(x[i], id));   // half away from 0
}

__device__ void q4_0(const float * x, uint8_t * o) {
    const float mx = signed_absmax(x, 32);
    const float d = __fdiv_rn(mx, -8.0f), id = safe_inv(d);
    put_f16(o, d);
    uint8_t q[32];
    for (int i = 0; i < 32; ++i) q[i] = (uint8_t) min(15, (int) truncf(__fadd_rn(__fmul_rn(x[i], id), 8.5f)));
    for (int j = 0; j < 16; ++j) o[2 + j] = (uint8_t) (q[j] | (q[16 + j] << 4));
}

__device__ void q4_1(const float * x, uint8_t * o) {
    float mn = x[0], mx = x[0];
    for (int i = 1; i < 32; ++i) { mn = fminf(mn, x[i]); mx = fmaxf(mx, x[i]); }
    const float d = __fdiv_rn(__fsub_rn(mx, mn), 15.0f), id = safe_inv(d);
    put_f16(o, d);
    put_f16(o + 2, mn);
    uint8_t q[32];
    for (int i = 0; i < 32; ++i)
        q[i] = (uint8_t) min(15, (int) truncf(__fadd_rn(__fmul_rn(__fsub_rn(x[i], mn), id), 0.5f)));
    for (int j = 0; j < 16; ++j) o[4 + j] = (uint8_t) (q[j] | (q[16 + j] << 4));
}

__device__ void q5_0(const float * x, uint8_t * o) {
    const float mx = signed_absmax(x, 32);
    const float d = __fdiv_rn(mx, -16.0f), id = safe_inv(d);
    put_f16(o, d);
    uint8_t q[32];
    uint32_t qh = 0;
    for (int i = 0; i < 32; ++i) {
        q[i] = (uint8_t) min(31, (int) truncf(__fadd_rn(__fmul_rn(x[i], id), 16.5f)));
        qh |= (uint32_t) (q[i] >> 4) << i;
    }
    for (int b = 0; b < 4; ++b) o[2 + b] = (uint8_t) (qh >> (8 * b));
    for (int j = 0; j < 16; ++j) o[6 + j] = (uint8_t) ((q[j] & 15) | (q[16 + j] << 4));
}

__device__ void q5_1(const float * x, uint8_t * o) {
    float mn = x[0], mx = x[0];
    for (int i = 1; i < 32; ++i) { mn = fminf(mn, x[i]); mx = fmaxf(mx, x[i]); }
    const float d = __fdiv_rn(__fsub_rn(mx, mn), 31.0f), id = safe_inv(d);
    put_f16(o, d);
    put_f16(o + 2, mn);
    uint8_t q[32];
    uint32_t qh = 0;
    for (int i = 0; i < 32; ++i) {
        q[i] = (uint8_t) min(31, (int) truncf(__fadd_rn(__fmul_rn(__fsub_rn(x[i], mn), id), 0.5f)));
        qh |= (uint32_t) (q[i] >> 4) << i;
    }
    for (int b = 0; b < 4; ++b) o[4 + b] = (uint8_t) (qh >> (8 * b));
    for (int j = 0; j < 16; ++j) o[8 + j] = (uint8_t) ((q[j] & 15) | (q[16 + j] << 4));
}

// round half to even, then clamp to [lo, hi] (numpy rint + clip); a value that is not a number
// (a 0 / 0 the encoders never use) gives lo
__device__ __forceinline__ int rint_clip(float v, int lo, int hi) {
    if (!(v == v)) return lo;
    return (int) fminf(fmaxf(rintf(v), (float) lo), (float) hi);
}

// ---- 256-value super-blocks
// Q4_K / Q5_K: 8 sub-blocks of 32, affine (scale and minimum), 6-bit codes of both under fp16 d / dmin
template <int LEVELS>
__device__ void affine_k(const float * x, uint8_t * o, uint8_t (&q)[256]) {
    float scale[8], mins[8], smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = x[32 * j], hi = x[32 * j];
        for (int i = 1; i < 32; ++i) { lo = fminf(lo, x[32 * j + i]); hi = fmaxf(hi, x[32 * j + i]); }
        lo = fminf(lo, 0.0f);
        scale[j] = __fdiv_rn(__fsub_rn(hi, lo), (float) LEVELS);
        mins[j] = __fsub_rn(0.0f, lo);                  // +0 (not -0) when lo is 0
        smax = fmaxf(smax, scale[j]);
        mmax = fmaxf(mmax, mins[j]);
    }
    const float d = f16r(__fdiv_rn(smax, 63.0f)), dmin = f16r(__fdiv_rn(mmax, 63.0f));
    put_f16(o, d);
    put_f16(o + 2, dmin);
    uint8_t sc[8], mq[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(scale[j], d), 0, 63) : 0;
        mq[j] = dmin > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(mins[j], dmin), 0, 63) : 0;
    }
    // the 12-byte scale / minimum packing of get_scale_min_k4
    for (int j = 0; j < 4; ++j) {
        o[4 + j] = (uint8_t) ((sc[j] & 63) | ((sc[4 + j] >> 4) << 6));
        o[8 + j] = (uint8_t) ((mq[j] & 63) | ((mq[4 + j] >> 4) << 6));
        o[12 + j] = (uint8_t) ((sc[4 + j] & 15) | ((mq[4 + j] & 15) << 4));
    }
    for (int j = 0; j < 8; ++j) {
        const float dsub = __fmul_rn(d, (float) sc[j]), dm = __fmul_rn(dmin, (float) mq[j]);
        for (int i = 0; i < 32; ++i)
            q[32 * j + i] = dsub > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(__fadd_rn(x[32 * j + i], dm), dsub), 0, LEVELS) : 0;
    }
}

__device__ void q4_k(const float * x, uint8_t * o) {
    uint8_t q[256];
    affine_k<15>(x, o, q);
    // qs: 4 groups of 64 values, byte i of group g = q[64g + i] | q[64g + 32 + i] << 4
    for (int g = 0; g < 4; ++g)
        for (int i = 0; i < 32; ++i) o[16 + 32 * g + i] = (uint8_t) (q[64 * g + i] | (q[64 * g + 32 + i] << 4));
}

__device__ void q5_k(const float * x, uint8_t * o) {
    uint8_t q[256];
    affine_k<31>(x, o, q);
    // qh[i] bit j = bit 4 of q[32j + i]; qs as Q4_K on the low 4 bits
    for (int i = 0; i < 32; ++i) {
        uint8_t h = 0;
        for (int j = 0; j < 8; ++j) h |= (uint8_t) (((q[32 * j + i] >> 4) & 1) << j);
        o[16 + i] = h;
    }
    for (int g = 0; g < 4; ++g)
        for (int i = 0; i < 32; ++i)
            o[48 + 32 * g + i] = (uint8_t) ((q[64 * g + i] & 15) | ((q[64 * g + 32 + i] & 15) << 4));
}

// Q6_K: 16 sub-blocks of 16, symmetric, int8 sub-block scales under an fp16 d, 6-bit codes
__device__ void q6_k(const float * x, uint8_t * o) {
    float s[16], smax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int i = 0; i < 16; ++i) a = fmaxf(a, fabsf(x[16 * j + i]));
        s[j] = __fdiv_rn(a, 31.0f);
        smax = fmaxf(smax, s[j]);
    }
    const float d = f16r(__fdiv_rn(smax, 127.0f));
    int8_t sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = d > 0.0f ? (int8_t) rint_clip(__fdiv_rn(s[j], d), -128, 127) : 0;
    uint8_t q[256];
    for (int j = 0; j < 16; ++j) {
        const float dsub = __fmul_rn(d, (float) sc[j]);
        for (int i = 0; i < 16; ++i)
            q[16 * j + i] = (uint8_t) ((dsub != 0.0f ? rint_clip(__fdiv_rn(x[16 * j + i], dsub), -32, 31) : 0) + 32);
    }
    // ql: per half h, byte r (0..63) = q[128h + r] & 15 | (q[128h + 64 + r] & 15) << 4
    // qh: per half h, byte r (0..31) = sum over k of ((q[128h + 32k + r] >> 4) & 3) << 2k
    for (int h = 0; h < 2; ++h) {
        for (int r = 0; r < 64; ++r)
            o[64 * h + r] = (uint8_t) ((q[128 * h + r] & 15) | ((q[128 * h + 64 + r] & 15) << 4));
        for (int r = 0; r < 32; ++r) {
            uint8_t b = 0;
            for (int k = 0; k < 4; ++k) b |= (uint8_t) (((q[128 * h + 32 * k + r] >> 4) & 3) << (2 * k));
            o[128 + 32 * h + r] = b;
        }
    }
    for (int j = 0; j < 16; ++j) o[192 + j] = (uint8_t) sc[j];
    put_f16(o + 208, d);
}

// Q2_K: 16 sub-blocks of 16, affine, 4-bit scale and minimum codes under fp16 d / dmin, 2-bit codes
__device__ void q2_k(const float * x, uint8_t * o) {
    float scale[16], mins[16], smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float lo = x[16 * j], hi = x[16 * j];
        for (int i = 1; i < 16; ++i) { lo = fminf(lo, x[16 * j + i]); hi = fmaxf(hi, x[16 * j + i]); }
        lo = fminf(lo, 0.0f);
        scale[j] = __fdiv_rn(__fsub_rn(hi, lo), 3.0f);
        mins[j] = __fsub_rn(0.0f, lo);                  // +0 (not -0) when lo is 0
        smax = fmaxf(smax, scale[j]);
        mmax = fmaxf(mmax, mins[j]);
    }
    const float d = f16r(__fdiv_rn(smax, 15.0f)), dmin = f16r(__fdiv_rn(mmax, 15.0f));
    uint8_t sc[16], mq[16], q[256];
    for (int j = 0; j < 16; ++j) {
        sc[j] = d > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(scale[j], d), 0, 15) : 0;
        mq[j] = dmin > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(mins[j], dmin), 0, 15) : 0;
        o[j] = (uint8_t) (sc[j] | (mq[j] << 4));
        const float dsub = __fmul_rn(d, (float) sc[j]), dm = __fmul_rn(dmin, (float) mq[j]);
        for (int i = 0; i < 16; ++i)
            q[16 * j + i] = dsub > 0.0f ? (uint8_t) rint_clip(__fdiv_rn(__fadd_rn(x[16 * j + i], dm), dsub), 0, 3) : 0;
    }
    // qs: per half h, byte p (0..31) = sum over k of q[128h + 32k + p] << 2k
    for (int h = 0; h < 2; ++h)
        for (int p = 0; p < 32; ++p) {
            uint8_t b = 0;
            for (int k = 0; k < 4; ++k) b |= (uint8_t) (q[128 * h + 32 * k + p] << (2 * k));
            o[16 + 32 * h + p] = b;
        }
    put_f16(o + 80, d);
    put_f16(o + 82, dmin);
}

// Q3_K: 16 sub-blocks of 16, symmetric, 6-bit sub-block scales (stored + 32) under an fp16 d,
// 3-bit codes q in [-4, 3] stored as q + 4: low 2 bits in qs, bit 2 in hmask
__device__ void q3_k(const float * x, uint8_t * o) {
    float s[16], smax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float a = 0.0f;
        for (int i = 0; i < 16; ++i) a = fmaxf(a, fabsf(x[16 * j + i]));
        s[j] = __fdiv_rn(a, 4.0f);
        smax = fmaxf(smax, s[j]);
    }
    const float d = f16r(__fdiv_rn(smax, 31.0f));
    uint8_t sc6[16], q[256];
    for (int j = 0; j < 16; ++j) {
        const int sc = d > 0.0f ? rint_clip(__fdiv_rn(s[j], d), -32, 31) : 0;
        sc6[j] = (uint8_t) (sc + 32);
        const float dsub = __fmul_rn(d, (float) sc);
        for (int i = 0; i < 16; ++i)
            q[16 * j + i] = (uint8_t) ((dsub != 0.0f ? rint_clip(__fdiv_rn(x[16 * j + i], dsub), -4, 3) : 0) + 4);
    }
    // hmask[p] bit (4h + k) = bit 2 of value 128h + 32k + p; qs as Q2_K on the low 2 bits
    for (int p = 0; p < 32; ++p) {
        uint8_t b = 0;
        for (int h = 0; h < 2; ++h)
            for (int k = 0; k < 4; ++k) b |= (uint8_t) (((q[128 * h + 32 * k + p] >> 2) & 1) << (4 * h + k));
        o[p] = b;
    }
    for (int h = 0; h < 2; ++h)
        for (int p = 0; p < 32; ++p) {
            uint8_t b = 0;
            for (int k = 0; k < 4; ++k) b |= (uint8_t) ((q[128 * h + 32 * k + p] & 3) << (2 * k));
            o[32 + 32 * h + p] = b;
        }
    // scales: bytes 0-7 low nibbles of sub-blocks 0-7 and (high nibble) 8-15; bytes 8-11 the
    // top 2 bits, sub-block s in byte 8 + s % 4 at bit 2 * (s / 4)
    uint8_t * scb = o + 96;
    for (int b = 0; b < 12; ++b) scb[b] = 0;
    for (int s_ = 0; s_ < 16; ++s_) {
        const uint8_t v = sc6[s_];
        if (s_ < 8) scb[s_] |= (uint8_t) (v & 15);
        else        scb[s_ - 8] |= (uint8_t) ((v & 15) << 4);
        scb[8 + (s_ % 4)] |= (uint8_t) (((v >> 4) & 3) << (2 * (s_ / 4)));
    }
    put_f16(o + 108, d);
}

__global__ void quantize_kernel(int type, const float * __restrict__ x, int64_t n_blocks, int bs, int tb,
                                uint8_t * __restrict__ out) {
    const int64_t b = blockIdx.x * (int64_t) blockDim.x + threadIdx.x;
    if (b >= n_blocks) return;
    const float * xb = x + b * bs;
    uint8_t * ob = out + b * tb;
    switch (type) {
        case T_Q8_0: q8_0(xb, ob); break;
        case T_Q4_0: q4_0(xb, ob); break;
        case T_Q4_1: q4_1(xb, ob); break;
        case T_Q5_0: q5_0(xb, ob); break;
        case T_Q5_1: q5_1(xb, ob); break;
        case T_Q2_K: q2_k(xb, ob); break;
        case T_Q3_K: q3_k(xb, ob); break;
        case T_Q4_K: q4_k(xb, ob); break;
        case T_Q5_K: q5_k(xb, ob); break;
        case T_Q6_K: q6_k(xb, ob); break;
        default: break;
    }
}

__global__ void f32_to_f16_kernel(const float * __restrict__ x, int64_t n, uint8_t * __restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x;
    if (i < n) put_f16(out + 2 * i, x[i]);
}

__global__ void f16_to_f32_kernel(const uint16_t * __restrict__ x, int64_t n, float * __restrict__ out) {
    const int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x;
    if (i < n) out[i] = f16_value(x[i]);
}

bool supported_target(int t) {
    switch (t) {
        case T_F16: case T_Q8_0: case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1:
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return true;
        default: return false;
    }
}

} // namespace quant
} // namespace nxk

extern "C" int nxk_quantize_rows(int type, const float * x, int64_t n_per_row, int64_t rows, void * out,
                                 void * stream) {
    using namespace nxk::quant;
    if (!supported_target(type) || n_per_row <= 0 || rows < 0 || !x || !out) return NXK_EINVAL;
    const int64_t bs = nxg::blck_size(type);
    if (bs <= 0 || n_per_row % bs) return NXK_EINVAL;
    if (rows == 0) return NXK_OK;
    cudaStream_t s = (cudaStream_t) stream;
    if (type == T_F16) {
        const int64_t n = n_per_row * rows;
        f32_to_f16_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(x, n, (uint8_t *) out);
    } else {
        const int64_t nb = n_per_row / bs * rows;
        quantize_kernel<<<(unsigned) ((nb + 127) / 128), 128, 0, s>>>(type, x, nb, (int) bs,
                                                                         (int) nxg::type_size(type), (uint8_t *) out);
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}

// ---------------------------------------------------------------------------
// nextera_quantize: the whole file (host)
// ---------------------------------------------------------------------------
namespace {

struct Preset {
    const char * name;
    uint32_t ftype;
    int base, more;
};

// tools/quantize.cpp:33-45 (llama.cpp's general.file_type numbering)
const Preset PRESETS[] = {
    {"F32", 0, 0, 0},        {"F16", 1, 1, 1},        {"Q8_0", 7, 8, 8},      {"Q6_K", 18, 14, 14},
    {"Q5_K_M", 17, 13, 14},  {"Q5_K_S", 16, 13, 13},  {"Q5_0", 8, 6, 6},      {"Q4_K_M", 15, 12, 14},
    {"Q4_K_S", 14, 12, 12},  {"Q4_0", 2, 2, 2},       {"Q3_K_M", 12, 11, 12},
};

const std::pair<const char *, int> TYPE_NAMES[] = {
    {"F32", 0}, {"F16", 1}, {"Q8_0", 8}, {"Q6_K", 14}, {"Q5_K", 13}, {"Q5_0", 6}, {"Q5_1", 7},
    {"Q4_K", 12}, {"Q4_0", 2}, {"Q4_1", 3}, {"Q3_K", 11}, {"Q2_K", 10},
};

const char * type_name(int t) {
    for (const auto & p : TYPE_NAMES)
        if (p.second == t) return p.first;
    return "?";
}

std::string upper(std::string s) {
    for (char & ch : s) ch = (char) toupper((unsigned char) ch);
    return s;
}

bool parse_type(const std::string & s, int & out) {
    for (const auto & t : TYPE_NAMES)
        if (upper(s) == t.first) { out = t.second; return true; }
    return false;
}

bool ends_with(const std::string & s, const char * suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// tools/quantize.cpp:75-83: the tensors the "_M" presets keep at the higher type
bool wants_more_bits(const std::string & n) {
    return ends_with(n, ".attn.c_proj.weight") || ends_with(n, ".mlp.c_proj.weight") ||
           ends_with(n, ".attn.c_v.weight") || ends_with(n, ".attn.c_gate.weight") || n == "mlm.dense.weight" ||
           n == "head.dense.weight" || n == "pooler.dense.weight";
}

// tools/quantize.cpp:87-98: K-quants for rows that are not a multiple of 256 fall back
int fallback_for_row(int t, int64_t n_per_row) {
    if (n_per_row % nxg::blck_size(t) == 0) return t;
    switch (t) {
        case 10: case 11: t = 2; break;     // Q2_K, Q3_K -> Q4_0
        case 12: t = 6; break;              // Q4_K -> Q5_0
        case 13: t = 7; break;              // Q5_K -> Q5_1
        case 14: t = 8; break;              // Q6_K -> Q8_0
        default: break;
    }
    return n_per_row % nxg::blck_size(t) == 0 ? t : 0;
}

// The raw layout of a GGUF: every key/value entry's bytes (to copy them as they are), the tensor
// records and the data section.
struct RawGguf {
    uint32_t version = 3, alignment = 32;
    std::vector<std::pair<std::string, std::vector<uint8_t>>> kv;   // key -> whole entry bytes
    std::vector<nxg::TensorInfo> tensors;
    uint64_t data_offset = 0;
    std::string error;
};

struct Reader {
    FILE * f;
    bool ok = true;
    std::vector<uint8_t> * rec = nullptr;      // bytes read are also appended here
    void rd(void * p, size_t n) {
        if (ok && fread(p, 1, n, f) != n) ok = false;
        if (ok && rec) rec->insert(rec->end(), (uint8_t *) p, (uint8_t *) p + n);
    }
    uint32_t u32() { uint32_t v = 0; rd(&v, 4); return v; }
    uint64_t u64() { uint64_t v = 0; rd(&v, 8); return v; }
    std::string str() {
        const uint64_t n = u64();
        if (!ok || n > (1ull << 31)) { ok = false; return {}; }
        std::string s(n, '\0');
        rd(&s[0], n);
        return s;
    }
};

size_t scalar_bytes(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

bool read_raw(const char * path, RawGguf & g) {
    FILE * f = fopen(path, "rb");
    if (!f) { g.error = "cannot open file"; return false; }
    Reader r{f};
    char magic[4];
    r.rd(magic, 4);
    if (!r.ok || memcmp(magic, "GGUF", 4) != 0) { fclose(f); g.error = "not a GGUF file"; return false; }
    g.version = r.u32();
    const uint64_t n_tensors = r.u64(), n_kv = r.u64();
    if (!r.ok || g.version < 2 || n_kv > 100000 || n_tensors > 1000000) { fclose(f); g.error = "bad GGUF header"; return false; }
    for (uint64_t i = 0; r.ok && i < n_kv; ++i) {
        std::vector<uint8_t> bytes;
        r.rec = &bytes;
        const std::string key = r.str();
        const uint32_t type = r.u32();
        if (type == 8) {
            r.str();
        } else if (type == 9) {
            const uint32_t at = r.u32();
            const uint64_t n = r.u64();
            if (n > (1ull << 28)) { r.ok = false; break; }
            if (at == 8) {
                for (uint64_t j = 0; r.ok && j < n; ++j) r.str();
            } else {
                const size_t es = scalar_bytes(at);
                if (!es) { r.ok = false; break; }
                std::vector<uint8_t> tmp(es * n);
                r.rd(tmp.data(), tmp.size());
            }
        } else {
            const size_t n = scalar_bytes(type);
            if (!n) { r.ok = false; break; }
            uint8_t tmp[8];
            r.rd(tmp, n);
            if (key == "general.alignment" && type == 4) memcpy(&g.alignment, tmp, 4);
        }
        r.rec = nullptr;
        g.kv.emplace_back(key, std::move(bytes));
    }
    for (uint64_t i = 0; r.ok && i < n_tensors; ++i) {
        nxg::TensorInfo t;
        t.name = r.str();
        t.n_dims = (int) r.u32();
        if (t.n_dims < 1 || t.n_dims > 4) { r.ok = false; break; }
        for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t) r.u64();
        t.type = (int) r.u32();
        t.offset = r.u64();
        t.nbytes = nxg::row_size(t.type, t.ne[0]) * (size_t) (t.ne[1] * t.ne[2] * t.ne[3]);
        if (!t.nbytes) { r.ok = false; break; }
        g.tensors.push_back(std::move(t));
    }
    if (!r.ok) { fclose(f); g.error = "truncated or malformed GGUF"; return false; }
    const uint64_t pos = (uint64_t) ftello(f);
    const uint64_t a = g.alignment ? g.alignment : 32;
    g.data_offset = (pos + a - 1) / a * a;
    fclose(f);
    return true;
}

void put_u32(std::vector<uint8_t> & b, uint32_t v) { b.insert(b.end(), (uint8_t *) &v, (uint8_t *) &v + 4); }
void put_u64(std::vector<uint8_t> & b, uint64_t v) { b.insert(b.end(), (uint8_t *) &v, (uint8_t *) &v + 8); }
void put_str(std::vector<uint8_t> & b, const std::string & s) {
    put_u64(b, s.size());
    b.insert(b.end(), s.begin(), s.end());
}
std::vector<uint8_t> kv_u32(const std::string & key, uint32_t v) {
    std::vector<uint8_t> b;
    put_str(b, key);
    put_u32(b, 4);
    put_u32(b, v);
    return b;
}

struct DeviceBuf {
    void * p = nullptr;
    size_t n = 0;
    ~DeviceBuf() { if (p) cudaFree(p); }
    bool reserve(size_t bytes) {
        if (bytes <= n) return true;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        if (cudaMalloc(&p, bytes) != cudaSuccess) { cudaGetLastError(); return false; }
        n = bytes;
        return true;
    }
};

} // namespace

extern "C" int32_t nextera_quantize(const char * in_path, const char * out_path, const char * ftype,
                                    int32_t n_overrides, const char * const * overrides) {
    using namespace nxk::quant;
    if (!in_path || !out_path || !ftype || n_overrides < 0 || (n_overrides > 0 && !overrides)) return 1;
    const Preset * ps = nullptr;
    for (const Preset & p : PRESETS)
        if (upper(ftype) == p.name) ps = &p;
    if (!ps) {
        fprintf(stderr, "nexterabert-quantize: unknown file type '%s'\n", ftype);
        return 1;
    }
    std::vector<std::pair<std::string, int>> ovr;
    for (int32_t i = 0; i < n_overrides; ++i) {
        const std::string v = overrides[i] ? overrides[i] : "";
        const size_t eq = v.rfind('=');
        int t = 0;
        if (eq == std::string::npos || !parse_type(v.substr(eq + 1), t)) {
            fprintf(stderr, "nexterabert-quantize: bad --tensor-type '%s'\n", v.c_str());
            return 1;
        }
        ovr.emplace_back(v.substr(0, eq), t);
    }
    RawGguf g;
    if (!read_raw(in_path, g)) {
        fprintf(stderr, "nexterabert-quantize: failed to read '%s' (%s)\n", in_path, g.error.c_str());
        return 1;
    }
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0) {
        cudaGetLastError();
        fprintf(stderr, "nexterabert-quantize: no CUDA device\n");
        return 3;
    }
    FILE * fin = fopen(in_path, "rb");
    if (!fin) return 1;
    std::unique_ptr<FILE, int (*)(FILE *)> fin_guard(fin, fclose);

    // output tensors: type per tensor, then offsets
    const uint64_t align = g.alignment ? g.alignment : 32;
    std::vector<int> target(g.tensors.size());
    std::vector<size_t> out_bytes(g.tensors.size());
    std::vector<uint64_t> out_off(g.tensors.size());
    uint64_t off = 0;
    for (size_t i = 0; i < g.tensors.size(); ++i) {
        const nxg::TensorInfo & t = g.tensors[i];
        const bool is_matrix = t.n_dims == 2 && ends_with(t.name, ".weight") && t.name != "classifier.weight" &&
                               t.ne[0] >= 32 && t.ne[1] >= 32 && (t.type == T_F32 || t.type == T_F16);
        int tt = t.type;
        if (is_matrix) {
            tt = wants_more_bits(t.name) ? ps->more : ps->base;
            for (const auto & o : ovr)
                if (t.name.find(o.first) != std::string::npos) tt = o.second;
            tt = fallback_for_row(tt, t.ne[0]);
        }
        target[i] = tt;
        out_bytes[i] = tt == t.type ? t.nbytes : nxg::row_size(tt, t.ne[0]) * (size_t) t.ne[1];
        out_off[i] = off;
        off += (out_bytes[i] + align - 1) / align * align;
    }

    // header, metadata (every key as it was, then the file type and quantization version), records
    std::vector<uint8_t> head;
    head.insert(head.end(), {'G', 'G', 'U', 'F'});
    put_u32(head, 3);
    put_u64(head, g.tensors.size());
    size_t n_kv = 0;
    std::vector<uint8_t> kvb;
    for (const auto & e : g.kv) {
        if (e.first == "general.file_type" || e.first == "general.quantization_version") continue;
        kvb.insert(kvb.end(), e.second.begin(), e.second.end());
        ++n_kv;
    }
    for (const auto & e : {kv_u32("general.file_type", ps->ftype), kv_u32("general.quantization_version", 2)}) {
        kvb.insert(kvb.end(), e.begin(), e.end());
        ++n_kv;
    }
    put_u64(head, n_kv);
    head.insert(head.end(), kvb.begin(), kvb.end());
    for (size_t i = 0; i < g.tensors.size(); ++i) {
        const nxg::TensorInfo & t = g.tensors[i];
        put_str(head, t.name);
        put_u32(head, (uint32_t) t.n_dims);
        for (int d = 0; d < t.n_dims; ++d) put_u64(head, (uint64_t) t.ne[d]);
        put_u32(head, (uint32_t) target[i]);
        put_u64(head, out_off[i]);
    }
    head.resize((head.size() + align - 1) / align * align, 0);

    const std::string tmp_path = std::string(out_path) + ".tmp";
    FILE * fo = fopen(tmp_path.c_str(), "wb");
    if (!fo) {
        fprintf(stderr, "nexterabert-quantize: failed to write '%s'\n", out_path);
        return 1;
    }
    bool ok = fwrite(head.data(), 1, head.size(), fo) == head.size();
    DeviceBuf d_in, d_f32, d_out;
    cudaStream_t s = nullptr;
    ok = ok && cudaStreamCreate(&s) == cudaSuccess;
    std::vector<uint8_t> src, dst;
    size_t bytes_in = 0, bytes_out = 0;
    int rc = 0;
    for (size_t i = 0; ok && i < g.tensors.size(); ++i) {
        const nxg::TensorInfo & t = g.tensors[i];
        src.resize(t.nbytes);
        if (fseeko(fin, (off_t) (g.data_offset + t.offset), SEEK_SET) != 0 || fread(src.data(), 1, t.nbytes, fin) != t.nbytes) {
            fprintf(stderr, "nexterabert-quantize: '%s': truncated tensor data\n", t.name.c_str());
            rc = 1;
            ok = false;
            break;
        }
        bytes_in += t.nbytes;
        const std::vector<uint8_t> * outp = &src;
        if (target[i] != t.type) {
            const int64_t n = t.ne[0] * t.ne[1];
            const float * xf = nullptr;
            if (!d_in.reserve(t.nbytes) || !d_out.reserve(out_bytes[i]) || (t.type == T_F16 && !d_f32.reserve(4 * (size_t) n))) {
                rc = 2;
                ok = false;
                break;
            }
            ok = cudaMemcpyAsync(d_in.p, src.data(), t.nbytes, cudaMemcpyHostToDevice, s) == cudaSuccess;
            if (t.type == T_F16) {
                f16_to_f32_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, s>>>((const uint16_t *) d_in.p, n, (float *) d_f32.p);
                xf = (const float *) d_f32.p;
            } else {
                xf = (const float *) d_in.p;
            }
            ok = ok && nxk_quantize_rows(target[i], xf, t.ne[0], t.ne[1], d_out.p, s) == NXK_OK;
            dst.resize(out_bytes[i]);
            ok = ok && cudaMemcpyAsync(dst.data(), d_out.p, out_bytes[i], cudaMemcpyDeviceToHost, s) == cudaSuccess &&
                 cudaStreamSynchronize(s) == cudaSuccess;
            if (!ok) {
                fprintf(stderr, "nexterabert-quantize: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
                rc = 3;
                break;
            }
            outp = &dst;
            printf("%-48s [%5lld x %5lld]  %-4s -> %-5s %8.2f MiB -> %7.2f MiB\n", t.name.c_str(), (long long) t.ne[0],
                   (long long) t.ne[1], type_name(t.type), type_name(target[i]), t.nbytes / 1048576.0,
                   out_bytes[i] / 1048576.0);
        }
        bytes_out += outp->size();
        ok = fwrite(outp->data(), 1, outp->size(), fo) == outp->size();
        const size_t pad = (size_t) ((outp->size() + align - 1) / align * align - outp->size());
        static const uint8_t zeros[256] = {0};
        ok = ok && (pad == 0 || fwrite(zeros, 1, pad, fo) == pad);
        if (!ok && rc == 0) rc = 1;
    }
    if (s) cudaStreamDestroy(s);
    if (fclose(fo) != 0 && ok) { ok = false; rc = 1; }
    if (!ok) {
        remove(tmp_path.c_str());
        if (rc == 0) rc = 1;
        fprintf(stderr, "nexterabert-quantize: failed to write '%s'\n", out_path);
        return rc;
    }
    if (rename(tmp_path.c_str(), out_path) != 0) {
        remove(tmp_path.c_str());
        fprintf(stderr, "nexterabert-quantize: failed to write '%s'\n", out_path);
        return 1;
    }
    printf("\n%s: %.1f MiB -> %.1f MiB  (%s)\n", out_path, bytes_in / 1048576.0, bytes_out / 1048576.0, ps->name);
    return 0;
}
