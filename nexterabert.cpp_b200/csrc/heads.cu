// The task heads on sm_100a: pooler_output, classify and mlm_logits
// (src/nexterabert.cpp:1296-1317, :1963-2011).
//
// A head is "transform" (an int8 linear, GELU(erf), LayerNorm times a gain)
// followed, for classify and the MLM, by a product with a weight that is NOT on
// the int8 path: the classifier (kept F32 or F16 by the quantizer) and the tied
// MLM decoder over the quantized embedding table.  The reference leaves those
// to ggml_mul_mat, whose CPU backend converts each activation row to the weight
// type's "vec_dot type" and then takes one dot product per weight row:
//
//   weight                      activation                 block dot
//   F32 / F16 / BF16            F32 / F16 / BF16 (RNE)     sum w*x
//   Q4_0 Q5_0 Q8_0              Q8_0 (32 per block)        d_w*d_x*isum
//   Q4_1 Q5_1                   Q8_1 (32 per block)        d_w*d_x*isum + m_w*s_x
//   Q2_K Q3_K Q4_K Q5_K Q6_K    Q8_K (256 per block)       d_x*d_w*isum - d_x*dmin_w*msum
//
// Both steps run here on the raw GGUF blocks: `act_prep_kernel` quantizes the
// activation rows exactly as ggml does (every code and scale bit-identical),
// and `mul_mat_kernel` decodes 32 weights per lane into packed int8 codes and
// takes each 32-weight chunk's integer dots with dp4a (exact).  From there the
// arithmetic is fp32, in another order than ggml's SIMD lanes.
//
// The MLM decoder reads its table (29 MB at Q4_K for 50368 x 1024) once per
// tile of 8 positions; four weight rows per warp share each activation load.
#include "common.cuh"
#include "dequant.cuh"
#include "nextera_kernels.h"

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nxk {
namespace {

enum : int { FAM_F32, FAM_F16, FAM_BF16, FAM_Q8_0, FAM_Q8_1, FAM_Q8_K, FAM_NONE };

__host__ __device__ constexpr int vec_dot_family(int type) {
    switch (type) {
        case T_F32: return FAM_F32;
        case T_F16: return FAM_F16;
        case T_BF16: return FAM_BF16;
        case T_Q4_0: case T_Q5_0: case T_Q8_0: return FAM_Q8_0;
        case T_Q4_1: case T_Q5_1: return FAM_Q8_1;
        case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return FAM_Q8_K;
        default: return FAM_NONE;
    }
}

// bytes of one activation row in the vec_dot type, padded to 16:
//   Q8_0 / Q8_1: int8 q[K] | float d[K/32] | float s[K/32] (Q8_1)
//   Q8_K:        int8 q[K] | float d[K/256] | int32 bsum[K/16]
//   F32/F16/BF16: float x[K] (rounded to the type)
__host__ __device__ inline size_t act_row_bytes(int fam, int K) {
    size_t b = 0;
    switch (fam) {
        case FAM_F32: case FAM_F16: case FAM_BF16: b = 4 * (size_t) K; break;
        case FAM_Q8_0: b = (size_t) K + 4 * (size_t) (K / 32); break;
        case FAM_Q8_1: b = (size_t) K + 8 * (size_t) (K / 32); break;
        case FAM_Q8_K: b = (size_t) K + 4 * (size_t) (K / 256) + 4 * (size_t) (K / 16); break;
        default: return 0;
    }
    return (b + 15) & ~(size_t) 15;
}

__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// ---------------------------------------------------------------------------
// activation rows -> vec_dot type.  One warp per row; lane L owns elements
// 256*i + 8L .. +7, so a 32-block is 4 lanes and a 16-group is 2 lanes.
// ---------------------------------------------------------------------------
template <int FAM>
__global__ void __launch_bounds__(256) act_prep_kernel(const float * __restrict__ x, int K, int M,
                                                       uint8_t * __restrict__ act, size_t stride) {
    const int m = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    const float * xr = x + (size_t) m * K;
    uint8_t * row = act + (size_t) m * stride;
    for (int base = 0; base < K; base += 256) {
        const int e0 = base + 8 * lane;
        const bool in = e0 < K;                 // K % 32 == 0: whole 4-lane groups are in or out
        float v[8];
        if (in) {
            const float4 a = *(const float4 *) (xr + e0), b = *(const float4 *) (xr + e0 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        if constexpr (FAM == FAM_F32 || FAM == FAM_F16 || FAM == FAM_BF16) {
            if (in) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if constexpr (FAM == FAM_F16) v[i] = round_f16(v[i]);
                    if constexpr (FAM == FAM_BF16) v[i] = round_bf16(v[i]);
                }
                float * o = (float *) row + e0;
                *(float4 *) o = make_float4(v[0], v[1], v[2], v[3]);
                *(float4 *) (o + 4) = make_float4(v[4], v[5], v[6], v[7]);
            }
        } else if constexpr (FAM == FAM_Q8_0 || FAM == FAM_Q8_1) {
            // d = amax / 127 (stored fp16), codes = rint(x * 127 / amax), s = fp16(d * sum of codes)
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            int sum = 0;
            uint32_t w0 = 0, w1 = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int q = __float2int_rn(__fmul_rn(v[i], id));
                sum += q;
                if (i < 4) w0 |= (uint32_t) (q & 255) << (8 * i);
                else       w1 |= (uint32_t) (q & 255) << (8 * (i - 4));
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            if (in) {
                *(uint2 *) (row + e0) = make_uint2(w0, w1);
                if ((lane & 3) == 0) {
                    float * dd = (float *) (row + K);
                    dd[e0 / 32] = round_f16(d);
                    if constexpr (FAM == FAM_Q8_1) dd[K / 32 + e0 / 32] = round_f16(__fmul_rn(d, (float) sum));
                }
            }
        } else {
            // Q8_K: scale -127 / (the value of largest magnitude, first one on ties)
            float amax = -1.0f, mx = 0.0f;
            int idx = 1 << 30;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float ax = fabsf(v[i]);
                if (ax > amax) { amax = ax; mx = v[i]; idx = e0 + i; }
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float a2 = __shfl_xor_sync(0xffffffffu, amax, o);
                const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
                if (a2 > amax || (a2 == amax && i2 < idx)) { amax = a2; mx = m2; idx = i2; }
            }
            int32_t * bsum = (int32_t *) (row + K + 4 * (size_t) (K / 256));
            float * dd = (float *) (row + K);
            const int blk = base / 256;
            if (amax == 0.0f) {
                *(uint2 *) (row + e0) = make_uint2(0u, 0u);
                if ((lane & 1) == 0) bsum[e0 / 16] = 0;
                if (lane == 0) dd[blk] = 0.0f;
            } else {
                const float iscale = __fdiv_rn(-127.0f, mx);
                int sum = 0;
                uint32_t w0 = 0, w1 = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int q = min(__float2int_rn(__fmul_rn(iscale, v[i])), 127);
                    sum += q;
                    if (i < 4) w0 |= (uint32_t) (q & 255) << (8 * i);
                    else       w1 |= (uint32_t) (q & 255) << (8 * (i - 4));
                }
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                *(uint2 *) (row + e0) = make_uint2(w0, w1);
                if ((lane & 1) == 0) bsum[e0 / 16] = sum;
                if (lane == 0) dd[blk] = __fdiv_rn(1.0f, iscale);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// 32 weights of one row as packed int8 codes plus their integer sub-scales
// (one per 16 weights) and sub-mins, and the block's fp32 d / dmin (or m).
// Loads are as wide as the block layout allows: a row starts 16-byte aligned
// and its blocks are 144 / 176 (16-aligned), 84 / 20 (4), 24 (8) or
// 210 / 110 / 34 / 22 / 18 bytes (2-aligned).
// ---------------------------------------------------------------------------
struct Chunk {
    uint32_t q[8];
    int sc0, sc1, mn0, mn1;
    float d, dm;
};

__device__ __forceinline__ uint32_t ld16(const uint8_t * p) { return __ldg((const unsigned short *) p); }
__device__ __forceinline__ uint32_t ld32(const uint8_t * p) { return __ldg((const unsigned int *) p); }
__device__ __forceinline__ uint32_t ld32_2(const uint8_t * p) { return ld16(p) | (ld16(p + 2) << 16); }
__device__ __forceinline__ float h2f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short) (h & 0xffffu))); }

// n 32-bit words from p, which is 16- / 4- / 2-byte aligned (ALIGN)
template <int ALIGN, int NW>
__device__ __forceinline__ void ldw(const uint8_t * p, uint32_t (&v)[8]) {
    if constexpr (ALIGN == 16) {
#pragma unroll
        for (int i = 0; i < NW / 4; ++i) {
            const uint4 a = __ldg((const uint4 *) p + i);
            v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
        }
    } else if constexpr (ALIGN == 4) {
#pragma unroll
        for (int i = 0; i < NW; ++i) v[i] = ld32(p + 4 * i);
    } else {
#pragma unroll
        for (int i = 0; i < NW; ++i) v[i] = ld32_2(p + 4 * i);
    }
}

// the four bits (x >> 4i) & 15 of x spread to bit 0 of four bytes
__device__ __forceinline__ uint32_t spread4(uint32_t x, int i) {
    const uint32_t b = (x >> (4 * i)) & 15u;
    return (b & 1u) | ((b & 2u) << 7) | ((b & 4u) << 14) | ((b & 8u) << 21);
}

// 12 scale bytes of a Q4_K / Q5_K block -> the 6-bit scale and min of sub-block j (k_scale_min)
__device__ __forceinline__ void scale_min_k(uint32_t s0, uint32_t s1, uint32_t s2, int j, int & sc, int & mn) {
    auto byte = [&](int x) -> int {
        const uint32_t w = x < 4 ? s0 : x < 8 ? s1 : s2;
        return (int) ((w >> (8 * (x & 3))) & 255u);
    };
    if (j < 4) {
        sc = byte(j) & 63;
        mn = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

template <int TYPE>
__device__ __forceinline__ void decode_chunk(const uint8_t * __restrict__ row, int c, Chunk & k) {
    k.sc0 = k.sc1 = 1;
    k.mn0 = k.mn1 = 0;
    k.dm = 0.0f;
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q4_1) {
        constexpr bool M1 = TYPE == T_Q4_1;
        const uint8_t * b = row + (size_t) c * (M1 ? 20 : 18);
        uint32_t v[8];
        if constexpr (M1) {
            const uint32_t dm = ld32(b);
            k.d = h2f(dm);
            k.dm = h2f(dm >> 16);
            ldw<4, 4>(b + 4, v);
        } else {
            k.d = h2f(ld16(b));
            ldw<2, 4>(b + 2, v);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = v[i] & 0x0f0f0f0fu, hi = (v[i] >> 4) & 0x0f0f0f0fu;
            k.q[i] = M1 ? lo : __vsub4(lo, 0x08080808u);
            k.q[i + 4] = M1 ? hi : __vsub4(hi, 0x08080808u);
        }
    } else if constexpr (TYPE == T_Q5_0 || TYPE == T_Q5_1) {
        constexpr bool M1 = TYPE == T_Q5_1;
        const uint8_t * b = row + (size_t) c * (M1 ? 24 : 22);
        uint32_t v[8], qh;
        if constexpr (M1) {
            const uint32_t dm = ld32(b);
            k.d = h2f(dm);
            k.dm = h2f(dm >> 16);
            qh = ld32(b + 4);
            ldw<4, 4>(b + 8, v);
        } else {
            k.d = h2f(ld16(b));
            qh = ld32_2(b + 2);
            ldw<2, 4>(b + 6, v);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = (v[i] & 0x0f0f0f0fu) | (spread4(qh, i) << 4);
            const uint32_t hi = ((v[i] >> 4) & 0x0f0f0f0fu) | (spread4(qh, i + 4) << 4);
            k.q[i] = M1 ? lo : __vsub4(lo, 0x10101010u);
            k.q[i + 4] = M1 ? hi : __vsub4(hi, 0x10101010u);
        }
    } else if constexpr (TYPE == T_Q8_0) {
        const uint8_t * b = row + (size_t) c * 34;
        k.d = h2f(ld16(b));
        ldw<2, 8>(b + 2, k.q);
    } else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        constexpr bool K5 = TYPE == T_Q5_K;
        const int j = c & 7;
        const uint8_t * b = row + (size_t) (c >> 3) * (K5 ? 176 : 144);
        const uint32_t dm = ld32(b);
        k.d = h2f(dm);
        k.dm = h2f(dm >> 16);
        int sc, mn;
        scale_min_k(ld32(b + 4), ld32(b + 8), ld32(b + 12), j, sc, mn);
        k.sc0 = k.sc1 = sc;
        k.mn0 = k.mn1 = mn;
        uint32_t v[8];
        ldw<16, 8>(b + (K5 ? 48 : 16) + 32 * (j >> 1), v);
        const int sh = 4 * (j & 1);
        if constexpr (K5) {
            uint32_t h[8];
            ldw<16, 8>(b + 16, h);
#pragma unroll
            for (int i = 0; i < 8; ++i) k.q[i] = ((v[i] >> sh) & 0x0f0f0f0fu) | (((h[i] >> j) & 0x01010101u) << 4);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) k.q[i] = (v[i] >> sh) & 0x0f0f0f0fu;
        }
    } else if constexpr (TYPE == T_Q6_K) {
        const int j = c & 7, h = j >> 2;
        const uint8_t * b = row + (size_t) (c >> 3) * 210;
        k.d = h2f(ld16(b + 208));
        const uint32_t sc = ld16(b + 192 + 2 * j);
        k.sc0 = (int) (int8_t) (sc & 255u);
        k.sc1 = (int) (int8_t) (sc >> 8);
        uint32_t lo[8], hi[8];
        ldw<2, 8>(b + 64 * h + 32 * (j & 1), lo);
        ldw<2, 8>(b + 128 + 32 * h, hi);
        const int lsh = 4 * ((j & 3) >> 1), hsh = 2 * (j & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            k.q[i] = __vsub4(((lo[i] >> lsh) & 0x0f0f0f0fu) | (((hi[i] >> hsh) & 0x03030303u) << 4), 0x20202020u);
    } else if constexpr (TYPE == T_Q2_K) {
        const int j = c & 7;
        const uint8_t * b = row + (size_t) (c >> 3) * 84;
        const uint32_t dm = ld32(b + 80);
        k.d = h2f(dm);
        k.dm = h2f(dm >> 16);
        const uint32_t sc = ld16(b + 2 * j);
        k.sc0 = (int) (sc & 15u);
        k.mn0 = (int) ((sc >> 4) & 15u);
        k.sc1 = (int) ((sc >> 8) & 15u);
        k.mn1 = (int) (sc >> 12);
        uint32_t v[8];
        ldw<4, 8>(b + 16 + 32 * (j >> 2), v);
        const int sh = 2 * (j & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i) k.q[i] = (v[i] >> sh) & 0x03030303u;
    } else if constexpr (TYPE == T_Q3_K) {
        const int j = c & 7;
        const uint8_t * b = row + (size_t) (c >> 3) * 110;
        k.d = h2f(ld16(b + 108));
        const uint32_t s01 = ld32_2(b + 96), s23 = ld32_2(b + 100), s45 = ld32_2(b + 104);
        auto byte = [&](int x) -> int {
            const uint32_t w = x < 4 ? s01 : x < 8 ? s23 : s45;
            return (int) ((w >> (8 * (x & 3))) & 255u);
        };
        auto scale = [&](int s) {
            const int lo = (byte(s & 7) >> (4 * (s >> 3))) & 15;
            const int hi = (byte(8 + (s & 3)) >> (2 * (s >> 2))) & 3;
            return (lo | (hi << 4)) - 32;
        };
        k.sc0 = scale(2 * j);
        k.sc1 = scale(2 * j + 1);
        uint32_t qs[8], hm[8];
        ldw<2, 8>(b + 32 + 32 * (j >> 2), qs);
        ldw<2, 8>(b, hm);
        const int sh = 2 * (j & 3);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            k.q[i] = __vsub4(((qs[i] >> sh) & 0x03030303u) | (((hm[i] >> j) & 0x01010101u) << 2), 0x04040404u);
    }
}

template <int TYPE>
__device__ __forceinline__ void decode_floats(const uint8_t * __restrict__ row, int c, float (&w)[32]) {
    if constexpr (TYPE == T_F32) {
        const float4 * p = (const float4 *) (row + (size_t) c * 128);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 a = __ldg(p + i);
            w[4 * i] = a.x; w[4 * i + 1] = a.y; w[4 * i + 2] = a.z; w[4 * i + 3] = a.w;
        }
    } else {
        const uint4 * p = (const uint4 *) (row + (size_t) c * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 a = __ldg(p + i);
            const uint32_t u[4] = { a.x, a.y, a.z, a.w };
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const uint32_t lo = u[h] & 0xffffu, hi = u[h] >> 16;
                if constexpr (TYPE == T_F16) {
                    w[8 * i + 2 * h] = __half2float(__ushort_as_half((unsigned short) lo));
                    w[8 * i + 2 * h + 1] = __half2float(__ushort_as_half((unsigned short) hi));
                } else {
                    w[8 * i + 2 * h] = __uint_as_float(lo << 16);
                    w[8 * i + 2 * h + 1] = __uint_as_float(hi << 16);
                }
            }
        }
    }
}

constexpr int MP = 8;       // activation rows per pass

// rows of W per warp: quantized weights share each activation load across 4 rows; float
// weights (the classifier, usually a handful of rows) take one
template <int TYPE> __host__ __device__ constexpr int rows_per_warp() { return vec_dot_family(TYPE) <= FAM_BF16 ? 1 : 4; }

// out[m][n] = W[n] . x[m] (+ bias[n]).  A warp takes R consecutive weight rows and 8 activation
// rows; lane L takes the 32-weight chunks L, L + 32, ... of those rows.  Each chunk of each row is
// decoded once (wide loads) and each 32-code activation chunk is loaded once for the R rows.  A
// chunk's dot products are exact integers (dp4a); its fp32 term (d_x * d * isum - d_x * dmin * msum
// for the K-quants, d_w * d_x * isum (+ m_w * s_x) for the legacy types) goes into the lane's sum,
// and the 32 lanes' sums are added at the end.  ggml's own SIMD kernels likewise turn per-lane
// integer sums into fp32 before adding them; only the order of the fp32 additions differs.
template <int TYPE>
__global__ void __launch_bounds__(256) mul_mat_kernel(const uint8_t * __restrict__ w, size_t row_bytes, int N, int K,
                                                      const uint8_t * __restrict__ act, size_t stride, int M,
                                                      const float * __restrict__ bias, float * __restrict__ out) {
    constexpr int FAM = vec_dot_family(TYPE);
    constexpr int R = rows_per_warp<TYPE>();
    const int lane = threadIdx.x & 31;
    const int n0 = (int) ((blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R);
    if (n0 >= N) return;                                   // warp-uniform
    const int m0 = blockIdx.x * MP;
    const int mcount = min(MP, M - m0);
    const int n_chunks = K / 32;
    // rows past N / M repeat the last one (computed, not stored), so every pass runs the same code
    const uint8_t * wr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wr[r] = w + (size_t) min(n0 + r, N - 1) * row_bytes;
    const uint8_t * ar[MP];
#pragma unroll
    for (int i = 0; i < MP; ++i) ar[i] = act + (size_t) min(m0 + i, M - 1) * stride;
    float acc[R][MP];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int i = 0; i < MP; ++i) acc[r][i] = 0.0f;

    for (int c = lane; c < n_chunks; c += 32) {
        if constexpr (FAM == FAM_F32 || FAM == FAM_F16 || FAM == FAM_BF16) {
            float wv[32];
            decode_floats<TYPE>(wr[0], c, wv);
#pragma unroll
            for (int i = 0; i < MP; ++i) {
                const float4 * xp = (const float4 *) ar[i] + 8 * c;
                float s = acc[0][i];
#pragma unroll
                for (int v4 = 0; v4 < 8; ++v4) {
                    const float4 a = __ldg(xp + v4);
                    s = __fmaf_rn(wv[4 * v4], a.x, s);
                    s = __fmaf_rn(wv[4 * v4 + 1], a.y, s);
                    s = __fmaf_rn(wv[4 * v4 + 2], a.z, s);
                    s = __fmaf_rn(wv[4 * v4 + 3], a.w, s);
                }
                acc[0][i] = s;
            }
        } else {
            Chunk k[R];
#pragma unroll
            for (int r = 0; r < R; ++r) decode_chunk<TYPE>(wr[r], c, k[r]);
#pragma unroll
            for (int i = 0; i < MP; ++i) {
                const uint4 a = __ldg((const uint4 *) (ar[i] + 32 * (size_t) c));
                const uint4 b = __ldg((const uint4 *) (ar[i] + 32 * (size_t) c) + 1);
                float dx, sx = 0.0f;
                int b0 = 0, b1 = 0;
                if constexpr (FAM == FAM_Q8_K) {
                    dx = __ldg((const float *) (ar[i] + K) + (c >> 3));
                    // bsum sits at K + 4 * (K / 256): 4-byte aligned only
                    const int32_t * bs = (const int32_t *) (ar[i] + K + 4 * (size_t) (K / 256)) + 2 * c;
                    b0 = __ldg(bs);
                    b1 = __ldg(bs + 1);
                } else {
                    dx = __ldg((const float *) (ar[i] + K) + c);
                    if constexpr (FAM == FAM_Q8_1) sx = __ldg((const float *) (ar[i] + K) + K / 32 + c);
                }
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    int s0 = __dp4a((int) k[r].q[0], (int) a.x, 0);
                    s0 = __dp4a((int) k[r].q[1], (int) a.y, s0);
                    s0 = __dp4a((int) k[r].q[2], (int) a.z, s0);
                    s0 = __dp4a((int) k[r].q[3], (int) a.w, s0);
                    int s1 = __dp4a((int) k[r].q[4], (int) b.x, 0);
                    s1 = __dp4a((int) k[r].q[5], (int) b.y, s1);
                    s1 = __dp4a((int) k[r].q[6], (int) b.z, s1);
                    s1 = __dp4a((int) k[r].q[7], (int) b.w, s1);
                    if constexpr (FAM == FAM_Q8_K) {
                        const int ip = k[r].sc0 * s0 + k[r].sc1 * s1;
                        const int mp = k[r].mn0 * b0 + k[r].mn1 * b1;
                        acc[r][i] = __fmaf_rn(__fmul_rn(dx, k[r].d), (float) ip, acc[r][i]);
                        acc[r][i] = __fmaf_rn(-__fmul_rn(dx, k[r].dm), (float) mp, acc[r][i]);
                    } else {
                        acc[r][i] = __fmaf_rn(__fmul_rn(k[r].d, dx), (float) (s0 + s1), acc[r][i]);
                        if constexpr (FAM == FAM_Q8_1) acc[r][i] = __fmaf_rn(k[r].dm, sx, acc[r][i]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int i = 0; i < MP; ++i) {
            float s = acc[r][i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
            const int n = n0 + r;
            if (lane == 0 && i < mcount && n < N) out[(size_t) (m0 + i) * N + n] = bias ? __fadd_rn(s, bias[n]) : s;
        }
    }
}

// ---------------------------------------------------------------------------
// transform's tail: GELU(erf) then ggml_norm (mean, variance in double) * gain
// ---------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// 0.5 * x * (1 + erf(x / sqrt(2))), each operation rounded as written
__device__ __forceinline__ float gelu_erf(float x) {
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erff(__fmul_rn(x, 0.70710678118654752f))));
}

__global__ void __launch_bounds__(256) gelu_norm_kernel(const float * __restrict__ x, const float * __restrict__ w,
                                                        float eps, int T, int C, float * __restrict__ out) {
    const int t = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float * xr = x + (size_t) t * C;
    float * o = out + (size_t) t * C;
    double s = 0.0;
    for (int c = lane; c < C; c += 32) {
        const float g = gelu_erf(xr[c]);
        o[c] = g;                                   // out may alias x: same element, same lane
        s += (double) g;
    }
    const float mean = (float) (warp_sum_d(s) / C);
    double s2 = 0.0;
    for (int c = lane; c < C; c += 32) {
        const float v = __fsub_rn(o[c], mean);
        s2 += (double) __fmul_rn(v, v);
    }
    const float variance = (float) (warp_sum_d(s2) / C);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    for (int c = lane; c < C; c += 32) {
        float y = __fmul_rn(__fsub_rn(o[c], mean), scale);
        if (w) y = __fmul_rn(y, w[c]);
        o[c] = y;
    }
}

__global__ void gather_rows_kernel(const float * __restrict__ x, int C, const int32_t * __restrict__ idx, int n,
                                   float * __restrict__ out) {
    const size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x;
    const size_t c4 = (size_t) C / 4;
    if (i >= (size_t) n * c4) return;
    const size_t r = i / c4, c = i % c4;
    ((float4 *) out)[r * c4 + c] = ((const float4 *) x)[(size_t) idx[r] * c4 + c];
}

inline cudaStream_t S(void * s) { return (cudaStream_t) s; }
inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH; }

template <int TYPE>
void launch_mul_mat(const void * w, int N, int K, const uint8_t * act, size_t stride, int M, const float * bias,
                    float * out, cudaStream_t st) {
    const size_t row_bytes = (size_t) K / blck_size(TYPE) * type_size(TYPE);
    const int rows = 8 * rows_per_warp<TYPE>();                // weight rows per 256-thread block
    const dim3 grid((unsigned) ((M + MP - 1) / MP), (unsigned) ((N + rows - 1) / rows));
    mul_mat_kernel<TYPE><<<grid, 256, 0, st>>>((const uint8_t *) w, row_bytes, N, K, act, stride, M, bias, out);
}

} // namespace
} // namespace nxk

using namespace nxk;

size_t nxk_mul_mat_workspace(int type, int K, int M) {
    const int fam = vec_dot_family(type);
    if (fam == FAM_NONE || K <= 0 || M < 0) return 0;
    return act_row_bytes(fam, K) * (size_t) M;
}

int nxk_mul_mat(int type, const void * w, int N, int K, const float * x, int M, const float * bias,
                void * workspace, float * out, void * stream) {
    const int fam = vec_dot_family(type);
    if (fam == FAM_NONE || N <= 0 || K <= 0 || M < 0 || (K & 31) || !w || !out || (M > 0 && (!x || !workspace)))
        return NXK_EINVAL;
    if (fam == FAM_Q8_K && (K & 255)) return NXK_EINVAL;
    // 16-byte loads of the weight rows, of x and of the converted rows
    if (((uintptr_t) w & 15) || ((uintptr_t) x & 15) || ((uintptr_t) workspace & 15) || ((uintptr_t) out & 3) ||
        ((uintptr_t) bias & 3))
        return NXK_EINVAL;
    if (N > 65535 * 8) return NXK_EINVAL;
    if (M == 0) return NXK_OK;
    const cudaStream_t st = S(stream);
    const size_t stride = act_row_bytes(fam, K);
    uint8_t * act = (uint8_t *) workspace;
    const unsigned pb = (unsigned) ((M + 7) / 8);
    switch (fam) {
        case FAM_F32:  act_prep_kernel<FAM_F32><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
        case FAM_F16:  act_prep_kernel<FAM_F16><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
        case FAM_BF16: act_prep_kernel<FAM_BF16><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
        case FAM_Q8_0: act_prep_kernel<FAM_Q8_0><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
        case FAM_Q8_1: act_prep_kernel<FAM_Q8_1><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
        default:       act_prep_kernel<FAM_Q8_K><<<pb, 256, 0, st>>>(x, K, M, act, stride); break;
    }
    switch (type) {
        case T_F32:  launch_mul_mat<T_F32>(w, N, K, act, stride, M, bias, out, st); break;
        case T_F16:  launch_mul_mat<T_F16>(w, N, K, act, stride, M, bias, out, st); break;
        case T_BF16: launch_mul_mat<T_BF16>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q4_0: launch_mul_mat<T_Q4_0>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q4_1: launch_mul_mat<T_Q4_1>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q5_0: launch_mul_mat<T_Q5_0>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q5_1: launch_mul_mat<T_Q5_1>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q8_0: launch_mul_mat<T_Q8_0>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q2_K: launch_mul_mat<T_Q2_K>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q3_K: launch_mul_mat<T_Q3_K>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q4_K: launch_mul_mat<T_Q4_K>(w, N, K, act, stride, M, bias, out, st); break;
        case T_Q5_K: launch_mul_mat<T_Q5_K>(w, N, K, act, stride, M, bias, out, st); break;
        default:     launch_mul_mat<T_Q6_K>(w, N, K, act, stride, M, bias, out, st); break;
    }
    return launched();
}

int nxk_gelu_norm(const float * x, const float * w, float eps, int T, int C, float * out, void * stream) {
    if (T < 0 || C <= 0 || !x || !out) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    gelu_norm_kernel<<<(unsigned) ((T + 7) / 8), 256, 0, S(stream)>>>(x, w, eps, T, C, out);
    return launched();
}

int nxk_gather_rows(const float * x, int C, const int32_t * idx, int n, float * out, void * stream) {
    if (n < 0 || C <= 0 || (C & 3) || !x || !idx || !out || ((uintptr_t) x & 15) || ((uintptr_t) out & 15))
        return NXK_EINVAL;
    if (n == 0) return NXK_OK;
    const size_t total = (size_t) n * (C / 4);
    gather_rows_kernel<<<(unsigned) ((total + 255) / 256), 256, 0, S(stream)>>>(x, C, idx, n, out);
    return launched();
}
