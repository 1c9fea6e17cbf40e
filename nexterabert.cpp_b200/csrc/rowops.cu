// Row ops, activation quantization, embedding gather, weight expansion,
// LayerNorm and pooling for sm_100a.
//
// All of these are HBM-bound.  Elementwise row ops run one warp per row with
// lane L owning the 8 consecutive columns 256*B + 8*L .. +7 of each 256-column
// block B (16-byte loads, one 8-byte store of int8 codes); the one reduction
// along a row that must follow the reference's order, op_rms_norm's dot
// product, reads the row the other way round first: lane L chains the
// elements 32*i + L, exactly one lane of the 32-lane dot_f32 accumulator
// (src/nexterabert.cpp:133-151).  The token convolutions stage their rows and
// halo in shared memory.  Every value is produced in the reference's operation
// order and, when the consumer is an int8 linear, quantized per (row,
// 256-column block) in the same pass (quantize_row, :378-403): the fp32 row
// never touches memory.
#include "common.cuh"
#include "dequant.cuh"
#include "nextera_kernels.h"

#include <cuda_runtime.h>

namespace nxk {

__device__ int g_error;
int gemm_take_error();      // gemm_i8.cu
int attn_take_error();      // attention.cu

constexpr int ROW_THREADS = 256;     // 8 rows per block

// eight consecutive floats (16-byte aligned)
__device__ __forceinline__ void ld8(const float * p, float (&v)[8]) {
    const float4 a = ((const float4 *) p)[0], b = ((const float4 *) p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

struct CopyOp {
    const float * x;
    __device__ void prepare(int, int, int) {}
    __device__ void value8(int t, int c0, int C, float (&v)[8]) const { ld8(x + (size_t) t * C + c0, v); }
};

// op_rms_norm (:464-482): x * (1 / sqrt(dot(x, x) / C + eps)) * g
struct RmsOp {
    const float * x;
    const float * g;
    float eps;
    float inv;
    __device__ void prepare(int t, int lane, int C) {
        const float * xr = x + (size_t) t * C;
        float acc = 0.0f;
        for (int i = 0; i < (C >> 5); ++i) {
            const float v = xr[32 * i + lane];
            acc = __fmaf_rn(v, v, acc);
        }
        const float dot = warp_dot_tree(acc);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(dot, (float) C), eps)));
    }
    __device__ void value8(int t, int c0, int C, float (&v)[8]) const {
        float gg[8];
        ld8(x + (size_t) t * C + c0, v);
        ld8(g + c0, gg);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(__fmul_rn(v[e], inv), gg[e]);
    }
};

// op_relu_sqr (:485-505)
struct ReluSqrOp {
    const float * x;
    __device__ void prepare(int, int, int) {}
    __device__ void value8(int t, int c0, int C, float (&v)[8]) const {
        ld8(x + (size_t) t * C + c0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float r = v[e] > 0.0f ? v[e] : 0.0f;
            v[e] = __fmul_rn(r, r);
        }
    }
};

// op_gate (:508-523): sigmoid(g) * y
struct GateOp {
    const float * g;
    const float * y;
    __device__ void prepare(int, int, int) {}
    __device__ void value8(int t, int c0, int C, float (&v)[8]) const {
        float gg[8];
        ld8(g + (size_t) t * C + c0, gg);
        ld8(y + (size_t) t * C + c0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(sigmoid8(gg[e]), v[e]);
    }
};

// op_block_mean (:642-660): mean over each HRA block's real tokens of h (* g)
struct BlockMeanOp {
    const float * h;
    const float * g;
    int block;
    const int32_t * doc_start;
    const int32_t * doc_len;
    const int32_t * bdoc_start;
    const int32_t * brow_doc;
    int ts, n;
    float inv;
    __device__ void prepare(int b, int, int) {
        const int d = brow_doc[b], bi = b - bdoc_start[d];
        ts = doc_start[d] + bi * block;
        n = min(block, doc_len[d] - bi * block);
        inv = __fdiv_rn(1.0f, (float) n);
    }
    __device__ void value8(int, int c0, int C, float (&v)[8]) const {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < n; ++i) {
            float hh[8], gg[8];
            ld8(h + (size_t) (ts + i) * C + c0, hh);
            if (g) ld8(g + (size_t) (ts + i) * C + c0, gg);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = g ? __fmaf_rn(hh[e], gg[e], acc[e]) : __fmaf_rn(1.0f, hh[e], acc[e]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(acc[e], inv);
    }
};

// op_upsample_add (:679-690)
struct UpsampleOp {
    const float * y;
    const float * r;
    int block;
    const int32_t * row_doc;
    const int32_t * doc_start;
    const int32_t * bdoc_start;
    int yb;
    __device__ void prepare(int t, int, int) {
        const int d = row_doc[t];
        yb = bdoc_start[d] + (t - doc_start[d]) / block;
    }
    __device__ void value8(int t, int c0, int C, float (&v)[8]) const {
        float rr[8];
        ld8(y + (size_t) yb * C + c0, v);
        ld8(r + (size_t) t * C + c0, rr);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], rr[e]);
    }
};

// ---------------------------------------------------------------------------
// Vectorised row emitter: lane L of the row's warp owns the 8 consecutive
// columns 256 * B + 8 * L .. + 7 of each 256-column block B, so every input is
// read with two 16-byte loads and the codes leave as one 8-byte store.  The
// per-element arithmetic is the scalar emitter's; only the lane that does it
// changes (the block's amax is a max, independent of order).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
    return (uint32_t) (uint8_t) act_code(a, inv) | ((uint32_t) (uint8_t) act_code(b, inv) << 8) |
           ((uint32_t) (uint8_t) act_code(c, inv) << 16) | ((uint32_t) (uint8_t) act_code(d, inv) << 24);
}

// one row's 8 values of a 256-column block -> fp32 or codes (+ the block scale from lane 0)
__device__ __forceinline__ void emit8(const float (&v)[8], bool on, int lane, size_t row_off, int c0, int blk,
                                      int n_blk, size_t t, float * __restrict__ out, int8_t * __restrict__ q,
                                      float * __restrict__ sx) {
    if (!q) {
        if (on) {
            float4 * o = (float4 *) (out + row_off + c0);
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        return;
    }
    float am = 0.0f;
    if (on) {
#pragma unroll
        for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(v[e]));
    }
    am = warp_max(am);
    const float inv = act_inv(am);
    if (lane == 0) sx[t * n_blk + blk] = act_scale(am);
    if (on) *(uint2 *) (q + row_off + c0) = make_uint2(pack4(v[0], v[1], v[2], v[3], inv), pack4(v[4], v[5], v[6], v[7], inv));
}

template <class Op>
__global__ void __launch_bounds__(ROW_THREADS) row8_kernel(Op op, int T, int C, float * __restrict__ out,
                                                           int8_t * __restrict__ q, float * __restrict__ sx) {
    const int t = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    op.prepare(t, lane, C);
    const int n_blk = (C + I8_BLOCK - 1) / I8_BLOCK;
    for (int B = 0; B < n_blk; ++B) {
        const int c0 = B * I8_BLOCK + 8 * lane;
        const bool on = c0 < C;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (on) op.value8(t, c0, C, v);
        emit8(v, on, lane, (size_t) t * C, c0, B, n_blk, (size_t) t, out, q, sx);
    }
}

template <class Op>
int launch_rows8(const Op & op, int T, int C, float * out, int8_t * q, float * sx, cudaStream_t s) {
    if (T < 0 || C <= 0 || (C & 31) || (!q && !out) || (q && !sx)) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    const int rows_per_block = ROW_THREADS / 32;
    const unsigned grid = (unsigned) ((T + rows_per_block - 1) / rows_per_block);
    row8_kernel<Op><<<grid, ROW_THREADS, 0, s>>>(op, T, C, out, q, sx);
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}

// ---------------------------------------------------------------------------
// Depthwise convolutions along the tokens of a document, tiled: a block owns
// CONV_ROWS rows x one 256-column block.  The rows it reads (its own plus k-1
// of halo) are staged in shared memory once, as x (op_dwconv, :528-544: every
// row of the tile by cp.async at once) or as the product a * x (op_lily_state,
// :548-579: through registers, a few rows per thread at a time), with the taps;
// each row's document bounds are looked up while the rows arrive; then each warp
// runs the tap loop of its rows from shared memory in the reference's order
// (taps ascending, only those inside the row's document) and emits the row's
// block as fp32 or codes.
//   dwconv  v = r (or 0);  v = fma(w[j], x[t + j - k/2], v)
//   lily    v = 0;         v = fma(w[j], (a * x)[t + j - k/2], v);  v = v * b[t]
// ---------------------------------------------------------------------------
constexpr int CONV_ROWS = 32;
static_assert(CONV_ROWS % 8 == 0, "the 8 warps of a block take the tile's rows in turn");
constexpr int CONV_KMAX = 64;

inline size_t conv_smem_bytes(int k) { return sizeof(float) * 256 * (size_t) (CONV_ROWS + 2 * k - 1); }

// KS > 0: the tap count is KS, and each lane keeps its 8 columns' taps in registers for rows whose
// taps all lie inside their document (the rest read them from shared memory)
template <bool LILY, int KS>
__global__ void __launch_bounds__(256) conv_kernel(const float * __restrict__ x, const float * __restrict__ a,
                                                   const float * __restrict__ r, const float * __restrict__ b,
                                                   const float * __restrict__ taps, int k, int halo,
                                                   const int32_t * __restrict__ row_doc,
                                                   const int32_t * __restrict__ doc_start,
                                                   const int32_t * __restrict__ doc_len, int T, int C, int ld,
                                                   float * __restrict__ out, int8_t * __restrict__ q,
                                                   float * __restrict__ sx) {
    extern __shared__ float4 conv_sm[];
    float * P = (float *) conv_sm;                              // [CONV_ROWS + k - 1][256]
    const int n_rows = CONV_ROWS + k - 1;
    float * W = P + (size_t) n_rows * 256;                      // [k][256]
    const int t0 = blockIdx.x * CONV_ROWS, cb = blockIdx.y * 256;
    const int ncol = min(256, C - cb);
    const int hk = k / 2;
    if (!LILY) {
        for (int i = threadIdx.x; i < n_rows * 64; i += blockDim.x) {
            const int rr = i >> 6, c4 = i & 63;
            const int tr = t0 - hk + rr;
            if (tr >= -halo && tr < T + halo && 4 * c4 < ncol)     // rows that exist
                cp_async16(P + 4 * i, x + (ptrdiff_t) tr * ld + cb + 4 * c4);
        }
        cp_async_commit();
    }
    // lane i < RPW: the taps of this warp's row i that lie inside the row's document, [j0, j1),
    // as j0 | j1 << 8 (k <= 64)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int RPW = CONV_ROWS / 8;                          // rows per warp (256 threads)
    static_assert(RPW <= 32, "one lane per row of the warp");
    int jr = 0;
    {
        const int t = t0 + warp + 8 * lane;
        if (lane < RPW && t < T) {
            const int d = row_doc[t];
            const int lo = doc_start[d], hi = lo + doc_len[d];
            jr = max(0, lo - (t - hk)) | min(k, hi - (t - hk)) << 8;
        }
    }
    // lily: staged in batches of 3 items per thread, every load of a batch issued before its first use
    if (LILY) {
        for (int i0 = threadIdx.x; i0 < n_rows * 64; i0 += 3 * blockDim.x) {
            float4 xv[3], av[3];
            bool ok[3];
#pragma unroll
            for (int z = 0; z < 3; ++z) {
                const int i = i0 + z * blockDim.x;
                const int rr = i >> 6, c4 = i & 63;
                const int tr = t0 - hk + rr;
                ok[z] = i < n_rows * 64 && tr >= -halo && tr < T + halo && 4 * c4 < ncol;   // rows that exist
                if (ok[z]) {
                    const ptrdiff_t off = (ptrdiff_t) tr * ld + cb + 4 * c4;
                    xv[z] = *(const float4 *) (x + off);
                    if (LILY) av[z] = *(const float4 *) (a + off);
                }
            }
#pragma unroll
            for (int z = 0; z < 3; ++z) {
                if (!ok[z]) continue;
                float4 p = xv[z];
                if (LILY)
                    p = make_float4(__fmul_rn(av[z].x, p.x), __fmul_rn(av[z].y, p.y), __fmul_rn(av[z].z, p.z),
                                    __fmul_rn(av[z].w, p.w));
                ((float4 *) P)[i0 + z * blockDim.x] = p;
            }
        }
    }
    for (int i = threadIdx.x; i < k * 64; i += blockDim.x) {
        const int j = i >> 6, c4 = i & 63;
        if (4 * c4 < ncol) ((float4 *) W)[i] = *(const float4 *) (taps + (size_t) j * C + cb + 4 * c4);
    }
    if (!LILY) cp_async_wait<0>();                             // this thread's copies have landed
    __syncthreads();
    const int c0 = 8 * lane;
    const bool on = c0 < ncol;
    const int n_blk = (C + I8_BLOCK - 1) / I8_BLOCK;
    float wr[KS > 0 ? KS : 1][8];
    if (KS > 0 && on) {
#pragma unroll
        for (int j = 0; j < (KS > 0 ? KS : 1); ++j) ld8(W + (size_t) j * 256 + c0, wr[j]);
    }
    for (int i = 0; i < RPW; ++i) {
        const int rr = warp + 8 * i, t = t0 + rr;
        if (t >= T) break;
        const int jv = __shfl_sync(0xffffffffu, jr, i);
        const int j0 = jv & 0xff, j1 = jv >> 8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (on) {
            float bv[8];
            if (LILY) ld8(b + (size_t) t * C + cb + c0, bv);          // issued before the tap loop
            if (!LILY && r) ld8(r + (size_t) t * ld + cb + c0, v);
            if (KS > 0 && j0 == 0 && j1 == KS) {
#pragma unroll
                for (int j = 0; j < (KS > 0 ? KS : 1); ++j) {
                    float pv[8];
                    ld8(P + (size_t) (rr + j) * 256 + c0, pv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __fmaf_rn(wr[j][e], pv[e], v[e]);
                }
            } else {
                for (int j = j0; j < j1; ++j) {
                    float pv[8], wv[8];
                    ld8(P + (size_t) (rr + j) * 256 + c0, pv);
                    ld8(W + (size_t) j * 256 + c0, wv);
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __fmaf_rn(wv[e], pv[e], v[e]);
                }
            }
            if (LILY) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], bv[e]);
            }
        }
        emit8(v, on, lane, (size_t) t * C + cb, c0, blockIdx.y, n_blk, (size_t) t, out, q, sx);
    }
}

// Narrow rows (C = 32, 64 or 128: the Lily low-rank conv): a row is C / 8 lanes, so a warp takes
// 256 / C rows at a time and a block 8 * 256 / C * NARROW_STEPS rows; otherwise as conv_kernel
// (dwconv only), with the row's quantization block (all C columns) reduced over its lanes.
constexpr int NARROW_STEPS = 4;

template <int C>
__global__ void __launch_bounds__(256) conv_narrow_kernel(const float * __restrict__ x, const float * __restrict__ r,
                                                          const float * __restrict__ taps, int k, int halo,
                                                          const int32_t * __restrict__ row_doc,
                                                          const int32_t * __restrict__ doc_start,
                                                          const int32_t * __restrict__ doc_len, int T, int ld,
                                                          float * __restrict__ out, int8_t * __restrict__ q,
                                                          float * __restrict__ sx) {
    constexpr int LPR = C / 8;                       // lanes per row
    constexpr int RPW = 32 / LPR;                    // rows per warp step
    constexpr int ROWS = 8 * RPW * NARROW_STEPS;     // rows per block
    extern __shared__ float4 conv_sm[];
    float * P = (float *) conv_sm;                   // [ROWS + k - 1][C]
    float * W = P + (size_t) (ROWS + k - 1) * C;     // [k][C]
    const int t0 = blockIdx.x * ROWS, hk = k / 2;
    const int n4 = (ROWS + k - 1) * (C / 4);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const int rr = i / (C / 4), c4 = i % (C / 4);
        const int tr = t0 - hk + rr;
        if (tr >= -halo && tr < T + halo) ((float4 *) P)[i] = *(const float4 *) (x + (ptrdiff_t) tr * ld + 4 * c4);
    }
    for (int i = threadIdx.x; i < k * (C / 4); i += blockDim.x) ((float4 *) W)[i] = ((const float4 *) taps)[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LPR, c0 = 8 * (lane % LPR);
    for (int step = 0; step < NARROW_STEPS; ++step) {
        const int rr = (step * 8 + warp) * RPW + sub;
        const int t = t0 + rr;
        const bool on = t < T;                                       // whole lane groups
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (on) {
            const int d = row_doc[t];
            const int lo = doc_start[d], hi = lo + doc_len[d];
            const int j0 = max(0, lo - (t - hk)), j1 = min(k, hi - (t - hk));
            if (r) ld8(r + (size_t) t * ld + c0, v);
            for (int j = j0; j < j1; ++j) {
                float pv[8], wv[8];
                ld8(P + (size_t) (rr + j) * C + c0, pv);
                ld8(W + (size_t) j * C + c0, wv);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fmaf_rn(wv[e], pv[e], v[e]);
            }
        }
        if (!q) {
            if (on) {
                float4 * o = (float4 *) (out + (size_t) t * C + c0);
                o[0] = make_float4(v[0], v[1], v[2], v[3]);
                o[1] = make_float4(v[4], v[5], v[6], v[7]);
            }
            continue;
        }
        // the row's maximum |v| over its LPR lanes (C <= 256: one quantization block)
        float am = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(v[e]));
#pragma unroll
        for (int o = 1; o < LPR; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        if (on) {
            const float inv = act_inv(am);
            if (lane % LPR == 0) sx[t] = act_scale(am);
            *(uint2 *) (q + (size_t) t * C + c0) =
                make_uint2(pack4(v[0], v[1], v[2], v[3], inv), pack4(v[4], v[5], v[6], v[7], inv));
        }
    }
}

// ld: floats between the rows of x (and a, r) of the dwconv; the outputs and lily's inputs are C wide
int launch_conv(bool lily, const float * x, const float * a, const float * r, const float * b, const float * taps,
                int k, int halo, const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len, int T,
                int C, int ld, float * out, int8_t * q, float * sx, cudaStream_t s) {
    if (T < 0 || C <= 0 || (C & 31) || k <= 0 || k > CONV_KMAX || halo < 0 || (!q && !out) || (q && !sx))
        return NXK_EINVAL;
    if (ld < C || (ld & 3) || (lily && ld != C)) return NXK_EINVAL;   // 16-byte row starts
    if (T == 0) return NXK_OK;
    if (!lily && (C == 32 || C == 64 || C == 128)) {
        auto narrow = [&](auto kern, int c) {
            const int rows = 8 * (256 / c) * NARROW_STEPS;
            const size_t smem = sizeof(float) * (size_t) c * (size_t) (rows + 2 * k - 1);
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            kern<<<(unsigned) ((T + rows - 1) / rows), 256, smem, s>>>(x, r, taps, k, halo, row_doc, doc_start,
                                                                       doc_len, T, ld, out, q, sx);
        };
        if (C == 32) narrow(conv_narrow_kernel<32>, 32);
        else if (C == 64) narrow(conv_narrow_kernel<64>, 64);
        else narrow(conv_narrow_kernel<128>, 128);
        return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
    }
    const dim3 grid((unsigned) ((T + CONV_ROWS - 1) / CONV_ROWS), (unsigned) ((C + 255) / 256));
    const size_t smem = conv_smem_bytes(k);
    auto go = [&](auto kern, const float * a_, const float * r_, const float * b_) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        kern<<<grid, 256, smem, s>>>(x, a_, r_, b_, taps, k, halo, row_doc, doc_start, doc_len, T, C, ld, out, q, sx);
    };
    if (lily) {
        if (k == 5) go(conv_kernel<true, 5>, a, nullptr, b);
        else go(conv_kernel<true, 0>, a, nullptr, b);
    } else {
        if (k == 5) go(conv_kernel<false, 5>, nullptr, r, nullptr);
        else go(conv_kernel<false, 0>, nullptr, r, nullptr);
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}

// ---------------------------------------------------------------------------
// q / k / v of one attention mixer from the fused projection [T][H*D + 2*G*D]:
// q and k heads through qk_prep's DyT + RoPE, q token-major [T][H][D], k and v
// head-major [G][T][D].  One warp per row (the document position and the RoPE
// row are looked up once for all heads); D = 64, lane i owns the pair (i, i+32).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qkv_prep_kernel(const float * __restrict__ x, int ldx,
                                                       const float * __restrict__ q_alpha,
                                                       const float * __restrict__ q_beta,
                                                       const float * __restrict__ k_alpha,
                                                       const float * __restrict__ k_beta,
                                                       const float * __restrict__ cos_t,
                                                       const float * __restrict__ sin_t,
                                                       const int32_t * __restrict__ row_doc,
                                                       const int32_t * __restrict__ doc_start, int T, int H, int G,
                                                       int Tk, int koff, float * __restrict__ q,
                                                       float * __restrict__ k, float * __restrict__ v) {
    const int t = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int i = threadIdx.x & 31;
    if (t >= T) return;
    const int pos = t - doc_start[row_doc[t]];
    const float c = cos_t[(size_t) pos * 32 + i], s = sin_t[(size_t) pos * 32 + i];
    const float * xr = x + (size_t) t * ldx;
    const float qa0 = q_alpha[i], qa1 = q_alpha[32 + i], qb0 = q_beta[i], qb1 = q_beta[32 + i];
    const float ka0 = k_alpha[i], ka1 = k_alpha[32 + i], kb0 = k_beta[i], kb1 = k_beta[32 + i];
#pragma unroll 4
    for (int h = 0; h < H; ++h) {
        const float x1 = xr[64 * h + i], x2 = xr[64 * h + 32 + i];
        const float a = __fmul_rn(qb0, tanh8(__fmul_rn(qa0, x1)));
        const float b = __fmul_rn(qb1, tanh8(__fmul_rn(qa1, x2)));
        float * y = q + ((size_t) t * H + h) * 64;
        y[i] = __fmaf_rn(a, c, __fmul_rn(b, s));
        y[32 + i] = __fmaf_rn(-a, s, __fmul_rn(b, c));
    }
    const float * xk = xr + 64 * H;
#pragma unroll 4
    for (int g = 0; g < G; ++g) {
        const float x1 = xk[64 * g + i], x2 = xk[64 * g + 32 + i];
        const float a = __fmul_rn(kb0, tanh8(__fmul_rn(ka0, x1)));
        const float b = __fmul_rn(kb1, tanh8(__fmul_rn(ka1, x2)));
        float * y = k + ((size_t) g * Tk + koff + t) * 64;
        y[i] = __fmaf_rn(a, c, __fmul_rn(b, s));
        y[32 + i] = __fmaf_rn(-a, s, __fmul_rn(b, c));
    }
    const float * xv = xk + 64 * G;
#pragma unroll 4
    for (int g = 0; g < G; ++g) {
        float * y = v + ((size_t) g * Tk + koff + t) * 64;
        y[i] = xv[64 * g + i];
        y[32 + i] = xv[64 * g + 32 + i];
    }
}

// ---------------------------------------------------------------------------
// qk_prep (:590-625): DyT then RoPE at the document-relative position.
// One warp per (row, head); lane i owns the pair (i, i + D/2).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) qk_prep_kernel(const float * __restrict__ x, const float * __restrict__ alpha,
                                                      const float * __restrict__ beta, const float * __restrict__ cos_t,
                                                      const float * __restrict__ sin_t, const int32_t * __restrict__ row_doc,
                                                      const int32_t * __restrict__ doc_start, int T, int H, int D,
                                                      int head_major, float * __restrict__ out) {
    const size_t w = (blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (size_t) T * H) return;
    const int t = (int) (w / H), h = (int) (w % H);
    const int half = D >> 1;
    const int pos = t - doc_start[row_doc[t]];
    const float * x1 = x + (size_t) t * H * D + (size_t) h * D;
    float * y1 = head_major ? out + ((size_t) h * T + t) * D : out + (size_t) t * H * D + (size_t) h * D;
    for (int i = lane; i < half; i += 32) {
        const float c = cos_t[(size_t) pos * half + i], s = sin_t[(size_t) pos * half + i];
        const float a = __fmul_rn(beta[i], tanh8(__fmul_rn(alpha[i], x1[i])));
        const float b = __fmul_rn(beta[half + i], tanh8(__fmul_rn(alpha[half + i], x1[half + i])));
        y1[i] = __fmaf_rn(a, c, __fmul_rn(b, s));
        y1[half + i] = __fmaf_rn(-a, s, __fmul_rn(b, c));
    }
}

__global__ void head_major_kernel(const float * __restrict__ x, int T, int H, int D, float * __restrict__ out) {
    const size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x;
    const size_t n = (size_t) T * H * D;
    if (i >= n) return;
    const int d = (int) (i % D);
    const size_t th = i / D;
    const int h = (int) (th % H), t = (int) (th / H);
    out[((size_t) h * T + t) * D + d] = x[i];
}

// ---------------------------------------------------------------------------
// LayerNorm (ggml_norm restated: mean and variance accumulated in double) * w + b
// ---------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(256) layer_norm_kernel(const float * __restrict__ x, const float * __restrict__ w,
                                                         const float * __restrict__ b, float eps, int T, int C,
                                                         float * __restrict__ out) {
    const int t = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float * xr = x + (size_t) t * C;
    double s = 0.0;
    for (int c = lane; c < C; c += 32) s += (double) xr[c];
    const float mean = (float) (warp_sum_d(s) / C);
    double s2 = 0.0;
    for (int c = lane; c < C; c += 32) {
        const float v = __fsub_rn(xr[c], mean);
        s2 += (double) __fmul_rn(v, v);
    }
    const float variance = (float) (warp_sum_d(s2) / C);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
    float * o = out + (size_t) t * C;
    for (int c = lane; c < C; c += 32) {
        float y = __fmul_rn(__fsub_rn(xr[c], mean), scale);
        if (w) y = __fmul_rn(y, w[c]);
        if (b) y = __fadd_rn(y, b[c]);
        o[c] = y;
    }
}

// ---------------------------------------------------------------------------
// pooling (:1903-1918): per (document, channel) sequential sum, then the scale
// ---------------------------------------------------------------------------
__global__ void pool_sum_kernel(const float * __restrict__ hidden, const int32_t * __restrict__ doc_start,
                                const int32_t * __restrict__ doc_len, int n_docs, int C, float * __restrict__ pooled) {
    const size_t i = blockIdx.x * (size_t) blockDim.x + threadIdx.x;
    if (i >= (size_t) n_docs * C) return;
    const int d = (int) (i / C), c = (int) (i % C);
    const float * h = hidden + (size_t) doc_start[d] * C + c;
    const int n = doc_len[d];
    float s = 0.0f;
    int t = 0;
    for (; t + 4 <= n; t += 4) {       // loads issued together, adds kept in order
        const float a0 = h[(size_t) t * C], a1 = h[(size_t) (t + 1) * C];
        const float a2 = h[(size_t) (t + 2) * C], a3 = h[(size_t) (t + 3) * C];
        s = __fadd_rn(s, a0);
        s = __fadd_rn(s, a1);
        s = __fadd_rn(s, a2);
        s = __fadd_rn(s, a3);
    }
    for (; t < n; ++t) s = __fadd_rn(s, h[(size_t) t * C]);
    pooled[i] = s;
}

// 1/n, or 1/||sum|| when normalizing, applied to one pooled row by one warp
__device__ __forceinline__ void pool_scale_row(float * pv, int n, int C, int normalize, int lane) {
    float scale = __fdiv_rn(1.0f, (float) n);
    if (normalize) {
        float acc = 0.0f;
        for (int i = 0; i < (C >> 5); ++i) {
            const float v = pv[32 * i + lane];
            acc = __fmaf_rn(v, v, acc);
        }
        const float nrm = __fsqrt_rn(warp_dot_tree(acc));
        scale = nrm > 0.0f ? __fdiv_rn(1.0f, nrm) : 0.0f;
    }
    for (int c = lane; c < C; c += 32) pv[c] = __fmul_rn(pv[c], scale);
}

__global__ void pool_scale_kernel(const int32_t * __restrict__ doc_len, int n_docs, int C, int normalize,
                                  float * __restrict__ pooled) {
    const int d = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (d >= n_docs) return;
    pool_scale_row(pooled + (size_t) d * C, doc_len[d], C, normalize, lane);
}

// pooled[c] += hidden[t][c] for t = 0 .. T-1 in order (the continuation of pool_sum_kernel's sum)
__global__ void pool_continue_kernel(const float * __restrict__ hidden, int T, int C, float * __restrict__ pooled) {
    const int c = (int) (blockIdx.x * (size_t) blockDim.x + threadIdx.x);
    if (c >= C) return;
    const float * h = hidden + c;
    float s = pooled[c];
    int t = 0;
    for (; t + 4 <= T; t += 4) {       // loads issued together, adds kept in order
        const float a0 = h[(size_t) t * C], a1 = h[(size_t) (t + 1) * C];
        const float a2 = h[(size_t) (t + 2) * C], a3 = h[(size_t) (t + 3) * C];
        s = __fadd_rn(s, a0);
        s = __fadd_rn(s, a1);
        s = __fadd_rn(s, a2);
        s = __fadd_rn(s, a3);
    }
    for (; t < T; ++t) s = __fadd_rn(s, h[(size_t) t * C]);
    pooled[c] = s;
}

__global__ void pool_finish_kernel(int n, int C, int normalize, float * __restrict__ pooled) {
    pool_scale_row(pooled, n, C, normalize, threadIdx.x & 31);
}

// ---------------------------------------------------------------------------
// embedding rows (get_rows + add of the segment embedding)
// ---------------------------------------------------------------------------
constexpr int ERR_TOKEN_RANGE = 0x201;

// One warp per token row: lane L decodes the 4 consecutive values 128 * i + 4L .. +3 (one 16-byte
// store each), the block type fixed at compile time so the decoding of a block's header is shared
// by the 4 values (each value is still the per-element formula of deq_elem).
template <int TYPE>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t * __restrict__ table, size_t row_bytes,
                                                    int n_rows, int C, const int32_t * __restrict__ tokens, int T,
                                                    int ttype, const uint8_t * __restrict__ ttable, size_t trow_bytes,
                                                    int tn_rows, const int32_t * __restrict__ types,
                                                    float * __restrict__ out) {
    const int t = (int) ((blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const int id = tokens[t];
    float * o = out + (size_t) t * C;
    if (id < 0 || id >= n_rows) {
        for (int c = 4 * lane; c < C; c += 128) *(float4 *) (o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane == 0) atomicExch(&g_error, ERR_TOKEN_RANGE);
        return;
    }
    const uint8_t * row = table + row_bytes * (size_t) id;
    int ty = -1;
    if (ttable) {
        ty = types[t];
        if (ty < 0 || ty >= tn_rows) {
            if (lane == 0) atomicExch(&g_error, ERR_TOKEN_RANGE);
            ty = -1;
        }
    }
    const uint8_t * trow = ty >= 0 ? ttable + trow_bytes * (size_t) ty : nullptr;
    for (int c = 4 * lane; c < C; c += 128) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = deq_elem(TYPE, row, c + e);
        if (trow) {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = __fadd_rn(v[e], deq_elem(ttype, trow, c + e));
        }
        *(float4 *) (o + c) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

// ---------------------------------------------------------------------------
// build_i8_weight (:1010-1049): one warp per (row, 256-block)
// ---------------------------------------------------------------------------
__global__ void expand_kernel(int type, const uint8_t * __restrict__ blocks, size_t row_bytes, int n_in, int n_out,
                              int8_t * __restrict__ w8, float * __restrict__ scale, int32_t * __restrict__ off) {
    const size_t wi = (blockIdx.x * (size_t) blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int n_blk = (n_in + I8_BLOCK - 1) / I8_BLOCK;
    if (wi >= (size_t) n_out * n_blk) return;
    const int r = (int) (wi / n_blk), B = (int) (wi % n_blk);
    const uint8_t * row = blocks + row_bytes * (size_t) r;
    float v[8];
    float am = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int e = B * I8_BLOCK + 32 * u + lane;
        v[u] = e < n_in ? deq_elem(type, row, e) : 0.0f;
        am = fmaxf(am, fabsf(v[u]));
    }
    am = warp_max(am);
    const float inv = am > 0.0f ? __fdiv_rn(127.0f, am) : 0.0f;
    int sum = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int e = B * I8_BLOCK + 32 * u + lane;
        if (e < n_in) {
            const int qv = (int) roundf(__fmul_rn(v[u], inv));      // lround: half away from zero
            w8[(size_t) r * n_in + e] = (int8_t) qv;
            sum += qv;
        }
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
        scale[(size_t) B * n_out + r] = __fdiv_rn(am, 127.0f);
        if (off) off[(size_t) B * n_out + r] = -128 * sum;
    }
}

} // namespace nxk

using namespace nxk;

static inline cudaStream_t S(void * s) { return (cudaStream_t) s; }
static inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH; }

extern "C" {

int32_t nxk_take_error(void * stream) {
    int v = 0, zero = 0;
    cudaStreamSynchronize(S(stream));
    cudaMemcpyFromSymbol(&v, g_error, sizeof(int));
    cudaMemcpyToSymbol(g_error, &zero, sizeof(int));
    const int g = gemm_take_error();        // the GEMM's own word (cleared as well)
    const int a = attn_take_error();        // the attention planner's word (cleared as well)
    return v ? v : g ? g : a;
}

int nxk_quantize(const float * x, int T, int C, int8_t * q, float * sx, void * stream) {
    return launch_rows8(CopyOp{x}, T, C, nullptr, q, sx, S(stream));
}

int nxk_rms_norm(const float * x, const float * gain, float eps, int T, int C, float * out, int8_t * q, float * sx,
                 void * stream) {
    return launch_rows8(RmsOp{x, gain, eps, 0.0f}, T, C, out, q, sx, S(stream));
}

int nxk_relu_sqr(const float * x, int T, int C, float * out, int8_t * q, float * sx, void * stream) {
    return launch_rows8(ReluSqrOp{x}, T, C, out, q, sx, S(stream));
}

int nxk_gate(const float * g, const float * y, int T, int C, float * out, int8_t * q, float * sx, void * stream) {
    return launch_rows8(GateOp{g, y}, T, C, out, q, sx, S(stream));
}

int nxk_dwconv(const float * x, const float * r, const float * taps, int k, const int32_t * row_doc,
               const int32_t * doc_start, const int32_t * doc_len, int T, int C, float * out, int8_t * q,
               float * sx, void * stream) {
    return launch_conv(false, x, nullptr, r, nullptr, taps, k, 0, row_doc, doc_start, doc_len, T, C, C, out, q, sx,
                       S(stream));
}

int nxk_dwconv_halo(const float * x, const float * r, const float * taps, int k, int halo, const int32_t * row_doc,
                    const int32_t * doc_start, const int32_t * doc_len, int T, int C, float * out, int8_t * q,
                    float * sx, void * stream) {
    return launch_conv(false, x, nullptr, r, nullptr, taps, k, halo, row_doc, doc_start, doc_len, T, C, C, out, q, sx,
                       S(stream));
}

int nxk_dwconv_halo_ld(const float * x, const float * r, int ld, const float * taps, int k, int halo,
                       const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len, int T, int C,
                       float * out, int8_t * q, float * sx, void * stream) {
    return launch_conv(false, x, nullptr, r, nullptr, taps, k, halo, row_doc, doc_start, doc_len, T, C, ld, out, q,
                       sx, S(stream));
}

int nxk_lily_state(const float * a, const float * x, const float * b, const float * taps, int k,
                   const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len, int T, int C,
                   float * out, int8_t * q, float * sx, void * stream) {
    return launch_conv(true, x, a, nullptr, b, taps, k, 0, row_doc, doc_start, doc_len, T, C, C, out, q, sx,
                       S(stream));
}

int nxk_lily_state_halo(const float * a, const float * x, const float * b, const float * taps, int k, int halo,
                        const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len, int T, int C,
                        float * out, int8_t * q, float * sx, void * stream) {
    return launch_conv(true, x, a, nullptr, b, taps, k, halo, row_doc, doc_start, doc_len, T, C, C, out, q, sx,
                       S(stream));
}

int nxk_block_mean(const float * h, const float * g, int C, int block, const int32_t * doc_start,
                   const int32_t * doc_len, const int32_t * bdoc_start, const int32_t * brow_doc, int n_brows,
                   float * out, int8_t * q, float * sx, void * stream) {
    if (block <= 0) return NXK_EINVAL;
    return launch_rows8(BlockMeanOp{h, g, block, doc_start, doc_len, bdoc_start, brow_doc, 0, 0, 0.0f},
                        n_brows, C, out, q, sx, S(stream));
}

int nxk_upsample_add(const float * y, const float * r, int C, int block, int T, const int32_t * row_doc,
                     const int32_t * doc_start, const int32_t * bdoc_start, float * out, void * stream) {
    if (block <= 0) return NXK_EINVAL;
    return launch_rows8(UpsampleOp{y, r, block, row_doc, doc_start, bdoc_start, 0}, T, C, out, nullptr, nullptr,
                        S(stream));
}

int nxk_qk_prep(const float * x, const float * alpha, const float * beta, const float * cos_t, const float * sin_t,
                const int32_t * row_doc, const int32_t * doc_start, int T, int H, int D, int head_major, float * out,
                void * stream) {
    if (T < 0 || H <= 0 || D <= 0 || (D & 1)) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    const size_t warps = (size_t) T * H;
    qk_prep_kernel<<<(unsigned) ((warps * 32 + 255) / 256), 256, 0, S(stream)>>>(
        x, alpha, beta, cos_t, sin_t, row_doc, doc_start, T, H, D, head_major, out);
    return launched();
}

int nxk_qkv_prep(const float * x, int ldx, const float * q_alpha, const float * q_beta, const float * k_alpha,
                 const float * k_beta, const float * cos_t, const float * sin_t, const int32_t * row_doc,
                 const int32_t * doc_start, int T, int H, int G, int D, float * q, float * k, float * v,
                 void * stream) {
    return nxk_qkv_prep_kv(x, ldx, q_alpha, q_beta, k_alpha, k_beta, cos_t, sin_t, row_doc, doc_start, T, H, G, D, T, 0,
                           q, k, v, stream);
}

int nxk_qkv_prep_kv(const float * x, int ldx, const float * q_alpha, const float * q_beta, const float * k_alpha,
                    const float * k_beta, const float * cos_t, const float * sin_t, const int32_t * row_doc,
                    const int32_t * doc_start, int T, int H, int G, int D, int Tk, int koff, float * q, float * k,
                    float * v, void * stream) {
    if (T < 0 || H <= 0 || G <= 0 || D != 64 || ldx < (H + 2 * G) * D || (ldx & 3)) return NXK_EINVAL;
    if (koff < 0 || (long long) koff + T > Tk) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    qkv_prep_kernel<<<(unsigned) (((size_t) T * 32 + 255) / 256), 256, 0, S(stream)>>>(
        x, ldx, q_alpha, q_beta, k_alpha, k_beta, cos_t, sin_t, row_doc, doc_start, T, H, G, Tk, koff, q, k, v);
    return launched();
}

int nxk_head_major(const float * x, int T, int H, int D, float * out, void * stream) {
    if (T < 0 || H <= 0 || D <= 0) return NXK_EINVAL;
    const size_t n = (size_t) T * H * D;
    if (!n) return NXK_OK;
    head_major_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, S(stream)>>>(x, T, H, D, out);
    return launched();
}

int nxk_layer_norm(const float * x, const float * w, const float * b, float eps, int T, int C, float * out,
                   void * stream) {
    if (T < 0 || C <= 0) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    layer_norm_kernel<<<(unsigned) ((T + 7) / 8), 256, 0, S(stream)>>>(x, w, b, eps, T, C, out);
    return launched();
}

int nxk_pool(const float * hidden, const int32_t * doc_start, const int32_t * doc_len, int n_docs, int C,
             int normalize, float * pooled, void * stream) {
    if (n_docs < 0 || C <= 0 || (C & 31)) return NXK_EINVAL;
    if (n_docs == 0) return NXK_OK;
    const size_t n = (size_t) n_docs * C;
    pool_sum_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, S(stream)>>>(hidden, doc_start, doc_len, n_docs, C, pooled);
    pool_scale_kernel<<<(unsigned) ((n_docs + 7) / 8), 256, 0, S(stream)>>>(doc_len, n_docs, C, normalize, pooled);
    return launched();
}

int nxk_pool_continue(const float * hidden, int T, int C, float * pooled, void * stream) {
    if (T < 0 || C <= 0) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    pool_continue_kernel<<<(unsigned) ((C + 255) / 256), 256, 0, S(stream)>>>(hidden, T, C, pooled);
    return launched();
}

int nxk_pool_finish(int n, int C, int normalize, float * pooled, void * stream) {
    if (n <= 0 || C <= 0 || (C & 31)) return NXK_EINVAL;
    pool_finish_kernel<<<1, 32, 0, S(stream)>>>(n, C, normalize, pooled);
    return launched();
}

int nxk_embed(int type, const void * table, int n_rows, int C, const int32_t * tokens, int T, int ttype,
              const void * ttable, int tn_rows, const int32_t * types, float * out, void * stream) {
    const int bs = blck_size(type);
    if (T < 0 || C <= 0 || n_rows <= 0 || bs <= 0 || C % bs) return NXK_EINVAL;
    if (ttable && (blck_size(ttype) <= 0 || C % blck_size(ttype) || !types)) return NXK_EINVAL;
    if (T == 0) return NXK_OK;
    const size_t rb = (size_t) (C / bs) * type_size(type);
    const size_t trb = ttable ? (size_t) (C / blck_size(ttype)) * type_size(ttype) : 0;
    if (((uintptr_t) out & 15) || (C & 3)) return NXK_EINVAL;           // 16-byte stores
    const unsigned grid = (unsigned) ((T + 7) / 8);
    auto go = [&](auto kern) {
        kern<<<grid, 256, 0, S(stream)>>>((const uint8_t *) table, rb, n_rows, C, tokens, T, ttype,
                                          (const uint8_t *) ttable, trb, tn_rows, types, out);
    };
    switch (type) {
        case T_F32: go(embed_kernel<T_F32>); break;
        case T_F16: go(embed_kernel<T_F16>); break;
        case T_BF16: go(embed_kernel<T_BF16>); break;
        case T_Q4_0: go(embed_kernel<T_Q4_0>); break;
        case T_Q4_1: go(embed_kernel<T_Q4_1>); break;
        case T_Q5_0: go(embed_kernel<T_Q5_0>); break;
        case T_Q5_1: go(embed_kernel<T_Q5_1>); break;
        case T_Q8_0: go(embed_kernel<T_Q8_0>); break;
        case T_Q2_K: go(embed_kernel<T_Q2_K>); break;
        case T_Q3_K: go(embed_kernel<T_Q3_K>); break;
        case T_Q4_K: go(embed_kernel<T_Q4_K>); break;
        case T_Q5_K: go(embed_kernel<T_Q5_K>); break;
        case T_Q6_K: go(embed_kernel<T_Q6_K>); break;
        default: return NXK_EINVAL;
    }
    return launched();
}

int nxk_expand_weight(int type, const void * blocks, int n_in, int n_out, int8_t * w8, float * scale, int32_t * off,
                      void * stream) {
    const int bs = blck_size(type);
    if (n_in <= 0 || n_out <= 0 || bs <= 0 || n_in % bs) return NXK_EINVAL;
    const size_t rb = (size_t) (n_in / bs) * type_size(type);
    const int n_blk = (n_in + I8_BLOCK - 1) / I8_BLOCK;
    const size_t warps = (size_t) n_out * n_blk;
    expand_kernel<<<(unsigned) ((warps * 32 + 255) / 256), 256, 0, S(stream)>>>(
        type, (const uint8_t *) blocks, rb, n_in, n_out, w8, scale, off);
    return launched();
}

} // extern "C"
