// Grouped-query attention over a packed, unpadded batch of documents,
// reproducing the reference's op_attention (src/nexterabert.cpp:698-852)
// operation for operation.
//
// Why exact: every linear layer re-quantizes its input to int8, so a rounding
// difference anywhere upstream flips int8 codes, and flips grow through the
// layers (a 1e-7 relative perturbation of the attention outputs alone moves the
// 18-layer random-init model's last hidden state by ~2e-2).  Matching the
// reference therefore means computing what it computes, in its order:
//   score(j)  lane l (0..7) chains q[8r+l]*k[8r+l] over r with fused multiply-adds
//             (NEXTERA_DOT64, :710-714); keys are grouped in 8s from the first
//             key the query sees: a full group reduces ((a0+a1)+(a2+a3)) +
//             ((a4+a5)+(a6+a7)), the n%8 keys after the last full group reduce
//             as hsum256; then * scale (:704-730)
//   softmax   m = max; full groups: e = exp256(s - m) (its Cephes polynomial),
//             summed per lane in key order, then hsum256; the tail keys: e =
//             exp(s - m) from the C library, added in order (:178-198); inv = 1/sum
//   values    o[d] = fma(e_j * inv, v_j[d], o[d]) over the keys in order (:733-754)
// The tail exp is computed in double precision and rounded to fp32 (correctly
// rounded), which equals glibc's expf on all but 8.7e-5 of arguments (counted
// over every float in [-90, 0]); every other operation is the same IEEE fp32
// operation, so the output is bit-identical except where such a tail exp differs.
//
// Work item = (document, 32-query tile, KV head g).  The CTA holds the H/G query
// heads that share g; two threads share one (query, head): thread `sub` keeps
// lanes 4*sub .. 4*sub+3 of the 8-lane accumulators (q and the output dims
// 8r + 4*sub + i).  Keys and values stream through shared memory in 32-key
// tiles.  The softmax max must be known before any exp, so the pass over the
// keys runs three times: max, then exp-sum, then the weighted sum of values
// (scores are recomputed each time; O(T) memory for any document length).
#include "common.cuh"
#include "nextera_kernels.h"

#include <algorithm>
#include <cuda_runtime.h>
#include <vector>

namespace nxk {
namespace attn {

constexpr int D = 64;
constexpr int QT = 32;      // queries per tile
constexpr int KT = 32;      // keys per shared-memory tile

struct Item {
    int q0, q1;      // query rows [q0, q1), all in one document
    int k0, k1;      // keys the tile may touch
    int doc;
};

// exp for the softmax tail: correctly rounded fp32 exp (see above)
__device__ __forceinline__ float exp_tail(float x) { return (float) exp((double) x); }

struct Lanes {
    float a[4];      // this thread's 4 of the 8 lane accumulators
};

// the thread's 4 lanes of NEXTERA_DOT64 for one key row
__device__ __forceinline__ void dot_lanes(const float (&q)[8][4], const float * krow, int sub, Lanes & r) {
#pragma unroll
    for (int r8 = 0; r8 < 8; ++r8) {
        const float4 kk = *(const float4 *) (krow + 8 * r8 + 4 * sub);
        if (r8 == 0) {
            r.a[0] = __fmul_rn(q[0][0], kk.x);
            r.a[1] = __fmul_rn(q[0][1], kk.y);
            r.a[2] = __fmul_rn(q[0][2], kk.z);
            r.a[3] = __fmul_rn(q[0][3], kk.w);
        } else {
            r.a[0] = __fmaf_rn(q[r8][0], kk.x, r.a[0]);
            r.a[1] = __fmaf_rn(q[r8][1], kk.y, r.a[1]);
            r.a[2] = __fmaf_rn(q[r8][2], kk.z, r.a[2]);
            r.a[3] = __fmaf_rn(q[r8][3], kk.w, r.a[3]);
        }
    }
}

// score of one key for both threads of the pair; `full`: the key is in a whole
// group of 8.  All 32 lanes of the warp must call this (shuffles).
__device__ __forceinline__ float pair_score(const Lanes & r, int sub, bool full, float scale) {
    // full group: each thread reduces its 4 lanes, the pair adds the halves
    const float half = __fadd_rn(__fadd_rn(r.a[0], r.a[1]), __fadd_rn(r.a[2], r.a[3]));
    const float other = __shfl_xor_sync(0xffffffffu, half, 1);
    const float t_full = sub == 0 ? __fadd_rn(half, other) : __fadd_rn(other, half);
    // tail key: hsum256 = ((a0+a4) + (a2+a6)) + ((a1+a5) + (a3+a7))
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, r.a[i], 1);
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = __fadd_rn(r.a[i], p[i]);
    const float t_tail = __fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3]));
    return full ? __fmul_rn(t_full, scale) : __fmul_rn(scale, t_tail);
}

template <int REP>
__global__ void __launch_bounds__(QT * REP * 2)
attn_kernel(const float * __restrict__ q, const float * __restrict__ k, const float * __restrict__ v,
            float * __restrict__ out, const Item * __restrict__ items, const float * __restrict__ scale,
            const int32_t * __restrict__ doc_start, const int32_t * __restrict__ doc_len, int T, int H, int half) {
    __shared__ __align__(16) float Ks[KT][D];
    __shared__ __align__(16) float Vs[KT][D];
    constexpr int NT = QT * REP * 2;

    const Item it = items[blockIdx.x];
    const int g = blockIdx.y;
    const int sub = threadIdx.x & 1, pair = threadIdx.x >> 1;
    const int hq = pair / QT, qi = pair % QT;
    const int h = g * REP + hq;
    const int t = it.q0 + qi;
    const bool valid = t < it.q1;
    const int dlo = doc_start[it.doc], dhi = dlo + doc_len[it.doc];
    int lo = dlo, hi = dhi;
    if (half >= 0) {
        lo = max(lo, t - half);
        hi = min(hi, t + half + 1);
    }
    if (!valid) { lo = 0; hi = 0; }
    const int n = hi - lo;
    const int full_end = lo + (n & ~7);          // keys before this are in whole groups of 8
    const float sc = scale[it.doc];

    float qv[8][4];
    {
        const float * qp = q + (size_t) (valid ? t : it.q0) * H * D + (size_t) h * D;
#pragma unroll
        for (int r8 = 0; r8 < 8; ++r8) {
            const float4 x = *(const float4 *) (qp + 8 * r8 + 4 * sub);
            qv[r8][0] = x.x; qv[r8][1] = x.y; qv[r8][2] = x.z; qv[r8][3] = x.w;
        }
    }
    const float * kg = k + (size_t) g * T * D;
    const float * vg = v + (size_t) g * T * D;

    auto load_tile = [&](int kt, int nk, bool with_v) {
        for (int i = threadIdx.x; i < KT * D / 4; i += NT) {
            const int j = i / (D / 4), d4 = i % (D / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (j < nk) {
                kv = ((const float4 *) (kg + (size_t) (kt + j) * D))[d4];
                if (with_v) vv = ((const float4 *) (vg + (size_t) (kt + j) * D))[d4];
            }
            ((float4 *) Ks[j])[d4] = kv;
            if (with_v) ((float4 *) Vs[j])[d4] = vv;
        }
    };

    // ---- pass 1: the maximum score (exact whatever the order)
    float m = -INFINITY;
    for (int kt = it.k0; kt < it.k1; kt += KT) {
        const int nk = min(KT, it.k1 - kt);
        load_tile(kt, nk, false);
        __syncthreads();
        for (int j = 0; j < nk; ++j) {
            Lanes r;
            dot_lanes(qv, Ks[j], sub, r);
            const int kj = kt + j;
            const float s = pair_score(r, sub, kj < full_end, sc);
            if (kj >= lo && kj < hi) m = (m < s) ? s : m;
        }
        __syncthreads();
    }

    // ---- pass 2: e = exp256(s - m) over whole groups, summed per lane in key order
    float vs[4] = {0.f, 0.f, 0.f, 0.f};       // lanes 4*sub .. 4*sub+3 of the 8 sum lanes
    for (int kt = it.k0; kt < it.k1; kt += KT) {
        const int nk = min(KT, it.k1 - kt);
        load_tile(kt, nk, false);
        __syncthreads();
        for (int j = 0; j < nk; ++j) {
            Lanes r;
            dot_lanes(qv, Ks[j], sub, r);
            const int kj = kt + j;
            const float s = pair_score(r, sub, true, sc);
            if (kj >= lo && kj < full_end) {
                const float e = exp8(__fsub_rn(s, m));
                const int l = (kj - lo) & 7;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (l == 4 * sub + i) vs[i] = __fadd_rn(vs[i], e);
                }
            }
        }
        __syncthreads();
    }
    // hsum256 of the 8 lanes, then the tail keys in order with the C library's exp
    float sum;
    {
        float p[4], x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, vs[i], 1);
#pragma unroll
        for (int i = 0; i < 4; ++i) x[i] = __fadd_rn(vs[i], p[i]);
        sum = __fadd_rn(__fadd_rn(x[0], x[2]), __fadd_rn(x[1], x[3]));
    }
    for (int i = 0; i < 7; ++i) {                 // warp-uniform trip count: the shuffles need every lane
        const int kj = full_end + i;
        const bool act = kj < hi;
        Lanes r;
        dot_lanes(qv, kg + (size_t) (act ? kj : 0) * D, sub, r);
        const float s = pair_score(r, sub, false, sc);
        if (act) sum = __fadd_rn(sum, exp_tail(__fsub_rn(s, m)));
    }
    const float inv = __fdiv_rn(1.0f, sum);

    // ---- pass 3: o[d] = fma(e_j * inv, v_j[d], o[d]) over the keys in order
    float o[8][4];
#pragma unroll
    for (int r8 = 0; r8 < 8; ++r8) {
#pragma unroll
        for (int i = 0; i < 4; ++i) o[r8][i] = 0.0f;
    }
    for (int kt = it.k0; kt < it.k1; kt += KT) {
        const int nk = min(KT, it.k1 - kt);
        load_tile(kt, nk, true);
        __syncthreads();
        for (int j = 0; j < nk; ++j) {
            Lanes r;
            dot_lanes(qv, Ks[j], sub, r);
            const int kj = kt + j;
            const bool full = kj < full_end;
            const float s = pair_score(r, sub, full, sc);
            if (kj >= lo && kj < hi) {
                const float x = __fsub_rn(s, m);
                const float c = __fmul_rn(full ? exp8(x) : exp_tail(x), inv);
#pragma unroll
                for (int r8 = 0; r8 < 8; ++r8) {
                    const float4 vv = *(const float4 *) (Vs[j] + 8 * r8 + 4 * sub);
                    o[r8][0] = __fmaf_rn(c, vv.x, o[r8][0]);
                    o[r8][1] = __fmaf_rn(c, vv.y, o[r8][1]);
                    o[r8][2] = __fmaf_rn(c, vv.z, o[r8][2]);
                    o[r8][3] = __fmaf_rn(c, vv.w, o[r8][3]);
                }
            }
        }
        __syncthreads();
    }
    if (valid) {
        float * op = out + (size_t) t * H * D + (size_t) h * D;
#pragma unroll
        for (int r8 = 0; r8 < 8; ++r8) {
            *(float4 *) (op + 8 * r8 + 4 * sub) = make_float4(o[r8][0], o[r8][1], o[r8][2], o[r8][3]);
        }
    }
}

// ---------------------------------------------------------------------------
// Stored-score kernel (used by nxk_attention).  Same arithmetic as attn_kernel;
// the difference is where the scores live.  One thread owns one (query, head) and
// all 64 lanes of its dot products (q in registers, keys broadcast from shared
// memory), computes every score once, and keeps it in a per-CTA scratch slot in
// global memory (sized for the longest key range of the launch; L2-resident for
// the band layers).  Pass 2 walks the thread's own scores in groups of 8 for the
// exp-sum and leaves each exp in place of its score; pass 3 scales them by
// 1/sum and accumulates the values.  Work units (tile, KV head) are spread over a persistent grid,
// longest first.
// ---------------------------------------------------------------------------
constexpr int QT3 = 64;            // queries per work unit

template <int REP>
__global__ void __launch_bounds__(QT3 * REP)
attn_scored_kernel(const float * __restrict__ q, const float * __restrict__ k, const float * __restrict__ v,
                   float * __restrict__ out, const Item * __restrict__ items, int n_units, int G,
                   const float * __restrict__ scale, const int32_t * __restrict__ doc_start,
                   const int32_t * __restrict__ doc_len, int T, int H, int half, float * __restrict__ scratch,
                   int slot_keys) {
    constexpr int NT = QT3 * REP;
    __shared__ __align__(16) float Ks[KT][D];
    __shared__ __align__(16) float Vs[KT][D];
    __shared__ float Cw[KT][NT];                                        // the tile's softmax weights
    float * sc_base = scratch + (size_t) blockIdx.x * slot_keys * NT;   // [key - k0][thread]

    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const Item it = items[u / G];
        const int g = u % G;
        const int hq = threadIdx.x / QT3, qi = threadIdx.x % QT3;
        const int h = g * REP + hq;
        const int t = it.q0 + qi;
        const bool valid = t < it.q1;
        int lo = doc_start[it.doc], hi = lo + doc_len[it.doc];
        if (half >= 0) {
            lo = max(lo, t - half);
            hi = min(hi, t + half + 1);
        }
        if (!valid) { lo = it.k0; hi = it.k0; }
        const int n = hi - lo;
        const int full_end = lo + (n & ~7);
        const float sc = scale[it.doc];
        const float * kg = k + (size_t) g * T * D;
        const float * vg = v + (size_t) g * T * D;

        // ---- pass 1: every score once (stored), and their maximum.  Lanes l and l+4 of
        // the 8-lane accumulator run as one packed pair (f32x2 FMA, each component an
        // IEEE fused multiply-add); key rows sit in shared memory interleaved to match.
        float m = -INFINITY;
        {
            float2 q2[8][4];            // q2[r][i] = (q[8r+i], q[8r+4+i])
            const float * qp = q + (size_t) (valid ? t : it.q0) * H * D + (size_t) h * D;
#pragma unroll
            for (int r8 = 0; r8 < 8; ++r8) {
                const float4 x0 = *(const float4 *) (qp + 8 * r8), x1 = *(const float4 *) (qp + 8 * r8 + 4);
                q2[r8][0] = make_float2(x0.x, x1.x); q2[r8][1] = make_float2(x0.y, x1.y);
                q2[r8][2] = make_float2(x0.z, x1.z); q2[r8][3] = make_float2(x0.w, x1.w);
            }
            for (int kt = it.k0; kt < it.k1; kt += KT) {
                const int nk = min(KT, it.k1 - kt);
                for (int i = threadIdx.x; i < KT * D / 8; i += NT) {
                    const int j = i / (D / 8), r8 = i % (D / 8);
                    float4 k0 = make_float4(0.f, 0.f, 0.f, 0.f), k1 = k0;
                    if (j < nk) {
                        k0 = ((const float4 *) (kg + (size_t) (kt + j) * D))[2 * r8];
                        k1 = ((const float4 *) (kg + (size_t) (kt + j) * D))[2 * r8 + 1];
                    }
                    ((float4 *) Ks[j])[2 * r8] = make_float4(k0.x, k1.x, k0.y, k1.y);
                    ((float4 *) Ks[j])[2 * r8 + 1] = make_float4(k0.z, k1.z, k0.w, k1.w);
                }
                __syncthreads();
#pragma unroll 2
                for (int j = 0; j < nk; ++j) {
                    float2 a[4];                // a[i] = (lane i, lane i+4)
#pragma unroll
                    for (int r8 = 0; r8 < 8; ++r8) {
                        const float4 p0 = ((const float4 *) Ks[j])[2 * r8];
                        const float4 p1 = ((const float4 *) Ks[j])[2 * r8 + 1];
                        const float2 kk[4] = { make_float2(p0.x, p0.y), make_float2(p0.z, p0.w),
                                               make_float2(p1.x, p1.y), make_float2(p1.z, p1.w) };
#pragma unroll
                        for (int i = 0; i < 4; ++i) a[i] = r8 == 0 ? __fmul2_rn(q2[0][i], kk[i]) : __ffma2_rn(q2[r8][i], kk[i], a[i]);
                    }
                    const int kj = kt + j;
                    float s;
                    if (kj < full_end) {
                        // ((a0+a1)+(a2+a3)) + ((a4+a5)+(a6+a7)), both halves at once
                        const float2 h = __fadd2_rn(__fadd2_rn(a[0], a[1]), __fadd2_rn(a[2], a[3]));
                        s = __fmul_rn(__fadd_rn(h.x, h.y), sc);
                    } else {
                        // hsum256: ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7))
                        const float tt = __fadd_rn(__fadd_rn(__fadd_rn(a[0].x, a[0].y), __fadd_rn(a[2].x, a[2].y)),
                                                   __fadd_rn(__fadd_rn(a[1].x, a[1].y), __fadd_rn(a[3].x, a[3].y)));
                        s = __fmul_rn(sc, tt);
                    }
                    if (kj >= lo && kj < hi) {
                        m = (m < s) ? s : m;
                        sc_base[(size_t) (kj - it.k0) * NT + threadIdx.x] = s;
                    }
                }
                __syncthreads();
            }
        }

        // ---- pass 2: e = exp256(s - m) over whole groups of 8, summed per lane in key order,
        // then the tail with the C library's exp; every e overwrites its score for pass 3
        float sum;
        {
            float vs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            float * sp = sc_base + (size_t) (lo - it.k0) * NT + threadIdx.x;
            const int nf = n & ~7;
            int j = 0;
            for (; j + 16 <= nf; j += 16) {                 // two groups per trip: 16 loads in flight
                float x[16];
#pragma unroll
                for (int l = 0; l < 16; ++l) x[l] = sp[(size_t) (j + l) * NT];
#pragma unroll
                for (int l = 0; l < 16; ++l) {
                    const float e = exp8(__fsub_rn(x[l], m));
                    vs[l & 7] = __fadd_rn(vs[l & 7], e);
                    sp[(size_t) (j + l) * NT] = e;
                }
            }
            for (; j < nf; j += 8) {
#pragma unroll
                for (int l = 0; l < 8; ++l) {
                    const float e = exp8(__fsub_rn(sp[(size_t) (j + l) * NT], m));
                    vs[l] = __fadd_rn(vs[l], e);
                    sp[(size_t) (j + l) * NT] = e;
                }
            }
            sum = __fadd_rn(__fadd_rn(__fadd_rn(vs[0], vs[4]), __fadd_rn(vs[2], vs[6])),
                            __fadd_rn(__fadd_rn(vs[1], vs[5]), __fadd_rn(vs[3], vs[7])));
            for (j = nf; j < n; ++j) {
                const float e = exp_tail(__fsub_rn(sp[(size_t) j * NT], m));
                sum = __fadd_rn(sum, e);
                sp[(size_t) j * NT] = e;
            }
        }
        const float inv = __fdiv_rn(1.0f, sum);

        // ---- pass 3: o[d] = fma(e_j * inv, v_j[d], o[d]) over the keys in order (dims in packed pairs)
        float2 o[D / 2];
#pragma unroll
        for (int d = 0; d < D / 2; ++d) o[d] = make_float2(0.0f, 0.0f);
        for (int kt = it.k0; kt < it.k1; kt += KT) {
            const int nk = min(KT, it.k1 - kt);
            for (int i = threadIdx.x; i < KT * D / 4; i += NT) {
                const int j = i / (D / 4), d4 = i % (D / 4);
                ((float4 *) Vs[j])[d4] = j < nk ? ((const float4 *) (vg + (size_t) (kt + j) * D))[d4]
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            __syncthreads();
            // this thread's weights for the tile's keys -> Cw (0 outside its range), then the values
#pragma unroll 8
            for (int j = 0; j < KT; ++j) {
                const int kj = kt + j;
                float c = 0.0f;
                if (j < nk && kj >= lo && kj < hi) c = __fmul_rn(sc_base[(size_t) (kj - it.k0) * NT + threadIdx.x], inv);
                Cw[j][threadIdx.x] = c;
            }
            __syncthreads();
            for (int j = 0; j < nk; ++j) {
                const int kj = kt + j;
                if (kj >= lo && kj < hi) {
                    const float c = Cw[j][threadIdx.x];
                    const float2 c2 = make_float2(c, c);
#pragma unroll
                    for (int d4 = 0; d4 < D / 4; ++d4) {
                        const float4 vv = ((const float4 *) Vs[j])[d4];
                        o[2 * d4]     = __ffma2_rn(c2, make_float2(vv.x, vv.y), o[2 * d4]);
                        o[2 * d4 + 1] = __ffma2_rn(c2, make_float2(vv.z, vv.w), o[2 * d4 + 1]);
                    }
                }
            }
            __syncthreads();
        }
        if (valid) {
            float4 * op = (float4 *) (out + (size_t) t * H * D + (size_t) h * D);
#pragma unroll
            for (int d4 = 0; d4 < D / 4; ++d4) {
                op[d4] = make_float4(o[2 * d4].x, o[2 * d4].y, o[2 * d4 + 1].x, o[2 * d4 + 1].y);
            }
        }
    }
}

// one qt-query tile per item; key range = document, or the band around the tile
void plan(const int32_t * start, const int32_t * len, int n_docs, int half, int qt, std::vector<Item> & items) {
    items.clear();
    for (int d = 0; d < n_docs; ++d) {
        const int lo = start[d], hi = lo + len[d];
        for (int q0 = lo; q0 < hi; q0 += qt) {
            const int q1 = std::min(hi, q0 + qt);
            Item it;
            it.q0 = q0;
            it.q1 = q1;
            it.doc = d;
            it.k0 = half < 0 ? lo : std::max(lo, q0 - half);
            it.k1 = half < 0 ? hi : std::min(hi, q1 - 1 + half + 1);
            items.push_back(it);
        }
    }
    std::stable_sort(items.begin(), items.end(),
                     [](const Item & a, const Item & b) { return (a.k1 - a.k0) > (b.k1 - b.k0); });
}

size_t n_items(const int32_t * len, int n_docs, int qt) {
    size_t n = 0;
    for (int d = 0; d < n_docs; ++d) n += (size_t) (len[d] + qt - 1) / qt;
    return n;
}

// Score scratch of the stored-score kernel: one slot per resident CTA, each
// holding (longest key range) x (threads) floats; threads sized for 4 heads per
// KV head (the most this build runs).  Slots: 4 per SM, at least one per SM,
// and no more than fit in 8 GiB.
constexpr int SLOTS_PER_SM = 4;
constexpr size_t SCRATCH_BUDGET = (size_t) 8 << 30;

struct Scratch {
    int slot_keys = 0;
    int slots = 0;
    size_t bytes = 0;
};

Scratch scratch_plan(const int32_t * len, int n_docs, int half) {
    int max_len = 0;
    for (int d = 0; d < n_docs; ++d) max_len = std::max(max_len, (int) len[d]);
    Scratch sp;
    sp.slot_keys = half < 0 ? max_len : std::min(max_len, QT3 + 2 * half);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    const size_t slot_bytes = (size_t) sp.slot_keys * QT3 * 4 * sizeof(float);
    size_t slots = (size_t) sms * SLOTS_PER_SM;
    if (slot_bytes > 0 && slots * slot_bytes > SCRATCH_BUDGET) slots = std::max((size_t) sms, SCRATCH_BUDGET / slot_bytes);
    sp.slots = (int) slots;
    sp.bytes = slots * slot_bytes;
    return sp;
}

} // namespace attn
} // namespace nxk

using namespace nxk;

extern "C" {

size_t nxk_attention_workspace(const int32_t * h_doc_len, int n_docs, int half) {
    const size_t items = attn::n_items(h_doc_len, n_docs, attn::QT3) * sizeof(attn::Item);
    return (items + 255) / 256 * 256 + attn::scratch_plan(h_doc_len, n_docs, half).bytes;
}

int nxk_attention(const float * q, const float * k, const float * v, int T, int H, int G, int D, int half,
                  const float * scale, const int32_t *, const int32_t * doc_start, const int32_t * doc_len,
                  int n_docs, const int32_t * h_doc_start, const int32_t * h_doc_len, void * workspace,
                  size_t workspace_bytes, float * out, void * stream) {
    if (T < 0 || H <= 0 || G <= 0 || H % G || D != attn::D || n_docs < 0) return NXK_EINVAL;
    const int rep = H / G;
    if (rep != 1 && rep != 2 && rep != 4) return NXK_EINVAL;     // 64 * rep threads per block
    if (T == 0 || n_docs == 0) return NXK_OK;
    std::vector<attn::Item> items;
    attn::plan(h_doc_start, h_doc_len, n_docs, half, attn::QT3, items);
    const attn::Scratch sp = attn::scratch_plan(h_doc_len, n_docs, half);
    const size_t item_bytes = (items.size() * sizeof(attn::Item) + 255) / 256 * 256;
    if (!workspace || workspace_bytes < item_bytes + sp.bytes) return NXK_EINVAL;
    cudaStream_t s = (cudaStream_t) stream;
    // from pageable memory: staged by CUDA before the call returns, so `items` may go
    if (cudaMemcpyAsync(workspace, items.data(), items.size() * sizeof(attn::Item), cudaMemcpyHostToDevice, s) !=
        cudaSuccess) {
        return NXK_ELAUNCH;
    }
    const attn::Item * it = (const attn::Item *) workspace;
    float * scratch = (float *) ((char *) workspace + item_bytes);
    const long long n_units = (long long) items.size() * G;
    if (n_units > INT32_MAX) return NXK_EINVAL;
    // persistent grid: no more CTAs than can be resident at once (each owns a scratch slot)
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    switch (rep) {
        case 1: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn::attn_scored_kernel<1>, attn::QT3, 0); break;
        case 2: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn::attn_scored_kernel<2>, attn::QT3 * 2, 0); break;
        default: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn::attn_scored_kernel<4>, attn::QT3 * 4, 0); break;
    }
    const long long resident = (long long) std::max(per_sm, 1) * std::max(sms, 1);
    const unsigned grid = (unsigned) std::min<long long>(std::min<long long>(n_units, sp.slots), resident);
    switch (rep) {
        case 1: attn::attn_scored_kernel<1><<<grid, attn::QT3 * 1, 0, s>>>(q, k, v, out, it, (int) n_units, G, scale,
                    doc_start, doc_len, T, H, half, scratch, sp.slot_keys); break;
        case 2: attn::attn_scored_kernel<2><<<grid, attn::QT3 * 2, 0, s>>>(q, k, v, out, it, (int) n_units, G, scale,
                    doc_start, doc_len, T, H, half, scratch, sp.slot_keys); break;
        default: attn::attn_scored_kernel<4><<<grid, attn::QT3 * 4, 0, s>>>(q, k, v, out, it, (int) n_units, G, scale,
                    doc_start, doc_len, T, H, half, scratch, sp.slot_keys); break;
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}

} // extern "C"

// ---------------------------------------------------------------------------
// nxk_attention_noalloc: the same attention without a caller-provided workspace.
//
// For callers that cannot allocate device memory at the point of the call: a
// host that hands this library pointers into a pool it manages itself (a
// serving framework's arena, a memory-mapped buffer shared with another
// process) and forbids cudaMalloc after start-up, or code that must not touch
// the allocator at all (a real-time path where cudaMalloc may block on the
// device).  nxk_attention needs a workspace for its work plan; this variant
// keeps the plan in a fixed array compiled into the library instead.
//
// The plan lives in g_noalloc_items, a file-scope __device__ array of
// NOALLOC_MAX_ITEMS items (20 bytes each, 2.5 MiB on every device that loads
// the library, held until exit).  One item is one 32-query tile of one
// document, so a batch may hold at most NOALLOC_MAX_ITEMS tiles (sum over the
// documents of ceil(len / 32)); larger batches are rejected with NXK_EINVAL and
// a message.  The plan is written on the device by a small planner kernel from
// doc_start / doc_len, in document order; every entry the attention kernel
// reads is written by the same call first, so nothing needs clearing.  All calls
// share the array: two calls whose work overlaps on the GPU (different streams,
// no ordering between them) race on it and must not be issued.
//
// Host code cannot use the array's name as a device address; its address is
// looked up once per device with cudaGetSymbolAddress on the first call made
// with that device current.  That first call should therefore come before any
// CUDA stream capture.  No device memory is allocated, and no host memory
// either.
// ---------------------------------------------------------------------------
#include <cstdio>
#include <mutex>

namespace nxk {
namespace attn {

constexpr int NOALLOC_MAX_ITEMS = 1 << 17;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) Item g_noalloc_items[NOALLOC_MAX_ITEMS];

// One block: each thread owns a contiguous run of documents, counts their tiles,
// the block scans the counts, then every thread writes its documents' items.
__global__ void __launch_bounds__(1024) plan_kernel(Item * __restrict__ items, const int32_t * __restrict__ doc_start,
                                                    const int32_t * __restrict__ doc_len, int n_docs, int half) {
    __shared__ int part[1024];
    const int tid = threadIdx.x, nt = blockDim.x;
    const int per = (n_docs + nt - 1) / nt;
    const int d0 = min(n_docs, tid * per), d1 = min(n_docs, d0 + per);
    int cnt = 0;
    for (int d = d0; d < d1; ++d) cnt += (doc_len[d] + QT - 1) / QT;
    part[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < nt; off <<= 1) {        // inclusive scan (Hillis-Steele)
        const int add = tid >= off ? part[tid - off] : 0;
        __syncthreads();
        part[tid] += add;
        __syncthreads();
    }
    int o = part[tid] - cnt;
    for (int d = d0; d < d1; ++d) {
        const int lo = doc_start[d], hi = lo + doc_len[d];
        for (int q0 = lo; q0 < hi; q0 += QT) {
            Item it;
            it.q0 = q0;
            it.q1 = min(hi, q0 + QT);
            it.doc = d;
            it.k0 = half < 0 ? lo : max(lo, q0 - half);
            it.k1 = half < 0 ? hi : min(hi, it.q1 - 1 + half + 1);
            items[o++] = it;
        }
    }
}

// address of g_noalloc_items on the current device (looked up once per device)
Item * noalloc_items() {
    static std::mutex mu;
    static Item * ptr[NOALLOC_MAX_DEVICES] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!ptr[dev]) {
        void * p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_items) != cudaSuccess) {
            fprintf(stderr, "nxk_attention_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
                    cudaGetErrorString(cudaGetLastError()));
            return nullptr;
        }
        ptr[dev] = (Item *) p;
    }
    return ptr[dev];
}

} // namespace attn
} // namespace nxk

extern "C" int nxk_attention_noalloc(const float * q, const float * k, const float * v, int T, int H, int G, int D,
                                     int half, const float * scale, const int32_t * doc_start,
                                     const int32_t * doc_len, int n_docs, const int32_t * h_doc_len, float * out,
                                     void * stream) {
    using namespace nxk::attn;
    if (T < 0 || H <= 0 || G <= 0 || H % G || D != nxk::attn::D || n_docs < 0 || !h_doc_len) return NXK_EINVAL;
    const int rep = H / G;
    if (rep != 1 && rep != 2 && rep != 4) return NXK_EINVAL;
    if (T == 0 || n_docs == 0) return NXK_OK;
    long long n_items = 0;
    for (int d = 0; d < n_docs; ++d) {
        if (h_doc_len[d] <= 0) return NXK_EINVAL;
        n_items += (h_doc_len[d] + QT - 1) / QT;
    }
    if (n_items > NOALLOC_MAX_ITEMS) {
        fprintf(stderr, "nxk_attention_noalloc: %lld query tiles exceed the fixed plan of %d "
                        "(at most %d tiles of %d queries per call)\n", n_items, NOALLOC_MAX_ITEMS,
                NOALLOC_MAX_ITEMS, QT);
        return NXK_EINVAL;
    }
    Item * items = noalloc_items();
    if (!items) return NXK_ELAUNCH;
    cudaStream_t s = (cudaStream_t) stream;
    plan_kernel<<<1, 1024, 0, s>>>(items, doc_start, doc_len, n_docs, half);
    const dim3 grid((unsigned) n_items, (unsigned) G);
    switch (rep) {
        case 1: attn_kernel<1><<<grid, QT * 2, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
        case 2: attn_kernel<2><<<grid, QT * 4, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
        default: attn_kernel<4><<<grid, QT * 8, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}
