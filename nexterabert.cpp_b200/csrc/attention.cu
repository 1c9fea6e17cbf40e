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
#include "attention_plan.hpp"
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
// Tiled kernel (used by nxk_attention).  Same arithmetic and order as
// attn_kernel; what changes is which thread does which operation.  A work unit
// is (64-query tile, KV head g) with the H/G query heads that share g; its
// scores live in a per-CTA scratch slot in global memory, [key - k0][query,
// head], L2-resident for the band layers.
//   pass 1  every score once, in register tiles: a thread owns 4 queries x 4
//           keys and runs the 8 lane chains of NEXTERA_DOT64 one lane after
//           the other (dims l, 8 + l, ..., 56 + l), folding each finished lane
//           into the full-group tree ((a0+a1)+(a2+a3)) + ((a4+a5)+(a6+a7)) as
//           it completes.  Queries and keys sit transposed in shared memory
//           ([dim][query], [dim][key]), so one float4 of each feeds 16 FMAs,
//           issued as 8 packed f32x2 multiply-adds (one query against a key
//           pair).
//           Partial maxima over the keys in whole groups go to shared memory.
//   pass 2  two threads per (query, head): the tail keys (the n % 8 after the
//           last whole group) are recomputed with the hsum256 tree, then the
//           exp-sum runs with lanes 0-3 of every group on one thread and lanes
//           4-7 on the other, each exp written over its score; 1 / sum.
//   pass 3  register tiles of 4 queries x 8 dims: o = fma(e * inv, v, o) over
//           the keys in order; the tile's weights are staged in shared memory,
//           zero outside a query's range (fma(0, v, o) leaves o unchanged).
// ---------------------------------------------------------------------------


template <int REP>
constexpr int tiled_smem_floats() {
    return REP * D * QT3 + D * KT + KT * D + KT * QT3 * REP + QT3 * REP;
}

template <int REP>
__global__ void __launch_bounds__(128 * REP, 4 / REP)
attn_tiled_kernel(const float * __restrict__ q, const float * __restrict__ k, const float * __restrict__ v,
                  float * __restrict__ out, const Item * __restrict__ items, int n_units, int G,
                  const float * __restrict__ scale, const int32_t * __restrict__ doc_start,
                  const int32_t * __restrict__ doc_len, int T, int Tk, int koff, int H, int half,
                  float * __restrict__ scratch, int slot_keys) {
    constexpr int NT = 128 * REP;
    constexpr int NQH = QT3 * REP;                                  // (query, head) pairs of a unit
    // pass-2 ring tile (band layers): two stages of [KT2][NQH] over the shared memory of pass 1
    // (all of it but invs)
    constexpr int KT2 = 2 * 64 * NQH <= REP * D * QT3 + 2 * D * KT + KT * NQH ? 64 : 32;
    static_assert(2 * KT2 * NQH <= REP * D * QT3 + 2 * D * KT + KT * NQH, "pass-2 ring overlaps invs");
    extern __shared__ __align__(16) float smem[];
    float (*Qs)[QT3] = reinterpret_cast<float (*)[QT3]>(smem);                       // [REP * D][QT3]
    float (*Ks)[KT] = reinterpret_cast<float (*)[KT]>(smem + REP * D * QT3);         // [D][KT]
    // [KT][D] after Ks: only the rings of passes 2-3 use it (a 64-key pass-2 tile needs it)
    float (*Cw)[NQH] = reinterpret_cast<float (*)[NQH]>(smem + REP * D * QT3 + 2 * D * KT);   // [KT][NQH]
    float * mx = &Cw[0][0];                                        // [8][NQH], passes 1-2 only
    float * invs = smem + REP * D * QT3 + 2 * D * KT + KT * NQH;    // [NQH]
    float * sc_base = scratch + (size_t) blockIdx.x * slot_keys * NQH;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hq = warp >> 2, w4 = warp & 3;                       // 4 warps per query head
    const int qa = 32 * (w4 & 1) + 4 * (lane & 7);                 // the thread's 4 queries
    const int kb = 16 * (w4 >> 1) + 4 * (lane >> 3);               // pass 1: its 4 keys of a tile
    const int kgrp = kb >> 2;                                      // 0..7
    const int db = 32 * (w4 >> 1) + 8 * (lane >> 3);               // pass 3: its 8 dims
    const int p_qh = tid >> 1, p_sub = tid & 1;                    // pass 2: the pair
    const int p_h = p_qh / QT3, p_qi = p_qh % QT3;
    const int c_qh = tid % NQH;                                    // pass 3: weight column it fills

    for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const Item it = items[u / G];
        const int g = u % G;
        const float sc = scale[it.doc];
        const int dlo = doc_start[it.doc], dhi = dlo + doc_len[it.doc];
        // key row j (relative to query row 0, may be negative) of head g is at kg + j * D
        const float * kg = k + ((ptrdiff_t) g * Tk + koff) * D;
        const float * vg = v + ((ptrdiff_t) g * Tk + koff) * D;
        // the key range [lo, hi) of query row q0 + qi (empty past q1)
        auto range = [&](int qi, int & lo, int & hi) {
            const int t = it.q0 + qi;
            lo = dlo;
            hi = dhi;
            if (half >= 0) {
                lo = max(lo, t - half);
                hi = min(hi, t + half + 1);
            }
            if (t >= it.q1) { lo = it.k0; hi = it.k0; }
        };

        // queries, transposed (zeros past q1); the previous unit's last reads of Qs
        // are in pass 2, which a barrier closes
        for (int i = tid; i < REP * QT3 * (D / 4); i += NT) {
            const int qi = i % QT3, r = i / QT3;
            const int h = r / (D / 4), d4 = r % (D / 4);
            const int t = it.q0 + qi;
            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < it.q1) x = *(const float4 *) (q + ((size_t) t * H + (size_t) g * REP + h) * D + 4 * d4);
            Qs[h * D + 4 * d4 + 0][qi] = x.x;
            Qs[h * D + 4 * d4 + 1][qi] = x.y;
            Qs[h * D + 4 * d4 + 2][qi] = x.z;
            Qs[h * D + 4 * d4 + 3][qi] = x.w;
        }

        // ---- pass 1
        int lo4[4], hi4[4], fe4[4];
        float ml[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            int lo, hi;
            range(qa + a, lo, hi);
            lo4[a] = lo;
            hi4[a] = hi;
            fe4[a] = lo + ((hi - lo) & ~7);
            ml[a] = -INFINITY;
        }
        // keys that any of this warp's 32 queries sees: [w_lo, w_hi) (ranges grow with the row)
        int w_lo = it.k0, w_hi = it.k0;
        {
            const int qb = 32 * (w4 & 1);
            const int last = min(qb + 31, it.q1 - it.q0 - 1);
            if (last >= qb) {
                int l0, h0, l1, h1;
                range(qb, l0, h0);
                range(last, l1, h1);
                w_lo = l0;
                w_hi = h1;
            }
        }
        const float (*Qh)[QT3] = Qs + hq * D;
        // key tiles: the next tile's rows arrive by cp.async in the [KT][D] region that pass 1 does
        // not otherwise use (row j's float4 d4 at j * D + 4 * (d4 ^ (j & 15)), so that the
        // transposing reads below, 8 rows per phase, hit distinct banks) while this one is used
        float * Kraw = smem + REP * D * QT3 + D * KT;
        constexpr int KPT = KT * D / 4 / NT;
        auto kissue = [&](int kt) {
            for (int i = tid; i < KT * D / 4; i += NT) {
                const int j = i / (D / 4), d4 = i % (D / 4);
                float * dst = Kraw + j * D + 4 * (d4 ^ (j & 15));
                if (kt + j < it.k1) cp_async16(dst, kg + (ptrdiff_t) (kt + j) * D + 4 * d4);
                else *(float4 *) dst = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            cp_async_commit();
        };
        // key tiles last to first: the maximum does not depend on the order, and pass 2 then starts
        // on the scores written last, which are the likeliest to be still in L2
        const int kt_last = it.k0 + (it.k1 - 1 - it.k0) / KT * KT;
        kissue(kt_last);
        for (int kt = kt_last; kt >= it.k0; kt -= KT) {
            const int nk = min(KT, it.k1 - kt);
            cp_async_wait<0>();
            __syncthreads();                                       // Kraw landed; Ks free; Qs written
#pragma unroll
            for (int z = 0; z < KPT; ++z) {
                const int i = tid + z * NT, j = i % KT, d4 = i / KT;
                const float4 x = *(const float4 *) (Kraw + j * D + 4 * (d4 ^ (j & 15)));
                Ks[4 * d4 + 0][j] = x.x;
                Ks[4 * d4 + 1][j] = x.y;
                Ks[4 * d4 + 2][j] = x.z;
                Ks[4 * d4 + 3][j] = x.w;
            }
            __syncthreads();                                       // Ks written; Kraw free
            if (kt - KT >= it.k0) kissue(kt - KT);
            // a warp whose 32 queries see none of its 16 keys (band layers) only stores zeros
            const bool live = kt + kb - 4 * (lane >> 3) < w_hi && kt + kb - 4 * (lane >> 3) + 16 > w_lo;
            // The 4 x 4 tile in packed pairs, so that one f32x2 multiply-add advances two scores'
            // chains (each half an IEEE fma, the same bits as two scalar ones): P[A][B][s] holds
            // query 2A + s against keys 2B and 2B + 1, the query's value in both halves.  Score
            // (a, b) is component b & 1 of P[a >> 1][b >> 1][a & 1].
            float2 y0123[2][2][2], x45[2][2][2], x6[2][2][2], x01[2][2][2], x2[2][2][2], x0[2][2][2], x4[2][2][2];
#pragma unroll
            for (int A = 0; A < 2; ++A)
#pragma unroll
                for (int B = 0; B < 2; ++B)
#pragma unroll
                    for (int s2 = 0; s2 < 2; ++s2) x0[A][B][s2] = make_float2(0.0f, 0.0f);
            if (live) {
            const float2 sc2 = make_float2(sc, sc);
#pragma unroll
            for (int l = 0; l < 8; ++l) {
                float2 acc[2][2][2];
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int d = 8 * r + l;
                    const float4 qv = *(const float4 *) &Qh[d][qa];
                    const float4 kv = *(const float4 *) &Ks[d][kb];
                    const float2 qp[2][2] = {{make_float2(qv.x, qv.x), make_float2(qv.y, qv.y)},
                                             {make_float2(qv.z, qv.z), make_float2(qv.w, qv.w)}};
                    const float2 kp2[2] = {make_float2(kv.x, kv.y), make_float2(kv.z, kv.w)};
#pragma unroll
                    for (int A = 0; A < 2; ++A)
#pragma unroll
                        for (int B = 0; B < 2; ++B)
#pragma unroll
                            for (int s2 = 0; s2 < 2; ++s2)
                                acc[A][B][s2] = r == 0 ? __fmul2_rn(qp[A][s2], kp2[B])
                                                       : __ffma2_rn(qp[A][s2], kp2[B], acc[A][B][s2]);
                }
#pragma unroll
                for (int A = 0; A < 2; ++A)
#pragma unroll
                    for (int B = 0; B < 2; ++B)
#pragma unroll
                        for (int s2 = 0; s2 < 2; ++s2) {
                            const float2 c = acc[A][B][s2];
                            switch (l) {
                                case 0: x0[A][B][s2] = c; break;
                                case 1: x01[A][B][s2] = __fadd2_rn(x0[A][B][s2], c); break;
                                case 2: x2[A][B][s2] = c; break;
                                case 3: y0123[A][B][s2] = __fadd2_rn(x01[A][B][s2], __fadd2_rn(x2[A][B][s2], c)); break;
                                case 4: x4[A][B][s2] = c; break;
                                case 5: x45[A][B][s2] = __fadd2_rn(x4[A][B][s2], c); break;
                                case 6: x6[A][B][s2] = c; break;
                                default:                           // the finished score
                                    x0[A][B][s2] = __fmul2_rn(__fadd2_rn(y0123[A][B][s2],
                                                                         __fadd2_rn(x45[A][B][s2],
                                                                                    __fadd2_rn(x6[A][B][s2], c))),
                                                              sc2);
                            }
                        }
            }
            }
            // stored: the score inside the query's key range, 0 outside (pass 3 reads them as weights)
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2) {
                const int kj = kt + kb + b2;
                if (kb + b2 < nk) {
                    float sv[4];
#pragma unroll
                    for (int a = 0; a < 4; ++a) {
                        const float2 pr = x0[a >> 1][b2 >> 1][a & 1];
                        const float x = (b2 & 1) ? pr.y : pr.x;
                        const bool in = kj >= lo4[a] && kj < hi4[a];
                        sv[a] = in ? x : 0.0f;
                        if (kj >= lo4[a] && kj < fe4[a]) ml[a] = (ml[a] < x) ? x : ml[a];
                    }
                    *(float4 *) (sc_base + (size_t) (kj - it.k0) * NQH + hq * QT3 + qa) =
                        make_float4(sv[0], sv[1], sv[2], sv[3]);
                }
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) mx[kgrp * NQH + hq * QT3 + qa + a] = ml[a];
        __syncthreads();

        // ---- pass 2
        {
            int lo, hi;
            range(p_qi, lo, hi);
            const int n = hi - lo, fe = lo + (n & ~7);
            float m = -INFINITY;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float x = mx[r * NQH + p_qh];
                m = (m < x) ? x : m;
            }
            float * sp = sc_base + p_qh;
            if (p_sub == 0) {
                // tail keys: hsum256 ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)), then * scale
                for (int kj = fe; kj < hi; ++kj) {
                    const float4 * kr = (const float4 *) (kg + (ptrdiff_t) kj * D);
                    float a8[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const float4 k0 = kr[2 * r], k1 = kr[2 * r + 1];
                        const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
                        for (int l = 0; l < 8; ++l) {
                            const float qv = Qs[p_h * D + 8 * r + l][p_qi];
                            a8[l] = r == 0 ? __fmul_rn(qv, kk[l]) : __fmaf_rn(qv, kk[l], a8[l]);
                        }
                    }
                    const float tt = __fadd_rn(__fadd_rn(__fadd_rn(a8[0], a8[4]), __fadd_rn(a8[2], a8[6])),
                                               __fadd_rn(__fadd_rn(a8[1], a8[5]), __fadd_rn(a8[3], a8[7])));
                    const float s = __fmul_rn(sc, tt);
                    sp[(size_t) (kj - it.k0) * NQH] = s;
                    m = (m < s) ? s : m;
                }
            }
            {
                const float o = __shfl_xor_sync(0xffffffffu, m, 1);
                m = (m < o) ? o : m;
            }
            // whole groups: this thread's lanes 4 * sub .. 4 * sub + 3, summed per lane in key order;
            // each exp is written back over its score
            float2 vs2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};   // lanes (0,1), (2,3) of this thread
            const int ng = n >> 3;
            if (half < 0) {
                // full layers (long key ranges): each thread streams its own scores, 16 loads in flight
                float * gp = sp + (size_t) (lo - it.k0 + 4 * p_sub) * NQH;
                int gi = 0;
                for (; gi + 4 <= ng; gi += 4) {
                    float x[16];
#pragma unroll
                    for (int z = 0; z < 16; ++z) x[z] = gp[(size_t) (8 * (gi + (z >> 2)) + (z & 3)) * NQH];
#pragma unroll
                    for (int z = 0; z < 16; z += 2) {           // two exps per packed evaluation; s - m <= 0
                        const float2 e = exp8x2<true>(__fadd2_rn(make_float2(x[z], x[z + 1]), make_float2(-m, -m)));
                        vs2[(z >> 1) & 1] = __fadd2_rn(vs2[(z >> 1) & 1], e);
                        gp[(size_t) (8 * (gi + (z >> 2)) + (z & 3)) * NQH] = e.x;
                        gp[(size_t) (8 * (gi + ((z + 1) >> 2)) + ((z + 1) & 3)) * NQH] = e.y;
                    }
                }
                for (; gi < ng; ++gi) {
#pragma unroll
                    for (int z = 0; z < 4; z += 2) {
                        float * p0 = gp + (size_t) (8 * gi + z) * NQH, * p1 = p0 + NQH;
                        const float2 e = exp8x2<true>(__fadd2_rn(make_float2(*p0, *p1), make_float2(-m, -m)));
                        vs2[z >> 1] = __fadd2_rn(vs2[z >> 1], e);
                        *p0 = e.x;
                        *p1 = e.y;
                    }
                }
            } else {
                // band layers (a few hundred keys, where the streamed loads above wait on their
                // latency): the unit's scores come through a 2-stage cp.async ring of [KT2 keys][NQH]
                // tiles over the shared memory of pass 1, free once every thread has read the maxima
                // and finished its tail keys
                __syncthreads();
                const int lb = lo + 4 * p_sub;                     // the thread's first key of group 0
                float * ring = smem;                               // [2][KT2][NQH]
                auto issue2 = [&](int kt, int st) {
                    const int nk = min(KT2, it.k1 - kt);
                    const float * src = sc_base + (size_t) (kt - it.k0) * NQH;
                    float * dst = ring + st * KT2 * NQH;
                    for (int i = tid; i < nk * (NQH / 4); i += NT) cp_async16(dst + 4 * i, src + 4 * i);
                    cp_async_commit();
                };
                issue2(it.k0, 0);
                int st2 = 0;
                for (int kt = it.k0; kt < it.k1; kt += KT2, st2 ^= 1) {
                    const int nk = min(KT2, it.k1 - kt);
                    if (kt + KT2 < it.k1) {
                        issue2(kt + KT2, st2 ^ 1);
                        cp_async_wait<1>();
                    } else {
                        cp_async_wait<0>();
                    }
                    __syncthreads();
                    const float * se = ring + st2 * KT2 * NQH + p_qh;
                    // groups i whose keys lb + 8i .. lb + 8i + 3 meet [kt, kt + nk)
                    const int i0 = max(0, (kt - lb + 4) >> 3);
                    const int i1 = min(ng, ((kt + nk - 1 - lb) >> 3) + 1);
                    for (int i = i0; i < i1; ++i) {
#pragma unroll
                        for (int z = 0; z < 4; z += 2) {
                            const int ka = lb + 8 * i + z;
                            const bool ia = ka >= kt && ka < kt + nk, ib = ka + 1 >= kt && ka + 1 < kt + nk;
                            const float xa = ia ? se[(ka - kt) * NQH] : m, xb = ib ? se[(ka + 1 - kt) * NQH] : m;
                            const float2 e = exp8x2<true>(__fadd2_rn(make_float2(xa, xb), make_float2(-m, -m)));
                            float * gq = sp + (size_t) (ka - it.k0) * NQH;
                            if (ia) {
                                vs2[z >> 1].x = __fadd_rn(vs2[z >> 1].x, e.x);
                                gq[0] = e.x;
                            }
                            if (ib) {
                                vs2[z >> 1].y = __fadd_rn(vs2[z >> 1].y, e.y);
                                gq[NQH] = e.y;
                            }
                        }
                    }
                    __syncthreads();
                }
            }
            // sum = ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)); lanes 4-7 are the partner's 0-3
            const float vs[4] = {vs2[0].x, vs2[0].y, vs2[1].x, vs2[1].y};
            float w[4];
#pragma unroll
            for (int z = 0; z < 4; ++z) w[z] = __shfl_xor_sync(0xffffffffu, vs[z], 1);
            if (p_sub == 0) {
                float sum = __fadd_rn(__fadd_rn(__fadd_rn(vs[0], w[0]), __fadd_rn(vs[2], w[2])),
                                      __fadd_rn(__fadd_rn(vs[1], w[1]), __fadd_rn(vs[3], w[3])));
                for (int kj = fe; kj < hi; ++kj) {
                    float * p = sp + (size_t) (kj - it.k0) * NQH;
                    const float e = exp_tail(__fsub_rn(*p, m));
                    sum = __fadd_rn(sum, e);
                    *p = e;
                }
                invs[p_qh] = __fdiv_rn(1.0f, sum);
            }
        }
        __syncthreads();

        // ---- pass 3: o = fma(e * inv, v, o) over the keys in order; e is 0 outside a query's range,
        // and fma(0, v, o) leaves o unchanged.  Value rows and exps arrive by cp.async in a 2-stage
        // ring laid over the shared memory of passes 1-2 (invs excepted).
        float2 o[4][4];                                            // [query][dim pair]
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int z = 0; z < 4; ++z) o[a][z] = make_float2(0.0f, 0.0f);
        float inv4[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) inv4[a] = invs[hq * QT3 + qa + a];
        constexpr int STAGE = KT * D + KT * NQH;                   // V tile [KT][D], exps [KT][NQH]
        static_assert(2 * STAGE <= REP * D * QT3 + 2 * D * KT + KT * NQH, "pass-3 ring overlaps invs");
        auto issue = [&](int kt, int st) {
            const int nk = min(KT, it.k1 - kt);
            float * sv = smem + st * STAGE;
            float * se = sv + KT * D;
            for (int i = tid; i < nk * (D / 4); i += NT) {
                const int j = i / (D / 4), d4 = i % (D / 4);
                cp_async16(sv + j * D + 4 * d4, vg + (ptrdiff_t) (kt + j) * D + 4 * d4);
            }
            const float * eg = sc_base + (size_t) (kt - it.k0) * NQH;
            for (int i = tid; i < nk * (NQH / 4); i += NT) cp_async16(se + 4 * i, eg + 4 * i);
            cp_async_commit();
        };
        issue(it.k0, 0);
        int st = 0;
        for (int kt = it.k0; kt < it.k1; kt += KT, st ^= 1) {
            const int nk = min(KT, it.k1 - kt);
            if (kt + KT < it.k1) {
                issue(kt + KT, st ^ 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
            const float * sv = smem + st * STAGE;
            const float * se = sv + KT * D;
            // only the keys some query of this warp sees (band layers skip the rest)
            const int jlo = max(0, w_lo - kt), jhi = min(nk, w_hi - kt);
#pragma unroll 2
            for (int j = jlo; j < jhi; ++j) {
                const float4 e = *(const float4 *) (se + j * NQH + hq * QT3 + qa);
                const float2 c01 = __fmul2_rn(make_float2(e.x, e.y), make_float2(inv4[0], inv4[1]));
                const float2 c23 = __fmul2_rn(make_float2(e.z, e.w), make_float2(inv4[2], inv4[3]));
                const float cc[4] = {c01.x, c01.y, c23.x, c23.y};
                const float4 v0 = *(const float4 *) (sv + j * D + db);
                const float4 v1 = *(const float4 *) (sv + j * D + db + 4);
                const float2 vv[4] = {make_float2(v0.x, v0.y), make_float2(v0.z, v0.w),
                                      make_float2(v1.x, v1.y), make_float2(v1.z, v1.w)};
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float2 c2 = make_float2(cc[a], cc[a]);
#pragma unroll
                    for (int z = 0; z < 4; ++z) o[a][z] = __ffma2_rn(c2, vv[z], o[a][z]);
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int t = it.q0 + qa + a;
            if (t < it.q1) {
                float4 * op = (float4 *) (out + ((size_t) t * H + (size_t) g * REP + hq) * D + db);
                op[0] = make_float4(o[a][0].x, o[a][0].y, o[a][1].x, o[a][1].y);
                op[1] = make_float4(o[a][2].x, o[a][2].y, o[a][3].x, o[a][3].y);
            }
        }
    }
}

// one qt-query tile per item; key range = document, or the band around the tile
// Query rows are limited to [0, T): a document may reach outside them (a shard of a longer
// sequence, whose keys lie in a gathered or halo-extended K / V).
void plan(const int32_t * start, const int32_t * len, int n_docs, int half, int qt, int T, std::vector<Item> & items) {
    items.clear();
    for (int d = 0; d < n_docs; ++d) {
        const int lo = start[d], hi = lo + len[d];
        for (int q0 = std::max(lo, 0); q0 < std::min(hi, T); q0 += qt) {
            const int q1 = std::min(std::min(hi, T), q0 + qt);
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
    for (int d = 0; d < n_docs; ++d) n += (size_t) (((long long) len[d] + qt - 1) / qt);
    return n;
}

// Score scratch of the tiled kernel: one slot per resident CTA, each holding
// (longest key range) x (query, head) floats, sized for 4 query heads per KV
// head (the most this build runs).  Slots: 4 per SM, at least one per SM,
// and no more than fit in 24 GiB (a 65,536-key range needs 64 MiB per slot).
constexpr int SLOTS_PER_SM = 4;
constexpr size_t SCRATCH_BUDGET = (size_t) 24 << 30;

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

int launch_planned(const float * q, const float * k, const float * v, int T, int Tk, int koff, int H, int G,
                   int half, const float * scale, const int32_t * doc_start, const int32_t * doc_len,
                   const Item * d_items, size_t n_items_, const Scratch & sp, float * scratch, float * out,
                   cudaStream_t s) {
    const int rep = H / G;
    if (rep != 1 && rep != 2 && rep != 4) return NXK_EINVAL;     // 128 * rep threads per block
    if (n_items_ == 0) return NXK_OK;
    const Item * it = d_items;
    const long long n_units = (long long) n_items_ * G;
    if (n_units > INT32_MAX) return NXK_EINVAL;
    // persistent grid: no more CTAs than can be resident at once (each owns a scratch slot)
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto launch = [&](auto kernel, int rep_) {
        const int threads = 128 * rep_;
        const size_t smem_bytes = sizeof(float) * (size_t) (rep_ == 1 ? tiled_smem_floats<1>()
                                                            : rep_ == 2 ? tiled_smem_floats<2>()
                                                                        : tiled_smem_floats<4>());
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem_bytes);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem_bytes);
        const long long resident = (long long) std::max(per_sm, 1) * std::max(sms, 1);
        const unsigned grid = (unsigned) std::min<long long>(std::min<long long>(n_units, sp.slots), resident);
        kernel<<<grid, threads, smem_bytes, s>>>(q, k, v, out, it, (int) n_units, G, scale, doc_start, doc_len, T, Tk,
                                                 koff, H, half, scratch, sp.slot_keys);
    };
    switch (rep) {
        case 1: launch(attn_tiled_kernel<1>, 1); break;
        case 2: launch(attn_tiled_kernel<2>, 2); break;
        default: launch(attn_tiled_kernel<4>, 4); break;
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
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
    return nxk_attention_kv(q, k, v, T, T, 0, H, G, D, half, scale, doc_start, doc_len, n_docs, h_doc_start,
                            h_doc_len, workspace, workspace_bytes, out, stream);
}

int nxk_attention_kv(const float * q, const float * k, const float * v, int T, int Tk, int koff, int H, int G,
                     int D, int half, const float * scale, const int32_t * doc_start, const int32_t * doc_len,
                     int n_docs, const int32_t * h_doc_start, const int32_t * h_doc_len, void * workspace,
                     size_t workspace_bytes, float * out, void * stream) {
    if (T < 0 || Tk < 0 || koff < 0 || koff > Tk || H <= 0 || G <= 0 || H % G || D != attn::D || n_docs < 0)
        return NXK_EINVAL;

    const int rep = H / G;
    if (rep != 1 && rep != 2 && rep != 4) return NXK_EINVAL;     // 64 * rep threads per block
    if (T == 0 || n_docs == 0) return NXK_OK;
    std::vector<attn::Item> items;
    attn::plan(h_doc_start, h_doc_len, n_docs, half, attn::QT3, T, items);
    if (items.empty()) return NXK_OK;
    // every key a tile touches must lie in [-koff, Tk - koff) relative to query row 0
    for (const attn::Item & x : items) {
        if (x.k0 < -koff || x.k1 > Tk - koff) return NXK_EINVAL;
    }
    const attn::Scratch sp = attn::scratch_plan(h_doc_len, n_docs, half);
    const size_t item_bytes = (items.size() * sizeof(attn::Item) + 255) / 256 * 256;
    if (!workspace || workspace_bytes < item_bytes + sp.bytes) return NXK_EINVAL;
    cudaStream_t s = (cudaStream_t) stream;
    // from pageable memory: staged by CUDA before the call returns, so `items` may go
    if (cudaMemcpyAsync(workspace, items.data(), items.size() * sizeof(attn::Item), cudaMemcpyHostToDevice, s) !=
        cudaSuccess) {
        return NXK_ELAUNCH;
    }
    return attn::launch_planned(q, k, v, T, Tk, koff, H, G, half, scale, doc_start, doc_len,
                                (const attn::Item *) workspace, items.size(), sp,
                                (float *) ((char *) workspace + item_bytes), out, s);
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
// a message.  The documents must lie inside the T query rows: the host checks
// that its copy of the lengths sums to at most T, and the planner checks every
// device-side document against [0, T) and its tile count against the host's.
// The plan is written on the device by that planner kernel from doc_start /
// doc_len, in document order; every entry the attention kernel reads is written
// by the same call first, so nothing needs clearing.  When the device lengths
// disagree with the host copy, the planner writes empty entries instead and
// sets the error word that nxk_take_error returns (0x301).  All calls share the
// array: two calls whose work overlaps on the GPU (different streams, no
// ordering between them) race on it and must not be issued.
//
// Host code cannot use the array's name as a device address; its address is
// looked up once per device with cudaGetSymbolAddress on the first call made
// with that device current.  That first call should therefore come before any
// CUDA stream capture.  The cached address belongs to the device's primary
// context: after cudaDeviceReset it is stale, so this entry point does not
// support a reset device.  No device memory is allocated, and no host memory
// either.
// ---------------------------------------------------------------------------
#include <cstdio>
#include <mutex>

namespace nxk {
namespace attn {

constexpr int NOALLOC_MAX_ITEMS = 1 << 17;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) Item g_noalloc_items[NOALLOC_MAX_ITEMS];

// this file's device error word (the no-workspace planner found a document it must not plan);
// nxk_take_error reads it through attn_take_error
__device__ int g_attn_error;
constexpr int ERR_NOALLOC_PLAN = 0x301;

// One block: each thread owns a contiguous run of documents, counts their tiles,
// the block scans the counts, then every thread writes its documents' items.
// The grid that follows has n_expect blocks, counted on the host from its copy
// of the lengths.  The plan is written only if the device lengths give that
// same count and every document lies inside [0, T); otherwise every one of the
// n_expect entries becomes an empty item (no query rows, no keys) and the error
// word is set, so no entry is ever written past the array and the attention
// kernel reads nothing outside the caller's buffers.
__global__ void __launch_bounds__(1024) plan_kernel(Item * __restrict__ items, const int32_t * __restrict__ doc_start,
                                                    const int32_t * __restrict__ doc_len, int n_docs, int half,
                                                    int T, int n_expect) {
    __shared__ long long part[1024];
    __shared__ int bad;
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) bad = 0;
    __syncthreads();
    const int per = (n_docs + nt - 1) / nt;
    const int d0 = min(n_docs, tid * per), d1 = min(n_docs, d0 + per);
    long long cnt = 0;
    for (int d = d0; d < d1; ++d) {
        const long long lo = doc_start[d], n = doc_len[d];
        if (n <= 0 || lo < 0 || lo + n > T) bad = 1;
        cnt += n > 0 ? (n + QT - 1) / QT : 0;
    }
    part[tid] = cnt;
    __syncthreads();
    for (int off = 1; off < nt; off <<= 1) {        // inclusive scan (Hillis-Steele)
        const long long add = tid >= off ? part[tid - off] : 0;
        __syncthreads();
        part[tid] += add;
        __syncthreads();
    }
    if (tid == nt - 1 && part[tid] != n_expect) bad = 1;
    __syncthreads();
    if (bad) {
        if (tid == 0) atomicExch(&g_attn_error, ERR_NOALLOC_PLAN);
        Item e;
        e.q0 = e.q1 = e.k0 = e.k1 = e.doc = 0;
        for (int i = tid; i < n_expect; i += nt) items[i] = e;
        return;
    }
    long long o = part[tid] - cnt;
    for (int d = d0; d < d1; ++d) {
        const int lo = doc_start[d], hi = lo + doc_len[d];
        for (int q0 = lo; q0 < hi && o < n_expect; q0 += QT) {
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

namespace nxk {
// reads and clears this file's device error word (called by nxk_take_error)
int attn_take_error() {
    int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, attn::g_attn_error, sizeof(int));
    cudaMemcpyToSymbol(attn::g_attn_error, &zero, sizeof(int));
    return v;
}
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
    long long n_items = 0, n_rows = 0;
    for (int d = 0; d < n_docs; ++d) {
        if (h_doc_len[d] <= 0) return NXK_EINVAL;
        n_rows += h_doc_len[d];
        n_items += ((long long) h_doc_len[d] + QT - 1) / QT;
    }
    if (n_rows > T) {
        fprintf(stderr, "nxk_attention_noalloc: the documents hold %lld rows, more than T = %d\n", n_rows, T);
        return NXK_EINVAL;
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
    plan_kernel<<<1, 1024, 0, s>>>(items, doc_start, doc_len, n_docs, half, T, (int) n_items);
    const dim3 grid((unsigned) n_items, (unsigned) G);
    switch (rep) {
        case 1: attn_kernel<1><<<grid, QT * 2, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
        case 2: attn_kernel<2><<<grid, QT * 4, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
        default: attn_kernel<4><<<grid, QT * 8, 0, s>>>(q, k, v, out, items, scale, doc_start, doc_len, T, H, half); break;
    }
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}
