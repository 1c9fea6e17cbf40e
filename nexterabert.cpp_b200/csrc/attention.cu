// Grouped-query attention over a packed, unpadded batch of documents.
//
// Computes what the reference's op_attention (src/nexterabert.cpp:785-852)
// computes -- for every query row t and head h, softmax(scale[doc] * q . k) over
// the keys of t's document (optionally only those with |i - j| <= half) applied
// to v -- without materialising the score matrix: keys are streamed through
// shared memory in tiles and the softmax is accumulated online (running max and
// sum, rescaled per tile).  All arithmetic is fp32; results agree with the
// reference's two-pass softmax to ~1e-6 relative (different summation order and
// exp implementation), checked against the oracle at 1e-4.
//
// Work item = (document, 64-query tile, KV head g).  The CTA holds 64 queries for
// each of the H/G query heads that share g, so every K/V tile loaded into
// shared memory serves all of them.  Thread = (query, head); q and the output
// accumulator live in registers.  Items are planned on the host (key range per
// tile: the whole document, or the band around the tile) and ordered longest
// first.
#include "common.cuh"
#include "nextera_kernels.h"

#include <algorithm>
#include <cuda_runtime.h>
#include <vector>

namespace nxk {
namespace attn {

constexpr int D = 64;
constexpr int QT = 64;      // queries per tile
constexpr int KT = 32;      // keys per shared-memory tile

struct Item {
    int q0, q1;      // query rows [q0, q1), all in one document
    int k0, k1;      // keys the tile may touch
    int doc;
};

template <int REP>
__global__ void __launch_bounds__(QT * REP)
attn_kernel(const float * __restrict__ q, const float * __restrict__ k, const float * __restrict__ v,
            float * __restrict__ out, const Item * __restrict__ items, const float * __restrict__ scale,
            const int32_t * __restrict__ doc_start, const int32_t * __restrict__ doc_len, int T, int H, int half) {
    __shared__ __align__(16) float Ks[KT][D];
    __shared__ __align__(16) float Vs[KT][D];

    const Item it = items[blockIdx.x];
    const int g = blockIdx.y;
    const int hq = threadIdx.x / QT, qi = threadIdx.x % QT;
    const int h = g * REP + hq;
    const int t = it.q0 + qi;
    const bool valid = t < it.q1;
    const int lo_d = doc_start[it.doc], hi_d = lo_d + doc_len[it.doc];
    int lo = lo_d, hi = hi_d;
    if (half >= 0) {
        lo = max(lo, t - half);
        hi = min(hi, t + half + 1);
    }
    const float sc = scale[it.doc] * 1.4426950408889634f;     // scores in log2 units

    float qr[D];
    if (valid) {
        const float4 * qp = (const float4 *) (q + (size_t) t * H * D + (size_t) h * D);
#pragma unroll
        for (int d4 = 0; d4 < D / 4; ++d4) {
            const float4 x = qp[d4];
            qr[4 * d4] = x.x; qr[4 * d4 + 1] = x.y; qr[4 * d4 + 2] = x.z; qr[4 * d4 + 3] = x.w;
        }
    } else {
#pragma unroll
        for (int d = 0; d < D; ++d) qr[d] = 0.0f;
    }
    float o[D];
#pragma unroll
    for (int d = 0; d < D; ++d) o[d] = 0.0f;
    float m = -INFINITY, l = 0.0f;

    const float * kg = k + (size_t) g * T * D;
    const float * vg = v + (size_t) g * T * D;
    for (int kt = it.k0; kt < it.k1; kt += KT) {
        const int nk = min(KT, it.k1 - kt);
        // cooperative load of the key / value tile (float4, zero-filled past nk)
        for (int i = threadIdx.x; i < KT * D / 4; i += QT * REP) {
            const int j = i / (D / 4), d4 = i % (D / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (j < nk) {
                kv = ((const float4 *) (kg + (size_t) (kt + j) * D))[d4];
                vv = ((const float4 *) (vg + (size_t) (kt + j) * D))[d4];
            }
            ((float4 *) Ks[j])[d4] = kv;
            ((float4 *) Vs[j])[d4] = vv;
        }
        __syncthreads();
        float s[KT];
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < KT; ++j) {
            float acc = 0.0f;
#pragma unroll
            for (int d4 = 0; d4 < D / 4; ++d4) {
                const float4 kk = ((const float4 *) Ks[j])[d4];
                acc = fmaf(qr[4 * d4], kk.x, acc);
                acc = fmaf(qr[4 * d4 + 1], kk.y, acc);
                acc = fmaf(qr[4 * d4 + 2], kk.z, acc);
                acc = fmaf(qr[4 * d4 + 3], kk.w, acc);
            }
            const int kj = kt + j;
            s[j] = (j < nk && kj >= lo && kj < hi) ? acc * sc : -INFINITY;
            mt = fmaxf(mt, s[j]);
        }
        const float mn = fmaxf(m, mt);
        if (mn != -INFINITY) {
            const float corr = exp2f(m - mn);          // m = -inf -> 0
            l *= corr;
#pragma unroll
            for (int d = 0; d < D; ++d) o[d] *= corr;
#pragma unroll
            for (int j = 0; j < KT; ++j) {
                const float p = exp2f(s[j] - mn);     // masked -> 0
                l += p;
#pragma unroll
                for (int d4 = 0; d4 < D / 4; ++d4) {
                    const float4 vv = ((const float4 *) Vs[j])[d4];
                    o[4 * d4]     = fmaf(p, vv.x, o[4 * d4]);
                    o[4 * d4 + 1] = fmaf(p, vv.y, o[4 * d4 + 1]);
                    o[4 * d4 + 2] = fmaf(p, vv.z, o[4 * d4 + 2]);
                    o[4 * d4 + 3] = fmaf(p, vv.w, o[4 * d4 + 3]);
                }
            }
            m = mn;
        }
        __syncthreads();
    }
    if (valid) {
        const float inv = 1.0f / l;
        float4 * op = (float4 *) (out + (size_t) t * H * D + (size_t) h * D);
#pragma unroll
        for (int d4 = 0; d4 < D / 4; ++d4) {
            op[d4] = make_float4(o[4 * d4] * inv, o[4 * d4 + 1] * inv, o[4 * d4 + 2] * inv, o[4 * d4 + 3] * inv);
        }
    }
}

// one 64-query tile per item; key range = document or band
void plan(const int32_t * start, const int32_t * len, int n_docs, int half, std::vector<Item> & items) {
    items.clear();
    for (int d = 0; d < n_docs; ++d) {
        const int lo = start[d], hi = lo + len[d];
        for (int q0 = lo; q0 < hi; q0 += QT) {
            const int q1 = std::min(hi, q0 + QT);
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

size_t n_items(const int32_t * len, int n_docs) {
    size_t n = 0;
    for (int d = 0; d < n_docs; ++d) n += (size_t) (len[d] + QT - 1) / QT;
    return n;
}

} // namespace attn
} // namespace nxk

using namespace nxk;

extern "C" {

size_t nxk_attention_workspace(const int32_t * h_doc_len, int n_docs, int) {
    return attn::n_items(h_doc_len, n_docs) * sizeof(attn::Item);
}

int nxk_attention(const float * q, const float * k, const float * v, int T, int H, int G, int D, int half,
                  const float * scale, const int32_t *, const int32_t * doc_start, const int32_t * doc_len,
                  int n_docs, const int32_t * h_doc_start, const int32_t * h_doc_len, void * workspace,
                  size_t workspace_bytes, float * out, void * stream) {
    if (T < 0 || H <= 0 || G <= 0 || H % G || D != attn::D || n_docs < 0) return NXK_EINVAL;
    const int rep = H / G;
    if (rep != 1 && rep != 2 && rep != 4) return NXK_EINVAL;     // thread count 64 * rep, registers bound rep <= 4
    if (T == 0 || n_docs == 0) return NXK_OK;
    std::vector<attn::Item> items;
    attn::plan(h_doc_start, h_doc_len, n_docs, half, items);
    const size_t bytes = items.size() * sizeof(attn::Item);
    if (!workspace || workspace_bytes < bytes) return NXK_EINVAL;
    cudaStream_t s = (cudaStream_t) stream;
    if (cudaMemcpyAsync(workspace, items.data(), bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) return NXK_ELAUNCH;
    const dim3 grid((unsigned) items.size(), (unsigned) G);
    const attn::Item * it = (const attn::Item *) workspace;
    switch (rep) {
        case 1: attn::attn_kernel<1><<<grid, attn::QT * 1, 0, s>>>(q, k, v, out, it, scale, doc_start, doc_len, T, H, half); break;
        case 2: attn::attn_kernel<2><<<grid, attn::QT * 2, 0, s>>>(q, k, v, out, it, scale, doc_start, doc_len, T, H, half); break;
        default: attn::attn_kernel<4><<<grid, attn::QT * 4, 0, s>>>(q, k, v, out, it, scale, doc_start, doc_len, T, H, half); break;
    }
    // the host item list may be freed on return: the copy above is from pageable
    // memory, which CUDA stages before cudaMemcpyAsync returns
    return cudaPeekAtLastError() == cudaSuccess ? NXK_OK : NXK_ELAUNCH;
}

} // extern "C"
