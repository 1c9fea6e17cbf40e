// Host side of the tiled attention kernel, shared by the C-ABI entry points
// (attention.cu) and the model (model.cpp), which plans every attention layer of
// a forward once and uploads the plans with the rest of the call's metadata.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <vector>

namespace nxk {
namespace attn {

constexpr int QT3 = 64;            // queries per work unit of the tiled kernel

struct Item {
    int q0, q1;      // query rows [q0, q1), all in one document
    int k0, k1;      // keys the tile may touch
    int doc;
};

// Score scratch of the tiled kernel: per-CTA slots of (longest key range) x (query, head) floats.
struct Scratch {
    int slot_keys = 0;
    int slots = 0;
    size_t bytes = 0;
};

// One QT3-query item per tile of each document's rows inside [0, T), longest key range first.
void plan(const int32_t * start, const int32_t * len, int n_docs, int half, int qt, int T, std::vector<Item> & items);
size_t n_items(const int32_t * len, int n_docs, int qt);
Scratch scratch_plan(const int32_t * len, int n_docs, int half);

// Launches the tiled kernel over a plan already in device memory (n_items items at d_items).
// Returns NXK_OK / NXK_EINVAL / NXK_ELAUNCH.
int launch_planned(const float * q, const float * k, const float * v, int T, int Tk, int koff, int H, int G,
                   int half, const float * scale, const int32_t * doc_start, const int32_t * doc_len,
                   const Item * d_items, size_t n_items, const Scratch & sp, float * scratch, float * out,
                   cudaStream_t s);

} // namespace attn
} // namespace nxk
