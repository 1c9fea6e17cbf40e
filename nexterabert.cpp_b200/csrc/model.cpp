// libnexterabert.so host side: the nexterabert.h C API on one CUDA device.
//
// Mirrors the reference runtime's structure (src/nexterabert.cpp) with the
// compute moved to sm_100a kernels (nextera_kernels.h):
//   nextera_load     GGUF parse, hparams / block types / required-tensor checks
//                    with the reference's messages (:1549-1775); quantized
//                    linear weights are uploaded in their file blocks and
//                    expanded to int8 + per-block scales on the device
//                    (build_i8_weight, :1010-1049); conv kernels go tap-major
//   nextera_encode   prepare_batch (:1341-1370), then the encoder of
//                    builder::encoder (:1271-1294) as a sequence of kernel
//                    launches on the context's stream, then pooling (:1903-1918)
// Activation buffers live in a grow-only device arena sized for the largest
// batch seen; a call runs with no device allocation once the arena is large
// enough.  Every row op that feeds only int8 linears writes int8 codes
// directly (the reference's int8_only, :1080-1085).
#include "nexterabert.h"
#include "nextera_kernels.h"
#include "gguf.hpp"
#include "nccl_dl.hpp"
#include "attention_plan.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

namespace {

enum mixer_type { MIX_LILY, MIX_SWA, MIX_ATTN, MIX_HRA };
enum ssmax_mode { SSMAX_SSSMAX, SSMAX_SSMAX, SSMAX_NONE };
enum cls_task { CLS_NONE, CLS_SEQUENCE, CLS_CHOICE, CLS_TOKEN, CLS_QA };
const char * const CLS_NAMES[] = { "", "sequence-classification", "multiple-choice", "token-classification",
                                   "question-answering" };
constexpr int I8_BLOCK = 256;
// rows of padding before and after Fa / Fb / Fc: the halo a sharded token convolution reads
constexpr int HALO_ROWS = 8;
// the load-time concatenation of an attention mixer's c_q, c_k and c_v (no such tensor in a file)
const char * const QKV_NAME = "c_qkv.weight#fused";
// Lily's in_proj and A: both read the layer's normalized input, so one linear computes both
// (rows of in_proj, then of A) when the narrow convolution can read its two column ranges
const char * const LTC_IN_NAME = "ltc_conv.in_A.weight#fused";

struct hparams {
    int32_t n_vocab = 0, n_embd = 0, n_layer = 0, n_inter = 0, n_head = 0, n_kv_head = 0, head_dim = 0;
    int32_t lily_rank = 0, lily_kernel = 0, hra_block = 0, swa_window = 0, ntk_train_len = 0;
    float rope_base = 100000.0f, swa_rope_base = 10000.0f, ssmax_base = 0.1f, rms_eps = 1e-8f, ln_eps = 1e-5f;
    ssmax_mode ssmax = SSMAX_SSSMAX;
    std::vector<mixer_type> block_types;
    int32_t cls_id = -1, sep_id = -1, pad_id = -1, mask_id = -1;
    bool has_mlm = false, has_pooler = false;
    int32_t n_types = 0;
    cls_task cls = CLS_NONE;
    int32_t n_labels = 0;
    std::vector<std::string> labels;
};

struct DevBuf {
    void * p = nullptr;
    size_t bytes = 0;
    ~DevBuf() { if (p) cudaFree(p); }
    bool alloc(size_t n) {
        if (p) { cudaFree(p); p = nullptr; bytes = 0; }
        if (!n) return true;
        if (cudaMalloc(&p, n) != cudaSuccess) { p = nullptr; cudaGetLastError(); return false; }
        bytes = n;
        return true;
    }
    bool reserve(size_t n) { return n <= bytes ? true : alloc(n); }
    template <class T> T * as() const { return (T *) p; }
};

struct I8Weight {
    int n_in = 0, n_out = 0;
    DevBuf w, scale;
};

struct RawTensor {          // a tensor kept in its file layout on the device
    int type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    DevBuf d;
};

struct ConvTaps {
    int k = 0, C = 0;
    DevBuf taps;             // [k][C] tap-major
};

// device time per kind of kernel, as the reference's profiler reports per kind of custom op
enum prof_kind { PROF_LINEAR, PROF_ATTN, PROF_ROWS, PROF_COUNT };
const char * const PROF_NAMES[PROF_COUNT] = { "int8 linear", "attention", "norm / conv / gate / quantize" };

struct profiler {
    bool enabled = false;
    double ms[PROF_COUNT] = {};
    double total_ms = 0.0;
    int64_t calls = 0;
    std::vector<std::pair<cudaEvent_t, int>> marks;   // event recorded before each launch group
};

} // namespace

struct nextera_context {
    hparams hp;
    std::string tokenizer_json, ftype, sysinfo, path;
    int device = 0;
    int n_threads = 1;
    cudaStream_t stream = nullptr;

    std::unordered_map<std::string, I8Weight> i8;
    std::unordered_map<std::string, DevBuf> f32;          // 1-D fp32 parameters on the device
    std::unordered_map<std::string, std::vector<float>> host_f32;   // the same, on the host (SSMax scalars)
    std::unordered_map<std::string, ConvTaps> taps;
    std::unordered_map<std::string, RawTensor> raw;       // embedding tables
    std::vector<std::string> names;                       // every tensor in the file

    // forward arena
    DevBuf X, X2, U, Fa, Fb, Fc, Q1, Q1s, Q2, Q2s;
    DevBuf meta, attn_ws, pooled;
    // heads: gathered / pooled rows, their codes and scales, the transform's output, the
    // mul_mat workspace and the head's output
    DevBuf head_x, head_q, head_qs, head_y, head_ws, head_out, head_idx;
    int64_t cap_T = 0, cap_docs = 0;
    // host staging (pinned)
    void * h_stage = nullptr;
    size_t h_stage_bytes = 0;
    // rope tables on the device: [0] attn / hra base (NTK-stretched when needed), [1] swa
    DevBuf rope_cos[2], rope_sin[2];
    int rope_n[2] = {0, 0};
    float rope_base_cached[2] = {0.0f, 0.0f};

    // sequence sharding (nextera_shard_init): this process's rank, the ranks and their communicator
    int shard_rank = 0, shard_world = 1;
    ncclComm_t shard_comm = nullptr;
    DevBuf kv_ext, kv_full;       // K / V with halo rows (band layers), gathered K / V (global, HRA)
    // one batch partitioned over the ranks (nextera_encode_partitioned*): this rank's token ids, the
    // pooled rows every rank sends to rank 0 (received there in rank order) and rank 0's row map
    DevBuf part_tok, part_rows, part_idx;
    int32_t * h_part_idx = nullptr;
    size_t h_part_idx_n = 0;

    int32_t debug_n_layers = -1;
    profiler prof;
    double last_ms = 0.0;
    int64_t launches = 0;          // kernels launched since load (all calls)
    size_t stage_need = 0;         // pinned staging bytes of the last batch laid out

    // Forwards of a batch shape seen before replay as a CUDA graph (host calls, up to GRAPH_MAX_T
    // tokens): the shape's metadata sits in its own pinned staging buffer, the graph's first node
    // uploads it (with the call's token ids written in first) and its last ones copy the results to
    // pinned buffers.  An entry is dropped when a device buffer it uses has been reallocated.
    struct GraphEntry {
        std::vector<int32_t> key;          // lengths, then a flags word
        cudaGraphExec_t exec = nullptr;
        void * stage = nullptr;
        float * h_pooled = nullptr, * h_hidden = nullptr;
        size_t o_tok = 0, o_typ = 0;
        std::vector<const void *> sig;     // the device buffers baked into the graph
        int64_t launches = 0;
        uint64_t used = 0;
    };
    std::vector<GraphEntry> graphs;
    std::vector<std::vector<int32_t>> seen;   // recent shapes (a graph is made on the second one)
    uint64_t graph_clock = 0;

    bool has(const std::string & n) const {
        return i8.count(n) || f32.count(n) || taps.count(n) || raw.count(n) ||
               std::find(names.begin(), names.end(), n) != names.end();
    }
};

namespace {

const char * ftype_name(uint32_t ft) {
    switch (ft) {
        case 0: return "F32"; case 1: return "F16"; case 2: return "Q4_0"; case 3: return "Q4_1";
        case 7: return "Q8_0"; case 8: return "Q5_0"; case 9: return "Q5_1"; case 10: return "Q2_K";
        case 11: return "Q3_K_S"; case 12: return "Q3_K_M"; case 13: return "Q3_K_L"; case 14: return "Q4_K_S";
        case 15: return "Q4_K_M"; case 16: return "Q5_K_S"; case 17: return "Q5_K_M"; case 18: return "Q6_K";
        default: return "unknown";
    }
}

bool ends_with(const std::string & s, const char * suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// Every tensor the encoder and the file's heads need (the reference's required_tensors, :1483-1516)
std::vector<std::string> required_tensors(const hparams & hp) {
    std::vector<std::string> r = { "embedding.weight", "out_norm.weight", "out_norm.bias" };
    auto add = [&r](const std::string & pre, std::initializer_list<const char *> names) {
        for (const char * n : names) r.push_back(pre + n);
    };
    for (int l = 0; l < hp.n_layer && l < (int) hp.block_types.size(); ++l) {
        const std::string blk = "blocks." + std::to_string(l) + ".", pre = blk + "attn.";
        add(blk, { "attn_norm.weight", "mlp_norm.weight", "mlp.c_fc.weight", "mlp.c_proj.weight" });
        add(pre, { "c_proj.weight" });
        const mixer_type mt = hp.block_types[l];
        if (mt == MIX_LILY) {
            add(pre, { "ltc_conv.in_proj.weight", "ltc_conv.A.weight", "ltc_conv.kernel", "ltc_conv.out_proj.weight",
                       "x_proj.weight", "B_proj.weight", "state_conv.depthwise.weight" });
            continue;
        }
        add(pre, { "c_q.weight", "c_k.weight", "c_v.weight", "c_gate.weight",
                   "q_norm.alpha", "q_norm.beta", "k_norm.alpha", "k_norm.beta" });
        if (mt == MIX_HRA) {
            add(pre, { "qkv_in.weight", "qkv_gate.weight", "c_C.weight",
                       "qkv_conv.depthwise.weight", "c_o.depthwise.weight" });
        }
        if (mt != MIX_SWA && hp.ssmax != SSMAX_NONE) {
            add(pre, { "scalable_factor.s" });
            if (hp.ssmax == SSMAX_SSSMAX) add(pre, { "scalable_factor.b" });
        }
    }
    if (hp.has_mlm) add("mlm.", { "dense.weight", "norm.weight", "bias" });
    if (hp.cls != CLS_NONE) {
        add("classifier.", { "weight", "bias" });
        const bool pooled = hp.cls == CLS_SEQUENCE || hp.cls == CLS_CHOICE;
        add(pooled ? "pooler." : "head.", { "dense.weight", "norm.weight" });
    }
    return r;
}

// fp32 cos / sin tables exactly as the reference builds them (build_rope, :1322-1338)
void rope_table(int n_pos, float base, int head_dim, std::vector<float> & c, std::vector<float> & s) {
    const int half = head_dim / 2;
    c.resize((size_t) n_pos * half);
    s.resize((size_t) n_pos * half);
    std::vector<float> inv(half);
    for (int i = 0; i < half; ++i) inv[i] = 1.0f / std::pow(base, (float) (2 * i) / (float) head_dim);
    for (int t = 0; t < n_pos; ++t) {
        for (int i = 0; i < half; ++i) {
            const float a = (float) t * inv[i];
            c[(size_t) t * half + i] = std::cos(a);
            s[(size_t) t * half + i] = std::sin(a);
        }
    }
}

bool check(int rc, const char * what) {
    if (rc != NXK_OK) {
        fprintf(stderr, "nexterabert: kernel '%s' rejected its arguments or failed to launch (%d)\n", what, rc);
        return false;
    }
    return true;
}


// Concatenates expanded int8 weights with the same input width along their output rows into
// one weight `name` (scales [block][row] likewise); the parts are released.
bool fuse_rows(nextera_context & c, const std::vector<std::string> & parts, const std::string & name) {
    int n_in = -1, n_out = 0;
    for (const std::string & p : parts) {
        auto it = c.i8.find(p);
        if (it == c.i8.end() || (n_in >= 0 && it->second.n_in != n_in)) return false;
        n_in = it->second.n_in;
        n_out += it->second.n_out;
    }
    I8Weight & f = c.i8[name];
    f.n_in = n_in;
    f.n_out = n_out;
    const int n_blk = (n_in + I8_BLOCK - 1) / I8_BLOCK;
    if (!f.w.alloc((size_t) n_in * n_out) || !f.scale.alloc(sizeof(float) * (size_t) n_blk * n_out)) return false;
    size_t row = 0;
    for (const std::string & p : parts) {
        const I8Weight & w = c.i8.at(p);
        cudaMemcpyAsync(f.w.as<int8_t>() + row * n_in, w.w.p, (size_t) w.n_in * w.n_out, cudaMemcpyDeviceToDevice,
                        c.stream);
        cudaMemcpy2DAsync(f.scale.as<float>() + row, sizeof(float) * n_out, w.scale.p, sizeof(float) * w.n_out,
                          sizeof(float) * w.n_out, n_blk, cudaMemcpyDeviceToDevice, c.stream);
        row += w.n_out;
    }
    if (cudaStreamSynchronize(c.stream) != cudaSuccess) return false;
    for (const std::string & p : parts) c.i8.erase(p);
    return true;
}

} // namespace

// ---------------------------------------------------------------------------
// C API
// ---------------------------------------------------------------------------

struct nextera_params nextera_default_params(void) {
    nextera_params p;
    p.n_threads = 0;
    p.use_repack = 1;
    p.use_int8 = 1;
    p.verbosity = 0;
    return p;
}

struct nextera_context * nextera_load(const char * path, struct nextera_params params) {
    const auto t_start = std::chrono::steady_clock::now();
    nxg::File gg;
    if (!gg.open(path)) {
        fprintf(stderr, "nexterabert: failed to open '%s' (%s)\n", path, gg.error.c_str());
        return nullptr;
    }
    if (gg.str("general.architecture", "") != "nexterabert") {
        fprintf(stderr, "nexterabert: '%s' is not a nexterabert GGUF (general.architecture = '%s')\n", path,
                gg.str("general.architecture", "").c_str());
        return nullptr;
    }
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || n_dev == 0) {
        cudaGetLastError();
        fprintf(stderr, "nexterabert: no CUDA device\n");
        return nullptr;
    }
    std::unique_ptr<nextera_context> c(new nextera_context());
    c->path = path;
    cudaGetDevice(&c->device);
    hparams & hp = c->hp;
    bool ok = true;
    auto req_u32 = [&](const char * key) -> int32_t {
        const nxg::Value * v = gg.get(key);
        if (!v) { fprintf(stderr, "nexterabert: missing key '%s'\n", key); ok = false; return 0; }
        return (int32_t) v->u;
    };
    hp.n_vocab = req_u32("nexterabert.vocab_size");
    hp.n_embd = req_u32("nexterabert.embedding_length");
    hp.n_layer = req_u32("nexterabert.block_count");
    hp.n_inter = req_u32("nexterabert.feed_forward_length");
    hp.n_head = req_u32("nexterabert.attention.head_count");
    hp.n_kv_head = req_u32("nexterabert.attention.head_count_kv");
    if (!ok) return nullptr;
    hp.head_dim = hp.n_head > 0 ? hp.n_embd / hp.n_head : 0;
    hp.lily_rank = (int32_t) gg.u32("nexterabert.lily.low_rank", (uint32_t) hp.head_dim);
    hp.lily_kernel = (int32_t) gg.u32("nexterabert.lily.kernel_size", 5);
    hp.hra_block = (int32_t) gg.u32("nexterabert.hra.block_size", 4);
    hp.swa_window = (int32_t) gg.u32("nexterabert.swa.window", 256);
    hp.ntk_train_len = (int32_t) gg.u32("nexterabert.rope.ntk_train_length", 0);
    hp.rope_base = gg.f32("nexterabert.rope.freq_base", 100000.0f);
    hp.swa_rope_base = gg.f32("nexterabert.swa.rope.freq_base", 10000.0f);
    hp.ssmax_base = gg.f32("nexterabert.ssmax.base", 0.1f);
    hp.rms_eps = gg.f32("nexterabert.rms_norm_epsilon", 1e-8f);
    hp.ln_eps = gg.f32("nexterabert.layer_norm_epsilon", 1e-5f);
    hp.cls_id = (int32_t) gg.u32("tokenizer.ggml.cls_token_id", (uint32_t) -1);
    hp.sep_id = (int32_t) gg.u32("tokenizer.ggml.seperator_token_id", (uint32_t) -1);
    hp.pad_id = (int32_t) gg.u32("tokenizer.ggml.padding_token_id", (uint32_t) -1);
    hp.mask_id = (int32_t) gg.u32("tokenizer.ggml.mask_token_id", (uint32_t) -1);
    if (const nxg::Value * v = gg.get("nexterabert.mlm_head")) hp.has_mlm = v->u != 0;
    const std::string task = gg.str("nexterabert.classifier.task", "");
    for (int i = CLS_SEQUENCE; i <= CLS_QA; ++i) {
        if (task == CLS_NAMES[i]) hp.cls = (cls_task) i;
    }
    if (const nxg::Value * v = gg.get("nexterabert.classifier.labels")) hp.labels = v->arr_s;
    const std::string mode = gg.str("nexterabert.ssmax.mode", "sssmax");
    hp.ssmax = mode == "none" ? SSMAX_NONE : mode == "ssmax" ? SSMAX_SSMAX : SSMAX_SSSMAX;
    if (!task.empty() && hp.cls == CLS_NONE) {
        fprintf(stderr, "nexterabert: unsupported classifier task '%s'\n", task.c_str());
        ok = false;
    }
    {
        const nxg::Value * v = gg.get("nexterabert.block_types");
        const size_t n = v ? v->arr_s.size() : 0;
        if ((int32_t) n != hp.n_layer) {
            fprintf(stderr, "nexterabert: block_types has %zu entries, expected %d\n", n, hp.n_layer);
            ok = false;
        }
        for (size_t i = 0; ok && i < n; ++i) {
            const std::string & t = v->arr_s[i];
            if (t == "lily") hp.block_types.push_back(MIX_LILY);
            else if (t == "swa") hp.block_types.push_back(MIX_SWA);
            else if (t == "attn") hp.block_types.push_back(MIX_ATTN);
            else if (t == "hra") hp.block_types.push_back(MIX_HRA);
            else { fprintf(stderr, "nexterabert: unsupported block type '%s'\n", t.c_str()); ok = false; }
        }
    }
    if (hp.head_dim % 2 != 0 || hp.n_kv_head <= 0 || hp.n_head % hp.n_kv_head != 0) {
        fprintf(stderr, "nexterabert: unsupported head layout\n");
        ok = false;
    }
    // limits of the device kernels
    if (ok && (hp.head_dim != 64 || hp.n_embd % 64 || hp.n_inter % 64 || (hp.n_head / hp.n_kv_head) > 4)) {
        fprintf(stderr, "nexterabert: this build runs head_dim 64, n_embd / n_inter multiples of 64 and at most "
                        "4 query heads per KV head (file: head_dim %d, n_embd %d, n_inter %d, %d:%d heads)\n",
                hp.head_dim, hp.n_embd, hp.n_inter, hp.n_head, hp.n_kv_head);
        ok = false;
    }
    c->tokenizer_json = gg.str("tokenizer.huggingface.json", "");
    c->ftype = ftype_name(gg.u32("general.file_type", 0));
    if (!ok) return nullptr;

    int hw = (int) std::max(1u, std::thread::hardware_concurrency());
    c->n_threads = params.n_threads > 0 ? params.n_threads : hw;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "nexterabert: cannot create a CUDA stream\n");
        return nullptr;
    }

    FILE * f = fopen(path, "rb");
    if (!f) {
        fprintf(stderr, "nexterabert: failed to open '%s'\n", path);
        return nullptr;
    }
    std::vector<uint8_t> tmp;
    DevBuf staging;
    size_t weight_bytes = 0;
    for (const nxg::TensorInfo & t : gg.tensors) {
        c->names.push_back(t.name);
        const size_t n = t.nbytes;
        tmp.resize(n ? n : 1);
        if (fseeko(f, (off_t) (gg.data_offset + t.offset), SEEK_SET) != 0 || fread(tmp.data(), 1, n, f) != n) {
            fprintf(stderr, "nexterabert: failed to read tensor '%s'\n", t.name.c_str());
            ok = false;
            break;
        }
        const int n_dims = t.ne[3] > 1 ? 4 : t.ne[2] > 1 ? 3 : t.ne[1] > 1 ? 2 : 1;
        const bool embedding = t.name == "embedding.weight" || t.name == "mlm.decoder.weight" ||
                               t.name == "token_type_embeddings.weight";
        const bool gemm = !embedding && n_dims == 2 && nxg::is_quantized(t.type);
        if (gemm && t.ne[0] % 32 == 0 && t.ne[1] % 4 == 0) {
            // int8 path (:1663-1667): blocks to the device, expanded there
            I8Weight & w = c->i8[t.name];
            w.n_in = (int) t.ne[0];
            w.n_out = (int) t.ne[1];
            const int n_blk = (w.n_in + I8_BLOCK - 1) / I8_BLOCK;
            if (!staging.reserve(n) || !w.w.alloc((size_t) w.n_in * w.n_out) ||
                !w.scale.alloc(sizeof(float) * (size_t) n_blk * w.n_out)) {
                fprintf(stderr, "nexterabert: out of device memory loading '%s'\n", t.name.c_str());
                ok = false;
                break;
            }
            cudaMemcpyAsync(staging.p, tmp.data(), n, cudaMemcpyHostToDevice, c->stream);
            if (!check(nxk_expand_weight(t.type, staging.p, w.n_in, w.n_out, w.w.as<int8_t>(), w.scale.as<float>(),
                                         nullptr, c->stream), "expand_weight")) {
                ok = false;
                break;
            }
            cudaStreamSynchronize(c->stream);   // staging is reused by the next tensor
            weight_bytes += (size_t) w.n_in * w.n_out + sizeof(float) * (size_t) n_blk * w.n_out;
            continue;
        }
        // head matrices off the int8 path (the classifier, float head weights) run on ggml_mul_mat in
        // the reference (:1140-1142) and are kept in their file layout, like the embedding tables
        const bool head_matrix = t.name == "classifier.weight" || t.name == "pooler.dense.weight" ||
                                 t.name == "head.dense.weight" || t.name == "mlm.dense.weight";
        if (embedding || head_matrix) {
            RawTensor & r = c->raw[t.name];
            r.type = t.type;
            memcpy(r.ne, t.ne, sizeof(r.ne));
            if (!r.d.alloc(n)) { ok = false; break; }
            cudaMemcpy(r.d.p, tmp.data(), n, cudaMemcpyHostToDevice);
            weight_bytes += n;
            continue;
        }
        if (ends_with(t.name, ".depthwise.weight") || ends_with(t.name, ".kernel")) {
            // conv kernels are stored (k, C) per channel; the kernels want one row per tap (:1702-1711)
            if (t.type != 0) {
                fprintf(stderr, "nexterabert: conv kernel '%s' must be F32\n", t.name.c_str());
                ok = false;
                break;
            }
            ConvTaps & ct = c->taps[t.name];
            ct.k = (int) t.ne[0];
            ct.C = (int) t.ne[1];
            std::vector<float> tm((size_t) ct.k * ct.C);
            const float * src = (const float *) tmp.data();
            for (int ch = 0; ch < ct.C; ++ch) {
                for (int j = 0; j < ct.k; ++j) tm[(size_t) j * ct.C + ch] = src[(size_t) ch * ct.k + j];
            }
            if (!ct.taps.alloc(tm.size() * sizeof(float))) { ok = false; break; }
            cudaMemcpy(ct.taps.p, tm.data(), tm.size() * sizeof(float), cudaMemcpyHostToDevice);
            continue;
        }
        if (n_dims == 1 && t.type == 0) {
            std::vector<float> & hv = c->host_f32[t.name];
            hv.assign((const float *) tmp.data(), (const float *) tmp.data() + t.ne[0]);
            DevBuf & d = c->f32[t.name];
            if (!d.alloc(n)) { ok = false; break; }
            cudaMemcpy(d.p, tmp.data(), n, cudaMemcpyHostToDevice);
            continue;
        }
        if (gemm || n_dims == 2) {
            // F32 / F16 matrices would run on ggml's mul_mat in the reference (:1140-1142)
            const bool needed_by_encoder = t.name.rfind("blocks.", 0) == 0;
            if (needed_by_encoder) {
                fprintf(stderr, "nexterabert: '%s' (type %d) is not a quantized matrix this build can expand to "
                                "int8; float and unaligned GEMM weights are not supported on the GPU path\n",
                        t.name.c_str(), t.type);
                ok = false;
                break;
            }
        }
    }
    fclose(f);
    if (ok && cudaStreamSynchronize(c->stream) != cudaSuccess) {
        fprintf(stderr, "nexterabert: device error while expanding weights: %s\n", cudaGetErrorString(cudaGetLastError()));
        ok = false;
    }
    if (!ok) return nullptr;

    hp.has_pooler = c->has("pooler.dense.weight") && c->has("pooler.norm.weight");
    if (c->raw.count("token_type_embeddings.weight")) hp.n_types = (int32_t) c->raw["token_type_embeddings.weight"].ne[1];
    if (hp.cls != CLS_NONE && c->host_f32.count("classifier.bias")) {
        hp.n_labels = (int32_t) c->host_f32["classifier.bias"].size();
        if ((int32_t) hp.labels.size() != hp.n_labels) hp.labels.clear();
    }
    for (const std::string & name : required_tensors(hp)) {
        if (c->has(name)) continue;
        fprintf(stderr, "nexterabert: '%s' has no tensor '%s': not a complete nexterabert file "
                        "(convert the checkpoint again with python/convert_hf_to_gguf.py)\n", path, name.c_str());
        return nullptr;
    }
    // every encoder linear must be on the int8 path
    for (int l = 0; l < hp.n_layer; ++l) {
        const std::string blk = "blocks." + std::to_string(l) + ".";
        for (const std::string & n : required_tensors(hp)) {
            if (n.rfind(blk, 0) == 0 && ends_with(n, ".weight") && !c->taps.count(n) && !c->f32.count(n) &&
                !c->i8.count(n)) {
                fprintf(stderr, "nexterabert: '%s' is not on the int8 path\n", n.c_str());
                return nullptr;
            }
        }
    }

    // attention mixers: c_q, c_k and c_v become one weight, rows in that order, so one GEMM
    // computes all three projections; Lily mixers: in_proj and A the same way, when their rank is
    // a width the narrow convolution takes (32, 64 or 128)
    const size_t n_file_linears = c->i8.size();
    for (int l = 0; l < hp.n_layer; ++l) {
        const std::string pre = "blocks." + std::to_string(l) + ".attn.";
        if (hp.block_types[l] == MIX_LILY) {
            auto ip = c->i8.find(pre + "ltc_conv.in_proj.weight"), ia = c->i8.find(pre + "ltc_conv.A.weight");
            if (ip == c->i8.end() || ia == c->i8.end()) continue;
            const int r = ip->second.n_out;
            if (ia->second.n_out != r || ia->second.n_in != ip->second.n_in || (r != 32 && r != 64 && r != 128))
                continue;
            if (!fuse_rows(*c, {pre + "ltc_conv.in_proj.weight", pre + "ltc_conv.A.weight"}, pre + LTC_IN_NAME)) {
                fprintf(stderr, "nexterabert: cannot build the fused in_proj/A weight of layer %d\n", l);
                return nullptr;
            }
            continue;
        }
        if (!fuse_rows(*c, {pre + "c_q.weight", pre + "c_k.weight", pre + "c_v.weight"}, pre + QKV_NAME)) {
            fprintf(stderr, "nexterabert: cannot build the fused q/k/v weight of layer %d\n", l);
            return nullptr;
        }
    }

    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, c->device);
    char info[512];
    snprintf(info, sizeof(info),
             "CUDA = 1 | device = %s (sm_%d%d, %d SMs) | linear layers: %d int8 (tcgen05 kind::i8), 0 ggml repack | "
             "custom ops: CUDA sm_100a",
             prop.name, prop.major, prop.minor, prop.multiProcessorCount, (int) n_file_linears);
    c->sysinfo = info;
    if (params.verbosity > 0) {
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_start).count();
        fprintf(stderr, "nexterabert: %s | %s | %d layers, n_embd %d | device weights %.1f MiB | loaded in %.0f ms\n",
                path, c->ftype.c_str(), hp.n_layer, hp.n_embd, weight_bytes / 1048576.0, ms);
        fprintf(stderr, "nexterabert: %s\n", c->sysinfo.c_str());
    }
    return c.release();
}

void nextera_free(struct nextera_context * c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto & g : c->graphs) {
        if (g.exec) cudaGraphExecDestroy(g.exec);
        if (g.stage) cudaFreeHost(g.stage);
        if (g.h_pooled) cudaFreeHost(g.h_pooled);
        if (g.h_hidden) cudaFreeHost(g.h_hidden);
    }
    for (auto & m : c->prof.marks) cudaEventDestroy(m.first);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->h_part_idx) cudaFreeHost(c->h_part_idx);
    if (c->shard_comm) nxs::nccl().comm_destroy(c->shard_comm);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

int32_t nextera_n_embd(const struct nextera_context * c) { return c->hp.n_embd; }
int32_t nextera_n_vocab(const struct nextera_context * c) { return c->hp.n_vocab; }
int32_t nextera_n_layer(const struct nextera_context * c) { return c->hp.n_layer; }
int32_t nextera_has_mlm_head(const struct nextera_context * c) { return c->hp.has_mlm ? 1 : 0; }
int32_t nextera_has_pooler(const struct nextera_context * c) { return c->hp.has_pooler ? 1 : 0; }
int32_t nextera_n_token_types(const struct nextera_context * c) { return c->hp.n_types; }
int32_t nextera_n_labels(const struct nextera_context * c) { return c->hp.n_labels; }
const char * nextera_classifier_task(const struct nextera_context * c) { return CLS_NAMES[c->hp.cls]; }
const char * nextera_label(const struct nextera_context * c, int32_t i) {
    return i >= 0 && i < (int32_t) c->hp.labels.size() ? c->hp.labels[i].c_str() : "";
}
int32_t nextera_token_cls(const struct nextera_context * c) { return c->hp.cls_id; }
int32_t nextera_token_sep(const struct nextera_context * c) { return c->hp.sep_id; }
int32_t nextera_token_pad(const struct nextera_context * c) { return c->hp.pad_id; }
int32_t nextera_token_mask(const struct nextera_context * c) { return c->hp.mask_id; }
const char * nextera_tokenizer_json(const struct nextera_context * c) { return c->tokenizer_json.c_str(); }
const char * nextera_ftype(const struct nextera_context * c) { return c->ftype.c_str(); }
const char * nextera_system_info(const struct nextera_context * c) { return c->sysinfo.c_str(); }
int32_t nextera_get_n_threads(const struct nextera_context * c) { return c->n_threads; }
double nextera_last_ms(const struct nextera_context * c) { return c->last_ms; }
void nextera_set_n_threads(struct nextera_context * c, int32_t n) {
    c->n_threads = n > 0 ? n : (int) std::max(1u, std::thread::hardware_concurrency());
}

void nextera_debug_set_layers(struct nextera_context * c, int32_t n_layers) { c->debug_n_layers = n_layers; }

int64_t nextera_debug_launches(const struct nextera_context * c) { return c->launches; }

int64_t nextera_debug_profile_get(const struct nextera_context * c, double * kind_ms, double * total_ms) {
    for (int i = 0; i < PROF_COUNT; ++i) kind_ms[i] = c->prof.ms[i];
    *total_ms = c->prof.total_ms;
    return c->prof.calls;
}

void nextera_debug_profile(struct nextera_context * c, int32_t enable) {
    for (auto & m : c->prof.marks) cudaEventDestroy(m.first);
    c->prof = profiler();
    c->prof.enabled = enable != 0;
}

void nextera_debug_profile_print(const struct nextera_context * c) {
    const profiler & pr = c->prof;
    if (!pr.calls) return;
    double sum = 0.0;
    fprintf(stderr, "profile over %lld forward passes (ms per pass, device time):\n", (long long) pr.calls);
    for (int i = 0; i < PROF_COUNT; ++i) {
        sum += pr.ms[i];
        fprintf(stderr, "  %-22s %8.3f  %5.1f%%\n", PROF_NAMES[i], pr.ms[i] / pr.calls,
                pr.total_ms > 0 ? 100.0 * pr.ms[i] / pr.total_ms : 0.0);
    }
    fprintf(stderr, "  %-22s %8.3f  %5.1f%%   (host work, copies, launch gaps)\n", "everything else",
            (pr.total_ms - sum) / pr.calls, pr.total_ms > 0 ? 100.0 * (pr.total_ms - sum) / pr.total_ms : 0.0);
    fprintf(stderr, "  %-22s %8.3f\n", "total", pr.total_ms / pr.calls);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
namespace {

struct Batch {
    int n_docs = 0, T = 0, nb = 0, max_len = 0;
    std::vector<int32_t> start, len, bstart, blen, row_doc, brow_doc;
};

// device views of one forward's layout
struct Layout {
    const int32_t * row_doc, * start, * len, * bstart, * blen, * brow_doc, * tokens, * types;
};

class Forward {
public:
    Forward(nextera_context & c, cudaStream_t s) : c_(c), s_(s), hp_(c.hp) {}

    bool ok = true;

    void mark(int kind) {
        if (!c_.prof.enabled) return;
        cudaEvent_t e;
        cudaEventCreate(&e);
        cudaEventRecord(e, s_);
        c_.prof.marks.emplace_back(e, kind);
    }

    // y = W x (+ res): x = (q, sx) with T rows
    void linear(const std::string & name, const int8_t * q, const float * sx, int T, const float * res, float * out) {
        if (!ok) return;
        auto it = c_.i8.find(name);
        if (it == c_.i8.end()) {
            fprintf(stderr, "nexterabert: missing tensor '%s'\n", name.c_str());
            ok = false;
            return;
        }
        mark(PROF_LINEAR);
        ++c_.launches;
        const I8Weight & w = it->second;
        ok = check(nxk_linear_i8(q, sx, T, w.w.as<int8_t>(), w.scale.as<float>(), w.n_in, w.n_out, res, out, s_),
                   name.c_str());
    }

    // y = W x followed by relu^2 (z == nullptr) or sigmoid(y) * z, quantized for the next linear:
    // codes and scales out; false when the shape needs the separate row op (N % 256 != 0)
    bool linear_q(const std::string & name, const int8_t * q, const float * sx, int T, const float * z,
                  int8_t * qo, float * so) {
        if (!ok) return true;
        auto it = c_.i8.find(name);
        if (it == c_.i8.end() || it->second.n_out % 256 != 0) return false;
        mark(PROF_LINEAR);
        ++c_.launches;
        const I8Weight & w = it->second;
        const int rc = z ? nxk_linear_i8_gate_q(q, sx, T, w.w.as<int8_t>(), w.scale.as<float>(), w.n_in, w.n_out, z, qo,
                                                so, s_)
                         : nxk_linear_i8_relu_sqr_q(q, sx, T, w.w.as<int8_t>(), w.scale.as<float>(), w.n_in,
                                                    w.n_out, qo, so, s_);
        ok = check(rc, name.c_str());
        return true;
    }

    int n_out(const std::string & name) const {
        auto it = c_.i8.find(name);
        return it == c_.i8.end() ? 0 : it->second.n_out;
    }

    const float * p(const std::string & name) {
        auto it = c_.f32.find(name);
        if (it == c_.f32.end()) {
            fprintf(stderr, "nexterabert: missing tensor '%s'\n", name.c_str());
            ok = false;
            return nullptr;
        }
        return it->second.as<float>();
    }

    const ConvTaps * taps(const std::string & name) {
        auto it = c_.taps.find(name);
        if (it == c_.taps.end()) {
            fprintf(stderr, "nexterabert: missing tensor '%s'\n", name.c_str());
            ok = false;
            return nullptr;
        }
        return &it->second;
    }

    // a row-op / attention / embedding launch (pooling launches two kernels)
    void rows(int rc, const char * what, int n_kernels = 1) {
        c_.launches += n_kernels;
        if (ok) ok = check(rc, what);
    }

    // Scalable-Softmax scale for n attended keys (ssmax_scale, :1174-1181)
    float ssmax_scale(const std::string & pre, int n) const {
        if (hp_.ssmax == SSMAX_NONE) return 1.0f;
        const float s = c_.host_f32.at(pre + "scalable_factor.s")[0];
        const float ln = std::log((float) std::max(n, 1));
        if (hp_.ssmax == SSMAX_SSMAX) return s * ln;
        const float b = c_.host_f32.at(pre + "scalable_factor.b")[0];
        return s * ln + hp_.ssmax_base + std::max(b, 0.0f);
    }

    nextera_context & c_;
    cudaStream_t s_;
    const hparams & hp_;
};

// Lays out the batch and checks it (prepare_batch :1341-1370, check_tokens / check_types :1843-1863)
int prepare(const nextera_context & c, const int32_t * tokens, const int32_t * types, const int32_t * lengths,
            int32_t n_seqs, bool tokens_on_host, Batch & b, float & rope0_base) {
    if (n_seqs <= 0 || !lengths) return 1;
    b.n_docs = n_seqs;
    b.start.resize(n_seqs);
    b.len.assign(lengths, lengths + n_seqs);
    b.bstart.resize(n_seqs);
    b.blen.resize(n_seqs);
    int64_t total = 0, btotal = 0;
    for (int i = 0; i < n_seqs; ++i) {
        if (lengths[i] <= 0) {
            fprintf(stderr, "nexterabert: empty sequence in batch\n");
            return 1;
        }
        b.start[i] = (int32_t) total;
        total += lengths[i];
        b.blen[i] = (lengths[i] + c.hp.hra_block - 1) / c.hp.hra_block;
        b.bstart[i] = (int32_t) btotal;
        btotal += b.blen[i];
        b.max_len = std::max(b.max_len, lengths[i]);
    }
    if (total > INT32_MAX / 4) {
        fprintf(stderr, "nexterabert: batch too large\n");
        return 1;
    }
    b.T = (int) total;
    b.nb = (int) btotal;
    b.row_doc.resize(b.T);
    b.brow_doc.resize(b.nb);
    for (int i = 0; i < n_seqs; ++i) {
        std::fill(b.row_doc.begin() + b.start[i], b.row_doc.begin() + b.start[i] + b.len[i], i);
        std::fill(b.brow_doc.begin() + b.bstart[i], b.brow_doc.begin() + b.bstart[i] + b.blen[i], i);
    }
    if (tokens_on_host) {
        for (int i = 0; i < b.T; ++i) {
            if (tokens[i] < 0 || tokens[i] >= c.hp.n_vocab) {
                fprintf(stderr, "nexterabert: token id %d out of range\n", tokens[i]);
                return 1;
            }
        }
        for (int i = 0; types && c.hp.n_types > 0 && i < b.T; ++i) {
            if (types[i] < 0 || types[i] >= c.hp.n_types) {
                fprintf(stderr, "nexterabert: token type id %d out of range\n", types[i]);
                return 1;
            }
        }
    }
    float base = c.hp.rope_base;
    if (c.hp.ntk_train_len > 0 && b.max_len > c.hp.ntk_train_len) {
        if (n_seqs > 1) {
            fprintf(stderr, "nexterabert: sequences beyond rope.ntk_train_length must be encoded one at a time\n");
            return 1;
        }
        const double d = c.hp.head_dim;
        base = (float) ((double) base * std::pow((double) b.max_len / c.hp.ntk_train_len, d / (d - 2.0)));
    }
    rope0_base = base;
    return 0;
}

bool ensure_rope(nextera_context & c, int which, int n_pos, float base) {
    if (c.rope_n[which] >= n_pos && c.rope_base_cached[which] == base) return true;
    const int n = std::max(n_pos, 1);
    std::vector<float> cs, sn;
    rope_table(n, base, c.hp.head_dim, cs, sn);
    if (!c.rope_cos[which].alloc(cs.size() * 4) || !c.rope_sin[which].alloc(sn.size() * 4)) return false;
    cudaMemcpy(c.rope_cos[which].p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(c.rope_sin[which].p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    c.rope_n[which] = n;
    c.rope_base_cached[which] = base;
    return true;
}

bool ensure_arena(nextera_context & c, const Batch & b) {
    const hparams & hp = c.hp;
    const int64_t T = std::max<int64_t>(b.T, 1), C = hp.n_embd, I = hp.n_inter;
    const int64_t HD = (int64_t) hp.n_head * hp.head_dim, GD = (int64_t) hp.n_kv_head * hp.head_dim;
    const int64_t wide = std::max<int64_t>(I, 2 * (HD + 2 * GD));     // q, k, v and their fused projection
    const int64_t nb_C = (C + I8_BLOCK - 1) / I8_BLOCK, nb_W = (std::max(I, C) + I8_BLOCK - 1) / I8_BLOCK;
    bool ok = c.X.reserve(sizeof(float) * T * C) && c.X2.reserve(sizeof(float) * T * C) &&
              c.U.reserve(sizeof(float) * T * wide) && c.Fa.reserve(sizeof(float) * (T + 2 * HALO_ROWS) * C) &&
              c.Fb.reserve(sizeof(float) * (T + 2 * HALO_ROWS) * C) &&
              c.Fc.reserve(sizeof(float) * (T + 2 * HALO_ROWS) * C) &&
              c.Q1.reserve((size_t) T * std::max(I, C)) && c.Q1s.reserve(sizeof(float) * T * nb_W) &&
              c.Q2.reserve((size_t) T * C) && c.Q2s.reserve(sizeof(float) * T * nb_C);
    // staged metadata: row_doc T, brow_doc nb, start / len / bstart / blen per document, tokens T,
    // types T (each padded to 64 entries), one SSMax scale per (attention layer, document), then the
    // attention plans (token rows banded and full, HRA block rows; 5 ints per item)
    const size_t plan_ints = 5 * (2 * nxk::attn::n_items(b.len.data(), b.n_docs, nxk::attn::QT3) +
                                  nxk::attn::n_items(b.blen.data(), b.n_docs, nxk::attn::QT3)) + 3 * 64;
    const size_t meta = sizeof(int32_t) * ((size_t) 3 * T + (size_t) b.nb + 4 * (size_t) b.n_docs + 9 * 64 +
                                           plan_ints) +
                        sizeof(float) * (size_t) b.n_docs * (size_t) std::max(hp.n_layer, 1) + 256;
    c.stage_need = meta;
    ok = ok && c.meta.reserve(meta);
    size_t ws = std::max(nxk_attention_workspace(b.len.data(), b.n_docs, -1),
                         nxk_attention_workspace(b.blen.data(), b.n_docs, -1));
    ok = ok && c.attn_ws.reserve(std::max<size_t>(ws, 256));
    ok = ok && c.pooled.reserve(sizeof(float) * (size_t) b.n_docs * C);
    const size_t stage = meta;
    if (ok && c.h_stage_bytes < stage) {
        if (c.h_stage) cudaFreeHost(c.h_stage);
        c.h_stage = nullptr;
        c.h_stage_bytes = 0;
        if (cudaMallocHost(&c.h_stage, stage) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
        } else {
            c.h_stage_bytes = stage;
        }
    }
    return ok;
}

// One forward pass.  tokens / types are device pointers when the layout says so.
// this rank's part of one sequence split over ranks (rows [offset, offset + Batch.T) of `total`)
struct ShardRun {
    int rank = 0, world = 1, offset = 0, total = 0;
    ncclComm_t comm = nullptr;
};

// Fills rows [-h, 0) of x from the previous rank's last h rows and rows [rows, rows + h) from the
// next rank's first h rows (x: rows of `width` floats).
bool halo_rows(const ShardRun & sh, float * x, int rows, int width, int h, cudaStream_t s) {
    if (h <= 0 || sh.world == 1) return true;
    const nxs::NcclApi & n = nxs::nccl();
    const size_t cnt = (size_t) h * width;
    bool ok = nxs::nccl_ok(n.group_start(), "group start");
    if (sh.rank > 0) {
        ok = ok && nxs::nccl_ok(n.send(x, cnt, ncclFloat32, sh.rank - 1, sh.comm, s), "halo send");
        ok = ok && nxs::nccl_ok(n.recv(x - cnt, cnt, ncclFloat32, sh.rank - 1, sh.comm, s), "halo recv");
    }
    if (sh.rank + 1 < sh.world) {
        ok = ok && nxs::nccl_ok(n.send(x + (size_t) (rows - h) * width, cnt, ncclFloat32, sh.rank + 1, sh.comm, s),
                                "halo send");
        ok = ok && nxs::nccl_ok(n.recv(x + (size_t) rows * width, cnt, ncclFloat32, sh.rank + 1, sh.comm, s),
                                "halo recv");
    }
    return nxs::nccl_ok(n.group_end(), "group end") && ok;
}

int run_encoder(nextera_context & c, const Batch & b, float rope0_base, const int32_t * tokens,
                const int32_t * types, bool on_host, cudaStream_t s, float * d_hidden_out, float * d_pooled_out,
                int normalize, float ** hidden_dev, const ShardRun * sh = nullptr, void * stage = nullptr,
                size_t * tok_off = nullptr, size_t * typ_off = nullptr) {
    const hparams & hp = c.hp;
    const int T = b.T, C = hp.n_embd, H = hp.n_head, G = hp.n_kv_head, D = hp.head_dim;
    if (!ensure_arena(c, b) || !ensure_rope(c, 0, b.max_len, rope0_base) ||
        !ensure_rope(c, 1, b.max_len, hp.swa_rope_base)) {
        fprintf(stderr, "nexterabert: failed to allocate the device buffers for %d tokens\n", T);
        return 2;
    }
    // stage the layout (and host tokens) in pinned memory, one copy to the device
    int32_t * hs = (int32_t *) (stage ? stage : c.h_stage);
    int32_t * dm = c.meta.as<int32_t>();
    size_t o = 0;
    auto put = [&](const int32_t * src, size_t n) {
        const size_t at = o;
        if (src) memcpy(hs + at, src, n * sizeof(int32_t));
        o += (n + 63) / 64 * 64;
        return at;
    };
    const size_t o_row = put(b.row_doc.data(), T);
    const size_t o_brow = put(b.brow_doc.data(), b.nb);
    const size_t o_start = put(b.start.data(), b.n_docs), o_len = put(b.len.data(), b.n_docs);
    const size_t o_bstart = put(b.bstart.data(), b.n_docs), o_blen = put(b.blen.data(), b.n_docs);
    size_t o_tok = 0, o_typ = 0;
    const bool use_types = types && hp.n_types > 0;
    if (on_host) {
        o_tok = put(tokens, T);
        if (use_types) o_typ = put(types, T);
    }
    if (tok_off) *tok_off = o_tok;
    if (typ_off) *typ_off = o_typ;
    // SSMax scales per attention layer and document (host math as in the reference)
    std::vector<int> scale_off(hp.n_layer, -1);
    float * hsc = (float *) (hs + o);
    size_t n_sc = 0;
    const float base_scale = 1.0f / std::sqrt((float) D);
    const int n_layer = c.debug_n_layers >= 0 ? std::min(c.debug_n_layers, hp.n_layer) : hp.n_layer;
    Forward fw(c, s);
    for (int l = 0; l < n_layer; ++l) {
        if (hp.block_types[l] == MIX_LILY) continue;
        const std::string pre = "blocks." + std::to_string(l) + ".attn.";
        const bool swa = hp.block_types[l] == MIX_SWA;
        scale_off[l] = (int) n_sc;
        for (int d = 0; d < b.n_docs; ++d) {
            const int n = hp.block_types[l] == MIX_HRA ? b.blen[d] : b.len[d];
            hsc[n_sc++] = base_scale * (swa ? 1.0f : fw.ssmax_scale(pre, n));
        }
    }
    // the attention plans of this batch (one per kind of rows and band the layers use), staged with
    // the rest so one copy uploads everything; sharded runs plan per call instead (nxk_attention_kv)
    struct APlan {
        bool blocks;
        int half;
        size_t n, off;
        nxk::attn::Scratch sp;
    };
    std::vector<APlan> aplans;
    size_t o_end = o + (n_sc + 63) / 64 * 64;
    if (!sh) {
        std::vector<nxk::attn::Item> items;
        for (int l = 0; l < n_layer; ++l) {
            const mixer_type mt = hp.block_types[l];
            if (mt == MIX_LILY) continue;
            const bool blocks = mt == MIX_HRA;
            const int half = mt == MIX_SWA ? std::max(1, hp.swa_window / 2) : -1;
            bool have = false;
            for (const APlan & p : aplans) have = have || (p.blocks == blocks && p.half == half);
            if (have) continue;
            const std::vector<int32_t> & st = blocks ? b.bstart : b.start, & ln = blocks ? b.blen : b.len;
            nxk::attn::plan(st.data(), ln.data(), b.n_docs, half, nxk::attn::QT3, blocks ? b.nb : T, items);
            aplans.push_back({blocks, half, items.size(), o_end, nxk::attn::scratch_plan(ln.data(), b.n_docs, half)});
            memcpy(hs + o_end, items.data(), items.size() * sizeof(nxk::attn::Item));
            o_end += (items.size() * sizeof(nxk::attn::Item) / sizeof(int32_t) + 63) / 64 * 64;
        }
    }
    const size_t stage_ints = sh ? o + n_sc : o_end;
    cudaMemcpyAsync(dm, hs, stage_ints * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    const float * d_scales = (const float *) (dm + o);
    Layout L;
    L.row_doc = dm + o_row;
    L.brow_doc = dm + o_brow;
    L.start = dm + o_start;
    L.len = dm + o_len;
    L.bstart = dm + o_bstart;
    L.blen = dm + o_blen;
    L.tokens = on_host ? dm + o_tok : tokens;
    L.types = use_types ? (on_host ? dm + o_typ : types) : nullptr;

    float * X = c.X.as<float>(), * X2 = c.X2.as<float>(), * U = c.U.as<float>();
    // row 0 of Fa / Fb / Fc comes after HALO_ROWS rows of padding (halo rows of a shard)
    float * Fa = c.Fa.as<float>() + (size_t) HALO_ROWS * C, * Fb = c.Fb.as<float>() + (size_t) HALO_ROWS * C;
    float * Fc = c.Fc.as<float>() + (size_t) HALO_ROWS * C;
    int8_t * Q1 = c.Q1.as<int8_t>(), * Q2 = c.Q2.as<int8_t>();
    float * Q1s = c.Q1s.as<float>(), * Q2s = c.Q2s.as<float>();

    // embedding (+ segment embedding)
    {
        const RawTensor & e = c.raw.at("embedding.weight");
        const RawTensor * tt = use_types ? &c.raw.at("token_type_embeddings.weight") : nullptr;
        fw.mark(PROF_ROWS);
        fw.rows(nxk_embed(e.type, e.d.p, (int) e.ne[1], C, L.tokens, T, tt ? tt->type : 0, tt ? tt->d.p : nullptr,
                          tt ? (int) tt->ne[1] : 0, L.types, X, s), "embed");
    }

    // attention of a mixer over `rows` rows laid out by (start, len, row_doc).  Sharded, the keys
    // come from beyond this rank's rows: band layers read `half` halo rows of the neighbours,
    // full layers the K / V of all ranks, gathered (tot_rows rows, this rank's at row_off).
    auto attention = [&](const std::string & pre, const int8_t * hq, const float * hsx, int rows,
                         const int32_t * start, const int32_t * len, const int32_t * row_doc,
                         const std::vector<int32_t> & h_start, const std::vector<int32_t> & h_len, int rope,
                         int half, const float * scale, float * y, int tot_rows, int row_off) {
        // c_q, c_k, c_v as one GEMM over their concatenated rows (each output column is the
        // same dot product as in the separate layers), then DyT + RoPE and the layouts in one pass
        const int ld = (H + 2 * G) * D;
        float * q = U;
        float * qkv = q + (size_t) rows * H * D;
        float * k, * v;
        int Tk, koff;
        if (!sh) {
            Tk = rows;
            koff = 0;
            k = qkv + (size_t) rows * ld;
        } else if (half >= 0) {
            Tk = rows + 2 * half;
            koff = half;
            k = c.kv_ext.as<float>();
        } else {
            Tk = tot_rows;
            koff = row_off;
            k = c.kv_full.as<float>();
        }
        v = k + (size_t) G * Tk * D;
        fw.linear(pre + QKV_NAME, hq, hsx, rows, nullptr, qkv);
        fw.mark(PROF_ROWS);
        fw.rows(nxk_qkv_prep_kv(qkv, ld, fw.p(pre + "q_norm.alpha"), fw.p(pre + "q_norm.beta"),
                                fw.p(pre + "k_norm.alpha"), fw.p(pre + "k_norm.beta"), c.rope_cos[rope].as<float>(),
                                c.rope_sin[rope].as<float>(), row_doc, start, rows, H, G, D, Tk, koff, q, k, v, s),
                "qkv_prep");
        fw.mark(PROF_ATTN);
        if (sh && fw.ok) {
            const nxs::NcclApi & n = nxs::nccl();
            bool ok = true;
            if (half >= 0) {
                for (int g = 0; ok && g < 2 * G; ++g)       // k heads, then v heads
                    ok = halo_rows(*sh, k + ((size_t) g * Tk + koff) * D, rows, D, half, s);
            } else {
                // in place: head g's rows of this rank already sit at row_off of the gathered buffer
                ok = nxs::nccl_ok(n.group_start(), "group start");
                for (int g = 0; ok && g < 2 * G; ++g) {
                    float * hb = k + (size_t) g * Tk * D;
                    ok = nxs::nccl_ok(n.all_gather(hb + (size_t) koff * D, hb, (size_t) rows * D, ncclFloat32,
                                                   sh->comm, s), "all-gather");
                }
                ok = nxs::nccl_ok(n.group_end(), "group end") && ok;
            }
            if (!ok) fw.ok = false;
        }
        if (sh) {
            fw.rows(nxk_attention_kv(q, k, v, rows, Tk, koff, H, G, D, half, scale, start, len, b.n_docs,
                                     h_start.data(), h_len.data(), c.attn_ws.p, c.attn_ws.bytes, y, s), "attention");
            return;
        }
        const bool blocks = &h_start == &b.bstart;
        const APlan * ap = nullptr;
        for (const APlan & p : aplans) if (p.blocks == blocks && p.half == half) ap = &p;
        if (!ap || ap->sp.bytes > c.attn_ws.bytes) {
            fprintf(stderr, "nexterabert: no attention plan for this layer\n");
            fw.ok = false;
            return;
        }
        fw.rows(nxk::attn::launch_planned(q, k, v, rows, Tk, koff, H, G, half, scale, start, len,
                                     (const nxk::attn::Item *) (dm + ap->off), ap->n, ap->sp, (float *) c.attn_ws.p, y, s),
                "attention");
    };

    // halo rows of a token convolution's input (sharded runs only); returns the halo to read
    auto conv_halo = [&](float * x, int width, int k) {
        if (!sh || !fw.ok) return 0;
        const int h = k / 2;
        if (!halo_rows(*sh, x, T, width, h, s)) fw.ok = false;
        return h;
    };

    // x + c_proj(sigmoid(c_gate(y)) * z)  (gated_out, :1209-1214); y, z: [T][C]
    auto gated_out = [&](const std::string & pre, const float * y, const float * z, float * gl) {
        fw.mark(PROF_ROWS);
        fw.rows(nxk_quantize(y, T, C, Q1, Q1s, s), "quantize");
        // (nxk_linear_i8_gate_q fuses the next two steps but is slower here: each epilogue lane
        // reads its own row of z, 32 rows per warp load)
        fw.linear(pre + "c_gate.weight", Q1, Q1s, T, nullptr, gl);
        fw.mark(PROF_ROWS);
        fw.rows(nxk_gate(gl, z, T, C, nullptr, Q1, Q1s, s), "gate");
        fw.linear(pre + "c_proj.weight", Q1, Q1s, T, X, X);       // x += c_proj(...), in place
    };

    for (int l = 0; l < n_layer && fw.ok; ++l) {
        const std::string blk = "blocks." + std::to_string(l) + ".", pre = blk + "attn.";
        const mixer_type mt = hp.block_types[l];
        fw.mark(PROF_ROWS);
        fw.rows(nxk_rms_norm(X, fw.p(blk + "attn_norm.weight"), hp.rms_eps, T, C, nullptr, Q2, Q2s, s), "rms_norm");
        if (mt == MIX_LILY) {
            const int r2 = fw.n_out(pre + LTC_IN_NAME);             // fused: in_proj | A, 2r columns
            const int r = r2 > 0 ? r2 / 2 : fw.n_out(pre + "ltc_conv.in_proj.weight");
            if (r2 > 0) {
                fw.linear(pre + LTC_IN_NAME, Q2, Q2s, T, nullptr, Fa);
            } else {
                fw.linear(pre + "ltc_conv.in_proj.weight", Q2, Q2s, T, nullptr, Fa);
                fw.linear(pre + "ltc_conv.A.weight", Q2, Q2s, T, nullptr, Fb);
            }
            const ConvTaps * k1 = fw.taps(pre + "ltc_conv.kernel");
            if (!fw.ok) break;
            fw.mark(PROF_ROWS);
            const int h1 = conv_halo(Fa, r2 > 0 ? r2 : r, k1->k);
            if (r2 > 0)
                fw.rows(nxk_dwconv_halo_ld(Fa, Fa + r, r2, k1->taps.as<float>(), k1->k, h1, L.row_doc, L.start, L.len,
                                           T, r, nullptr, Q1, Q1s, s), "dwconv");
            else
                fw.rows(nxk_dwconv_halo(Fa, Fb, k1->taps.as<float>(), k1->k, h1, L.row_doc, L.start, L.len, T, r,
                                        nullptr, Q1, Q1s, s), "dwconv");
            fw.linear(pre + "ltc_conv.out_proj.weight", Q1, Q1s, T, nullptr, Fa);
            fw.linear(pre + "x_proj.weight", Q2, Q2s, T, nullptr, Fb);
            fw.linear(pre + "B_proj.weight", Q2, Q2s, T, nullptr, Fc);
            const ConvTaps * k2 = fw.taps(pre + "state_conv.depthwise.weight");
            if (!fw.ok) break;
            fw.mark(PROF_ROWS);
            const int h2 = conv_halo(Fa, C, k2->k);
            conv_halo(Fb, C, k2->k);
            fw.rows(nxk_lily_state_halo(Fa, Fb, Fc, k2->taps.as<float>(), k2->k, h2, L.row_doc, L.start, L.len, T, C,
                                        nullptr, Q1, Q1s, s), "lily_state");
            fw.linear(pre + "c_proj.weight", Q1, Q1s, T, X, X);      // x += c_proj(...), in place
        } else if (mt == MIX_SWA || mt == MIX_ATTN) {
            const bool swa = mt == MIX_SWA;
            const int half = swa ? std::max(1, hp.swa_window / 2) : -1;
            attention(pre, Q2, Q2s, T, L.start, L.len, L.row_doc, b.start, b.len, swa ? 1 : 0, half,
                      d_scales + scale_off[l], Fb, sh ? sh->total : 0, sh ? sh->offset : 0);
            gated_out(pre, Fb, Fb, Fa);
        } else {
            // HRA (mix_hra, :1246-1264)
            fw.linear(pre + "qkv_in.weight", Q2, Q2s, T, nullptr, Fa);
            const ConvTaps * kq = fw.taps(pre + "qkv_conv.depthwise.weight");
            if (!fw.ok) break;
            fw.mark(PROF_ROWS);
            const int hq = conv_halo(Fa, C, kq->k);
            fw.rows(nxk_dwconv_halo(Fa, nullptr, kq->taps.as<float>(), kq->k, hq, L.row_doc, L.start, L.len, T, C, Fb,
                                    nullptr, nullptr, s), "dwconv");
            fw.linear(pre + "qkv_gate.weight", Q2, Q2s, T, nullptr, Fa);
            fw.mark(PROF_ROWS);
            fw.rows(nxk_block_mean(Fb, Fa, C, hp.hra_block, L.start, L.len, L.bstart, L.brow_doc, b.nb, nullptr, Q1, Q1s,
                                   s), "block_mean");
            attention(pre, Q1, Q1s, b.nb, L.bstart, L.blen, L.brow_doc, b.bstart, b.blen, 0, -1,
                      d_scales + scale_off[l], Fa, sh ? sh->total / hp.hra_block : 0, sh ? sh->offset / hp.hra_block : 0);
            fw.linear(pre + "c_C.weight", Q2, Q2s, T, nullptr, Fb);
            fw.mark(PROF_ROWS);
            fw.rows(nxk_upsample_add(Fa, Fb, C, hp.hra_block, T, L.row_doc, L.start, L.bstart, Fc, s), "upsample_add");
            const ConvTaps * ko = fw.taps(pre + "c_o.depthwise.weight");
            if (!fw.ok) break;
            fw.mark(PROF_ROWS);
            const int ho = conv_halo(Fc, C, ko->k);
            fw.rows(nxk_dwconv_halo(Fc, nullptr, ko->taps.as<float>(), ko->k, ho, L.row_doc, L.start, L.len, T, C, Fb,
                                    nullptr, nullptr, s), "dwconv");
            gated_out(pre, Fc, Fb, Fa);
        }
        // MLP (:1284-1289)
        fw.mark(PROF_ROWS);
        fw.rows(nxk_rms_norm(X, fw.p(blk + "mlp_norm.weight"), hp.rms_eps, T, C, nullptr, Q2, Q2s, s), "rms_norm");
        const int I = fw.n_out(blk + "mlp.c_fc.weight");
        // c_fc, relu^2 and its quantization in one kernel when I is a multiple of 256
        if (!fw.linear_q(blk + "mlp.c_fc.weight", Q2, Q2s, T, nullptr, Q1, Q1s)) {
            fw.linear(blk + "mlp.c_fc.weight", Q2, Q2s, T, nullptr, U);
            fw.mark(PROF_ROWS);
            fw.rows(nxk_relu_sqr(U, T, I, nullptr, Q1, Q1s, s), "relu_sqr");
        }
        fw.linear(blk + "mlp.c_proj.weight", Q1, Q1s, T, X, X);      // x += c_proj(...), in place
    }
    if (!fw.ok) return 3;
    float * hidden = X;
    if (c.debug_n_layers < 0) {
        fw.mark(PROF_ROWS);
        fw.rows(nxk_layer_norm(X, fw.p("out_norm.weight"), fw.p("out_norm.bias"), hp.ln_eps, T, C, X2, s), "layer_norm");
        hidden = X2;
    }
    float * pooled = d_pooled_out ? d_pooled_out : c.pooled.as<float>();
    fw.mark(PROF_ROWS);
    if (!sh) {
        fw.rows(nxk_pool(hidden, L.start, L.len, b.n_docs, C, normalize, pooled, s), "pool", 2);
    } else if (fw.ok) {
        // the reference sums the sequence's rows in order: the running sum goes from rank to rank,
        // each continuing it over its rows; the last rank scales it and sends it to all
        const nxs::NcclApi & n = nxs::nccl();
        bool ok = true;
        if (sh->rank == 0) ok = cudaMemsetAsync(pooled, 0, sizeof(float) * C, s) == cudaSuccess;
        else ok = nxs::nccl_ok(n.recv(pooled, C, ncclFloat32, sh->rank - 1, sh->comm, s), "pool recv");
        if (ok) fw.rows(nxk_pool_continue(hidden, T, C, pooled, s), "pool");
        if (ok && sh->rank + 1 < sh->world)
            ok = nxs::nccl_ok(n.send(pooled, C, ncclFloat32, sh->rank + 1, sh->comm, s), "pool send");
        if (ok && sh->rank + 1 == sh->world) fw.rows(nxk_pool_finish(sh->total, C, normalize, pooled, s), "pool");
        if (ok)
            ok = nxs::nccl_ok(n.broadcast(pooled, pooled, C, ncclFloat32, sh->world - 1, sh->comm, s), "broadcast");
        if (!ok) fw.ok = false;
    }
    if (d_hidden_out) cudaMemcpyAsync(d_hidden_out, hidden, sizeof(float) * (size_t) T * C, cudaMemcpyDeviceToDevice, s);
    fw.mark(-1);
    if (!fw.ok) return 3;
    *hidden_dev = hidden;
    return 0;
}

void collect_profile(nextera_context & c) {
    profiler & pr = c.prof;
    if (!pr.enabled || pr.marks.size() < 2) return;
    cudaEventSynchronize(pr.marks.back().first);
    for (size_t i = 0; i + 1 < pr.marks.size(); ++i) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, pr.marks[i].first, pr.marks[i + 1].first);
        if (pr.marks[i].second >= 0) pr.ms[pr.marks[i].second] += ms;
    }
    for (auto & m : pr.marks) cudaEventDestroy(m.first);
    pr.marks.clear();
}

constexpr int GRAPH_MAX_T = 32768;       // larger batches keep the GPU busy without graphs
constexpr size_t GRAPH_CACHE = 8;

std::vector<const void *> graph_sig(const nextera_context & c) {
    return { c.X.p, c.X2.p, c.U.p, c.Fa.p, c.Fb.p, c.Fc.p, c.Q1.p, c.Q1s.p, c.Q2.p, c.Q2s.p, c.meta.p,
             c.attn_ws.p, c.pooled.p, c.rope_cos[0].p, c.rope_cos[1].p, c.rope_sin[0].p, c.rope_sin[1].p };
}

void drop_graph(nextera_context::GraphEntry & g) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.stage) cudaFreeHost(g.stage);
    if (g.h_pooled) cudaFreeHost(g.h_pooled);
    if (g.h_hidden) cudaFreeHost(g.h_hidden);
    g = nextera_context::GraphEntry();
}

// Records the forward of batch b as a graph (the same shape has run eagerly before, so the arena,
// rope tables and pinned staging already fit it and nothing below allocates device memory).
// Returns the new entry, or nullptr (and the call runs eagerly) if capture fails.
nextera_context::GraphEntry * capture_graph(nextera_context * c, const Batch & b, float rope0,
                                            const int32_t * tokens, const int32_t * types, bool want_hidden,
                                            int32_t normalize, std::vector<int32_t> key) {
    const int C = c->hp.n_embd;
    // the same sizing calls run_encoder makes, outside the capture (no-ops when they already fit)
    if (!ensure_arena(*c, b) || !ensure_rope(*c, 0, b.max_len, rope0) ||
        !ensure_rope(*c, 1, b.max_len, c->hp.swa_rope_base))
        return nullptr;
    nextera_context::GraphEntry g;
    g.key = std::move(key);
    if (cudaMallocHost(&g.stage, c->stage_need) != cudaSuccess ||
        cudaMallocHost((void **) &g.h_pooled, sizeof(float) * (size_t) b.n_docs * C) != cudaSuccess ||
        (want_hidden && cudaMallocHost((void **) &g.h_hidden, sizeof(float) * (size_t) b.T * C) != cudaSuccess)) {
        cudaGetLastError();
        drop_graph(g);
        return nullptr;
    }
    const int64_t l0 = c->launches;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        drop_graph(g);
        return nullptr;
    }
    float * hid = nullptr;
    int rc = run_encoder(*c, b, rope0, tokens, types, true, c->stream, nullptr, nullptr, normalize, &hid, nullptr,
                         g.stage, &g.o_tok, &g.o_typ);
    if (rc == 0) {
        cudaMemcpyAsync(g.h_pooled, c->pooled.p, sizeof(float) * (size_t) b.n_docs * C, cudaMemcpyDeviceToHost,
                        c->stream);
        if (want_hidden)
            cudaMemcpyAsync(g.h_hidden, hid, sizeof(float) * (size_t) b.T * C, cudaMemcpyDeviceToHost, c->stream);
    }
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    if (rc != 0 || e != cudaSuccess || !graph || cudaGraphInstantiate(&g.exec, graph, 0) != cudaSuccess) {
        cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        drop_graph(g);
        return nullptr;
    }
    cudaGraphDestroy(graph);
    g.launches = c->launches - l0;
    g.sig = graph_sig(*c);
    if (c->graphs.size() >= GRAPH_CACHE) {
        size_t old = 0;
        for (size_t i = 1; i < c->graphs.size(); ++i)
            if (c->graphs[i].used < c->graphs[old].used) old = i;
        drop_graph(c->graphs[old]);
        c->graphs.erase(c->graphs.begin() + (ptrdiff_t) old);
    }
    c->graphs.push_back(std::move(g));
    return &c->graphs.back();
}

int32_t encode_host(nextera_context * c, const int32_t * tokens, const int32_t * types, const int32_t * lengths,
                    int32_t n_seqs, float * hidden, float * pooled, int32_t normalize) {
    const auto t0 = std::chrono::steady_clock::now();
    cudaSetDevice(c->device);
    Batch b;
    float rope0 = 0.0f;
    if (!tokens) return 1;
    int rc = prepare(*c, tokens, types, lengths, n_seqs, true, b, rope0);
    if (rc) return rc;
    const bool use_types = types && c->hp.n_types > 0;
    if (!c->prof.enabled && b.T <= GRAPH_MAX_T) {
        std::vector<int32_t> key(b.len);
        key.push_back((use_types ? 1 : 0) | (hidden ? 2 : 0) | (normalize ? 4 : 0) | ((c->debug_n_layers + 1) << 3));
        nextera_context::GraphEntry * g = nullptr;
        for (auto & e : c->graphs) if (e.key == key) g = &e;
        if (g && g->sig != graph_sig(*c)) {
            drop_graph(*g);
            c->graphs.erase(c->graphs.begin() + (g - c->graphs.data()));
            g = nullptr;
        }
        if (!g && std::find(c->seen.begin(), c->seen.end(), key) != c->seen.end())
            g = capture_graph(c, b, rope0, tokens, types, hidden != nullptr, normalize, key);
        if (g) {
            const int C = c->hp.n_embd;
            g->used = ++c->graph_clock;
            memcpy((int32_t *) g->stage + g->o_tok, tokens, sizeof(int32_t) * (size_t) b.T);
            if (use_types) memcpy((int32_t *) g->stage + g->o_typ, types, sizeof(int32_t) * (size_t) b.T);
            rc = 0;
            if (cudaGraphLaunch(g->exec, c->stream) != cudaSuccess || cudaStreamSynchronize(c->stream) != cudaSuccess) {
                fprintf(stderr, "nexterabert: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
                rc = 3;
            } else if (int32_t e = nxk_take_error(c->stream)) {
                fprintf(stderr, "nexterabert: a kernel timed out waiting on its pipeline (code 0x%x)\n", e);
                rc = 3;
            }
            c->launches += g->launches;
            if (rc == 0) {
                if (pooled) memcpy(pooled, g->h_pooled, sizeof(float) * (size_t) n_seqs * C);
                if (hidden) memcpy(hidden, g->h_hidden, sizeof(float) * (size_t) b.T * C);
            }
            c->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            return rc;
        }
        if (std::find(c->seen.begin(), c->seen.end(), key) == c->seen.end()) {
            if (c->seen.size() >= 32) c->seen.erase(c->seen.begin());
            c->seen.push_back(std::move(key));
        }
    }
    float * hid = nullptr;
    rc = run_encoder(*c, b, rope0, tokens, types, true, c->stream, nullptr, nullptr, normalize, &hid);
    if (rc == 0) {
        if (hidden) cudaMemcpyAsync(hidden, hid, sizeof(float) * (size_t) b.T * c->hp.n_embd, cudaMemcpyDeviceToHost, c->stream);
        if (pooled) cudaMemcpyAsync(pooled, c->pooled.p, sizeof(float) * (size_t) n_seqs * c->hp.n_embd,
                                    cudaMemcpyDeviceToHost, c->stream);
        if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
            fprintf(stderr, "nexterabert: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
            rc = 3;
        } else if (int32_t e = nxk_take_error(c->stream)) {
            fprintf(stderr, "nexterabert: a kernel timed out waiting on its pipeline (code 0x%x)\n", e);
            rc = 3;
        }
    }
    collect_profile(*c);
    c->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (c->prof.enabled) {
        c->prof.total_ms += c->last_ms;
        c->prof.calls++;
    }
    return rc;
}

// y = W x (+ bias) for M rows of x (K floats each) into out (M rows of W's n_out): the int8 linear
// when W is on the int8 path (x quantized first, as the qcache's op_copy does, :1125-1130), else
// ggml_mul_mat on W's blocks (:1140-1142).  Returns W's n_out, or 0 after printing why.
int head_linear(nextera_context & c, Forward & fw, const std::string & name, const float * x, int M, int K,
                const float * bias, float * out, cudaStream_t s) {
    auto it = c.i8.find(name);
    if (it != c.i8.end()) {
        const I8Weight & w = it->second;
        if (w.n_in != K || bias) {
            fprintf(stderr, "nexterabert: '%s' cannot run on the int8 path here (%s)\n", name.c_str(),
                    bias ? "a biased int8 linear" : "input width");
            return 0;
        }
        const int nb = (K + I8_BLOCK - 1) / I8_BLOCK;
        if (!c.head_q.reserve((size_t) M * K) || !c.head_qs.reserve(sizeof(float) * (size_t) (M + 3) / 4 * 4 * nb)) {
            fprintf(stderr, "nexterabert: failed to allocate the head's buffers\n");
            return 0;
        }
        fw.mark(PROF_ROWS);
        fw.rows(nxk_quantize(x, M, K, c.head_q.as<int8_t>(), c.head_qs.as<float>(), s), "quantize");
        fw.linear(name, c.head_q.as<int8_t>(), c.head_qs.as<float>(), M, nullptr, out);
        return fw.ok ? w.n_out : 0;
    }
    auto rt = c.raw.find(name);
    if (rt == c.raw.end()) {
        fprintf(stderr, "nexterabert: missing tensor '%s'\n", name.c_str());
        return 0;
    }
    const RawTensor & r = rt->second;
    const size_t ws = nxk_mul_mat_workspace(r.type, K, M);
    if (r.ne[0] != K || ws == 0) {
        fprintf(stderr, "nexterabert: '%s' (type %d, %lld inputs) cannot multiply rows of %d\n", name.c_str(), r.type,
                (long long) r.ne[0], K);
        return 0;
    }
    if (!c.head_ws.reserve(ws)) {
        fprintf(stderr, "nexterabert: failed to allocate the head's buffers\n");
        return 0;
    }
    fw.mark(PROF_ROWS);
    fw.rows(nxk_mul_mat(r.type, r.d.p, (int) r.ne[1], K, x, M, bias, c.head_ws.p, out, s), name.c_str(), 2);
    return fw.ok ? (int) r.ne[1] : 0;
}

// transform(pre, x) (:1296-1301): dense (no bias) -> GELU(erf) -> ggml_norm * norm.weight, on M rows
// of C floats; the result in c.head_y (M rows of C)
float * head_transform(nextera_context & c, Forward & fw, const std::string & pre, const float * x, int M,
                       cudaStream_t s) {
    const int C = c.hp.n_embd;
    if (!c.head_y.reserve(sizeof(float) * (size_t) M * C)) {
        fprintf(stderr, "nexterabert: failed to allocate the head's buffers\n");
        return nullptr;
    }
    float * y = c.head_y.as<float>();
    const int n = head_linear(c, fw, pre + "dense.weight", x, M, C, nullptr, y, s);
    if (n != C) {
        if (n) fprintf(stderr, "nexterabert: '%sdense.weight' has %d outputs, not %d\n", pre.c_str(), n, C);
        return nullptr;
    }
    fw.mark(PROF_ROWS);
    fw.rows(nxk_gelu_norm(y, fw.p(pre + "norm.weight"), c.hp.ln_eps, M, C, y, s), "gelu_norm");
    return fw.ok ? y : nullptr;
}

// copies a head's output to the host, waits, and reports device errors (as encode_host)
int32_t finish_head(nextera_context & c, const float * d_out, size_t n, float * out,
                    std::chrono::steady_clock::time_point t0) {
    cudaMemcpyAsync(out, d_out, sizeof(float) * n, cudaMemcpyDeviceToHost, c.stream);
    int32_t rc = 0;
    if (cudaStreamSynchronize(c.stream) != cudaSuccess) {
        fprintf(stderr, "nexterabert: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
        rc = 3;
    } else if (int32_t e = nxk_take_error(c.stream)) {
        fprintf(stderr, "nexterabert: a kernel timed out waiting on its pipeline (code 0x%x)\n", e);
        rc = 3;
    }
    collect_profile(c);
    c.last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (c.prof.enabled) {
        c.prof.total_ms += c.last_ms;
        c.prof.calls++;
    }
    return rc;
}

enum head_kind { HEAD_POOLER, HEAD_CLASSIFIER };

// run_forward with a head (:1866-1925): the encoder, then pooler (:1304-1310) or classifier (:1313-1317)
int32_t run_head(nextera_context * c, const int32_t * tokens, const int32_t * types, const int32_t * lengths,
                 int32_t n_seqs, head_kind head, float * out) {
    const auto t0 = std::chrono::steady_clock::now();
    cudaSetDevice(c->device);
    if (!tokens || !out) return 1;
    Batch b;
    float rope0 = 0.0f;
    int rc = prepare(*c, tokens, types, lengths, n_seqs, true, b, rope0);
    if (rc) return rc;
    const hparams & hp = c->hp;
    const int C = hp.n_embd;
    const bool pooled = head == HEAD_POOLER || hp.cls == CLS_SEQUENCE || hp.cls == CLS_CHOICE;
    // the encoder's per-document pooling with the 1/n scale is op_doc_mean (:662-674)
    float * hid = nullptr;
    rc = run_encoder(*c, b, rope0, tokens, types, true, c->stream, nullptr, nullptr, 0, &hid);
    if (rc) return rc;
    Forward fw(*c, c->stream);
    const int M = pooled ? b.n_docs : b.T;
    float * h = head_transform(*c, fw, pooled ? "pooler." : "head.", pooled ? c->pooled.as<float>() : hid, M,
                               c->stream);
    if (!h) return fw.ok ? 2 : 3;
    if (head == HEAD_POOLER) {
        fw.mark(-1);
        return finish_head(*c, h, (size_t) M * C, out, t0);
    }
    const int L = hp.n_labels;
    if (!c->head_out.reserve(sizeof(float) * (size_t) M * std::max(L, 1))) return 2;
    const int n = head_linear(*c, fw, "classifier.weight", h, M, C, fw.p("classifier.bias"), c->head_out.as<float>(),
                              c->stream);
    fw.mark(-1);
    if (n != L) {
        if (n) fprintf(stderr, "nexterabert: the classifier has %d outputs for %d labels\n", n, L);
        return 3;
    }
    return finish_head(*c, c->head_out.as<float>(), (size_t) M * L, out, t0);
}

} // namespace

int32_t nextera_encode(struct nextera_context * c, const int32_t * tokens, const int32_t * lengths, int32_t n_seqs,
                       float * hidden, float * pooled, int32_t normalize) {
    return encode_host(c, tokens, nullptr, lengths, n_seqs, hidden, pooled, normalize);
}

int32_t nextera_encode_segments(struct nextera_context * c, const int32_t * tokens, const int32_t * token_types,
                                const int32_t * lengths, int32_t n_seqs, float * hidden, float * pooled,
                                int32_t normalize) {
    return encode_host(c, tokens, token_types, lengths, n_seqs, hidden, pooled, normalize);
}

int32_t nextera_encode_device(struct nextera_context * c, const int32_t * d_tokens, const int32_t * d_token_types,
                              const int32_t * lengths, int32_t n_seqs, float * d_hidden, float * d_pooled,
                              int32_t normalize, void * stream) {
    cudaSetDevice(c->device);
    Batch b;
    float rope0 = 0.0f;
    if (!d_tokens) return 1;
    int rc = prepare(*c, nullptr, nullptr, lengths, n_seqs, false, b, rope0);
    if (rc) return rc;
    float * hid = nullptr;
    return run_encoder(*c, b, rope0, d_tokens, d_token_types, false, (cudaStream_t) stream, d_hidden, d_pooled,
                       normalize, &hid);
}

int32_t nextera_shard_unique_id(uint8_t * id) {
    if (!id) return 1;
    const nxs::NcclApi & n = nxs::nccl();
    if (!n.ok) return 3;
    ncclUniqueId u;
    if (!nxs::nccl_ok(n.get_unique_id(&u), "get unique id")) return 3;
    memcpy(id, &u, sizeof(u));
    return 0;
}

int32_t nextera_shard_init(struct nextera_context * c, int32_t rank, int32_t world, const uint8_t * id) {
    if (!c || !id || world < 1 || rank < 0 || rank >= world) return 1;
    const nxs::NcclApi & n = nxs::nccl();
    if (!n.ok) return 3;
    cudaSetDevice(c->device);
    if (c->shard_comm) {
        n.comm_destroy(c->shard_comm);
        c->shard_comm = nullptr;
    }
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    if (!nxs::nccl_ok(n.comm_init_rank(&c->shard_comm, world, u, rank), "init")) {
        c->shard_comm = nullptr;
        return 3;
    }
    c->shard_rank = rank;
    c->shard_world = world;
    return 0;
}

int32_t nextera_encode_sharded(struct nextera_context * c, const int32_t * d_tokens, int32_t n_local, int32_t n_total,
                               float * d_hidden, float * d_pooled, int32_t normalize, void * stream) {
    if (!c || !d_tokens) return 1;
    if (!c->shard_comm) {
        fprintf(stderr, "nexterabert: nextera_encode_sharded before nextera_shard_init\n");
        return 1;
    }
    const hparams & hp = c->hp;
    const int world = c->shard_world, rank = c->shard_rank;
    const int half = std::max(1, hp.swa_window / 2);
    if (n_local <= 0 || (int64_t) n_local * world != n_total || n_local % hp.hra_block != 0 || n_local < half ||
        n_local < HALO_ROWS) {
        fprintf(stderr, "nexterabert: a sharded sequence needs n_total = %d x n_local, n_local a multiple of %d "
                        "and at least %d (got n_local %d, n_total %d)\n",
                world, hp.hra_block, std::max(half, HALO_ROWS), n_local, n_total);
        return 1;
    }
    for (const auto & kv : c->taps) {
        if (kv.second.k / 2 > HALO_ROWS) {
            fprintf(stderr, "nexterabert: a convolution of %d taps is wider than the shard halo\n", kv.second.k);
            return 1;
        }
    }
    cudaSetDevice(c->device);
    ShardRun sh;
    sh.rank = rank;
    sh.world = world;
    sh.offset = rank * n_local;
    sh.total = n_total;
    sh.comm = c->shard_comm;
    // one document relative to this rank's first row: [-offset, total - offset)
    Batch b;
    b.n_docs = 1;
    b.T = n_local;
    b.nb = n_local / hp.hra_block;
    b.max_len = n_total;
    b.start = {-sh.offset};
    b.len = {n_total};
    b.bstart = {-sh.offset / hp.hra_block};
    b.blen = {n_total / hp.hra_block};
    b.row_doc.assign(b.T, 0);
    b.brow_doc.assign(b.nb, 0);
    float rope0 = hp.rope_base;
    if (hp.ntk_train_len > 0 && n_total > hp.ntk_train_len) {
        const double d = hp.head_dim;
        rope0 = (float) ((double) rope0 * std::pow((double) n_total / hp.ntk_train_len, d / (d - 2.0)));
    }
    const size_t G = hp.n_kv_head, D = hp.head_dim;
    if (!c->kv_ext.reserve(sizeof(float) * 2 * G * (size_t) (n_local + 2 * half) * D) ||
        !c->kv_full.reserve(sizeof(float) * 2 * G * (size_t) n_total * D)) {
        fprintf(stderr, "nexterabert: failed to allocate the shard's K / V buffers\n");
        return 2;
    }
    float * hid = nullptr;
    return run_encoder(*c, b, rope0, d_tokens, nullptr, false, (cudaStream_t) stream, d_hidden, d_pooled, normalize,
                       &hid, &sh);
}

// ---------------------------------------------------------------------------
// one batch of documents partitioned over ranks
// ---------------------------------------------------------------------------
namespace {

// Estimated device time of one document of length L, in units of the per-token work of the linear
// layers and row ops: that work, plus the attention kernel's work per (row of its 64-query tiles,
// key in the tile's range) over every attention layer (band, full and, at block level, HRA).  The
// weight of a tile-key against a token, 3.9e-4 at 16 heads, is the ratio of the two measured on
// B200 for the 4096-document batch (attention 987 ms over 6.62e9 tile-keys, the rest 651 ms over
// 1.69e6 tokens).
double doc_cost(const hparams & hp, int64_t L) {
    const int64_t QT = nxk::attn::QT3;
    const int64_t half = std::max(1, hp.swa_window / 2);
    const int64_t tiles = (L + QT - 1) / QT;
    double keys = 0.0;
    for (mixer_type m : hp.block_types) {
        if (m == MIX_SWA) {
            for (int64_t i = 0; i < tiles; ++i) {
                const int64_t q0 = i * QT, q1 = std::min(L, q0 + QT);
                keys += (double) QT * (double) (std::min(L, q1 + half) - std::max<int64_t>(0, q0 - half));
            }
        } else if (m == MIX_ATTN) {
            keys += (double) tiles * QT * (double) L;
        } else if (m == MIX_HRA) {
            const int64_t nb = (L + hp.hra_block - 1) / hp.hra_block;
            keys += (double) ((nb + QT - 1) / QT) * QT * (double) nb;
        }
    }
    return (double) L + 3.9e-4 * keys * (double) hp.n_head / 16.0;
}

// The partition of a batch and, for rank 0, where each document's pooled row arrives.
struct PartPlan {
    std::vector<int32_t> part;         // rank of each document
    std::vector<int32_t> mine;         // this rank's documents, in batch order
    std::vector<int32_t> counts;       // documents per rank
    std::vector<int32_t> row_of;       // document -> row of the rank-ordered concatenation
    int64_t my_tokens = 0;
};

// Longest-first greedy assignment: documents in order of falling cost (ties: batch order), each to
// the rank with the least cost so far (ties: the lowest rank).  Deterministic, so every rank
// computes the same partition from the same lengths.
void partition(const hparams & hp, const int32_t * lengths, int32_t n, int32_t parts, int32_t * part) {
    std::vector<double> cost((size_t) n);
    for (int32_t i = 0; i < n; ++i) cost[(size_t) i] = doc_cost(hp, lengths[i]);
    std::vector<int32_t> order((size_t) n);
    for (int32_t i = 0; i < n; ++i) order[(size_t) i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return cost[(size_t) a] > cost[(size_t) b]; });
    std::vector<double> load((size_t) parts, 0.0);
    for (int32_t i : order) {
        int32_t best = 0;
        for (int32_t r = 1; r < parts; ++r)
            if (load[(size_t) r] < load[(size_t) best]) best = r;
        part[(size_t) i] = best;
        load[(size_t) best] += cost[(size_t) i];
    }
}

int make_part_plan(const nextera_context & c, const int32_t * lengths, int32_t n, int rank, int world, PartPlan & pp) {
    if (!lengths || n <= 0) return 1;
    for (int32_t i = 0; i < n; ++i) {
        if (lengths[i] <= 0) {
            fprintf(stderr, "nexterabert: empty sequence in batch\n");
            return 1;
        }
    }
    pp.part.assign((size_t) n, 0);
    if (world > 1) partition(c.hp, lengths, n, world, pp.part.data());
    pp.counts.assign((size_t) world, 0);
    pp.mine.clear();
    pp.my_tokens = 0;
    for (int32_t i = 0; i < n; ++i) {
        pp.counts[(size_t) pp.part[(size_t) i]]++;
        if (pp.part[(size_t) i] == rank) {
            pp.mine.push_back(i);
            pp.my_tokens += lengths[i];
        }
    }
    std::vector<int32_t> next((size_t) world, 0);
    for (int r = 1; r < world; ++r) next[(size_t) r] = next[(size_t) r - 1] + pp.counts[(size_t) r - 1];
    pp.row_of.resize((size_t) n);
    for (int32_t i = 0; i < n; ++i) pp.row_of[(size_t) i] = next[(size_t) pp.part[(size_t) i]]++;
    return 0;
}

// After this rank's forward left its documents' pooled rows in c.pooled (batch order among its
// own): every rank sends them to rank 0, which receives all ranks' rows in rank order and writes
// each document's row to d_out in batch order.  Enqueued on s; every rank must call it.
int gather_pooled(nextera_context & c, const PartPlan & pp, int n_seqs, float * d_out, cudaStream_t s) {
    const int C = c.hp.n_embd, world = c.shard_world, rank = c.shard_rank;
    const size_t row = (size_t) C;
    if (world == 1) {
        if (d_out != c.pooled.as<float>() &&
            cudaMemcpyAsync(d_out, c.pooled.p, sizeof(float) * row * (size_t) n_seqs, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return 3;
        return 0;
    }
    const nxs::NcclApi & n = nxs::nccl();
    if (rank == 0) {
        if (!c.part_rows.reserve(sizeof(float) * row * (size_t) n_seqs) || !c.part_idx.reserve(sizeof(int32_t) * (size_t) n_seqs))
            return 2;
        if (c.h_part_idx_n < (size_t) n_seqs) {
            if (c.h_part_idx) cudaFreeHost(c.h_part_idx);
            c.h_part_idx = nullptr;
            c.h_part_idx_n = 0;
            if (cudaMallocHost((void **) &c.h_part_idx, sizeof(int32_t) * (size_t) n_seqs) != cudaSuccess) {
                cudaGetLastError();
                return 2;
            }
            c.h_part_idx_n = (size_t) n_seqs;
        }
    }
    float * rows = c.part_rows.as<float>();
    bool ok = nxs::nccl_ok(n.group_start(), "group start");
    if (rank == 0) {
        size_t at = (size_t) pp.counts[0];
        for (int r = 1; r < world; ++r) {
            const size_t cnt = (size_t) pp.counts[(size_t) r];
            if (cnt) ok = ok && nxs::nccl_ok(n.recv(rows + at * row, cnt * row, ncclFloat32, r, c.shard_comm, s), "recv");
            at += cnt;
        }
    } else if (pp.counts[(size_t) rank]) {
        ok = ok && nxs::nccl_ok(n.send(c.pooled.p, (size_t) pp.counts[(size_t) rank] * row, ncclFloat32, 0, c.shard_comm, s),
                                "send");
    }
    ok = nxs::nccl_ok(n.group_end(), "group end") && ok;
    if (!ok) return 3;
    if (rank != 0) return 0;
    if (pp.counts[0] &&
        cudaMemcpyAsync(rows, c.pooled.p, sizeof(float) * row * (size_t) pp.counts[0], cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess)
        return 3;
    // the row map as a gather: output row i (document i) takes received row row_of[i]
    memcpy(c.h_part_idx, pp.row_of.data(), sizeof(int32_t) * (size_t) n_seqs);
    if (cudaMemcpyAsync(c.part_idx.p, c.h_part_idx, sizeof(int32_t) * (size_t) n_seqs, cudaMemcpyHostToDevice, s) !=
        cudaSuccess)
        return 3;
    ++c.launches;
    return nxk_gather_rows(rows, C, c.part_idx.as<int32_t>(), n_seqs, d_out, s) == NXK_OK ? 0 : 3;
}

// This rank's forward over its documents (token ids on the host or the device, in batch order of
// its own documents), pooled rows into c.pooled.
int run_part(nextera_context & c, const PartPlan & pp, const int32_t * lengths, const int32_t * tokens,
             const int32_t * types, bool on_host, int32_t normalize, cudaStream_t s) {
    if (pp.mine.empty()) return 0;
    std::vector<int32_t> len;
    len.reserve(pp.mine.size());
    for (int32_t i : pp.mine) len.push_back(lengths[i]);
    Batch b;
    float rope0 = 0.0f;
    int rc = prepare(c, tokens, types, len.data(), (int32_t) len.size(), on_host, b, rope0);
    if (rc) return rc;
    float * hid = nullptr;
    return run_encoder(c, b, rope0, tokens, types, on_host, s, nullptr, nullptr, normalize, &hid);
}

} // namespace

int32_t nextera_partition(const struct nextera_context * c, const int32_t * lengths, int32_t n_seqs, int32_t n_parts,
                          int32_t * part) {
    if (!c || !lengths || !part || n_seqs < 0 || n_parts < 1) return 1;
    for (int32_t i = 0; i < n_seqs; ++i)
        if (lengths[i] <= 0) return 1;
    partition(c->hp, lengths, n_seqs, n_parts, part);
    return 0;
}

int32_t nextera_encode_partitioned(struct nextera_context * c, const int32_t * tokens, const int32_t * token_types,
                                   const int32_t * lengths, int32_t n_seqs, float * pooled, int32_t normalize) {
    if (!c || !tokens) return 1;
    const auto t0 = std::chrono::steady_clock::now();
    const int world = c->shard_comm ? c->shard_world : 1, rank = c->shard_comm ? c->shard_rank : 0;
    const int C = c->hp.n_embd;
    cudaSetDevice(c->device);
    PartPlan pp;
    int rc = make_part_plan(*c, lengths, n_seqs, rank, world, pp);
    if (rc) return rc;
    // the whole batch is checked on every rank, so bad input fails on all ranks alike, before any
    // of them communicates
    std::vector<int64_t> start((size_t) n_seqs + 1, 0);
    for (int32_t i = 0; i < n_seqs; ++i) start[(size_t) i + 1] = start[(size_t) i] + lengths[i];
    const bool use_types = token_types && c->hp.n_types > 0;
    for (int64_t t = 0; t < start[(size_t) n_seqs]; ++t) {
        if (tokens[t] < 0 || tokens[t] >= c->hp.n_vocab) {
            fprintf(stderr, "nexterabert: token id %d out of range\n", tokens[t]);
            return 1;
        }
        if (use_types && (token_types[t] < 0 || token_types[t] >= c->hp.n_types)) {
            fprintf(stderr, "nexterabert: token type id %d out of range\n", token_types[t]);
            return 1;
        }
    }
    // this rank's ids (and segment ids) in its documents' batch order
    std::vector<int32_t> tok, typ;
    tok.reserve((size_t) pp.my_tokens);
    if (use_types) typ.reserve((size_t) pp.my_tokens);
    for (int32_t i : pp.mine) {
        tok.insert(tok.end(), tokens + start[(size_t) i], tokens + start[(size_t) i + 1]);
        if (use_types) typ.insert(typ.end(), token_types + start[(size_t) i], token_types + start[(size_t) i + 1]);
    }
    rc = run_part(*c, pp, lengths, tok.data(), use_types ? typ.data() : nullptr, true, normalize, c->stream);
    if (rc == 0 && rank == 0 && !c->part_tok.reserve(sizeof(float) * (size_t) n_seqs * C)) rc = 2;
    if (rc == 0 && cudaStreamSynchronize(c->stream) != cudaSuccess) {
        fprintf(stderr, "nexterabert: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
        rc = 3;
    }
    if (rc == 0) {
        if (int32_t e = nxk_take_error(c->stream)) {
            fprintf(stderr, "nexterabert: a kernel reported device error 0x%x\n", e);
            rc = 3;
        }
    }
    collect_profile(*c);
    // the ranks agree on the outcome (the largest code wins) before rows move
    if (world > 1) {
        const nxs::NcclApi & n = nxs::nccl();
        int32_t * st = c->part_idx.reserve(sizeof(int32_t) * (size_t) std::max(world, n_seqs)) ? c->part_idx.as<int32_t>()
                                                                                                 : nullptr;
        std::vector<int32_t> all((size_t) world, 3);
        if (!st || cudaMemcpy(st + rank, &rc, sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess ||
            !nxs::nccl_ok(n.all_gather(st + rank, st, 1, ncclInt32, c->shard_comm, c->stream), "all-gather") ||
            cudaMemcpyAsync(all.data(), st, sizeof(int32_t) * (size_t) world, cudaMemcpyDeviceToHost, c->stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(c->stream) != cudaSuccess) {
            cudaGetLastError();
            return 3;
        }
        for (int32_t x : all) rc = std::max(rc, x);
    }
    if (rc) return rc;
    float * dst = rank == 0 ? c->part_tok.as<float>() : nullptr;
    rc = gather_pooled(*c, pp, n_seqs, dst, c->stream);
    if (rc == 0 && rank == 0 && pooled &&
        cudaMemcpyAsync(pooled, dst, sizeof(float) * (size_t) n_seqs * C, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        rc = 3;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess && rc == 0) {
        fprintf(stderr, "nexterabert: device error: %s\n", cudaGetErrorString(cudaGetLastError()));
        rc = 3;
    }
    c->last_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (c->prof.enabled) {
        c->prof.total_ms += c->last_ms;
        c->prof.calls++;
    }
    return rc;
}

int32_t nextera_encode_partitioned_device(struct nextera_context * c, const int32_t * d_tokens, const int32_t * lengths,
                                          int32_t n_seqs, float * d_pooled, int32_t normalize, void * stream) {
    if (!c) return 1;
    const int world = c->shard_comm ? c->shard_world : 1, rank = c->shard_comm ? c->shard_rank : 0;
    if (rank == 0 && !d_pooled) return 1;
    cudaSetDevice(c->device);
    PartPlan pp;
    int rc = make_part_plan(*c, lengths, n_seqs, rank, world, pp);
    if (rc) return rc;
    if (!d_tokens && pp.my_tokens > 0) return 1;       // a rank given no sequences may pass NULL
    cudaStream_t s = (cudaStream_t) stream;
    rc = run_part(*c, pp, lengths, d_tokens, nullptr, false, normalize, s);
    if (rc) return rc;
    return gather_pooled(*c, pp, n_seqs, rank == 0 ? d_pooled : nullptr, s);
}

int32_t nextera_pooler_output(struct nextera_context * c, const int32_t * tokens, const int32_t * token_types,
                              const int32_t * lengths, int32_t n_seqs, float * out) {
    if (!c->hp.has_pooler) {
        fprintf(stderr, "nexterabert: this file has no pooler\n");
        return 1;
    }
    return run_head(c, tokens, token_types, lengths, n_seqs, HEAD_POOLER, out);
}

int32_t nextera_classify(struct nextera_context * c, const int32_t * tokens, const int32_t * token_types,
                         const int32_t * lengths, int32_t n_seqs, float * logits) {
    if (c->hp.cls == CLS_NONE) {
        fprintf(stderr, "nexterabert: this file has no classifier head\n");
        return 1;
    }
    return run_head(c, tokens, token_types, lengths, n_seqs, HEAD_CLASSIFIER, logits);
}

// nextera_mlm_logits (:1963-2011): one sequence; transform("mlm.") of the selected rows, then the
// decoder (the embedding table, or mlm.decoder.weight when untied) plus mlm.bias
int32_t nextera_mlm_logits(struct nextera_context * c, const int32_t * tokens, int32_t n_tokens,
                           const int32_t * positions, int32_t n_pos, float * logits) {
    const auto t0 = std::chrono::steady_clock::now();
    if (!c->hp.has_mlm) {
        fprintf(stderr, "nexterabert: this file has no MLM head\n");
        return 1;
    }
    if (n_pos <= 0 || !tokens || !positions || !logits) return 1;
    cudaSetDevice(c->device);
    Batch b;
    float rope0 = 0.0f;
    int rc = prepare(*c, tokens, nullptr, &n_tokens, 1, true, b, rope0);
    if (rc) return rc;
    for (int32_t i = 0; i < n_pos; ++i) {
        if (positions[i] < 0 || positions[i] >= n_tokens) return 1;
    }
    const hparams & hp = c->hp;
    const int C = hp.n_embd;
    float * hid = nullptr;
    rc = run_encoder(*c, b, rope0, tokens, nullptr, true, c->stream, nullptr, nullptr, 0, &hid);
    if (rc) return rc;
    if (!c->head_idx.reserve(sizeof(int32_t) * (size_t) n_pos) || !c->head_x.reserve(sizeof(float) * (size_t) n_pos * C) ||
        !c->head_out.reserve(sizeof(float) * (size_t) n_pos * hp.n_vocab))
        return 2;
    Forward fw(*c, c->stream);
    cudaMemcpyAsync(c->head_idx.p, positions, sizeof(int32_t) * (size_t) n_pos, cudaMemcpyHostToDevice, c->stream);
    fw.mark(PROF_ROWS);
    fw.rows(nxk_gather_rows(hid, C, c->head_idx.as<int32_t>(), n_pos, c->head_x.as<float>(), c->stream), "get_rows");
    float * h = fw.ok ? head_transform(*c, fw, "mlm.", c->head_x.as<float>(), n_pos, c->stream) : nullptr;
    if (!h) return fw.ok ? 2 : 3;
    const std::string dec = c->raw.count("mlm.decoder.weight") ? "mlm.decoder.weight" : "embedding.weight";
    const int n = head_linear(*c, fw, dec, h, n_pos, C, fw.p("mlm.bias"), c->head_out.as<float>(), c->stream);
    fw.mark(-1);
    if (n != hp.n_vocab) {
        if (n) fprintf(stderr, "nexterabert: the MLM decoder has %d outputs for %d tokens\n", n, hp.n_vocab);
        return 3;
    }
    return finish_head(*c, c->head_out.as<float>(), (size_t) n_pos * hp.n_vocab, logits, t0);
}
