// Implementation of the minimal ggml / gguf stand-in (see ggml.h): enough of a
// tensor / graph runtime for the reference's src/nexterabert.cpp to load a GGUF
// file and run its encoder on the CPU.  Test infrastructure only.
//
// What the reference delegates to ggml is restated here, not taken from ggml
// (which is not available): block dequantization (oracle/dequant.c, pinned
// against gguf-py), get_rows, add / mul with row broadcast, LayerNorm
// (mean / variance in double), mul_mat with ggml's activation conversion to the
// weight's vec_dot type (oracle/vecdot.c) and GELU(erf).  The graph
// runs its nodes in order; each custom op is called as fn(dst, ith, nth, ud) on
// every thread of the pool, exactly as the reference expects.
#include "ggml.h"
#include "ggml-alloc.h"
#include "ggml-backend.h"
#include "ggml-cpu.h"
#include "gguf.h"

extern "C" {
#include "../gguf_min.h"
#include "../oracle.h"
}

#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

struct ggml_context {
    bool no_alloc = false;
    std::vector<ggml_tensor *> tensors;
    std::vector<void *> allocs;
    std::vector<ggml_cgraph *> graphs;
};

struct ggml_cgraph {
    std::vector<ggml_tensor *> nodes;
    std::unordered_set<ggml_tensor *> seen;
};

struct ggml_backend_buffer {
    std::vector<void *> allocs;
    size_t size = 0;
};

struct ggml_backend_buffer_type { int dummy; };
struct ggml_backend_device { int dummy; };
struct ggml_backend_reg { int dummy; };

// --------------------------------------------------------------------------
// thread pool: run(fn) calls fn(ith, nth) on every thread and waits
// --------------------------------------------------------------------------
struct ggml_threadpool {
    int n = 1;
    std::vector<std::thread> th;
    std::mutex mu;
    std::condition_variable cv, done_cv;
    std::function<void(int, int)> job;
    uint64_t gen = 0;
    int pending = 0;
    bool stop = false;

    explicit ggml_threadpool(int n_threads) : n(n_threads < 1 ? 1 : n_threads) {
        for (int i = 1; i < n; ++i) {
            th.emplace_back([this, i]() {
                uint64_t seen = 0;
                for (;;) {
                    std::function<void(int, int)> fn;
                    {
                        std::unique_lock<std::mutex> lk(mu);
                        cv.wait(lk, [&] { return stop || gen != seen; });
                        if (stop) return;
                        seen = gen;
                        fn = job;
                    }
                    fn(i, n);
                    std::lock_guard<std::mutex> lk(mu);
                    if (--pending == 0) done_cv.notify_all();
                }
            });
        }
    }
    ~ggml_threadpool() {
        {
            std::lock_guard<std::mutex> lk(mu);
            stop = true;
        }
        cv.notify_all();
        for (auto & t : th) t.join();
    }
    void run(const std::function<void(int, int)> & fn) {
        {
            std::lock_guard<std::mutex> lk(mu);
            job = fn;
            pending = n - 1;
            ++gen;
        }
        cv.notify_all();
        fn(0, n);
        std::unique_lock<std::mutex> lk(mu);
        done_cv.wait(lk, [&] { return pending == 0; });
    }
};

struct ggml_backend {
    int n_threads = 1;
    ggml_threadpool * tp = nullptr;
};

struct ggml_gallocr {
    std::vector<void *> allocs;
    void release() {
        for (void * p : allocs) free(p);
        allocs.clear();
    }
};

struct gguf_context {
    gm_file * f = nullptr;
};

// --------------------------------------------------------------------------
// types
// --------------------------------------------------------------------------
template <int T>
static void to_float_t(const void * x, float * y, int64_t k) { or_dequant_row(T, x, y, k); }

static ggml_type_traits make_traits(const char * name, int type, ggml_to_float_t fn) {
    ggml_type_traits t;
    t.type_name = name;
    t.blck_size = gm_blck_size(type);
    t.type_size = gm_type_size(type);
    t.is_quantized = gm_is_quantized(type) != 0;
    t.to_float = fn;
    return t;
}

const struct ggml_type_traits * ggml_get_type_traits(enum ggml_type type) {
    static ggml_type_traits table[GGML_TYPE_COUNT];
    static bool init = false;
    if (!init) {
        table[GGML_TYPE_F32]  = make_traits("f32", 0, to_float_t<0>);
        table[GGML_TYPE_F16]  = make_traits("f16", 1, to_float_t<1>);
        table[GGML_TYPE_Q4_0] = make_traits("q4_0", 2, to_float_t<2>);
        table[GGML_TYPE_Q4_1] = make_traits("q4_1", 3, to_float_t<3>);
        table[GGML_TYPE_Q5_0] = make_traits("q5_0", 6, to_float_t<6>);
        table[GGML_TYPE_Q5_1] = make_traits("q5_1", 7, to_float_t<7>);
        table[GGML_TYPE_Q8_0] = make_traits("q8_0", 8, to_float_t<8>);
        table[GGML_TYPE_Q2_K] = make_traits("q2_K", 10, to_float_t<10>);
        table[GGML_TYPE_Q3_K] = make_traits("q3_K", 11, to_float_t<11>);
        table[GGML_TYPE_Q4_K] = make_traits("q4_K", 12, to_float_t<12>);
        table[GGML_TYPE_Q5_K] = make_traits("q5_K", 13, to_float_t<13>);
        table[GGML_TYPE_Q6_K] = make_traits("q6_K", 14, to_float_t<14>);
        table[GGML_TYPE_I32]  = make_traits("i32", 26, nullptr);
        table[GGML_TYPE_BF16] = make_traits("bf16", 30, to_float_t<30>);
        init = true;
    }
    return &table[(int) type];
}

size_t ggml_row_size(enum ggml_type type, int64_t ne) { return gm_row_size((int) type, ne); }
bool ggml_is_quantized(enum ggml_type type) { return gm_is_quantized((int) type) != 0; }

void ggml_fp16_to_fp32_row(const ggml_fp16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = or_fp16_to_fp32(x[i]);
}

// --------------------------------------------------------------------------
// contexts and tensors
// --------------------------------------------------------------------------
struct ggml_context * ggml_init(struct ggml_init_params params) {
    ggml_context * c = new ggml_context();
    c->no_alloc = params.no_alloc;
    return c;
}

void ggml_free(struct ggml_context * ctx) {
    if (!ctx) return;
    for (ggml_tensor * t : ctx->tensors) free(t);
    for (void * p : ctx->allocs) free(p);
    for (ggml_cgraph * g : ctx->graphs) delete g;
    delete ctx;
}

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor) + 16; }
size_t ggml_graph_overhead_custom(size_t size, bool) { return 1024 + size * 4 * sizeof(void *); }

size_t ggml_nbytes(const struct ggml_tensor * t) {
    return ggml_row_size(t->type, t->ne[0]) * (size_t) (t->ne[1] * t->ne[2] * t->ne[3]);
}

int ggml_n_dims(const struct ggml_tensor * t) {
    for (int i = 3; i >= 1; --i) {
        if (t->ne[i] > 1) return i + 1;
    }
    return 1;
}

static ggml_tensor * new_tensor(ggml_context * ctx, ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3) {
    ggml_tensor * t = (ggml_tensor *) calloc(1, sizeof(ggml_tensor));
    t->type = type;
    t->ne[0] = ne0; t->ne[1] = ne1; t->ne[2] = ne2; t->ne[3] = ne3;
    const size_t ts = gm_type_size((int) type);
    t->nb[0] = ts;
    t->nb[1] = ggml_row_size(type, ne0);
    t->nb[2] = t->nb[1] * (size_t) ne1;
    t->nb[3] = t->nb[2] * (size_t) ne2;
    t->op = SHIM_OP_NONE;
    ctx->tensors.push_back(t);
    if (!ctx->no_alloc) {
        t->data = calloc(1, ggml_nbytes(t) + 64);
        ctx->allocs.push_back(t->data);
    }
    return t;
}

struct ggml_tensor * ggml_new_tensor_1d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0) {
    return new_tensor(ctx, type, ne0, 1, 1, 1);
}
struct ggml_tensor * ggml_new_tensor_2d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0, int64_t ne1) {
    return new_tensor(ctx, type, ne0, ne1, 1, 1);
}
struct ggml_tensor * ggml_dup_tensor(struct ggml_context * ctx, const struct ggml_tensor * src) {
    return new_tensor(ctx, src->type, src->ne[0], src->ne[1], src->ne[2], src->ne[3]);
}

struct ggml_tensor * ggml_get_tensor(struct ggml_context * ctx, const char * name) {
    for (ggml_tensor * t : ctx->tensors) {
        if (strcmp(t->name, name) == 0) return t;
    }
    return nullptr;
}

struct ggml_tensor * ggml_set_name(struct ggml_tensor * t, const char * name) {
    snprintf(t->name, sizeof(t->name), "%s", name);
    return t;
}

void ggml_set_input(struct ggml_tensor *) {}
void ggml_set_output(struct ggml_tensor *) {}

static std::chrono::steady_clock::time_point g_t0 = std::chrono::steady_clock::now();
void ggml_time_init(void) {}
int64_t ggml_time_us(void) {
    return std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - g_t0).count();
}

void ggml_log_set(ggml_log_callback, void *) {}
FILE * ggml_fopen(const char * fname, const char * mode) { return fopen(fname, mode); }

// --------------------------------------------------------------------------
// ops (graph construction)
// --------------------------------------------------------------------------
static ggml_tensor * op_node(ggml_context * ctx, shim_op op, ggml_type type, const int64_t * ne,
                             ggml_tensor * a, ggml_tensor * b) {
    ggml_tensor * t = new_tensor(ctx, type, ne[0], ne[1], ne[2], ne[3]);
    t->op = op;
    t->src[0] = a;
    t->src[1] = b;
    return t;
}

struct ggml_tensor * ggml_get_rows(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b) {
    const int64_t ne[4] = { a->ne[0], b->ne[0], 1, 1 };
    return op_node(ctx, SHIM_OP_GET_ROWS, GGML_TYPE_F32, ne, a, b);
}
struct ggml_tensor * ggml_add(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b) {
    return op_node(ctx, SHIM_OP_ADD, GGML_TYPE_F32, a->ne, a, b);
}
struct ggml_tensor * ggml_mul(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b) {
    return op_node(ctx, SHIM_OP_MUL, GGML_TYPE_F32, a->ne, a, b);
}
struct ggml_tensor * ggml_norm(struct ggml_context * ctx, struct ggml_tensor * a, float eps) {
    ggml_tensor * t = op_node(ctx, SHIM_OP_NORM, GGML_TYPE_F32, a->ne, a, nullptr);
    t->f_param = eps;
    return t;
}
struct ggml_tensor * ggml_mul_mat(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b) {
    const int64_t ne[4] = { a->ne[1], b->ne[1], 1, 1 };
    return op_node(ctx, SHIM_OP_MUL_MAT, GGML_TYPE_F32, ne, a, b);
}
struct ggml_tensor * ggml_gelu_erf(struct ggml_context * ctx, struct ggml_tensor * a) {
    return op_node(ctx, SHIM_OP_GELU_ERF, GGML_TYPE_F32, a->ne, a, nullptr);
}
struct ggml_tensor * ggml_custom_4d(struct ggml_context * ctx, enum ggml_type type,
                                    int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                                    struct ggml_tensor ** args, int n_args,
                                    ggml_custom_op_t fun, int n_tasks, void * userdata) {
    ggml_tensor * t = new_tensor(ctx, type, ne0, ne1, ne2, ne3);
    t->op = SHIM_OP_CUSTOM;
    for (int i = 0; i < n_args && i < GGML_MAX_SRC; ++i) t->src[i] = args[i];
    t->custom_fn = fun;
    t->custom_ud = userdata;
    t->n_tasks = n_tasks;
    return t;
}

// --------------------------------------------------------------------------
// graphs and allocation
// --------------------------------------------------------------------------
struct ggml_cgraph * ggml_new_graph_custom(struct ggml_context * ctx, size_t, bool) {
    ggml_cgraph * g = new ggml_cgraph();
    ctx->graphs.push_back(g);
    return g;
}

static void visit(ggml_cgraph * g, ggml_tensor * t) {
    if (!t || g->seen.count(t)) return;
    g->seen.insert(t);
    for (int i = 0; i < GGML_MAX_SRC; ++i) visit(g, t->src[i]);
    g->nodes.push_back(t);   // leaves too: the allocator needs them, compute skips them
}

void ggml_build_forward_expand(struct ggml_cgraph * gf, struct ggml_tensor * t) { visit(gf, t); }

ggml_gallocr_t ggml_gallocr_new(ggml_backend_buffer_type_t) { return new ggml_gallocr(); }
void ggml_gallocr_free(ggml_gallocr_t a) {
    if (!a) return;
    a->release();
    delete a;
}

bool ggml_gallocr_alloc_graph(ggml_gallocr_t a, struct ggml_cgraph * g) {
    a->release();
    for (ggml_tensor * t : g->nodes) {
        if (t->data) continue;
        t->data = calloc(1, ggml_nbytes(t) + 64);
        if (!t->data) return false;
        a->allocs.push_back(t->data);
    }
    return true;
}

// --------------------------------------------------------------------------
// compute
// --------------------------------------------------------------------------
static void parallel_rows(ggml_threadpool * tp, int64_t n, const std::function<void(int64_t)> & fn) {
    if (!tp || tp->n == 1) {
        for (int64_t i = 0; i < n; ++i) fn(i);
        return;
    }
    tp->run([&](int ith, int nth) {
        for (int64_t i = ith; i < n; i += nth) fn(i);
    });
}

static void compute_node(ggml_backend * be, ggml_tensor * t) {
    ggml_threadpool * tp = be->tp;
    switch (t->op) {
        case SHIM_OP_NONE:
            return;
        case SHIM_OP_CUSTOM:
            if (tp && tp->n > 1) {
                tp->run([&](int ith, int nth) { t->custom_fn(t, ith, nth, t->custom_ud); });
            } else {
                t->custom_fn(t, 0, 1, t->custom_ud);
            }
            return;
        case SHIM_OP_GET_ROWS: {
            const ggml_tensor * a = t->src[0], * b = t->src[1];
            const size_t rs = ggml_row_size(a->type, a->ne[0]);
            const int32_t * idx = (const int32_t *) b->data;
            parallel_rows(tp, t->ne[1], [&](int64_t i) {
                or_dequant_row((int) a->type, (const uint8_t *) a->data + rs * (size_t) idx[i],
                               (float *) t->data + i * t->ne[0], a->ne[0]);
            });
            return;
        }
        case SHIM_OP_ADD:
        case SHIM_OP_MUL: {
            const ggml_tensor * a = t->src[0], * b = t->src[1];
            const int64_t C = t->ne[0], rows = t->ne[1] * t->ne[2] * t->ne[3];
            const int64_t brows = b->ne[1] * b->ne[2] * b->ne[3];
            const bool add = t->op == SHIM_OP_ADD;
            parallel_rows(tp, rows, [&](int64_t r) {
                const float * x = (const float *) a->data + r * C;
                const float * y = (const float *) b->data + (brows == 1 ? 0 : r) * C;
                float * o = (float *) t->data + r * C;
                for (int64_t i = 0; i < C; ++i) o[i] = add ? x[i] + y[i] : x[i] * y[i];
            });
            return;
        }
        case SHIM_OP_NORM: {
            const ggml_tensor * a = t->src[0];
            const int64_t C = t->ne[0], rows = t->ne[1];
            parallel_rows(tp, rows, [&](int64_t r) {
                or_layer_norm((const float *) a->data + r * C, nullptr, nullptr, t->f_param, 1, (int) C,
                              (float *) t->data + r * C);
            });
            return;
        }
        case SHIM_OP_MUL_MAT: {
            // ggml's CPU mul_mat: the activation row goes to the weight type's vec_dot
            // type first (Q8_K / Q8_0 / Q8_1 / F16 ...), then one dot per weight row
            // (oracle/vecdot.c)
            const ggml_tensor * a = t->src[0], * b = t->src[1];
            const int64_t K = a->ne[0], N = a->ne[1], M = b->ne[1];
            const size_t rs = ggml_row_size(a->type, K);
            const size_t ab = or_act_bytes((int) a->type, K);
            GGML_ASSERT(ab > 0);
            std::vector<uint8_t> act(ab * (size_t) M);
            parallel_rows(tp, M, [&](int64_t m) {
                GGML_ASSERT(or_quantize_act((int) a->type, (const float *) b->data + m * K, K, act.data() + ab * m) == 0);
            });
            parallel_rows(tp, N, [&](int64_t n) {
                const uint8_t * wr = (const uint8_t *) a->data + rs * (size_t) n;
                for (int64_t m = 0; m < M; ++m) {
                    ((float *) t->data)[m * N + n] = or_vec_dot((int) a->type, wr, act.data() + ab * m, K);
                }
            });
            return;
        }
        case SHIM_OP_GELU_ERF: {
            const ggml_tensor * a = t->src[0];
            or_gelu_erf((const float *) a->data, t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3], (float *) t->data);
            return;
        }
    }
}

enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph * graph) {
    for (ggml_tensor * t : graph->nodes) compute_node(backend, t);
    return GGML_STATUS_SUCCESS;
}

// --------------------------------------------------------------------------
// backend plumbing
// --------------------------------------------------------------------------
ggml_backend_t ggml_backend_cpu_init(void) {
    ggml_backend * b = new ggml_backend();
    b->n_threads = (int) std::max(1u, std::thread::hardware_concurrency());
    return b;
}
void ggml_backend_free(ggml_backend_t backend) { delete backend; }
void ggml_backend_cpu_set_n_threads(ggml_backend_t b, int n) { b->n_threads = n; }
void ggml_backend_cpu_set_threadpool(ggml_backend_t b, struct ggml_threadpool * tp) { b->tp = tp; }

void ggml_backend_tensor_set(struct ggml_tensor * t, const void * data, size_t offset, size_t size) {
    memcpy((uint8_t *) t->data + offset, data, size);
}

static ggml_backend_device g_dev;
static ggml_backend_reg g_reg;
static ggml_backend_buffer_type g_buft;

ggml_backend_dev_t ggml_backend_dev_by_type(enum ggml_backend_dev_type) { return &g_dev; }
ggml_backend_reg_t ggml_backend_dev_backend_reg(ggml_backend_dev_t) { return &g_reg; }
void * ggml_backend_reg_get_proc_address(ggml_backend_reg_t, const char *) { return nullptr; }
bool ggml_backend_dev_supports_op(ggml_backend_dev_t, const struct ggml_tensor *) { return false; }
ggml_backend_buffer_type_t ggml_backend_cpu_buffer_type(void) { return &g_buft; }

ggml_backend_buffer_t ggml_backend_buft_alloc_buffer(ggml_backend_buffer_type_t, size_t size) {
    ggml_backend_buffer * b = new ggml_backend_buffer();
    b->size = size;
    if (size) b->allocs.push_back(calloc(1, size));
    return b;
}

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors_from_buft(struct ggml_context * ctx, ggml_backend_buffer_type_t) {
    ggml_backend_buffer * b = new ggml_backend_buffer();
    for (ggml_tensor * t : ctx->tensors) {
        if (t->data) continue;
        const size_t n = ggml_nbytes(t);
        t->data = calloc(1, n + 64);
        b->allocs.push_back(t->data);
        b->size += n;
    }
    return b;
}

size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t b) { return b ? b->size : 0; }
void ggml_backend_buffer_free(ggml_backend_buffer_t b) {
    if (!b) return;
    for (void * p : b->allocs) free(p);
    delete b;
}

struct ggml_threadpool_params ggml_threadpool_params_default(int n_threads) {
    ggml_threadpool_params p;
    p.n_threads = n_threads;
    return p;
}
struct ggml_threadpool * ggml_threadpool_new(struct ggml_threadpool_params * params) {
    return new ggml_threadpool(params->n_threads);
}
void ggml_threadpool_free(struct ggml_threadpool * tp) { delete tp; }

#if defined(__AVX2__)
int ggml_cpu_has_avx2(void) { return 1; }
#else
int ggml_cpu_has_avx2(void) { return 0; }
#endif
#if defined(__AVXVNNI__)
int ggml_cpu_has_avx_vnni(void) { return 1; }
#else
int ggml_cpu_has_avx_vnni(void) { return 0; }
#endif
#if defined(__FMA__)
int ggml_cpu_has_fma(void) { return 1; }
#else
int ggml_cpu_has_fma(void) { return 0; }
#endif
#if defined(__F16C__)
int ggml_cpu_has_f16c(void) { return 1; }
#else
int ggml_cpu_has_f16c(void) { return 0; }
#endif
#if defined(__AVX512F__)
int ggml_cpu_has_avx512(void) { return 1; }
#else
int ggml_cpu_has_avx512(void) { return 0; }
#endif
int ggml_cpu_has_neon(void) { return 0; }
int ggml_cpu_has_llamafile(void) { return 0; }

// --------------------------------------------------------------------------
// gguf
// --------------------------------------------------------------------------
struct gguf_context * gguf_init_from_file(const char * fname, struct gguf_init_params params) {
    gm_file * f = gm_open(fname);
    if (!f) return nullptr;
    gguf_context * g = new gguf_context();
    g->f = f;
    if (params.ctx) {
        ggml_init_params ip = { 0, nullptr, true };
        ggml_context * meta = ggml_init(ip);
        for (int64_t i = 0; i < f->n_tensors; ++i) {
            const gm_tensor * gt = &f->tensors[i];
            ggml_tensor * t = new_tensor(meta, (ggml_type) gt->type, gt->ne[0], gt->ne[1], gt->ne[2], gt->ne[3]);
            ggml_set_name(t, gt->name);
        }
        *params.ctx = meta;
    }
    return g;
}

void gguf_free(struct gguf_context * g) {
    if (!g) return;
    gm_close(g->f);
    delete g;
}

int64_t gguf_find_key(const struct gguf_context * g, const char * key) { return gm_find_key(g->f, key); }
uint32_t gguf_get_val_u32(const struct gguf_context * g, int64_t id) { return (uint32_t) g->f->kv[id].v.u; }
float gguf_get_val_f32(const struct gguf_context * g, int64_t id) { return (float) g->f->kv[id].v.f; }
bool gguf_get_val_bool(const struct gguf_context * g, int64_t id) { return g->f->kv[id].v.u != 0; }
const char * gguf_get_val_str(const struct gguf_context * g, int64_t id) {
    return g->f->kv[id].str ? g->f->kv[id].str : "";
}
size_t gguf_get_arr_n(const struct gguf_context * g, int64_t id) { return (size_t) g->f->kv[id].arr_n; }
const char * gguf_get_arr_str(const struct gguf_context * g, int64_t id, size_t i) { return g->f->kv[id].arr_str[i]; }
int64_t gguf_get_n_tensors(const struct gguf_context * g) { return g->f->n_tensors; }
const char * gguf_get_tensor_name(const struct gguf_context * g, int64_t i) { return g->f->tensors[i].name; }
size_t gguf_get_tensor_offset(const struct gguf_context * g, int64_t i) { return (size_t) g->f->tensors[i].offset; }
size_t gguf_get_data_offset(const struct gguf_context * g) { return (size_t) g->f->data_offset; }
