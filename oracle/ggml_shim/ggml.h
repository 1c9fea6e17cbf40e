// Minimal stand-in for the ggml / gguf C API, written for this repository's
// test oracle only.  It declares exactly the types and functions that the
// reference's src/nexterabert.cpp uses, so that file compiles unmodified with
// g++ when ggml itself (fetched over the network by the reference's CMake,
// CMakeLists.txt:51-57) is not available.  The implementation is
// ggml_shim.cpp; it is test infrastructure and never part of the product.
//
// Enumerations that are part of the GGUF file format (ggml_type ids) keep the
// values that format defines; everything else is this shim's own.
#pragma once

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_ASSERT(x) do { if (!(x)) { fprintf(stderr, "GGML_ASSERT(%s) failed at %s:%d\n", #x, __FILE__, __LINE__); abort(); } } while (0)
#define GGML_N_TASKS_MAX (-1)
#define GGML_MAX_SRC 10

// tensor element types: the GGUF file format's type ids
enum ggml_type {
    GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6, GGML_TYPE_Q5_1 = 7, GGML_TYPE_Q8_0 = 8, GGML_TYPE_Q8_1 = 9,
    GGML_TYPE_Q2_K = 10, GGML_TYPE_Q3_K = 11, GGML_TYPE_Q4_K = 12, GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14, GGML_TYPE_Q8_K = 15, GGML_TYPE_I8 = 24, GGML_TYPE_I16 = 25,
    GGML_TYPE_I32 = 26, GGML_TYPE_I64 = 27, GGML_TYPE_F64 = 28, GGML_TYPE_BF16 = 30,
    GGML_TYPE_COUNT = 40,
};

enum ggml_log_level {
    GGML_LOG_LEVEL_NONE = 0, GGML_LOG_LEVEL_DEBUG = 1, GGML_LOG_LEVEL_INFO = 2,
    GGML_LOG_LEVEL_WARN = 3, GGML_LOG_LEVEL_ERROR = 4, GGML_LOG_LEVEL_CONT = 5,
};

enum ggml_status { GGML_STATUS_FAILED = -1, GGML_STATUS_SUCCESS = 0 };

enum ggml_backend_dev_type { GGML_BACKEND_DEVICE_TYPE_CPU = 0 };

typedef uint16_t ggml_fp16_t;

struct ggml_tensor;
struct ggml_context;
struct ggml_cgraph;
struct gguf_context;
struct ggml_threadpool;
struct ggml_backend;
struct ggml_backend_device;
struct ggml_backend_reg;
struct ggml_backend_buffer;
struct ggml_backend_buffer_type;
struct ggml_gallocr;

typedef struct ggml_backend * ggml_backend_t;
typedef struct ggml_backend_device * ggml_backend_dev_t;
typedef struct ggml_backend_reg * ggml_backend_reg_t;
typedef struct ggml_backend_buffer * ggml_backend_buffer_t;
typedef struct ggml_backend_buffer_type * ggml_backend_buffer_type_t;
typedef struct ggml_gallocr * ggml_gallocr_t;

typedef void (*ggml_custom_op_t)(struct ggml_tensor * dst, int ith, int nth, void * userdata);
typedef void (*ggml_log_callback)(enum ggml_log_level level, const char * text, void * user_data);
typedef ggml_backend_buffer_type_t * (*ggml_backend_dev_get_extra_bufts_t)(ggml_backend_dev_t device);
typedef void (*ggml_to_float_t)(const void * x, float * y, int64_t k);

enum shim_op { SHIM_OP_NONE, SHIM_OP_GET_ROWS, SHIM_OP_ADD, SHIM_OP_MUL, SHIM_OP_NORM,
               SHIM_OP_MUL_MAT, SHIM_OP_GELU_ERF, SHIM_OP_CUSTOM };

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t  nb[4];
    void *  data;
    struct ggml_tensor * src[GGML_MAX_SRC];
    char    name[128];
    // shim-private
    enum shim_op op;
    ggml_custom_op_t custom_fn;
    void *  custom_ud;
    float   f_param;
    int     n_tasks;
    int     visited;
    struct ggml_backend_buffer * buffer;
};

struct ggml_init_params {
    size_t mem_size;
    void * mem_buffer;
    bool   no_alloc;
};

struct gguf_init_params {
    bool no_alloc;
    struct ggml_context ** ctx;
};

struct ggml_threadpool_params {
    int n_threads;
};

struct ggml_type_traits {
    const char *    type_name;
    int64_t         blck_size;
    size_t          type_size;
    bool            is_quantized;
    ggml_to_float_t to_float;
};

// core
struct ggml_context * ggml_init(struct ggml_init_params params);
void    ggml_free(struct ggml_context * ctx);
size_t  ggml_tensor_overhead(void);
size_t  ggml_graph_overhead_custom(size_t size, bool grads);
struct ggml_tensor * ggml_new_tensor_1d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor * ggml_new_tensor_2d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor * ggml_dup_tensor(struct ggml_context * ctx, const struct ggml_tensor * src);
struct ggml_tensor * ggml_get_tensor(struct ggml_context * ctx, const char * name);
struct ggml_tensor * ggml_set_name(struct ggml_tensor * t, const char * name);
void    ggml_set_input(struct ggml_tensor * t);
void    ggml_set_output(struct ggml_tensor * t);
size_t  ggml_nbytes(const struct ggml_tensor * t);
int     ggml_n_dims(const struct ggml_tensor * t);
size_t  ggml_row_size(enum ggml_type type, int64_t ne);
bool    ggml_is_quantized(enum ggml_type type);
const struct ggml_type_traits * ggml_get_type_traits(enum ggml_type type);
void    ggml_fp16_to_fp32_row(const ggml_fp16_t * x, float * y, int64_t n);
void    ggml_time_init(void);
int64_t ggml_time_us(void);
void    ggml_log_set(ggml_log_callback cb, void * user_data);
FILE *  ggml_fopen(const char * fname, const char * mode);

// ops
struct ggml_tensor * ggml_get_rows(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_add(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_mul(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_norm(struct ggml_context * ctx, struct ggml_tensor * a, float eps);
struct ggml_tensor * ggml_mul_mat(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_gelu_erf(struct ggml_context * ctx, struct ggml_tensor * a);
struct ggml_tensor * ggml_custom_4d(struct ggml_context * ctx, enum ggml_type type,
                                    int64_t ne0, int64_t ne1, int64_t ne2, int64_t ne3,
                                    struct ggml_tensor ** args, int n_args,
                                    ggml_custom_op_t fun, int n_tasks, void * userdata);

// graphs
struct ggml_cgraph * ggml_new_graph_custom(struct ggml_context * ctx, size_t size, bool grads);
void    ggml_build_forward_expand(struct ggml_cgraph * gf, struct ggml_tensor * t);

// allocation
ggml_gallocr_t ggml_gallocr_new(ggml_backend_buffer_type_t buft);
void    ggml_gallocr_free(ggml_gallocr_t galloc);
bool    ggml_gallocr_alloc_graph(ggml_gallocr_t galloc, struct ggml_cgraph * graph);

// backend
ggml_backend_t ggml_backend_cpu_init(void);
void    ggml_backend_free(ggml_backend_t backend);
void    ggml_backend_cpu_set_n_threads(ggml_backend_t backend, int n_threads);
void    ggml_backend_cpu_set_threadpool(ggml_backend_t backend, struct ggml_threadpool * tp);
enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph * graph);
void    ggml_backend_tensor_set(struct ggml_tensor * t, const void * data, size_t offset, size_t size);
ggml_backend_dev_t ggml_backend_dev_by_type(enum ggml_backend_dev_type type);
ggml_backend_reg_t ggml_backend_dev_backend_reg(ggml_backend_dev_t dev);
void *  ggml_backend_reg_get_proc_address(ggml_backend_reg_t reg, const char * name);
bool    ggml_backend_dev_supports_op(ggml_backend_dev_t dev, const struct ggml_tensor * op);
ggml_backend_buffer_type_t ggml_backend_cpu_buffer_type(void);
ggml_backend_buffer_t ggml_backend_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size);
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors_from_buft(struct ggml_context * ctx, ggml_backend_buffer_type_t buft);
size_t  ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer);
void    ggml_backend_buffer_free(ggml_backend_buffer_t buffer);

// threads
struct ggml_threadpool_params ggml_threadpool_params_default(int n_threads);
struct ggml_threadpool * ggml_threadpool_new(struct ggml_threadpool_params * params);
void    ggml_threadpool_free(struct ggml_threadpool * tp);

// CPU feature report
int ggml_cpu_has_avx2(void);
int ggml_cpu_has_avx_vnni(void);
int ggml_cpu_has_fma(void);
int ggml_cpu_has_f16c(void);
int ggml_cpu_has_avx512(void);
int ggml_cpu_has_neon(void);
int ggml_cpu_has_llamafile(void);

// gguf
struct gguf_context * gguf_init_from_file(const char * fname, struct gguf_init_params params);
void    gguf_free(struct gguf_context * ctx);
int64_t gguf_find_key(const struct gguf_context * ctx, const char * key);
uint32_t gguf_get_val_u32(const struct gguf_context * ctx, int64_t key_id);
float   gguf_get_val_f32(const struct gguf_context * ctx, int64_t key_id);
bool    gguf_get_val_bool(const struct gguf_context * ctx, int64_t key_id);
const char * gguf_get_val_str(const struct gguf_context * ctx, int64_t key_id);
size_t  gguf_get_arr_n(const struct gguf_context * ctx, int64_t key_id);
const char * gguf_get_arr_str(const struct gguf_context * ctx, int64_t key_id, size_t i);
int64_t gguf_get_n_tensors(const struct gguf_context * ctx);
const char * gguf_get_tensor_name(const struct gguf_context * ctx, int64_t tensor_id);
size_t  gguf_get_tensor_offset(const struct gguf_context * ctx, int64_t tensor_id);
size_t  gguf_get_data_offset(const struct gguf_context * ctx);

#ifdef __cplusplus
}
#endif
