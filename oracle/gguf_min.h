/* Minimal GGUF (v2/v3) reader for the CPU oracle and the ggml shim.
 *
 * Test infrastructure only: the product library has its own reader.  The file
 * format (magic, key/value types, tensor info records, data alignment) is the
 * published GGUF layout that gguf-py writes (gguf 0.19.0, gguf_writer.py).
 */
#ifndef NEXTERA_ORACLE_GGUF_MIN_H
#define NEXTERA_ORACLE_GGUF_MIN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum gm_vtype { GM_U8 = 0, GM_I8, GM_U16, GM_I16, GM_U32, GM_I32, GM_F32, GM_BOOL, GM_STR,
                GM_ARR, GM_U64, GM_I64, GM_F64 };

typedef struct gm_kv {
    char *   key;
    int      type;        /* enum gm_vtype */
    int      arr_type;    /* element type when type == GM_ARR */
    uint64_t arr_n;
    union { uint64_t u; int64_t i; double f; } v;   /* scalar value (bool/ints/floats) */
    char *   str;         /* GM_STR value */
    char **  arr_str;     /* GM_ARR of GM_STR */
    void *   arr_raw;     /* GM_ARR of scalars, packed as stored */
} gm_kv;

typedef struct gm_tensor {
    char *   name;
    int      n_dims;
    int64_t  ne[4];
    int      type;        /* ggml type id */
    uint64_t offset;      /* from the start of the data section */
    size_t   nbytes;
} gm_tensor;

typedef struct gm_file {
    uint32_t   version;
    int64_t    n_kv, n_tensors;
    gm_kv *    kv;
    gm_tensor * tensors;
    uint64_t   data_offset;   /* absolute file offset of the data section */
    uint32_t   alignment;
} gm_file;

/* Returns NULL (and prints why) on a malformed or unreadable file. */
gm_file * gm_open(const char * path);
void      gm_close(gm_file * f);
int64_t   gm_find_key(const gm_file * f, const char * key);
int64_t   gm_find_tensor(const gm_file * f, const char * name);

/* block size and bytes per block of a ggml type id; 0 if unknown */
int64_t   gm_blck_size(int type);
size_t    gm_type_size(int type);
size_t    gm_row_size(int type, int64_t ne0);
int       gm_is_quantized(int type);

#ifdef __cplusplus
}
#endif

#endif
