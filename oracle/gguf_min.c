/* Minimal GGUF reader for the CPU oracle (test infrastructure, see gguf_min.h). */
#define _FILE_OFFSET_BITS 64
#include "gguf_min.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* (block size, bytes per block) of the GGUF tensor types this model family uses */
int64_t gm_blck_size(int t) {
    switch (t) {
        case 0: case 1: case 24: case 25: case 26: case 27: case 28: case 30: return 1;
        case 2: case 3: case 6: case 7: case 8: case 9: return 32;
        case 10: case 11: case 12: case 13: case 14: case 15: return 256;
        default: return 0;
    }
}

size_t gm_type_size(int t) {
    switch (t) {
        case 0: return 4;          /* F32 */
        case 1: return 2;          /* F16 */
        case 2: return 18;         /* Q4_0 */
        case 3: return 20;         /* Q4_1 */
        case 6: return 22;         /* Q5_0 */
        case 7: return 24;         /* Q5_1 */
        case 8: return 34;         /* Q8_0 */
        case 9: return 36;         /* Q8_1 */
        case 10: return 84;        /* Q2_K */
        case 11: return 110;       /* Q3_K */
        case 12: return 144;       /* Q4_K */
        case 13: return 176;       /* Q5_K */
        case 14: return 210;       /* Q6_K */
        case 15: return 292;       /* Q8_K */
        case 24: return 1;
        case 25: return 2;
        case 26: return 4;
        case 27: return 8;
        case 28: return 8;
        case 30: return 2;         /* BF16 */
        default: return 0;
    }
}

size_t gm_row_size(int type, int64_t ne0) {
    const int64_t bs = gm_blck_size(type);
    if (bs <= 0) return 0;
    return (size_t) (ne0 / bs) * gm_type_size(type);
}

int gm_is_quantized(int t) {
    return t == 2 || t == 3 || t == 6 || t == 7 || t == 8 || t == 9 || (t >= 10 && t <= 15);
}

typedef struct { FILE * f; int ok; } rd;

static void rd_bytes(rd * r, void * dst, size_t n) {
    if (r->ok && fread(dst, 1, n, r->f) != n) r->ok = 0;
}
static uint64_t rd_u64(rd * r) { uint64_t v = 0; rd_bytes(r, &v, 8); return v; }
static uint32_t rd_u32(rd * r) { uint32_t v = 0; rd_bytes(r, &v, 4); return v; }

static char * rd_str(rd * r) {
    const uint64_t n = rd_u64(r);
    if (!r->ok || n > (1ull << 31)) { r->ok = 0; return NULL; }
    char * s = (char *) malloc(n + 1);
    rd_bytes(r, s, n);
    s[n] = 0;
    return s;
}

static size_t scalar_size(int t) {
    switch (t) {
        case GM_U8: case GM_I8: case GM_BOOL: return 1;
        case GM_U16: case GM_I16: return 2;
        case GM_U32: case GM_I32: case GM_F32: return 4;
        case GM_U64: case GM_I64: case GM_F64: return 8;
        default: return 0;
    }
}

static void rd_scalar(rd * r, int t, gm_kv * kv) {
    unsigned char b[8] = {0};
    const size_t n = scalar_size(t);
    if (!n) { r->ok = 0; return; }
    rd_bytes(r, b, n);
    switch (t) {
        case GM_U8: case GM_BOOL: kv->v.u = b[0]; break;
        case GM_I8: kv->v.i = (int8_t) b[0]; break;
        case GM_U16: { uint16_t x; memcpy(&x, b, 2); kv->v.u = x; break; }
        case GM_I16: { int16_t x; memcpy(&x, b, 2); kv->v.i = x; break; }
        case GM_U32: { uint32_t x; memcpy(&x, b, 4); kv->v.u = x; break; }
        case GM_I32: { int32_t x; memcpy(&x, b, 4); kv->v.i = x; break; }
        case GM_F32: { float x; memcpy(&x, b, 4); kv->v.f = x; break; }
        case GM_U64: { uint64_t x; memcpy(&x, b, 8); kv->v.u = x; break; }
        case GM_I64: { int64_t x; memcpy(&x, b, 8); kv->v.i = x; break; }
        case GM_F64: { double x; memcpy(&x, b, 8); kv->v.f = x; break; }
    }
}

gm_file * gm_open(const char * path) {
    FILE * fp = fopen(path, "rb");
    if (!fp) { fprintf(stderr, "gguf: cannot open '%s'\n", path); return NULL; }
    rd r = { fp, 1 };
    char magic[4];
    rd_bytes(&r, magic, 4);
    if (!r.ok || memcmp(magic, "GGUF", 4) != 0) {
        fprintf(stderr, "gguf: '%s' is not a GGUF file\n", path);
        fclose(fp);
        return NULL;
    }
    gm_file * g = (gm_file *) calloc(1, sizeof(gm_file));
    g->version   = rd_u32(&r);
    g->n_tensors = (int64_t) rd_u64(&r);
    g->n_kv      = (int64_t) rd_u64(&r);
    g->alignment = 32;
    if (!r.ok || g->version < 2 || g->n_kv < 0 || g->n_kv > 100000 || g->n_tensors < 0 || g->n_tensors > 1000000) {
        fprintf(stderr, "gguf: bad header in '%s'\n", path);
        fclose(fp);
        free(g);
        return NULL;
    }
    g->kv = (gm_kv *) calloc((size_t) g->n_kv + 1, sizeof(gm_kv));
    for (int64_t i = 0; r.ok && i < g->n_kv; ++i) {
        gm_kv * kv = &g->kv[i];
        kv->key  = rd_str(&r);
        kv->type = (int) rd_u32(&r);
        if (kv->type == GM_STR) {
            kv->str = rd_str(&r);
        } else if (kv->type == GM_ARR) {
            kv->arr_type = (int) rd_u32(&r);
            kv->arr_n    = rd_u64(&r);
            if (kv->arr_n > (1ull << 28)) { r.ok = 0; break; }
            if (kv->arr_type == GM_STR) {
                kv->arr_str = (char **) calloc(kv->arr_n + 1, sizeof(char *));
                for (uint64_t j = 0; r.ok && j < kv->arr_n; ++j) kv->arr_str[j] = rd_str(&r);
            } else {
                const size_t es = scalar_size(kv->arr_type);
                if (!es) { r.ok = 0; break; }
                kv->arr_raw = malloc(es * kv->arr_n + 1);
                rd_bytes(&r, kv->arr_raw, es * kv->arr_n);
            }
        } else {
            rd_scalar(&r, kv->type, kv);
        }
        if (kv->key && strcmp(kv->key, "general.alignment") == 0 && kv->type == GM_U32) {
            g->alignment = (uint32_t) kv->v.u;
        }
    }
    g->tensors = (gm_tensor *) calloc((size_t) g->n_tensors + 1, sizeof(gm_tensor));
    for (int64_t i = 0; r.ok && i < g->n_tensors; ++i) {
        gm_tensor * t = &g->tensors[i];
        t->name   = rd_str(&r);
        t->n_dims = (int) rd_u32(&r);
        if (t->n_dims < 1 || t->n_dims > 4) { r.ok = 0; break; }
        for (int d = 0; d < 4; ++d) t->ne[d] = 1;
        for (int d = 0; d < t->n_dims; ++d) t->ne[d] = (int64_t) rd_u64(&r);
        t->type   = (int) rd_u32(&r);
        t->offset = rd_u64(&r);
        const size_t rs = gm_row_size(t->type, t->ne[0]);
        t->nbytes = rs * (size_t) (t->ne[1] * t->ne[2] * t->ne[3]);
    }
    if (!r.ok) {
        fprintf(stderr, "gguf: truncated or malformed '%s'\n", path);
        fclose(fp);
        gm_close(g);
        return NULL;
    }
    const long pos = ftell(fp);
    const uint64_t a = g->alignment ? g->alignment : 32;
    g->data_offset = ((uint64_t) pos + a - 1) / a * a;
    fclose(fp);
    return g;
}

void gm_close(gm_file * g) {
    if (!g) return;
    for (int64_t i = 0; g->kv && i < g->n_kv; ++i) {
        gm_kv * kv = &g->kv[i];
        free(kv->key);
        free(kv->str);
        if (kv->arr_str) {
            for (uint64_t j = 0; j < kv->arr_n; ++j) free(kv->arr_str[j]);
            free(kv->arr_str);
        }
        free(kv->arr_raw);
    }
    for (int64_t i = 0; g->tensors && i < g->n_tensors; ++i) free(g->tensors[i].name);
    free(g->kv);
    free(g->tensors);
    free(g);
}

int64_t gm_find_key(const gm_file * g, const char * key) {
    for (int64_t i = 0; i < g->n_kv; ++i) {
        if (g->kv[i].key && strcmp(g->kv[i].key, key) == 0) return i;
    }
    return -1;
}

int64_t gm_find_tensor(const gm_file * g, const char * name) {
    for (int64_t i = 0; i < g->n_tensors; ++i) {
        if (g->tensors[i].name && strcmp(g->tensors[i].name, name) == 0) return i;
    }
    return -1;
}
