/* CPU oracle for the NexteraBERT encoder hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * A scalar C restatement of the reference runtime's arithmetic
 * (Rikka-Botan/NexteraBERT.cpp, src/nexterabert.cpp), written to reproduce its
 * AVX2 / AVX-VNNI fp32 operation order exactly: lane-for-lane accumulators,
 * the same horizontal-sum trees, the same fused multiply-adds, the same
 * Cephes-style exp.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline may load it, and only as the checker; the product never links it.
 *
 * Pinning: every op here is compared bit-for-bit against the reference's own
 * functions compiled from its source (oracle/_ref, see oracle/Makefile) and
 * against committed fixtures that build wrote (tests/golden/).  Arithmetic that
 * the reference delegates to ggml (block dequantization, get_rows, ggml_norm)
 * is restated from gguf-py / the published algorithm and is pinned only
 * against gguf-py (dequantization); ggml_norm is unpinned.
 */
#ifndef NEXTERA_ORACLE_H
#define NEXTERA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml / GGUF tensor type ids */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7, OR_Q8_0 = 8,
       OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14, OR_BF16 = 30 };

#define OR_I8_BLOCK 256
#define OR_ACT_MAX 127

float or_fp16_to_fp32(uint16_t h);
/* one row of n values of `type` -> fp32; returns 0, or -1 for an unknown type */
int   or_dequant_row(int type, const void * src, float * y, int64_t n);

/* ---- arithmetic building blocks (src/nexterabert.cpp:78-198) ---- */
float or_exp8(float x);                  /* one lane of exp256 (:81-99) */
float or_tanh8(float x);                 /* one lane of tanh256 (:103-117) */
float or_sigmoid8(float x);              /* one lane of sigmoid256 (:119-122) */
float or_dot_f32(const float * a, const float * b, int n);   /* dot_f32 (:133-151) */

/* ---- int8 linear (nexterabert.cpp:854-1049) ----
 * Activations are stored as s8 = u8 - 128 (the reference's u8 code minus its
 * +128 offset) with one fp32 scale per (token, 256-block): sx[t * n_blk + B].
 * Weights: s8 w[n_out][n_in], scale[n_blk][n_out], off[n_blk][n_out]. */
int  or_build_i8_weight(int type, const void * data, int n_in, int n_out,
                        int8_t * w, float * scale, int32_t * off);
void or_quantize_rows(const float * x, int T, int n_in, int8_t * q, float * sx);
void or_linear_i8(const int8_t * xq, const float * sx, int T, const int8_t * w, const float * sw,
                  int n_in, int n_out, const float * res, float * out,
                  int32_t * block_sums /* optional [T][n_out][n_blk] */);

/* ---- row ops (nexterabert.cpp:463-690); rows of C floats, row t at x + t*C ---- */
void or_rms_norm(const float * x, const float * gain, float eps, int T, int C, float * out);
void or_relu_sqr(const float * x, int T, int C, float * out);
void or_gate(const float * g, const float * y, int T, int C, float * out);
/* doc_start/doc_len per document; row_doc per row */
void or_dwconv(const float * x, const float * r, const float * taps /* [k][C] */, int k,
               const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
               int T, int C, float * out);
void or_lily_state(const float * a, const float * x, const float * b, const float * taps, int k,
                   const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                   int T, int C, float * out);
/* DyT + RoPE; head_major: write [H][T][D] instead of [T][H][D] */
void or_qk_prep(const float * x, const float * alpha, const float * beta,
                const float * cos_t, const float * sin_t /* [n_pos][D/2] */,
                const int32_t * row_doc, const int32_t * doc_start,
                int T, int H, int D, int head_major, float * out);
void or_head_major(const float * x, int T, int H, int D, float * out);
void or_block_mean(const float * h, const float * g /* may be NULL */, int C, int block,
                   const int32_t * doc_start, const int32_t * doc_len,
                   const int32_t * bdoc_start, const int32_t * brow_doc, int n_brows, float * out);
void or_upsample_add(const float * y, const float * r, int C, int block, int T,
                     const int32_t * row_doc, const int32_t * doc_start, const int32_t * bdoc_start,
                     float * out);
/* grouped-query attention inside each document; q [T][H*D], k/v head-major [G][T][D];
 * half < 0: full; scale[doc] per document (nexterabert.cpp:759-852) */
void or_attention(const float * q, const float * k, const float * v, int T, int H, int G, int D,
                  int half, const float * scale, const int32_t * row_doc, const int32_t * doc_start,
                  const int32_t * doc_len, float * out);
/* ggml_norm (LayerNorm without affine), restated; then * w + b when w/b given */
void or_layer_norm(const float * x, const float * w, const float * b, float eps, int T, int C, float * out);
/* host pooling of run_forward (:1903-1918) */
void or_pool(const float * hidden, const int32_t * lengths, int n_seqs, int C, int normalize, float * pooled);
/* rope table (build_rope :1322-1338) */
void or_rope_table(int n_pos, float base, int head_dim, float * cos_t, float * sin_t);

/* ---- ggml_mul_mat on a weight off the int8 path (vecdot.c; ggml restated, unpinned) ---- */
uint16_t or_fp32_to_fp16(float f);
int    or_vec_dot_family(int type);
size_t or_act_bytes(int type, int64_t K);
int    or_quantize_act(int type, const float * x, int64_t K, void * out);
float  or_vec_dot(int type, const void * wrow, const void * xact, int64_t K);
int    or_mul_mat(int type, const void * w, int64_t N, int64_t K, const float * x, int64_t M, float * out);
/* GELU(erf) as ggml_gelu_erf: 0.5 x (1 + erf(x / sqrt 2)) */
void   or_gelu_erf(const float * x, int64_t n, float * out);

/* ---- whole encoder (builder::encoder :1271-1294 + run_forward) ---- */
typedef struct or_model or_model;
or_model * or_load(const char * path);
void       or_free(or_model * m);
int        or_n_embd(const or_model * m);
/* returns 0, or the reference's error codes (1 bad input) */
int        or_encode(or_model * m, const int32_t * tokens, const int32_t * types, const int32_t * lengths,
                     int n_seqs, float * hidden, float * pooled, int normalize, int n_layers);
/* expanded int8 weight of a named tensor (NULL if not on the int8 path) */
int        or_get_i8(const or_model * m, const char * name, int * n_in, int * n_out,
                     const int8_t ** w, const float ** scale, const int32_t ** off);
void       or_set_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
