/* nextera_kernels.h -- the thin C-ABI kernel layer of libnexterabert.so (sm_100a).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void *; NULL = the legacy default stream) and only
 * enqueues work: nothing here synchronises or allocates unless it says so.
 * The host library (nexterabert.h) is built on these; tests and benchmarks call
 * them directly to check one kernel at a time.  Each function names the
 * reference routine (src/nexterabert.cpp of Rikka-Botan/NexteraBERT.cpp) whose
 * results it reproduces.
 *
 * Data layouts (row t of a [T][C] tensor starts at t * C):
 *   fp32 activations  [T][C]
 *   int8 activations  q [T][C] as s8 codes (the reference's u8 code minus 128)
 *                     sx [T][n_blk] fp32, n_blk = ceil(C / 256)
 *   int8 weights      w [N][K] s8, sw [n_blk][N] fp32 (off [n_blk][N] int32 optional)
 *   attention         q [T][H*D] row-major, k / v head-major [G][T][D]
 *   documents         doc_start[n_docs], doc_len[n_docs], row_doc[T]
 *
 * Return value: 0 on success, NXK_EINVAL for arguments the kernels do not
 * support, NXK_ELAUNCH when the launch itself failed.  Kernels that wait on
 * a pipeline report a timed-out wait through nxk_take_error().
 */
#ifndef NEXTERA_KERNELS_H
#define NEXTERA_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#include "nexterabert.h"   /* NEXTERA_API */

#ifdef __cplusplus
extern "C" {
#endif

#define NXK_OK       0
#define NXK_EINVAL  (-1)
#define NXK_ELAUNCH (-2)

/* device-side error word of the current device: returns it and clears it
 * (synchronises the stream).  Nonzero = a kernel gave up on a bounded wait. */
NEXTERA_API int32_t nxk_take_error(void * stream);
/* Failure-path self-test: one thread waits up to limit_ns (<= 1 s) on an mbarrier that nothing
 * completes, with the GEMM pipeline's bounded wait, then records a timeout (0x1ff) in the error
 * word that nxk_take_error returns.  The context stays usable. */
NEXTERA_API int nxk_selftest_wait(int64_t limit_ns, void * stream);

/* Tensor-pipe rate probe for the int8 GEMM's roofline (no counterpart in the reference): n_ctas
 * CTAs (one per SM when n_ctas <= the SM count), each issuing iters x 4 tcgen05.mma.kind::i8 of
 * M 128 x N 256 x K 32 on operands resident in shared memory, with no copies and no epilogue.
 * Work per launch: 2 * 128 * 256 * 128 * iters * n_ctas int ops.  Time it with events. */
NEXTERA_API int nxk_i8_mma_rate_probe(int n_ctas, int iters, void * stream);

/* ---- weights: build_i8_weight (:1010-1049), on the device ----
 * blocks: n_out rows of GGUF blocks of `type` (any of F32 F16 BF16 Q4_0 Q4_1
 * Q5_0 Q5_1 Q8_0 Q2_K Q3_K Q4_K Q5_K Q6_K); writes w8, scale and (if not NULL) off. */
NEXTERA_API int nxk_expand_weight(int type, const void * blocks, int n_in, int n_out,
                                  int8_t * w8, float * scale, int32_t * off, void * stream);

/* ---- quantization of fp32 rows into GGUF blocks (the block encoders behind nextera_quantize,
 * tools/quantize.cpp's ggml_quantize_chunk) ----
 * x: rows x n_per_row fp32 (device); out: rows x row_size(type) bytes of `type` blocks (F16 Q8_0
 * Q4_0 Q4_1 Q5_0 Q5_1 Q2_K Q3_K Q4_K Q5_K Q6_K; ggml type ids).  n_per_row must be a multiple of the
 * block size (32, or 256 for the K-quants).  The legacy types are bit-identical to ggml's reference
 * quantizers as gguf-py restates them; the K-quants are a direct per-sub-block fit in the published
 * layouts (valid encodings, not ggml's iterative scale search). */
NEXTERA_API int nxk_quantize_rows(int type, const float * x, int64_t n_per_row, int64_t rows, void * out,
                                  void * stream);

/* ---- embedding: ggml_get_rows (+ ggml_add of segment rows), :1272-1273 ----
 * table: n_rows rows of C values in blocks of `type`.  An id outside [0, n_rows)
 * yields a zero row and sets the device error word (ids are checked on the host
 * before host-memory calls; device-resident ids are checked here). */
NEXTERA_API int nxk_embed(int type, const void * table, int n_rows, int C, const int32_t * tokens, int T,
                          int ttype, const void * ttable, int tn_rows, const int32_t * types, float * out,
                          void * stream);

/* ---- int8 linear: op_linear_i8 (:969-1007) ----
 * out[t][n] = (res[t][n] +) sum_B fma(float(S_B) * sx[t][B], sw[B][n], .), S_B the
 * int32 dot product of block B.  tcgen05 kind::i8 kernel; res may be NULL. */
NEXTERA_API int nxk_linear_i8(const int8_t * xq, const float * sx, int T, const int8_t * w8, const float * sw,
                              int K, int N, const float * res, float * out, void * stream);
/* the same result from a plain CUDA-core kernel (validation only) */
NEXTERA_API int nxk_linear_i8_simt(const int8_t * xq, const float * sx, int T, const int8_t * w8, const float * sw,
                                   int K, int N, const float * res, float * out, void * stream);
/* The int8 linear followed by the row op the reference applies to its output and by quantize_row
 * (:378-403) for the next int8 linear, in one kernel: codes q [T][N] (s8, the reference's u8 - 128)
 * and scales sq [T][N/256]; N must be a multiple of 256.
 *   relu_sqr_q:  v = relu(y)^2              (op_relu_sqr, :485-505)
 *   gate_q:      v = sigmoid(y) * z[t][n]   (op_gate, :508-523), z [T][N] fp32
 * Same codes and scales as nxk_linear_i8 then nxk_relu_sqr / nxk_gate with int8 output. */
NEXTERA_API int nxk_linear_i8_relu_sqr_q(const int8_t * xq, const float * sx, int T, const int8_t * w8,
                                         const float * sw, int K, int N, int8_t * q, float * sq, void * stream);
NEXTERA_API int nxk_linear_i8_gate_q(const int8_t * xq, const float * sx, int T, const int8_t * w8,
                                     const float * sw, int K, int N, const float * z, int8_t * q, float * sq,
                                     void * stream);
/* int32 block sums S_B, [T][N][n_blk] (validation of the integer path) */
NEXTERA_API int nxk_block_sums(const int8_t * xq, int T, const int8_t * w8, int K, int N, int32_t * sums, void * stream);

/* ---- row ops (:453-690).  q / sx NULL: fp32 `out`; otherwise int8 output ---- */
NEXTERA_API int nxk_quantize(const float * x, int T, int C, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_rms_norm(const float * x, const float * gain, float eps, int T, int C,
                             float * out, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_relu_sqr(const float * x, int T, int C, float * out, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_gate(const float * g, const float * y, int T, int C, float * out, int8_t * q, float * sx,
                         void * stream);
NEXTERA_API int nxk_dwconv(const float * x, const float * r, const float * taps, int k,
                           const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                           int T, int C, float * out, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_lily_state(const float * a, const float * x, const float * b, const float * taps, int k,
                               const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                               int T, int C, float * out, int8_t * q, float * sx, void * stream);
/* The two token convolutions where the inputs x (and a) also hold halo rows: rows
 * [-halo, T + halo) relative to the pointer may be read (those the documents reach); outputs
 * are rows [0, T).  With halo = 0 these are nxk_dwconv / nxk_lily_state. */
NEXTERA_API int nxk_dwconv_halo(const float * x, const float * r, const float * taps, int k, int halo,
                                const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                                int T, int C, float * out, int8_t * q, float * sx, void * stream);
/* nxk_dwconv_halo over inputs whose rows are ld floats apart (ld >= C, a multiple of 4): x and r may be
 * column ranges of one wider matrix, e.g. two linears fused into one.  Outputs stay C wide. */
NEXTERA_API int nxk_dwconv_halo_ld(const float * x, const float * r, int ld, const float * taps, int k, int halo,
                                   const int32_t * row_doc, const int32_t * doc_start, const int32_t * doc_len,
                                   int T, int C, float * out, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_lily_state_halo(const float * a, const float * x, const float * b, const float * taps, int k,
                                    int halo, const int32_t * row_doc, const int32_t * doc_start,
                                    const int32_t * doc_len, int T, int C, float * out, int8_t * q, float * sx,
                                    void * stream);
NEXTERA_API int nxk_qk_prep(const float * x, const float * alpha, const float * beta,
                            const float * cos_t, const float * sin_t, const int32_t * row_doc,
                            const int32_t * doc_start, int T, int H, int D, int head_major, float * out,
                            void * stream);
NEXTERA_API int nxk_head_major(const float * x, int T, int H, int D, float * out, void * stream);
/* q, k and v of one mixer from its fused projection x [T][ldx] (columns: H q heads, G k heads,
 * G v heads): qk_prep on q (token-major [T][H][D]) and on k (head-major [G][T][D]), v copied
 * head-major; D must be 64.  Same values as nxk_qk_prep / nxk_head_major on the split columns. */
NEXTERA_API int nxk_qkv_prep(const float * x, int ldx, const float * q_alpha, const float * q_beta,
                             const float * k_alpha, const float * k_beta, const float * cos_t,
                             const float * sin_t, const int32_t * row_doc, const int32_t * doc_start,
                             int T, int H, int G, int D, float * q, float * k, float * v, void * stream);
/* nxk_qkv_prep writing k and v into buffers of Tk rows per head at rows koff .. koff + T - 1
 * (the layout nxk_attention_kv reads). */
NEXTERA_API int nxk_qkv_prep_kv(const float * x, int ldx, const float * q_alpha, const float * q_beta,
                                const float * k_alpha, const float * k_beta, const float * cos_t,
                                const float * sin_t, const int32_t * row_doc, const int32_t * doc_start,
                                int T, int H, int G, int D, int Tk, int koff, float * q, float * k, float * v,
                                void * stream);
NEXTERA_API int nxk_block_mean(const float * h, const float * g, int C, int block,
                               const int32_t * doc_start, const int32_t * doc_len,
                               const int32_t * bdoc_start, const int32_t * brow_doc, int n_brows,
                               float * out, int8_t * q, float * sx, void * stream);
NEXTERA_API int nxk_upsample_add(const float * y, const float * r, int C, int block, int T,
                                 const int32_t * row_doc, const int32_t * doc_start, const int32_t * bdoc_start,
                                 float * out, void * stream);
/* ggml_norm * w + b (:1292-1293); w / b may be NULL */
NEXTERA_API int nxk_layer_norm(const float * x, const float * w, const float * b, float eps, int T, int C,
                               float * out, void * stream);
/* run_forward's pooling (:1903-1918): per-document sum, then 1/n or 1/||sum|| */
NEXTERA_API int nxk_pool(const float * hidden, const int32_t * doc_start, const int32_t * doc_len, int n_docs,
                         int C, int normalize, float * pooled, void * stream);
/* The two halves of nxk_pool for a document split over several calls (shards in order):
 * pooled[c] continues the sequential sum from its current value over hidden rows [0, T);
 * nxk_pool_finish then applies 1/n (n = the whole length) or 1/||sum||. */
NEXTERA_API int nxk_pool_continue(const float * hidden, int T, int C, float * pooled, void * stream);
NEXTERA_API int nxk_pool_finish(int n, int C, int normalize, float * pooled, void * stream);

/* ---- heads (builder::transform / pooler / classifier :1296-1317, nextera_mlm_logits :1963-2011) ---- */
/* transform's tail: GELU(erf) (ggml_gelu_erf), then ggml_norm * w (w may be NULL); out may be x */
NEXTERA_API int nxk_gelu_norm(const float * x, const float * w, float eps, int T, int C, float * out, void * stream);
/* out[i] = x[idx[i]] for rows of C floats (ggml_get_rows on the hidden state, :1995) */
NEXTERA_API int nxk_gather_rows(const float * x, int C, const int32_t * idx, int n, float * out, void * stream);
/* ggml_mul_mat (:1140-1142) on a weight off the int8 path, in GGUF blocks of `type`
 * (F32 F16 BF16 Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 Q2_K Q3_K Q4_K Q5_K Q6_K):
 * out[m][n] = W[n] . x[m] (+ bias[n]) for N weight rows of K inputs and M rows of x,
 * with x first converted to the type's vec_dot type as ggml's CPU backend does
 * (Q8_K / Q8_0 / Q8_1 codes, or F16 / BF16 rounding).  `workspace` holds the
 * converted rows: nxk_mul_mat_workspace(type, K, M) bytes (0 = unsupported type).
 * K must be a multiple of 32 (256 for the K-quants); N <= 524280; w, x and workspace
 * 16-byte aligned. */
NEXTERA_API size_t nxk_mul_mat_workspace(int type, int K, int M);
NEXTERA_API int nxk_mul_mat(int type, const void * w, int N, int K, const float * x, int M, const float * bias,
                            void * workspace, float * out, void * stream);

/* ---- attention: op_attention (:785-852), varlen GQA over packed documents ----
 * half < 0: full attention inside each document, else the band |i - j| <= half.
 * scale[n_docs] on the device.  h_doc_start / h_doc_len: the same layout in host
 * memory, used to plan the work; the plan (nxk_attention_workspace bytes) is
 * written to `workspace` on the device. */
NEXTERA_API size_t nxk_attention_workspace(const int32_t * h_doc_len, int n_docs, int half);
NEXTERA_API int nxk_attention(const float * q, const float * k, const float * v, int T, int H, int G, int D,
                              int half, const float * scale, const int32_t * row_doc,
                              const int32_t * doc_start, const int32_t * doc_len, int n_docs,
                              const int32_t * h_doc_start, const int32_t * h_doc_len,
                              void * workspace, size_t workspace_bytes, float * out, void * stream);

/* nxk_attention with K / V in a buffer of Tk rows per head in which key row 0 (the row of query
 * row 0) is row koff: a document's keys may then lie before or after the query rows, as for a
 * shard of a long sequence whose K / V were gathered from all shards (Tk = total length, koff =
 * the shard's offset) or extended by the neighbours' rows (a halo).  Documents are given relative
 * to query row 0 and may start before it; only query rows [0, T) are computed.  Keys a tile needs
 * outside [-koff, Tk - koff) give NXK_EINVAL. */
NEXTERA_API int nxk_attention_kv(const float * q, const float * k, const float * v, int T, int Tk, int koff,
                                 int H, int G, int D, int half, const float * scale,
                                 const int32_t * doc_start, const int32_t * doc_len, int n_docs,
                                 const int32_t * h_doc_start, const int32_t * h_doc_len,
                                 void * workspace, size_t workspace_bytes, float * out, void * stream);

/* nxk_attention without a workspace argument, for callers that cannot allocate
 * device memory when they call (a host that hands this library pointers into a
 * pool it manages itself and forbids cudaMalloc after start-up, or a path where a
 * blocking allocation is not allowed).  No counterpart in the reference, whose
 * CPU attention needs no device memory.  Its work plan lives in a fixed array
 * inside the library (2.5 MiB on each device that loads it, kept until exit):
 * at most 131072 query tiles per call, i.e. sum over documents of
 * ceil(len / 32) <= 131072; larger batches return NXK_EINVAL.  h_doc_len is the
 * host copy of doc_len and must equal it; the documents must lie in [0, T)
 * (a host total above T returns NXK_EINVAL; a device copy that disagrees leaves
 * the output unwritten and sets error word 0x301, read by nxk_take_error).  The
 * array's device address is looked up on the first call made with each device
 * current, so make that first call before any stream capture; a device reset
 * (cudaDeviceReset) is not supported afterwards.  Calls share the array: two
 * calls in flight at the same time race. */
NEXTERA_API int nxk_attention_noalloc(const float * q, const float * k, const float * v, int T, int H, int G, int D,
                                      int half, const float * scale, const int32_t * doc_start,
                                      const int32_t * doc_len, int n_docs, const int32_t * h_doc_len, float * out,
                                      void * stream);

#ifdef __cplusplus
}
#endif

#endif
