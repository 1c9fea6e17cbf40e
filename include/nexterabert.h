/* nexterabert.h -- public C API of libnexterabert.so, the B200 (sm_100a) build.
 *
 * Drop-in for the reference runtime's API (Rikka-Botan/NexteraBERT.cpp,
 * src/nexterabert.h:28-123): the same functions, argument meanings, return codes
 * and ownership rules, so tools/cli.cpp and python/nexterabert_cpp.py of the
 * reference run unchanged against this library.  The function names, the
 * nextera_params layout and the NEXTERA_API visibility macro must stay
 * identical to the reference's for that reason; the comments below describe
 * this implementation.
 *
 * Execution model: nextera_load expands every quantized linear weight to int8
 * on the current CUDA device; each call then runs the whole encoder on that
 * device and copies results to the caller's host arrays before returning.
 * One call at a time per context.
 */
#ifndef NEXTERABERT_H
#define NEXTERABERT_H

#include <stddef.h>
#include <stdint.h>

#if defined(NEXTERA_SHARED)
#  if defined(_WIN32)
#    if defined(NEXTERA_BUILD)
#      define NEXTERA_API __declspec(dllexport)
#    else
#      define NEXTERA_API __declspec(dllimport)
#    endif
#  else
#    define NEXTERA_API __attribute__((visibility("default")))
#  endif
#else
#  define NEXTERA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

struct nextera_context;

/* reference: src/nexterabert.h:30-36 */
struct nextera_params {
    int32_t n_threads;   /* host threads for load-time work; <= 0: all cores */
    int32_t use_int8;    /* accepted for compatibility; linear layers always run int8 on the GPU */
    int32_t use_repack;  /* accepted for compatibility; no effect */
    int32_t verbosity;   /* 0 silent, 1 load summary on stderr */
};

/* reference: src/nexterabert.h:38 */
NEXTERA_API struct nextera_params nextera_default_params(void);

/* Loads a nexterabert GGUF onto the current CUDA device.  NULL on failure, with
 * the reason on stderr (bad file, unsupported tensor type, no CUDA device).
 * reference: src/nexterabert.h:40-42 */
NEXTERA_API struct nextera_context * nextera_load(const char * path, struct nextera_params params);
NEXTERA_API void nextera_free(struct nextera_context * ctx);

/* model facts (reference: src/nexterabert.h:44-66) */
NEXTERA_API int32_t nextera_n_embd(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_n_vocab(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_n_layer(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_has_mlm_head(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_has_pooler(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_n_token_types(const struct nextera_context * ctx);
NEXTERA_API const char * nextera_classifier_task(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_n_labels(const struct nextera_context * ctx);
NEXTERA_API const char * nextera_label(const struct nextera_context * ctx, int32_t i);
NEXTERA_API int32_t nextera_token_cls(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_token_sep(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_token_pad(const struct nextera_context * ctx);
NEXTERA_API int32_t nextera_token_mask(const struct nextera_context * ctx);
NEXTERA_API const char * nextera_tokenizer_json(const struct nextera_context * ctx);
NEXTERA_API const char * nextera_ftype(const struct nextera_context * ctx);
/* keeps the reference's "linear layers: N int8 (...)" fragment (parsed by its python/bench.py) */
NEXTERA_API const char * nextera_system_info(const struct nextera_context * ctx);

/* host threads for load-time work (reference: src/nexterabert.h:68-69) */
NEXTERA_API void    nextera_set_n_threads(struct nextera_context * ctx, int32_t n_threads);
NEXTERA_API int32_t nextera_get_n_threads(const struct nextera_context * ctx);

/* Encodes n_seqs unpadded sequences in one forward pass (reference:
 * src/nexterabert.h:71-87).  tokens: sum(lengths) ids; hidden (optional):
 * sum(lengths) x n_embd; pooled (optional): n_seqs x n_embd mean, L2-normalised
 * when normalize != 0.  Host memory.  A sequence's result does not depend on
 * the rest of the batch.  0 ok, 1 bad input, 2 allocation failure, 3 device failure. */
NEXTERA_API int32_t nextera_encode(struct nextera_context * ctx,
                                   const int32_t * tokens, const int32_t * lengths, int32_t n_seqs,
                                   float * hidden, float * pooled, int32_t normalize);

/* nextera_encode with optional segment ids (reference: src/nexterabert.h:95-98) */
NEXTERA_API int32_t nextera_encode_segments(struct nextera_context * ctx,
                                            const int32_t * tokens, const int32_t * token_types,
                                            const int32_t * lengths, int32_t n_seqs,
                                            float * hidden, float * pooled, int32_t normalize);

/* Heads (reference: src/nexterabert.h:100-121), on the GPU: the encoder, then the
 * pooler / classifier / MLM transform and decoder.  1 when the file has no such head. */
NEXTERA_API int32_t nextera_pooler_output(struct nextera_context * ctx,
                                          const int32_t * tokens, const int32_t * token_types,
                                          const int32_t * lengths, int32_t n_seqs, float * out);
NEXTERA_API int32_t nextera_classify(struct nextera_context * ctx,
                                     const int32_t * tokens, const int32_t * token_types,
                                     const int32_t * lengths, int32_t n_seqs, float * logits);
NEXTERA_API int32_t nextera_mlm_logits(struct nextera_context * ctx,
                                       const int32_t * tokens, int32_t n_tokens,
                                       const int32_t * positions, int32_t n_pos,
                                       float * logits);

/* wall time of the last encode call in ms, host copies included (reference: src/nexterabert.h:124) */
NEXTERA_API double nextera_last_ms(const struct nextera_context * ctx);

/* ---- outside the reference's public header ---- */

/* Exported by the reference without a header declaration (src/nexterabert.cpp:1818-1841);
 * its CLI and Python binding bind them.  set_layers: run only the first n blocks and
 * skip out_norm (-1: whole model).  profile: per-kind device time (int8 linear /
 * attention / row ops) measured with CUDA events, printed by profile_print. */
NEXTERA_API void nextera_debug_set_layers(struct nextera_context * ctx, int32_t n_layers);
NEXTERA_API void nextera_debug_profile(struct nextera_context * ctx, int32_t enable);
NEXTERA_API void nextera_debug_profile_print(const struct nextera_context * ctx);
/* Number of device kernels this context has launched since nextera_load (no
 * counterpart in the reference; lets a benchmark count the launches it timed). */
NEXTERA_API int64_t nextera_debug_launches(const struct nextera_context * ctx);
/* The profile's totals as numbers: kind_ms[3] = device ms in int8 linear / attention /
 * row ops, *total_ms = wall ms of the profiled calls; returns the number of calls. */
NEXTERA_API int64_t nextera_debug_profile_get(const struct nextera_context * ctx, double * kind_ms, double * total_ms);

/* Device-resident variant of nextera_encode_segments: tokens / token_types are
 * device pointers, hidden / pooled device pointers (either may be NULL), lengths
 * host memory; work is enqueued on `stream` (cudaStream_t as void *) and this
 * call returns once it is enqueued.  No counterpart in the reference (its data
 * never leaves the host); used to time the forward with inputs already in HBM. */
NEXTERA_API int32_t nextera_encode_device(struct nextera_context * ctx,
                                          const int32_t * d_tokens, const int32_t * d_token_types,
                                          const int32_t * lengths, int32_t n_seqs,
                                          float * d_hidden, float * d_pooled, int32_t normalize,
                                          void * stream);

/* ---- one sequence split over several GPUs (one process per GPU) ----
 * No counterpart in the reference, which runs on one host.  Each rank encodes a
 * contiguous, equal part of the sequence; neighbours exchange the halo rows of the
 * token convolutions and of the band-attention K / V, the full-attention layers
 * gather every rank's K / V, and the pooled vector is summed rank after rank in the
 * sequence's order, so every rank's rows and the pooled vector are the ones the whole
 * sequence gives on one GPU.  Communication is NCCL (libnccl.so.2, loaded on first use). */

/* Writes the 128-byte NCCL id for a new group; call on one rank and pass the bytes to all. */
NEXTERA_API int32_t nextera_shard_unique_id(uint8_t * id);
/* Joins the group (rank in [0, world)) on the context's device; every rank calls it with the
 * same id.  Blocks until all ranks have joined.  0 on success. */
NEXTERA_API int32_t nextera_shard_init(struct nextera_context * ctx, int32_t rank, int32_t world,
                                       const uint8_t * id);
/* Encodes this rank's n_local ids (device memory) of a sequence of n_total = world * n_local ids;
 * n_local must be a multiple of the HRA block and at least the band half-width.  d_hidden
 * ([n_local][n_embd], this rank's rows) and d_pooled ([n_embd], the whole sequence, on every rank)
 * are device pointers, either may be NULL.  Enqueued on `stream`; every rank must call it. */
NEXTERA_API int32_t nextera_encode_sharded(struct nextera_context * ctx, const int32_t * d_tokens, int32_t n_local,
                                           int32_t n_total, float * d_hidden, float * d_pooled, int32_t normalize,
                                           void * stream);

/* ---- one batch of sequences split over several GPUs (one process per GPU) ----
 * No counterpart in the reference, which runs on one host.  The reference's batch contract
 * (src/nexterabert.h:69-84: a sequence's result does not depend on the rest of the batch) lets
 * the sequences of one batch run on different GPUs: each rank encodes a share of them on its own
 * model replica, and the pooled rows come back to rank 0 in the batch's order, bit for bit what
 * one GPU gives.  The ranks are the group of nextera_shard_init; without it the whole batch runs
 * on this context's device. */

/* The partition every rank uses: part[i] = the rank of sequence i.  Longest-first greedy on an
 * estimate of each sequence's device time (tokens through the linear layers and row ops, plus
 * query-tile x key pairs through every attention layer), so the ranks finish together.  Depends
 * only on the lengths and the model, so all ranks compute the same one.  0 ok, 1 bad input. */
NEXTERA_API int32_t nextera_partition(const struct nextera_context * ctx, const int32_t * lengths, int32_t n_seqs,
                                      int32_t n_parts, int32_t * part);
/* nextera_encode_segments over a batch partitioned across the ranks, pooled output only.  Every
 * rank calls it with the same host arrays (tokens, token_types (may be NULL), lengths); each
 * encodes its share and rank 0 receives all pooled rows into `pooled` (n_seqs x n_embd, host
 * memory; other ranks may pass NULL).  The whole batch is checked on every rank first, and the
 * ranks agree on the outcome before rows move, so all ranks return the same code. */
NEXTERA_API int32_t nextera_encode_partitioned(struct nextera_context * ctx, const int32_t * tokens,
                                               const int32_t * token_types, const int32_t * lengths,
                                               int32_t n_seqs, float * pooled, int32_t normalize);
/* Device-resident variant: d_tokens holds only this rank's sequences (those with
 * nextera_partition(...)[i] == rank, concatenated in batch order) in device memory; lengths is
 * the whole batch (host memory); rank 0's d_pooled (device, n_seqs x n_embd) receives every
 * sequence's pooled row in batch order.  A rank that the partition gives no sequence may pass
 * d_tokens = NULL.  Enqueued on `stream`; every rank must call it. */
NEXTERA_API int32_t nextera_encode_partitioned_device(struct nextera_context * ctx, const int32_t * d_tokens,
                                                      const int32_t * lengths, int32_t n_seqs, float * d_pooled,
                                                      int32_t normalize, void * stream);

/* ---- the model quantizer (reference: tools/quantize.cpp, a separate program there) ----
 * Re-encodes the 2-D weights of an F32 / F16 GGUF (in_path) into out_path with the file type
 * `ftype` (F32 F16 Q8_0 Q6_K Q5_K_M Q5_K_S Q5_0 Q4_K_M Q4_K_S Q4_0 Q3_K_M) and the reference tool's
 * rules: which tensors are quantized, the "_M" presets' extra bits, the row-size fallback of the
 * K-quants, and overrides "SUBSTRING=TYPE" (its --tensor-type).  The block encoding runs on the
 * current CUDA device; the other tensors and every metadata key are copied.  Prints one line per
 * re-encoded tensor on stdout.  0 ok, 1 bad input or file error, 2 allocation failure, 3 device
 * failure.  No context is needed. */
NEXTERA_API int32_t nextera_quantize(const char * in_path, const char * out_path, const char * ftype,
                                     int32_t n_overrides, const char * const * overrides);

#ifdef __cplusplus
}
#endif

#endif /* NEXTERABERT_H */
