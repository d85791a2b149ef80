/*
 * eif_cuda.h -- B200 (sm_100a) token-mixing hot path of bitllm.c behind a C99 ABI.
 *
 * The engine keeps its C99 host code; the GQA attention over the KV cache and the Gated DeltaNet
 * state update run on the GPU through these entry points.  The header sits next to the engine's
 * eif_gpu.h and follows its conventions (include/eif_gpu.h:31-61 in bitllm.c): an opaque context,
 * one command stream per context, a context is not thread-safe.  Unlike eif_gpu there is no CPU
 * fallback: every failure comes back as an eif_status_t and the caller decides.
 *
 * Device mirrors keep the engine's layouts unchanged:
 *   KV cache   per layer, per sequence: [max_seq_len][n_kv_heads * head_dim], row t holds the
 *              rotated key / value of position t (qwen35_attn_state_t, include/eif_qwen35.h:204-208;
 *              tinyllm key_cache/value_cache, src/eif_tinyllm.c:415-418), fp32 or bf16.
 *   DeltaNet   per layer, per sequence: S [n_v_heads][d_k][d_v] fp32, d_v contiguous, and the
 *              conv window [conv_dim][conv_k] fp32 (qwen35_delta_state_t, include/eif_qwen35.h:199-202).
 *   Sequences of one batch are stacked: sequence b of layer l starts at b * (one sequence's size).
 *
 * Pointer conventions: arguments are HOST pointers unless the entry point's name ends in `_dev`,
 * in which case they are device pointers and the call is asynchronous on the context's stream.
 * Host entry points copy their inputs in, run, copy the outputs back and wait (with the context's
 * timeout) before returning.  Reference paths (file:line) are relative to the bitllm.c root.
 */
#ifndef EIF_CUDA_H
#define EIF_CUDA_H

#include <stddef.h>
#include <stdint.h>

/* Status codes: the engine's own eif_status_t (include/eif_status.h:8-19).  When the engine's header
 * is reachable it is used as is; otherwise the same enumerators are declared here under the same
 * include guard, so either header may come first. */
#if defined(__has_include)
#if __has_include("eif_status.h")
#include "eif_status.h"
#endif
#endif
#ifndef EIF_STATUS_H
#define EIF_STATUS_H
typedef enum {
    EIF_STATUS_OK = 0,
    EIF_STATUS_ERROR = -1,
    EIF_STATUS_INVALID_ARGUMENT = -2,
    EIF_STATUS_OUT_OF_MEMORY = -3,
    EIF_STATUS_NOT_IMPLEMENTED = -4,
    EIF_STATUS_NOT_SUPPORTED = -5,
    EIF_STATUS_TIMEOUT = -6,
    EIF_STATUS_INTERNAL_ERROR = -7,
    EIF_STATUS_INVALID_LAYER = -8,
    EIF_STATUS_SHAPE_MISMATCH = -9
} eif_status_t;
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct eif_cuda_ctx eif_cuda_ctx_t;      /* one device, one stream; not thread-safe */
typedef struct eif_cuda_kv eif_cuda_kv_t;        /* device KV cache of n_layers x batch sequences */
typedef struct eif_cuda_delta eif_cuda_delta_t;  /* device DeltaNet states of n_layers x batch sequences */

/* KV cache element type.  EIF_CUDA_INT8 is tinyllm's quantised cache (kv_type 1, src/eif_tinyllm.c:136-143):
 * int8 rows plus one fp32 scale per (row, kv head) for K and one for V; head_dim 64, 128 or 256. */
typedef enum { EIF_CUDA_F32 = 0, EIF_CUDA_BF16 = 1, EIF_CUDA_INT8 = 2 } eif_cuda_dtype_t;

/* SubLN applied after the attention output gate (src/eif_qwen35.c:779-789). */
typedef enum {
    EIF_CUDA_SUBLN_NONE = 0,  /* plain_linear: copy (also the tinyllm path, which has no SubLN) */
    EIF_CUDA_SUBLN_RMS = 1,   /* !plain_linear without a sub_norm weight: x * rsqrt(mean(x^2) + 1e-6) */
    EIF_CUDA_SUBLN_WEIGHT = 2 /* x * rsqrt(mean(x^2) + 1e-6) * sub_norm */
} eif_cuda_subln_t;

/* ---------------------------------------------------------------------------------------------
 * Context  (replaces eif_gpu_init / eif_gpu_shutdown for this path, include/eif_gpu.h:44-50)
 * ------------------------------------------------------------------------------------------- */

/* Number of visible CUDA devices (0 without a driver or with BITLLM_NO_CUDA=1). */
int eif_cuda_device_count(void);

/* Create a context on `device`.  Returns EIF_STATUS_NOT_SUPPORTED when there is no device, the device
 * is not sm_100 (B200) or BITLLM_NO_CUDA=1 is set. */
eif_status_t eif_cuda_init(eif_cuda_ctx_t **ctx, int device);
/* Free every KV cache, DeltaNet state and projection matrix made on the context before the context itself. */
void eif_cuda_free(eif_cuda_ctx_t *ctx);

/* Message of the last failure on this context ("" if none).  Valid until the next call. */
const char *eif_cuda_last_error(const eif_cuda_ctx_t *ctx);

/* Stream used by `_dev` calls: a cudaStream_t passed as void* (NULL = the context's own stream). */
eif_status_t eif_cuda_set_stream(eif_cuda_ctx_t *ctx, void *stream);
void *eif_cuda_get_stream(const eif_cuda_ctx_t *ctx);

/* Host waits poll the stream until done or `timeout_ms` elapses (EIF_STATUS_TIMEOUT); 0 = no limit. */
eif_status_t eif_cuda_set_timeout(eif_cuda_ctx_t *ctx, int timeout_ms);
eif_status_t eif_cuda_synchronize(eif_cuda_ctx_t *ctx);

/* Number of kernels this context has launched since it was created (instrumentation). */
uint64_t eif_cuda_launch_count(const eif_cuda_ctx_t *ctx);

/* ---------------------------------------------------------------------------------------------
 * KV cache mirror  (qwen35_attn_state_t, include/eif_qwen35.h:204-208; tinyllm_state_t key/value
 * caches, src/eif_tinyllm.c:131-134).  The reference keeps fp32 only (Qwen3.5) or fp32/INT8
 * (tinyllm); bf16 is the B200 storage type for long contexts.
 * ------------------------------------------------------------------------------------------- */

eif_status_t eif_cuda_kv_alloc(eif_cuda_ctx_t *ctx, int n_layers, int batch, int max_seq_len, int n_kv_heads,
                               int head_dim, eif_cuda_dtype_t dtype, eif_cuda_kv_t **kv);
void eif_cuda_kv_free(eif_cuda_kv_t *kv);

/* Zero every row of every layer (the KV part of qwen35_reset, src/eif_qwen35.c:1483-1497). */
eif_status_t eif_cuda_kv_reset(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv);

/* Copy rows [row0, row0+n_rows) of (layer, seq) from / to host fp32 arrays [n_rows][n_kv_heads*head_dim].
 * A bf16 cache converts on the device (round to nearest even) and widens on download.  An INT8 cache
 * quantises each (row, kv head) on upload exactly as tinyllm's cache write does (src/eif_tinyllm.c:509-553)
 * and returns code * scale on download. */
eif_status_t eif_cuda_kv_upload(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0, int n_rows,
                                const float *k_rows, const float *v_rows);
eif_status_t eif_cuda_kv_download(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                  int n_rows, float *k_rows, float *v_rows);

/* Device base pointers of one layer: [batch][max_seq_len][n_kv_heads][head_dim] of the cache dtype. */
eif_status_t eif_cuda_kv_layer_ptrs(const eif_cuda_kv_t *kv, int layer, void **k_dev, void **v_dev);

/* INT8 caches: the raw codes [n_rows][n_kv_heads*head_dim] and scales [n_rows][n_kv_heads] of rows
 * [row0, row0+n_rows) of (layer, seq) -- tinyllm_state_t's key_cache_i8 / value_cache_i8 rows and its
 * key_scale / value_scale entries (include/eif_tinyllm.h:153-157, indexed as src/eif_tinyllm.c:511-520).
 * EIF_STATUS_INVALID_ARGUMENT for another dtype. */
eif_status_t eif_cuda_kv_download_int8(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                       int n_rows, int8_t *k_codes, int8_t *v_codes, float *k_scale,
                                       float *v_scale);
/* Device pointers of one INT8 layer's scales, head-major: [batch][n_kv_heads][stride] fp32 with stride =
 * max_seq_len rounded up to 64 (entry (b, h, t) scales row t of kv head h of sequence b). */
eif_status_t eif_cuda_kv_layer_scales(const eif_cuda_kv_t *kv, int layer, float **k_scale_dev,
                                      float **v_scale_dev);

/* Append the new token's rotated k / v ([batch][n_kv_heads*head_dim] fp32) at row pos[b] of every
 * sequence -- the memcpy into the cache at src/eif_qwen35.c:734-736 and src/eif_tinyllm.c:417-418. */
eif_status_t eif_cuda_kv_append(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const int *pos, const float *k,
                                const float *v);
eif_status_t eif_cuda_kv_append_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const int *pos_dev,
                                    const float *k_dev, const float *v_dev);

/* tinyllm RoPE (src/eif_tinyllm.c:395-405, 481-507): the per-position cos / sin tables of the model's theta
 * (freq_j = 1 / theta^(2j/head_dim), the reference's float formula, computed on the host for every position
 * of the cache) and the pair convention: interleaved = 0 rotates (j, j + head_dim/2) (NeoX, Qwen2),
 * interleaved != 0 rotates (2j, 2j+1) (llama-style GGUF).  Call once per cache before the rope_append calls. */
eif_status_t eif_cuda_kv_set_rope(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, float theta, int interleaved);

/* RoPE of the new token's q and k at pos[b], and the cache write of k (rotated) and v at row pos[b]:
 * tinyllm_forward_embedding_ex's rotation (:481-507) plus its cache write (:415-418), one launch.
 *   q, q_out [batch][n_heads*head_dim]; k, v [batch][n_kv_heads*head_dim]
 * _dev: fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_rope_append(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, const float *k,
                                  const float *v, const int *pos, int n_heads, float *q_out);
eif_status_t eif_cuda_rope_append_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                      const float *k_dev, const float *v_dev, const int *pos_dev, int n_heads,
                                      float *q_out_dev);

/* The same for a prefill chunk: token i of every sequence at position start_pos + i (the per-token tables of
 * the batched prefill, src/eif_tinyllm.c:994-1006).
 *   q, q_out [batch][n_tok][n_heads*head_dim]; k, v [batch][n_tok][n_kv_heads*head_dim]
 * _dev: q_out in the input type of eif_cuda_attend_prefill_dev for this cache (bf16 for a bf16 cache, fp32 for
 * fp32 and INT8 caches), the rest fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_rope_append_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                          const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                          float *q_out);
eif_status_t eif_cuda_rope_append_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                              const float *k_dev, const float *v_dev, int n_tok, int start_pos,
                                              int n_heads, void *q_out_dev);

/*
 * A whole tinyllm decode step of one layer in one call: RoPE of the new q and k, the write of the new K / V row at
 * pos[b], and GQA attention over rows [0, pos[b]] for every head -- src/eif_tinyllm.c:480-507 (rotation and cache
 * write, :509-549 for an INT8 cache) then the head loop :555-656, i.e. eif_cuda_rope_append followed by
 * eif_cuda_attend_decode (no gate, no SubLN) without the rotated q leaving the device.  Small batches (fp32 or bf16
 * cache, head_dim 64 / 128, at most 8 q heads per kv head) run as ONE launch with a thread-block cluster per
 * (sequence, kv head); other shapes run the two calls' kernels.  Needs eif_cuda_kv_set_rope.
 *   q [batch][n_heads*head_dim], k, v [batch][n_kv*head_dim] fp32 (un-rotated); out [batch][n_heads*head_dim].
 * _dev: device arrays, asynchronous; max_pos bounds every pos[b] (as in eif_cuda_attend_decode_dev).
 */
eif_status_t eif_cuda_decode_step(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, const float *k,
                                  const float *v, const int *pos, int n_heads, float scale, float *out);
eif_status_t eif_cuda_decode_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                      const float *k_dev, const float *v_dev, const int *pos_dev, int max_pos,
                                      int n_heads, float scale, float *out_dev);

/* ---------------------------------------------------------------------------------------------
 * Decode attention: one new query token per sequence over cache rows [0, pos[b]].
 * Replaces the head loop of fullatt_attend (src/eif_qwen35.c:741-790) and the inline tinyllm decode
 * attention (src/eif_tinyllm.c:555-656):
 *   q        [batch][n_heads * head_dim] fp32, rotated (kv head of q head h = h / (n_heads/n_kv_heads))
 *   scale    score multiplier (1/sqrt(head_dim) in both engines)
 *   gate     NULL, or [batch][n_heads*head_dim]: out *= sigmoid(gate)  (src/eif_qwen35.c:773-777)
 *   subln    SubLN of the whole gated output row (src/eif_qwen35.c:779-789); sub_norm [n_heads*head_dim]
 *            is read only for EIF_CUDA_SUBLN_WEIGHT
 *   out      [batch][n_heads * head_dim] fp32
 * pos[b] must satisfy 0 <= pos[b] < max_seq_len (the bound tinyllm_forward enforces,
 * src/eif_tinyllm.c:387-389); violations return EIF_STATUS_INVALID_ARGUMENT before any launch.
 * ------------------------------------------------------------------------------------------- */
eif_status_t eif_cuda_attend_decode(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                    const int *pos, int n_heads, float scale, const float *gate,
                                    eif_cuda_subln_t subln, const float *sub_norm, float *out);
/* Device-pointer variant; max_pos is an upper bound of pos_dev[] (used to size the split over the KV
 * length: rows beyond a sequence's own pos are never read).  A pos_dev[b] above max_pos (or outside the
 * cache) is not computed: that sequence's output is zeros and the next synchronising call returns
 * EIF_STATUS_INVALID_ARGUMENT.  The TMA-fed kernels bulk-copy each item's query rows, so they need q_dev
 * 16-byte aligned; an unaligned q_dev runs the (slower) SIMT kernel with the same results. */
eif_status_t eif_cuda_attend_decode_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                        const int *pos_dev, int max_pos, int n_heads, float scale,
                                        const float *gate_dev, eif_cuda_subln_t subln, const float *sub_norm_dev,
                                        float *out_dev);

/* The split decode attention would use for this cache layer, n_heads and max_pos: key chunks per (sequence,
 * kv head) in *n_chunks, keys per chunk in *chunk_keys, and the device scratch its partials need in
 * *scratch_bytes.  noalloc != 0 answers for eif_cuda_attend_decode_noalloc_dev (split capped to its fixed
 * array; *scratch_bytes above that array means the call would be refused).  Launches nothing.  No counterpart
 * in the reference: it lets a caller size memory up front and lets tests pin the split regime. */
eif_status_t eif_cuda_attend_decode_plan(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_heads, int max_pos,
                                         int noalloc, int *n_chunks, int *chunk_keys, size_t *scratch_bytes);

/* ---------------------------------------------------------------------------------------------
 * Causal prefill attention: n_tok new tokens per sequence at positions start_pos .. start_pos+n_tok-1,
 * token i attending to cache rows 0 .. start_pos+i.  Replaces the batched prefill attention of
 * tinyllm_forward_batch_embeddings (src/eif_tinyllm.c:1158-1268) and the per-token fullatt_attend of
 * Qwen3.5's prefill_chunk (src/eif_qwen35.c:1122-1133, without gate / SubLN).  The chunk's k / v rows must
 * already be in the cache (kv_upload, kv_append, rope_append_prefill).  head_dim 64, 128 or 256.
 *   q   [batch][n_tok][n_heads*head_dim], out the same shape
 * A bf16 cache runs the tensor-core causal kernels: _dev takes bf16 device arrays (16-byte aligned) and the
 * host variant rounds q to bf16 on the device and widens the output back.  An fp32 or INT8 cache (tinyllm's
 * kv_type 1, read as src/eif_tinyllm.c:1172-1235 reads it) runs every token as one decode row at its own
 * position, in fp32 arithmetic over the cache's own values: _dev takes fp32 device arrays.
 * _dev calls are asynchronous; the host variant takes fp32 host arrays.
 * ------------------------------------------------------------------------------------------- */
eif_status_t eif_cuda_attend_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, int n_tok,
                                     int start_pos, int n_heads, float scale, float *out);
eif_status_t eif_cuda_attend_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const void *q_dev,
                                         int n_tok, int start_pos, int n_heads, float scale, void *out_dev);

/* Qwen3.5 gated prefill attention: what prefill_chunk gets from fullatt_attend per token
 * (src/eif_qwen35.c:1122-1133 -> :741-789), i.e. the causal prefill above followed, row by row, by the
 * output gate and SubLN of eif_cuda_attend_decode (out = SubLN(o * sigmoid(gate))).
 *   gate  NULL, or [batch][n_tok][n_heads*head_dim] fp32; sub_norm [n_heads*head_dim] for EIF_CUDA_SUBLN_WEIGHT
 *   out   [batch][n_tok][n_heads*head_dim] fp32
 * _dev: q bf16 (16-byte aligned) for a bf16 cache, fp32 for an fp32 cache; gate / sub_norm / out fp32 device
 * arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_attend_prefill_gated(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                           int n_tok, int start_pos, int n_heads, float scale, const float *gate,
                                           eif_cuda_subln_t subln, const float *sub_norm, float *out);
eif_status_t eif_cuda_attend_prefill_gated_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                               const void *q_dev, int n_tok, int start_pos, int n_heads, float scale,
                                               const float *gate_dev, eif_cuda_subln_t subln,
                                               const float *sub_norm_dev, float *out_dev);

/* Same computation and arguments as eif_cuda_attend_decode_dev, for callers that may not allocate device
 * memory after start-up (an engine whose device memory is all reserved up front, or one running under a
 * fixed memory budget).  No counterpart in the reference.  It calls no cudaMalloc / cudaFree: the split-K
 * partials go to one 16 MiB array compiled into the library (reserved on every GPU that loads it, until
 * exit); shapes whose partials do not fit even unsplit return EIF_STATUS_INVALID_ARGUMENT.  The first call
 * on a device looks the array's address up, so make it before any stream capture; the address belongs to
 * the device's primary context (the CUDA runtime's), so do not use this entry from another driver context or
 * after a cudaDeviceReset.  All calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller. */
eif_status_t eif_cuda_attend_decode_noalloc_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                const float *q_dev, const int *pos_dev, int max_pos, int n_heads,
                                                float scale, const float *gate_dev, eif_cuda_subln_t subln,
                                                const float *sub_norm_dev, float *out_dev);

/* ---------------------------------------------------------------------------------------------
 * Gated DeltaNet state mirror (qwen35_delta_state_t, include/eif_qwen35.h:199-202)
 * ------------------------------------------------------------------------------------------- */

/* n_heads = lin_n_v_heads = lin_n_k_heads (deltanet_core indexes q/k by the v head,
 * src/eif_qwen35.c:601-605).  conv_k may be 0 when only the delta rule is used. */
eif_status_t eif_cuda_delta_alloc(eif_cuda_ctx_t *ctx, int n_layers, int batch, int n_heads, int d_k, int d_v,
                                  int conv_k, eif_cuda_delta_t **st);
void eif_cuda_delta_free(eif_cuda_delta_t *st);
/* Zero S and the conv windows (the DeltaNet part of qwen35_reset, src/eif_qwen35.c:1483-1497). */
eif_status_t eif_cuda_delta_reset(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st);
/* Copy one sequence's S [n_heads][d_k][d_v] and / or conv window [conv_dim][conv_k] (either may be NULL). */
eif_status_t eif_cuda_delta_upload(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int seq, const float *S,
                                   const float *conv_state);
eif_status_t eif_cuda_delta_download(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int seq, float *S,
                                     float *conv_state);
/* Device base pointers of one layer: S [batch][n_heads][d_k][d_v], conv [batch][conv_dim][conv_k]. */
eif_status_t eif_cuda_delta_layer_ptrs(const eif_cuda_delta_t *st, int layer, float **S_dev, float **conv_dev);

/*
 * Delta rule of one token for every sequence and head (src/eif_qwen35.c:594-639), in the reference's
 * order: S <- exp(g) S; e = S^T k; S <- S + beta k (v - e)^T; o = S^T (q_scale q).
 *   q, k [batch][n_heads*d_k] (L2-normalised by the caller as at src/eif_qwen35.c:579-585)
 *   v, o [batch][n_heads*d_v]; beta, g [batch][n_heads]
 */
eif_status_t eif_cuda_deltanet_step(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q,
                                    const float *k, const float *v, const float *beta, const float *g,
                                    float q_scale, float *o);
eif_status_t eif_cuda_deltanet_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q_dev,
                                        const float *k_dev, const float *v_dev, const float *beta_dev,
                                        const float *g_dev, float q_scale, float *o_dev);

/*
 * The whole DeltaNet mixer of one token per sequence after the input projections: deltanet_core
 * (src/eif_qwen35.c:546-656) -- causal conv1d over the window + SiLU, q/k L2 norm, q *= 1/sqrt(d_k),
 * beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias), the delta rule, gated RMSNorm.
 * The layer's weights come first (eif_cuda_delta_set_weights); the state needs conv_k > 0.
 *   qkv [batch][2*H*d_k + H*d_v] (the qkv projection, conv input), z [batch][H*d_v],
 *   b_raw, a_raw [batch][H] (proj_b / proj_a outputs), out [batch][H*d_v] (input of out_proj)
 * Supported: d_k = d_v = 128 (Qwen3.5) or 64.
 */
eif_status_t eif_cuda_delta_set_weights(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                        const float *conv_w /*[conv_dim][conv_k]*/, const float *dt_bias /*[H]*/,
                                        const float *A_log /*[H]*/, const float *norm_w /*[d_v]*/);
eif_status_t eif_cuda_deltanet_core(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv,
                                    const float *z, const float *b_raw, const float *a_raw, float *out);
eif_status_t eif_cuda_deltanet_core_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv_dev,
                                        const float *z_dev, const float *b_dev, const float *a_dev, float *out_dev);

/* The whole DeltaNet mixer over a prefill chunk of n_tok tokens per sequence: what prefill_chunk gets from
 * calling deltanet_core once per token (src/eif_qwen35.c:1104-1106 -> :546-656), with the delta rule in
 * the chunked WY / UT form.  Conv window, S and the output are those of n_tok consecutive
 * eif_cuda_deltanet_core calls; q / k / v reach the rule as bf16 (the prefill tolerance, not the fp32 one).
 *   qkv [batch][n_tok][conv_dim], z / out [batch][n_tok][n_heads*d_v], b, a [batch][n_tok][n_heads]
 * Needs the layer's weights (eif_cuda_delta_set_weights), d_k = 128, d_v a multiple of 64 up to 256.
 * _dev: fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_deltanet_prefill_core(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv,
                                            const float *z, const float *b_raw, const float *a_raw, int n_tok,
                                            float *out);
eif_status_t eif_cuda_deltanet_prefill_core_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                const float *qkv_dev, const float *z_dev, const float *b_dev,
                                                const float *a_dev, int n_tok, float *out_dev);

/*
 * DeltaNet prefill of n_tok tokens per sequence in the chunked WY / UT form (64-token chunks, the chunk
 * products on tensor cores, fp32 state carried across chunks), starting from and updating the layer's S.
 * Algebraically the token-by-token rule the engine runs in prefill_chunk (src/eif_qwen35.c:1104-1106
 * calling :594-639 per token); q and k are L2-normalised by the caller, q is multiplied by q_scale.
 *   q, k [batch][n_tok][H][d_k], v, o [batch][n_tok][H][d_v]; beta, g [batch][n_tok][H] (decay = exp(g))
 * _dev: bf16 q / k / v / o (16-byte aligned), fp32 beta / g, asynchronous.  Host variant: fp32 arrays.
 * Supported: d_k = 128, d_v a multiple of 64 up to 256.
 */
eif_status_t eif_cuda_deltanet_prefill(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q,
                                       const float *k, const float *v, const float *beta, const float *g, int n_tok,
                                       float q_scale, float *o);
eif_status_t eif_cuda_deltanet_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const void *q_dev,
                                           const void *k_dev, const void *v_dev, const float *beta_dev,
                                           const float *g_dev, int n_tok, float q_scale, void *o_dev);

/*
 * Qwen3.5 attention prep of one token per sequence: fullatt_prep (src/eif_qwen35.c:699-737) -- split the
 * interleaved [q | gate] heads, RMSNorm q and k per head with the layer's q_norm / k_norm (eps 1e-6),
 * partial RoPE on the first head_dim/4 dims (theta 1e7, rope_partial :502-535; the cos / sin table is
 * computed once on the host by the reference's formula), and write k, v into cache row pos[b].
 *   qg [batch][n_heads][2*head_dim], k, v [batch][n_kv*head_dim], pos [batch]
 *   q_out, gate_out [batch][n_heads*head_dim] (the inputs of eif_cuda_attend_decode)
 */
eif_status_t eif_cuda_kv_set_norms(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_norm,
                                   const float *k_norm);
eif_status_t eif_cuda_fullatt_prep(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg, const float *k,
                                   const float *v, const int *pos, int n_heads, float *q_out, float *gate_out);
eif_status_t eif_cuda_fullatt_prep_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg_dev,
                                       const float *k_dev, const float *v_dev, const int *pos_dev, int n_heads,
                                       float *q_out_dev, float *gate_out_dev);

/* fullatt_prep for a prefill chunk: token i of every sequence at position start_pos + i (the per-token
 * fullatt_prep calls of prefill_chunk, src/eif_qwen35.c:1122-1133), one launch.
 *   qg [batch][n_tok][n_heads*2*head_dim], k, v [batch][n_tok][n_kv_heads*head_dim];
 *   q_out, gate_out [batch][n_tok][n_heads*head_dim]
 * _dev: q_out in the input type of eif_cuda_attend_prefill_gated_dev for this cache (bf16 for a bf16 cache, fp32
 * for an fp32 cache), the rest fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_fullatt_prep_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                           const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                           float *q_out, float *gate_out);
eif_status_t eif_cuda_fullatt_prep_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                               const float *qg_dev, const float *k_dev, const float *v_dev, int n_tok,
                                               int start_pos, int n_heads, void *q_out_dev, float *gate_out_dev);

/* The whole Qwen3.5 attention mixer of one token per sequence in one call: fullatt_prep then fullatt_attend,
 * as fullatt_fwd calls them (src/eif_qwen35.c:819-820 -> :699-737, :741-790) -- eif_cuda_fullatt_prep followed
 * by eif_cuda_attend_decode with the gate and SubLN, with q and the gate kept on the device between the two.
 *   qg [batch][n_heads][2*head_dim], k, v [batch][n_kv*head_dim] (the projections), pos [batch] (the new row;
 *   the attention spans rows [0, pos[b]]), sub_norm [n_heads*head_dim] for EIF_CUDA_SUBLN_WEIGHT,
 *   out [batch][n_heads*head_dim] (the input of o_proj).  Needs eif_cuda_kv_set_norms.
 * _dev: device arrays, asynchronous; max_pos bounds every pos_dev[b] as in eif_cuda_attend_decode_dev. */
eif_status_t eif_cuda_fullatt_decode(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg, const float *k,
                                     const float *v, const int *pos, int n_heads, float scale, eif_cuda_subln_t subln,
                                     const float *sub_norm, float *out);
eif_status_t eif_cuda_fullatt_decode_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg_dev,
                                         const float *k_dev, const float *v_dev, const int *pos_dev, int max_pos,
                                         int n_heads, float scale, eif_cuda_subln_t subln, const float *sub_norm_dev,
                                         float *out_dev);

/* The whole Qwen3.5 attention block of a prefill chunk in one call: fullatt_prep of every token, then the gated
 * causal attention -- prefill_chunk's attention layer (src/eif_qwen35.c:1118-1133) -- i.e.
 * eif_cuda_fullatt_prep_prefill followed by eif_cuda_attend_prefill_gated with q and the gate kept on the device.
 *   qg [batch][n_tok][n_heads*2*head_dim], k, v [batch][n_tok][n_kv*head_dim], out [batch][n_tok][n_heads*head_dim]
 * A bf16 cache runs the tensor-core prefill (bf16 q, the prefill tolerance); an fp32 cache the exact per-token
 * path.  _dev: fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_fullatt_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                      const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                      float scale, eif_cuda_subln_t subln, const float *sub_norm, float *out);
eif_status_t eif_cuda_fullatt_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg_dev,
                                          const float *k_dev, const float *v_dev, int n_tok, int start_pos,
                                          int n_heads, float scale, eif_cuda_subln_t subln, const float *sub_norm_dev,
                                          float *out_dev);

/* The whole tinyllm attention block of a prefill chunk in one call: RoPE of the chunk's q and k and the (plain or
 * quantised) cache writes, then causal attention -- tinyllm_forward_batch_embeddings for one layer
 * (src/eif_tinyllm.c:1086-1268) -- i.e. eif_cuda_rope_append_prefill then eif_cuda_attend_prefill with the
 * rotated queries kept on the device.  Needs eif_cuda_kv_set_rope.
 *   q [batch][n_tok][n_heads*head_dim], k, v [batch][n_tok][n_kv*head_dim] (un-rotated), out like q
 * _dev: fp32 device arrays, asynchronous.  Host variant: fp32 host arrays. */
eif_status_t eif_cuda_prefill_step(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, const float *k,
                                   const float *v, int n_tok, int start_pos, int n_heads, float scale, float *out);
eif_status_t eif_cuda_prefill_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                       const float *k_dev, const float *v_dev, int n_tok, int start_pos, int n_heads,
                                       float scale, float *out_dev);

/* ---------------------------------------------------------------------------------------------
 * Projections  (replace linear_gemv, src/eif_qwen35.c:422-443, its batched twin linear_gemm :1033-1063, and the
 * INT8 LM head int8_gemv :384-420; the mixers' q/k/v/z/a/b/o and FFN projections and the logits)
 * ------------------------------------------------------------------------------------------- */

/* Weight formats: the engine's quant types (include/eif_qwen35.h:83-86) and the INT8 LM head.  The engine's
 * packed quant type is passed unchanged: base = quant_type & 0xff, and for EIF_CUDA_W_TERNARY2 the scale group
 * in the upper bits, group = quant_type >> 8 (0: one scale a row; src/eif_qwen35.c:100-101). */
typedef enum {
    EIF_CUDA_W_F32 = 0,           /* fp32 rows, no scale (f32_gemv, :355-382) */
    EIF_CUDA_W_INT4 = 1,          /* two a byte, even column in the high nibble, value - 8; a scale a row (:293-352) */
    EIF_CUDA_W_TERNARY2 = 2,      /* four a byte, column c at bits 2(c mod 4), code 1 = +1, 2 = -1, else 0; a scale a
                                     row, or a scale per `group` columns (src/eif_quantize_bitnet.c:834-889, 1356-1420) */
    EIF_CUDA_W_TERNARY_DENSE = 3, /* five base-3 digits a byte, least significant first, 1 = +1, 2 = -1; a scale a row
                                     (bitnet_gemv_dense, src/eif_qwen35.c:148-180) */
    EIF_CUDA_W_INT8 = 4           /* int8, a scale a row: the LM head (int8_gemv) */
} eif_cuda_wtype_t;

typedef struct eif_cuda_linear eif_cuda_linear_t; /* one weight matrix resident on the context's device */

/* Upload a [rows][cols] weight matrix in the engine's packed row layout (row_bytes, src/eif_qwen35.c:110-116:
 * fp32 4*cols, INT4 (cols+1)/2, ternary (cols+3)/4, dense (cols+4)/5, INT8 cols bytes a row) and its scales (rows
 * floats; rows * cols/group for grouped ternary; NULL for fp32).  A group must be a multiple of 16 dividing cols
 * (the engine's loader accepts multiples of 32, src/eif_qwen35.c:1265); cols up to 12288.  Synchronous. */
eif_status_t eif_cuda_linear_upload(eif_cuda_ctx_t *ctx, int quant_type, int rows, int cols, const void *W,
                                    const float *scales, eif_cuda_linear_t **out);
/* Waits for the context's queued work, then frees the matrix; call it before eif_cuda_free of its context. */
void eif_cuda_linear_free(eif_cuda_linear_t *lin);

/* out[t][rows] = W x[t] for n tokens x[n][cols] (n = 1: linear_gemv; n > 1: linear_gemm), fp32 arithmetic: CUDA
 * cores below four tokens, tensor cores from four on for INT8 / INT4 / ungrouped 2-bit weights (exact integer
 * weights, x split into two f16 parts, fp32 accumulation).  The kernels are launched as programmatic dependents
 * of the previous kernel on the stream: they fetch weights early and wait for that kernel before reading x.
 * _dev: device arrays, asynchronous.  Host variant: host arrays, returns when out is written. */
eif_status_t eif_cuda_linear_forward(eif_cuda_ctx_t *ctx, const eif_cuda_linear_t *lin, const float *x, int n,
                                     float *out);
eif_status_t eif_cuda_linear_forward_dev(eif_cuda_ctx_t *ctx, const eif_cuda_linear_t *lin, const float *x_dev, int n,
                                         float *out_dev);

#ifdef __cplusplus
}
#endif

#endif /* EIF_CUDA_H */
