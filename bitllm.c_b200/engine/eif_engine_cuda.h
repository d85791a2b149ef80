/*
 * eif_engine_cuda.h -- the bitllm.c engines' token mixers on the GPU, at the engines' own call sites.
 *
 * C99.  Compiled with the engine sources patched by bitllm_cuda.patch (every hunk adds lines under
 * #ifdef BITLLM_CUDA; nothing of the engine is removed), and linked with libeif_cuda.so.  An application loads
 * a model as before (qwen35_load, tinyllm_init / tinyllm_load_model), then attaches it to a GPU:
 *
 *     qwen35_t m;  qwen35_load(&m, path, state, state_sz);
 *     eif_q35_cuda_attach(&m, 0, EIF_CUDA_F32, 0);        // the 18 DeltaNet states and 6 KV caches move to GPU 0
 *     qwen35_forward(&m, tok, pos);                        // unchanged API: the mixers now run on the GPU
 *
 * From then on the engine's deltanet_core / fullatt_prep / fullatt_attend calls (src/eif_qwen35.c:690, 819-820),
 * its prefill_chunk loops (:1104-1106, :1118-1133), tinyllm's per-token attention block (src/eif_tinyllm.c:481-657)
 * and its batched prefill attention (:1088-1268) run on the device through eif_cuda.h; the projections stay on
 * the host unless eif_q35_cuda_set_projections turns them on, the norms and the FFN's activations always do.  The device copies of the recurrent states and KV caches are authoritative while a
 * model is attached (the host copies are no longer updated).  A device failure is sticky: the forward functions
 * return NULL (prefill_chunk -1) from then on, and eif_*_cuda_error() says why; there is no silent CPU fallback.
 *
 * Each hook returns 1 when it ran the call on the GPU and 0 when the model is not attached (the engine then runs
 * its own loop), so an unattached model behaves exactly as the unpatched engine.  One attached model per
 * engine object; several models may be attached at once.  Not thread-safe (the engines are not either).
 */
#ifndef EIF_ENGINE_CUDA_H
#define EIF_ENGINE_CUDA_H

#include "eif_cuda.h"
#include "eif_qwen35.h"
#include "eif_tinyllm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* How the Qwen3.5 prefill runs its DeltaNet layers: the chunked WY / UT form on the tensor cores (bf16 q / k / v,
 * the prefill tolerance), or deltanet_core token by token on the device (the reference's fp32 recurrence). */
enum { EIF_ENGINE_PREFILL_CHUNKED = 0, EIF_ENGINE_PREFILL_TOKENWISE = 1 };

/* ---- Qwen3.5 (src/eif_qwen35.c) ---- */

/* Create device mirrors of m's DeltaNet states (S, conv windows), KV caches (kv_dtype EIF_CUDA_F32, the reference's
 * own cache type, or EIF_CUDA_BF16) and mixer weights on `device`, copying the current host state.  Needs
 * lin_n_k_heads == lin_n_v_heads, d_k = d_v = 128 (or 64 with prefill_mode TOKENWISE), head_dim 64 / 128 / 256.
 * Returns 0, or an eif_status_t (< 0) with the reason in eif_q35_cuda_error(m). */
int eif_q35_cuda_attach(qwen35_t *m, int device, eif_cuda_dtype_t kv_dtype, int prefill_mode);
void eif_q35_cuda_detach(qwen35_t *m);
int eif_q35_cuda_failed(const qwen35_t *m);
const char *eif_q35_cuda_error(const qwen35_t *m);
/* Zero the device states (called by qwen35_reset). */
void eif_q35_cuda_reset(qwen35_t *m);

/* Also run the model's projections on the device (on != 0): linear_gemv, linear_gemm and the INT8 LM head
 * int8_gemv (src/eif_qwen35.c:384-443, 1033-1063).  Each weight matrix is recognised by its address inside the
 * model's image and uploaded in the engine's packed layout on first use (eif_cuda_linear_upload); every call then
 * copies x in and the output back.  Off by default: the attachment moves only the token mixers. */
int eif_q35_cuda_set_projections(qwen35_t *m, int on);

/* Hooks at the engine's call sites. */
int eif_q35_cuda_linear(const void *W, const float *sc, int quant_type, int rows, int cols, const float *x, int n,
                        float *out);
int eif_q35_cuda_deltanet(const qwen35_delta_state_t *st, const float *qkv, const float *z, const float *b,
                          const float *a, float *out);
int eif_q35_cuda_fullatt(const qwen35_attn_state_t *st, const float *qg, const float *k, const float *v, int pos,
                         float *out);
int eif_q35_cuda_deltanet_chunk(const qwen35_delta_state_t *st, const float *qkv, const float *z, const float *b,
                                const float *a, int n, float *out);
int eif_q35_cuda_fullatt_chunk(const qwen35_attn_state_t *st, const float *qg, const float *k, const float *v, int n,
                               int start_pos, float *out);

/* ---- tinyllm (src/eif_tinyllm.c: Qwen2 / 2.5, LLaMA-family) ---- */

/* Device KV cache of llm's layers (fp32, or INT8 when llm->config.kv_type == 1, or bf16 when kv_dtype says so),
 * with the engine's RoPE tables (theta and pair layout as tinyllm_forward computes them).  Attach before the first
 * token (an INT8 host cache cannot be copied over); an fp32 host cache's rows are copied.  0 or eif_status_t. */
int eif_tl_cuda_attach(tinyllm_t *llm, int device, eif_cuda_dtype_t kv_dtype);
void eif_tl_cuda_detach(tinyllm_t *llm);
int eif_tl_cuda_active(const tinyllm_t *llm);
int eif_tl_cuda_failed(const tinyllm_t *llm);
const char *eif_tl_cuda_error(const tinyllm_t *llm);
void eif_tl_cuda_reset(tinyllm_t *llm);

/* One decode token's attention block of layer l: q, k, v un-rotated (k, v: the projections as the engine wrote
 * them into its host cache row), out [n_heads*head_dim]. */
int eif_tl_cuda_attention(tinyllm_t *llm, int layer, int pos, const float *q, const float *k, const float *v,
                          float *out);
/* A prefill chunk's attention of layer l: q [n][q_dim] un-rotated, k_rows / v_rows the chunk's host cache rows
 * (un-rotated projections), out rows of `out_stride` floats. */
int eif_tl_cuda_prefill_attention(tinyllm_t *llm, int layer, int n, int start_pos, const float *q,
                                  const float *k_rows, const float *v_rows, float *out, int out_stride);

#ifdef __cplusplus
}
#endif

#endif /* EIF_ENGINE_CUDA_H */
