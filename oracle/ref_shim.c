/*
 * ref_shim.c -- exposes the reference's own static hot-path functions for testing.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is compiled by oracle/Makefile together with the reference
 * sources where they lie (the reference tree is NOT copied into this repository) into
 * oracle/_ref/libbitllm_ref.so.  It reaches deltanet_core / fullatt_prep / fullatt_attend the way
 * the reference's own tests/test_q35_int4.c:41 reaches static functions: by including the .c file.
 *
 * Each ref_* wrapper builds the reference's config / weight / state structs around caller buffers
 * and calls the reference function unchanged.
 */
#include "eif_qwen35.c"

#define REF_EXPORT __attribute__((visibility("default")))

/* deltanet_core (src/eif_qwen35.c:546-656) for one token of one sequence, n_k_heads == n_v_heads == H. */
REF_EXPORT void ref_deltanet_core(float *qkv_raw, float *z, float *b_raw, float *a_raw, float *conv_state,
                                  float *S, const float *conv_w, const float *dt_bias, const float *A_log,
                                  const float *norm_w, float *out, int H, int dk, int dv, int conv_k)
{
    qwen35_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.lin_n_k_heads = H;
    cfg.lin_k_head_dim = dk;
    cfg.lin_n_v_heads = H;
    cfg.lin_v_head_dim = dv;
    cfg.conv_k_size = conv_k;
    qwen35_delta_weights_t w;
    memset(&w, 0, sizeof w);
    w.conv = conv_w;
    w.dt_bias = dt_bias;
    w.A_log = A_log;
    for (int h = 0; h < H && h < 64; h++) w.a_exp[h] = expf(A_log[h]); /* as the loader does, :1362 */
    w.norm_w = norm_w;
    qwen35_delta_state_t st;
    st.S = S;
    st.conv_state = conv_state;
    float *e = (float *)malloc(sizeof(float) * (size_t)H * dv);
    deltanet_core(qkv_raw, z, b_raw, a_raw, out, e, &w, &st, &cfg);
    free(e);
}

/* fullatt_prep (src/eif_qwen35.c:699-737). */
REF_EXPORT void ref_fullatt_prep(const float *qg, float *k, const float *v, float *q_out, float *gate_out,
                                 const float *q_norm, const float *k_norm, float *k_cache, float *v_cache, int pos,
                                 int nh, int nkv, int hd)
{
    qwen35_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.n_heads = nh;
    cfg.n_kv_heads = nkv;
    cfg.head_dim = hd;
    qwen35_attn_weights_t w;
    memset(&w, 0, sizeof w);
    w.q_norm = q_norm;
    w.k_norm = k_norm;
    qwen35_attn_state_t st;
    st.k_cache = k_cache;
    st.v_cache = v_cache;
    fullatt_prep(qg, k, v, q_out, gate_out, &w, &st, pos, &cfg);
}

/*
 * fullatt_attend (src/eif_qwen35.c:741-790): GQA over cache[0..pos], sigmoid gate, SubLN.
 * sub_norm may be NULL; plain_linear selects the copy branch when sub_norm is NULL.
 */
REF_EXPORT void ref_fullatt_attend(const float *q, const float *gate, float *o_in, float *k_cache, float *v_cache,
                                   const float *sub_norm, int plain_linear, int pos, int nh, int nkv, int hd)
{
    qwen35_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.n_heads = nh;
    cfg.n_kv_heads = nkv;
    cfg.head_dim = hd;
    cfg.plain_linear = plain_linear;
    qwen35_attn_state_t st;
    st.k_cache = k_cache;
    st.v_cache = v_cache;
    float *attn_out = (float *)malloc(sizeof(float) * (size_t)nh * hd);
    float *att = (float *)malloc(sizeof(float) * (size_t)nh * (pos + 1));
    fullatt_attend(q, gate, o_in, attn_out, att, &st, sub_norm, pos, &cfg);
    free(attn_out);
    free(att);
}

/*
 * tinyllm decode attention, reached through the reference's own public forward
 * (tinyllm_forward_embedding_ex, src/eif_tinyllm.c:371-857) on a one-layer fp32 model built so that the
 * attention is observable:
 *   - wq / wk / wv are zero and the Qwen QKV biases (:467-479) carry the caller's q / k / v of the step, so
 *     q = bq, k = bk, v = bv exactly before the reference's RoPE (:481-507);
 *   - kv_type 1 quantises k / v into the INT8 cache with per-(row, kv head) scales (:509-553);
 *   - wo is the identity, so s->xb2 (:676, untouched by the FFN) is the attention output exactly;
 *   - w1 / w3 / w2 are zero (the FFN adds 0).
 * Per step t the outputs are the rotated q (s->q), the rotated k and v rows (cache row t; for kv_type 1 the
 * fp32 row of t >= 1, which the INT8 rows alias only from the next steps on), the INT8 rows and scales, and
 * the attention output.  All buffers are [n_steps][...]; the INT8 ones are left alone for kv_type 0.
 * Returns 0, or -1 when the reference rejects the configuration.
 */
#include "eif_tinyllm.h"

REF_EXPORT int ref_tinyllm_decode_steps(int n_heads, int n_kv, int hd, int seq_len, float theta, int interleaved,
                                        int kv_type, int n_steps, const float *q_in, const float *k_in,
                                        const float *v_in, float *q_rot, float *k_row, float *v_row,
                                        int8_t *k_i8, int8_t *v_i8, float *k_scale, float *v_scale, float *attn)
{
    const int dim = n_heads * hd, kv_dim = n_kv * hd, hidden = 8;
    tinyllm_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.dim = dim;
    cfg.hidden_dim = hidden;
    cfg.n_layers = 1;
    cfg.n_heads = n_heads;
    cfg.n_kv_heads = n_kv;
    cfg.vocab_size = 8;
    cfg.seq_len = seq_len;
    cfg.qtype = TINYLLM_QTYPE_FP32;
    cfg.rope_interleaved = interleaved;
    cfg.rope_theta = theta;
    cfg.kv_type = kv_type;
    const size_t pool_bytes = tinyllm_memory_size(&cfg);
    void *pool = calloc(1, pool_bytes);
    tinyllm_t *llm = (tinyllm_t *)calloc(1, sizeof(tinyllm_t));
    if (!pool || !llm || tinyllm_init(llm, &cfg, pool, pool_bytes) != 0) {
        free(pool);
        free(llm);
        return -1;
    }
    float *ones = (float *)malloc(sizeof(float) * dim);
    for (int i = 0; i < dim; i++) ones[i] = 1.0f;
    float *wq = (float *)calloc((size_t)dim * dim, sizeof(float));
    float *wkv = (float *)calloc((size_t)dim * kv_dim, sizeof(float));
    float *wo = (float *)calloc((size_t)dim * dim, sizeof(float));
    for (int i = 0; i < dim; i++) wo[(size_t)i * dim + i] = 1.0f;
    float *wffn = (float *)calloc((size_t)dim * hidden, sizeof(float));
    float *bq = (float *)malloc(sizeof(float) * dim);
    float *bk = (float *)malloc(sizeof(float) * kv_dim);
    float *bv = (float *)malloc(sizeof(float) * kv_dim);
    float *x0 = (float *)calloc(dim, sizeof(float));
    tinyllm_weights_t *w = &llm->weights;
    w->rms_att_weight = ones;
    w->rms_ffn_weight = ones;
    w->rms_final_weight = ones;
    w->wq = wq;
    w->wk = wkv;
    w->wv = wkv;
    w->wo = wo;
    w->w1 = wffn;
    w->w3 = wffn;
    w->w2 = wffn;
    w->bq = bq;
    w->bk = bk;
    w->bv = bv;
    int rc = 0;
    for (int t = 0; t < n_steps && rc == 0; t++) {
        memcpy(bq, q_in + (size_t)t * dim, sizeof(float) * dim);
        memcpy(bk, k_in + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        memcpy(bv, v_in + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        if (!tinyllm_forward_embedding_ex(llm, x0, t, false)) {
            rc = -1;
            break;
        }
        tinyllm_state_t *s = &llm->state;
        memcpy(q_rot + (size_t)t * dim, s->q, sizeof(float) * dim);
        memcpy(k_row + (size_t)t * kv_dim, s->key_cache + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        memcpy(v_row + (size_t)t * kv_dim, s->value_cache + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        if (kv_type == 1) {
            memcpy(k_i8 + (size_t)t * kv_dim, s->key_cache_i8 + (size_t)t * kv_dim, kv_dim);
            memcpy(v_i8 + (size_t)t * kv_dim, s->value_cache_i8 + (size_t)t * kv_dim, kv_dim);
            memcpy(k_scale + (size_t)t * n_kv, s->key_scale + (size_t)t * n_kv, sizeof(float) * n_kv);
            memcpy(v_scale + (size_t)t * n_kv, s->value_scale + (size_t)t * n_kv, sizeof(float) * n_kv);
        }
        memcpy(attn + (size_t)t * dim, s->xb2, sizeof(float) * dim);
    }
    tinyllm_free(llm);
    free(llm);
    free(pool);
    free(ones);
    free(wq);
    free(wkv);
    free(wo);
    free(wffn);
    free(bq);
    free(bk);
    free(bv);
    free(x0);
    return rc;
}

/* Number of OpenMP threads the reference code will use (for reporting the CPU baseline). */
REF_EXPORT int ref_omp_threads(void)
{
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Set the OpenMP thread count the reference code uses in this process. */
REF_EXPORT void ref_set_threads(int n)
{
#if defined(_OPENMP)
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
