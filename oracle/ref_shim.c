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
#include <time.h>

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

/* A one-layer fp32 tinyllm model built so that its attention is observable: zero q / k / v projections whose
 * Qwen biases carry the step's q / k / v (src/eif_tinyllm.c:467-479), an identity wo (s->xb2 is the attention
 * output), a zero FFN. */
typedef struct {
    tinyllm_t *llm;
    void *pool;
    float *ones, *wq, *wkv, *wo, *wffn, *bq, *bk, *bv, *x0;
    int dim, kv_dim;
} tl_model_t;

static void tl_model_free(tl_model_t *m)
{
    if (m->llm) {
        tinyllm_free(m->llm);
        free(m->llm);
    }
    free(m->pool);
    free(m->ones);
    free(m->wq);
    free(m->wkv);
    free(m->wo);
    free(m->wffn);
    free(m->bq);
    free(m->bk);
    free(m->bv);
    free(m->x0);
    memset(m, 0, sizeof *m);
}

static int tl_model_make(tl_model_t *m, int n_heads, int n_kv, int hd, int seq_len, float theta, int interleaved,
                         int kv_type)
{
    memset(m, 0, sizeof *m);
    const int dim = n_heads * hd, kv_dim = n_kv * hd, hidden = 8;
    m->dim = dim;
    m->kv_dim = kv_dim;
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
    m->pool = calloc(1, pool_bytes);
    tinyllm_t *llm = (tinyllm_t *)calloc(1, sizeof(tinyllm_t));
    if (!m->pool || !llm || tinyllm_init(llm, &cfg, m->pool, pool_bytes) != 0) {
        free(llm);
        tl_model_free(m);
        return -1;
    }
    m->llm = llm;
    m->ones = (float *)malloc(sizeof(float) * dim);
    for (int i = 0; i < dim; i++) m->ones[i] = 1.0f;
    m->wq = (float *)calloc((size_t)dim * dim, sizeof(float));
    m->wkv = (float *)calloc((size_t)dim * kv_dim, sizeof(float));
    m->wo = (float *)calloc((size_t)dim * dim, sizeof(float));
    for (int i = 0; i < dim; i++) m->wo[(size_t)i * dim + i] = 1.0f;
    m->wffn = (float *)calloc((size_t)dim * hidden, sizeof(float));
    m->bq = (float *)malloc(sizeof(float) * dim);
    m->bk = (float *)malloc(sizeof(float) * kv_dim);
    m->bv = (float *)malloc(sizeof(float) * kv_dim);
    m->x0 = (float *)calloc(dim, sizeof(float));
    tinyllm_weights_t *w = &llm->weights;
    w->rms_att_weight = m->ones;
    w->rms_ffn_weight = m->ones;
    w->rms_final_weight = m->ones;
    w->wq = m->wq;
    w->wk = m->wkv;
    w->wv = m->wkv;
    w->wo = m->wo;
    w->w1 = m->wffn;
    w->w3 = m->wffn;
    w->w2 = m->wffn;
    w->bq = m->bq;
    w->bk = m->bk;
    w->bv = m->bv;
    return 0;
}

REF_EXPORT int ref_tinyllm_decode_steps(int n_heads, int n_kv, int hd, int seq_len, float theta, int interleaved,
                                        int kv_type, int n_steps, const float *q_in, const float *k_in,
                                        const float *v_in, float *q_rot, float *k_row, float *v_row,
                                        int8_t *k_i8, int8_t *v_i8, float *k_scale, float *v_scale, float *attn)
{
    tl_model_t m;
    if (tl_model_make(&m, n_heads, n_kv, hd, seq_len, theta, interleaved, kv_type) != 0) return -1;
    const int dim = m.dim, kv_dim = m.kv_dim;
    int rc = 0;
    for (int t = 0; t < n_steps && rc == 0; t++) {
        memcpy(m.bq, q_in + (size_t)t * dim, sizeof(float) * dim);
        memcpy(m.bk, k_in + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        memcpy(m.bv, v_in + (size_t)t * kv_dim, sizeof(float) * kv_dim);
        if (!tinyllm_forward_embedding_ex(m.llm, m.x0, t, false)) {
            rc = -1;
            break;
        }
        tinyllm_state_t *s = &m.llm->state;
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
    tl_model_free(&m);
    return rc;
}

/* Seconds the reference's own tinyllm forward takes for n_steps decode steps at position pos (each step writes
 * row pos and attends over rows [0, pos]) of the model above, on a cache whose rows [0, pos) were filled with
 * pseudo-random contents: fp32 rows in [-1, 1), or (kv_type 1) INT8 codes in [-127, 127] with scales in
 * [0.005, 0.03).  For timing the CPU baseline; -1 on failure. */
REF_EXPORT double ref_tinyllm_decode_time(int n_heads, int n_kv, int hd, int seq_len, float theta, int kv_type,
                                          int pos, int n_steps)
{
    if (pos < 0 || pos >= seq_len || n_steps < 1) return -1.0;
    tl_model_t m;
    if (tl_model_make(&m, n_heads, n_kv, hd, seq_len, theta, 0, kv_type) != 0) return -1.0;
    tinyllm_state_t *s = &m.llm->state;
    uint32_t x = 12345u;
    for (size_t i = 0; i < (size_t)pos * m.kv_dim; i++) {
        x = x * 1664525u + 1013904223u;
        if (kv_type == 1) {
            s->key_cache_i8[i] = (int8_t)((int)((x >> 24) % 255u) - 127);
            s->value_cache_i8[i] = (int8_t)((int)(((x >> 8) & 0xffu) % 255u) - 127);
        } else {
            s->key_cache[i] = (float)(x >> 8) * (2.0f / 16777216.0f) - 1.0f;
            s->value_cache[i] = (float)((x * 747796405u) >> 8) * (2.0f / 16777216.0f) - 1.0f;
        }
    }
    if (kv_type == 1)
        for (size_t i = 0; i < (size_t)pos * n_kv; i++) {
            x = x * 1664525u + 1013904223u;
            s->key_scale[i] = 0.005f + 0.025f * (float)(x >> 8) / 16777216.0f;
            s->value_scale[i] = 0.005f + 0.025f * (float)((x * 747796405u) >> 8) / 16777216.0f;
        }
    for (int i = 0; i < m.dim; i++) m.bq[i] = (float)((i * 37) % 11) * 0.1f - 0.5f;
    for (int i = 0; i < m.kv_dim; i++) m.bk[i] = m.bv[i] = (float)((i * 13) % 7) * 0.1f - 0.3f;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    int ok = 1;
    for (int t = 0; t < n_steps && ok; t++) ok = tinyllm_forward_embedding_ex(m.llm, m.x0, pos, false);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    tl_model_free(&m);
    if (!ok) return -1.0;
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
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

/* The projections as the engine runs them: linear_gemv (src/eif_qwen35.c:422-443) for one token, linear_gemm
 * (:1033-1063) for n > 1, and the INT8 LM head int8_gemv (:384-420) token by token (quant type 4). */
REF_EXPORT void ref_linear(float *out, const void *W, const float *sc, const float *x, int n, int rows, int cols,
                           int quant_type)
{
    if (quant_type == 4) {
        for (int t = 0; t < n; t++)
            int8_gemv(out + (size_t)t * rows, (const int8_t *)W, sc, x + (size_t)t * cols, rows, cols);
    } else if (n == 1) {
        linear_gemv(out, W, sc, x, rows, cols, quant_type);
    } else {
        linear_gemm(out, W, sc, x, n, rows, cols, quant_type);
    }
}

/* Seconds for `reps` calls of ref_linear (the CPU baseline of the projection workload). */
REF_EXPORT double ref_linear_time(float *out, const void *W, const float *sc, const float *x, int n, int rows,
                                  int cols, int quant_type, int reps)
{
    struct timespec a, b;
    clock_gettime(CLOCK_MONOTONIC, &a);
    for (int i = 0; i < reps; i++) ref_linear(out, W, sc, x, n, rows, cols, quant_type);
    clock_gettime(CLOCK_MONOTONIC, &b);
    return (double)(b.tv_sec - a.tv_sec) + 1e-9 * (double)(b.tv_nsec - a.tv_nsec);
}
