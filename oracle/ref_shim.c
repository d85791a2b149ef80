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
