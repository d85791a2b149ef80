/*
 * eif_engine_cuda.c -- device mirrors of a bitllm.c engine's token-mixer state, and the hooks its patched call
 * sites use (eif_engine_cuda.h).  C99; everything on the device goes through eif_cuda.h.
 */
#include "eif_engine_cuda.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAX_ATTACHED 16

/* ================================================================================================
 * Qwen3.5
 * ============================================================================================== */

#define MAX_MATRICES 512  /* a Qwen3.5 model has 5 / 4 mixer projections a layer, 3 FFN ones and the head */

typedef struct {
    const void *W;  /* the engine's weight pointer (inside the model image) */
    int quant_type, rows, cols;
    eif_cuda_linear_t *lin;
} q35_matrix_t;

typedef struct {
    qwen35_t *m;
    eif_cuda_ctx_t *ctx;
    eif_cuda_kv_t *kv;       /* n_full layers, batch 1 */
    eif_cuda_delta_t *dn;    /* n_delta layers, batch 1 */
    int prefill_mode;
    int projections;         /* linear_gemv / linear_gemm / int8_gemv on the device too */
    int n_mat;
    q35_matrix_t mat[MAX_MATRICES];
    int failed;
    char err[256];
} q35_dev_t;

static q35_dev_t g_q35[MAX_ATTACHED];

static q35_dev_t *q35_of_model(const qwen35_t *m) {
    for (int i = 0; i < MAX_ATTACHED; i++)
        if (g_q35[i].m && g_q35[i].m == m) return &g_q35[i];
    return NULL;
}

/* The attachment whose model holds this DeltaNet state, and the state's layer index. */
static q35_dev_t *q35_of_delta(const qwen35_delta_state_t *st, int *layer) {
    for (int i = 0; i < MAX_ATTACHED; i++) {
        qwen35_t *m = g_q35[i].m;
        if (m && st >= m->state.delta && st < m->state.delta + m->config.n_delta) {
            *layer = (int)(st - m->state.delta);
            return &g_q35[i];
        }
    }
    return NULL;
}

static q35_dev_t *q35_of_attn(const qwen35_attn_state_t *st, int *layer) {
    for (int i = 0; i < MAX_ATTACHED; i++) {
        qwen35_t *m = g_q35[i].m;
        if (m && st >= m->state.attn && st < m->state.attn + m->config.n_full) {
            *layer = (int)(st - m->state.attn);
            return &g_q35[i];
        }
    }
    return NULL;
}

/* Record the first device failure of an attachment (sticky) and say the hook ran (the engine must not run its
 * own loop on host state that is no longer current). */
static int q35_status(q35_dev_t *d, eif_status_t st, const char *what) {
    if (st != EIF_STATUS_OK && !d->failed) {
        d->failed = 1;
        snprintf(d->err, sizeof d->err, "%s: status %d (%s)", what, (int)st, eif_cuda_last_error(d->ctx));
    }
    return 1;
}

int eif_q35_cuda_set_projections(qwen35_t *m, int on) {
    q35_dev_t *d = q35_of_model(m);
    if (!d) return EIF_STATUS_INVALID_ARGUMENT;
    d->projections = on != 0;
    return EIF_STATUS_OK;
}

/* The projection hook: the attachment whose model image holds W (with projections on) runs out = W x for n
 * tokens on its device, uploading the matrix on first use; 0 when no attachment owns W. */
int eif_q35_cuda_linear(const void *W, const float *sc, int quant_type, int rows, int cols, const float *x, int n,
                        float *out) {
    q35_dev_t *d = NULL;
    for (int i = 0; i < MAX_ATTACHED && !d; i++) {
        const qwen35_t *m = g_q35[i].m;
        if (m && g_q35[i].projections && m->file_data && (const uint8_t *)W >= (const uint8_t *)m->file_data &&
            (const uint8_t *)W < (const uint8_t *)m->file_data + m->file_size)
            d = &g_q35[i];
    }
    if (!d) return 0;
    if (d->failed) return 1;
    q35_matrix_t *e = NULL;
    for (int i = 0; i < d->n_mat && !e; i++)
        if (d->mat[i].W == W && d->mat[i].quant_type == quant_type && d->mat[i].rows == rows && d->mat[i].cols == cols)
            e = &d->mat[i];
    if (!e) {
        if (d->n_mat == MAX_MATRICES) return q35_status(d, EIF_STATUS_OUT_OF_MEMORY, "projection table full");
        e = &d->mat[d->n_mat];
        eif_status_t st = eif_cuda_linear_upload(d->ctx, quant_type, rows, cols, W, sc, &e->lin);
        if (st != EIF_STATUS_OK) return q35_status(d, st, "linear_upload");
        e->W = W;
        e->quant_type = quant_type;
        e->rows = rows;
        e->cols = cols;
        d->n_mat++;
    }
    return q35_status(d, eif_cuda_linear_forward(d->ctx, e->lin, x, n, out), "linear_forward");
}

static eif_cuda_subln_t q35_subln(const qwen35_t *m, int fa) {
    /* fullatt_attend's epilogue (src/eif_qwen35.c:779-789) */
    if (m->weights.full[fa].sub_norm) return EIF_CUDA_SUBLN_WEIGHT;
    return m->config.plain_linear ? EIF_CUDA_SUBLN_NONE : EIF_CUDA_SUBLN_RMS;
}

void eif_q35_cuda_detach(qwen35_t *m) {
    q35_dev_t *d = q35_of_model(m);
    if (!d) return;
    for (int i = 0; i < d->n_mat; i++) eif_cuda_linear_free(d->mat[i].lin);
    if (d->kv) eif_cuda_kv_free(d->kv);
    if (d->dn) eif_cuda_delta_free(d->dn);
    if (d->ctx) eif_cuda_free(d->ctx);
    memset(d, 0, sizeof *d);
}

int eif_q35_cuda_attach(qwen35_t *m, int device, eif_cuda_dtype_t kv_dtype, int prefill_mode) {
    if (!m) return EIF_STATUS_INVALID_ARGUMENT;
    eif_q35_cuda_detach(m);
    q35_dev_t *d = NULL;
    for (int i = 0; i < MAX_ATTACHED && !d; i++)
        if (!g_q35[i].m) d = &g_q35[i];
    if (!d) return EIF_STATUS_OUT_OF_MEMORY;
    memset(d, 0, sizeof *d);
    const qwen35_config_t *c = &m->config;
    if (c->lin_n_k_heads != c->lin_n_v_heads) return EIF_STATUS_NOT_SUPPORTED;
    if (kv_dtype != EIF_CUDA_F32 && kv_dtype != EIF_CUDA_BF16) return EIF_STATUS_NOT_SUPPORTED;
    const int H = c->lin_n_v_heads, dk = c->lin_k_head_dim, dv = c->lin_v_head_dim, ck = c->conv_k_size;
    const int conv_dim = 2 * H * dk + H * dv, kv_dim = c->n_kv_heads * c->head_dim;
    eif_status_t st = eif_cuda_init(&d->ctx, device);
    if (st == EIF_STATUS_OK && c->n_full > 0)
        st = eif_cuda_kv_alloc(d->ctx, c->n_full, 1, c->max_seq_len, c->n_kv_heads, c->head_dim, kv_dtype, &d->kv);
    if (st == EIF_STATUS_OK && c->n_delta > 0) st = eif_cuda_delta_alloc(d->ctx, c->n_delta, 1, H, dk, dv, ck, &d->dn);
    for (int l = 0; st == EIF_STATUS_OK && l < c->n_delta; l++) {
        const qwen35_delta_weights_t *w = &m->weights.delta[l];
        st = eif_cuda_delta_set_weights(d->ctx, d->dn, l, w->conv, w->dt_bias, w->A_log, w->norm_w);
        if (st == EIF_STATUS_OK)
            st = eif_cuda_delta_upload(d->ctx, d->dn, l, 0, m->state.delta[l].S, m->state.delta[l].conv_state);
    }
    for (int l = 0; st == EIF_STATUS_OK && l < c->n_full; l++) {
        const qwen35_attn_weights_t *w = &m->weights.full[l];
        st = eif_cuda_kv_set_norms(d->ctx, d->kv, l, w->q_norm, w->k_norm);
        if (st == EIF_STATUS_OK)
            st = eif_cuda_kv_upload(d->ctx, d->kv, l, 0, 0, c->max_seq_len, m->state.attn[l].k_cache,
                                    m->state.attn[l].v_cache);
    }
    (void)conv_dim;
    (void)kv_dim;
    d->m = m;
    d->prefill_mode = prefill_mode;
    if (st != EIF_STATUS_OK) {
        fprintf(stderr, "[eif_engine_cuda] Qwen3.5 attach failed: %s\n", d->ctx ? eif_cuda_last_error(d->ctx) : "");
        eif_q35_cuda_detach(m);
    }
    return st;
}

int eif_q35_cuda_failed(const qwen35_t *m) {
    const q35_dev_t *d = q35_of_model(m);
    return d ? d->failed : 0;
}

const char *eif_q35_cuda_error(const qwen35_t *m) {
    const q35_dev_t *d = q35_of_model(m);
    return d ? d->err : "";
}

void eif_q35_cuda_reset(qwen35_t *m) {
    q35_dev_t *d = q35_of_model(m);
    if (!d) return;
    if (d->kv) q35_status(d, eif_cuda_kv_reset(d->ctx, d->kv), "kv_reset");
    if (d->dn) q35_status(d, eif_cuda_delta_reset(d->ctx, d->dn), "delta_reset");
}

int eif_q35_cuda_deltanet(const qwen35_delta_state_t *st, const float *qkv, const float *z, const float *b,
                          const float *a, float *out) {
    int l;
    q35_dev_t *d = q35_of_delta(st, &l);
    if (!d) return 0;
    if (d->failed) return 1;
    return q35_status(d, eif_cuda_deltanet_core(d->ctx, d->dn, l, qkv, z, b, a, out), "deltanet_core");
}

int eif_q35_cuda_fullatt(const qwen35_attn_state_t *st, const float *qg, const float *k, const float *v, int pos,
                         float *out) {
    int l;
    q35_dev_t *d = q35_of_attn(st, &l);
    if (!d) return 0;
    if (d->failed) return 1;
    const qwen35_config_t *c = &d->m->config;
    const float scale = 1.0f / sqrtf((float)c->head_dim);
    return q35_status(d, eif_cuda_fullatt_decode(d->ctx, d->kv, l, qg, k, v, &pos, c->n_heads, scale,
                                                 q35_subln(d->m, l), d->m->weights.full[l].sub_norm, out),
                      "fullatt_decode");
}

int eif_q35_cuda_deltanet_chunk(const qwen35_delta_state_t *st, const float *qkv, const float *z, const float *b,
                                const float *a, int n, float *out) {
    int l;
    q35_dev_t *d = q35_of_delta(st, &l);
    if (!d) return 0;
    if (d->failed) return 1;
    if (d->prefill_mode == EIF_ENGINE_PREFILL_CHUNKED)
        return q35_status(d, eif_cuda_deltanet_prefill_core(d->ctx, d->dn, l, qkv, z, b, a, n, out),
                          "deltanet_prefill_core");
    const qwen35_config_t *c = &d->m->config;
    const int H = c->lin_n_v_heads, conv_dim = 2 * H * c->lin_k_head_dim + H * c->lin_v_head_dim;
    const int val_dim = H * c->lin_v_head_dim;
    for (int t = 0; t < n && !d->failed; t++)
        q35_status(d, eif_cuda_deltanet_core(d->ctx, d->dn, l, qkv + (size_t)t * conv_dim, z + (size_t)t * val_dim,
                                             b + (size_t)t * H, a + (size_t)t * H, out + (size_t)t * val_dim),
                   "deltanet_core");
    return 1;
}

int eif_q35_cuda_fullatt_chunk(const qwen35_attn_state_t *st, const float *qg, const float *k, const float *v, int n,
                               int start_pos, float *out) {
    int l;
    q35_dev_t *d = q35_of_attn(st, &l);
    if (!d) return 0;
    if (d->failed) return 1;
    const qwen35_config_t *c = &d->m->config;
    const float scale = 1.0f / sqrtf((float)c->head_dim);
    return q35_status(d, eif_cuda_fullatt_prefill(d->ctx, d->kv, l, qg, k, v, n, start_pos, c->n_heads, scale,
                                                  q35_subln(d->m, l), d->m->weights.full[l].sub_norm, out),
                      "fullatt_prefill");
}

/* ================================================================================================
 * tinyllm
 * ============================================================================================== */

typedef struct {
    tinyllm_t *llm;
    eif_cuda_ctx_t *ctx;
    eif_cuda_kv_t *kv;
    int failed;
    char err[256];
    float *qbuf, *kbuf, *vbuf, *obuf;  /* host staging of a prefill chunk (contiguous rows) */
    size_t cap;
} tl_dev_t;

static tl_dev_t g_tl[MAX_ATTACHED];

static tl_dev_t *tl_of(const tinyllm_t *llm) {
    for (int i = 0; i < MAX_ATTACHED; i++)
        if (g_tl[i].llm && g_tl[i].llm == llm) return &g_tl[i];
    return NULL;
}

static int tl_status(tl_dev_t *d, eif_status_t st, const char *what) {
    if (st != EIF_STATUS_OK && !d->failed) {
        d->failed = 1;
        snprintf(d->err, sizeof d->err, "%s: status %d (%s)", what, (int)st, eif_cuda_last_error(d->ctx));
    }
    return 1;
}

static int tl_head_dim(const tinyllm_config_t *p) { return p->head_dim > 0 ? p->head_dim : p->dim / p->n_heads; }

void eif_tl_cuda_detach(tinyllm_t *llm) {
    tl_dev_t *d = tl_of(llm);
    if (!d) return;
    if (d->kv) eif_cuda_kv_free(d->kv);
    if (d->ctx) eif_cuda_free(d->ctx);
    free(d->qbuf);
    memset(d, 0, sizeof *d);
}

int eif_tl_cuda_attach(tinyllm_t *llm, int device, eif_cuda_dtype_t kv_dtype) {
    if (!llm) return EIF_STATUS_INVALID_ARGUMENT;
    eif_tl_cuda_detach(llm);
    tl_dev_t *d = NULL;
    for (int i = 0; i < MAX_ATTACHED && !d; i++)
        if (!g_tl[i].llm) d = &g_tl[i];
    if (!d) return EIF_STATUS_OUT_OF_MEMORY;
    memset(d, 0, sizeof *d);
    const tinyllm_config_t *p = &llm->config;
    const int hd = tl_head_dim(p), kv_dim = p->n_kv_heads * hd;
    if (p->kv_type == 1) kv_dtype = EIF_CUDA_INT8;
    /* the engine's RoPE base (src/eif_tinyllm.c:399) */
    const float theta = p->rope_theta > 0.0f ? p->rope_theta
                        : (p->vocab_size > 120000 ? 5000000.0f : (p->vocab_size > 60000 ? 100000.0f : 10000.0f));
    eif_status_t st = eif_cuda_init(&d->ctx, device);
    if (st == EIF_STATUS_OK)
        st = eif_cuda_kv_alloc(d->ctx, p->n_layers, 1, p->seq_len, p->n_kv_heads, hd, kv_dtype, &d->kv);
    if (st == EIF_STATUS_OK) st = eif_cuda_kv_set_rope(d->ctx, d->kv, theta, p->rope_interleaved);
    if (st == EIF_STATUS_OK && kv_dtype != EIF_CUDA_INT8)
        for (int l = 0; l < p->n_layers && st == EIF_STATUS_OK; l++) {
            const size_t loff = (size_t)l * p->seq_len * kv_dim;
            st = eif_cuda_kv_upload(d->ctx, d->kv, l, 0, 0, p->seq_len, llm->state.key_cache + loff,
                                    llm->state.value_cache + loff);
        }
    d->llm = llm;
    if (st != EIF_STATUS_OK) {
        fprintf(stderr, "[eif_engine_cuda] tinyllm attach failed: %s\n", d->ctx ? eif_cuda_last_error(d->ctx) : "");
        eif_tl_cuda_detach(llm);
    }
    return st;
}

int eif_tl_cuda_active(const tinyllm_t *llm) { return tl_of(llm) != NULL; }

int eif_tl_cuda_failed(const tinyllm_t *llm) {
    const tl_dev_t *d = tl_of(llm);
    return d ? d->failed : 0;
}

const char *eif_tl_cuda_error(const tinyllm_t *llm) {
    const tl_dev_t *d = tl_of(llm);
    return d ? d->err : "";
}

void eif_tl_cuda_reset(tinyllm_t *llm) {
    tl_dev_t *d = tl_of(llm);
    if (d) tl_status(d, eif_cuda_kv_reset(d->ctx, d->kv), "kv_reset");
}

int eif_tl_cuda_attention(tinyllm_t *llm, int layer, int pos, const float *q, const float *k, const float *v,
                          float *out) {
    tl_dev_t *d = tl_of(llm);
    if (!d) return 0;
    if (d->failed) return 1;
    const tinyllm_config_t *p = &llm->config;
    const float scale = 1.0f / sqrtf((float)tl_head_dim(p));
    return tl_status(d, eif_cuda_decode_step(d->ctx, d->kv, layer, q, k, v, &pos, p->n_heads, scale, out),
                     "decode_step");
}

int eif_tl_cuda_prefill_attention(tinyllm_t *llm, int layer, int n, int start_pos, const float *q,
                                  const float *k_rows, const float *v_rows, float *out, int out_stride) {
    tl_dev_t *d = tl_of(llm);
    if (!d) return 0;
    if (d->failed) return 1;
    const tinyllm_config_t *p = &llm->config;
    const int hd = tl_head_dim(p), q_dim = p->n_heads * hd;
    const float scale = 1.0f / sqrtf((float)hd);
    const size_t need = (size_t)n * q_dim;
    if (need > d->cap) {
        free(d->qbuf);
        d->qbuf = (float *)malloc(need * sizeof(float));
        d->cap = d->qbuf ? need : 0;
        if (!d->qbuf) return tl_status(d, EIF_STATUS_OUT_OF_MEMORY, "prefill staging");
    }
    eif_status_t st = eif_cuda_prefill_step(d->ctx, d->kv, layer, q, k_rows, v_rows, n, start_pos, p->n_heads, scale,
                                            d->qbuf);
    if (st == EIF_STATUS_OK)
        for (int t = 0; t < n; t++) memcpy(out + (size_t)t * out_stride, d->qbuf + (size_t)t * q_dim, q_dim * 4);
    return tl_status(d, st, "prefill_step");
}
