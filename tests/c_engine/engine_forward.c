/*
 * engine_forward.c -- the bitllm.c engines, patched at their token-mixer call sites (bitllm.c_b200/engine/),
 * run one synthetic model twice: once on the host as the reference runs it, once attached to the GPU
 * (eif_*_cuda_attach), and compare the logits.  Built by bitllm.c_b200/engine/Makefile; run by
 * tests/test_engine_integration.py.
 *
 *   engine_forward qwen35 <f32|bf16> <tokenwise|chunked>     24-layer Qwen3.5 model from a synthetic GGUF
 *   engine_forward tinyllm <f32|bf16|int8>                   fp32 tinyllm model (Qwen2 shape, NeoX RoPE)
 *
 * Prints one line per phase -- the worst rel-L2 of the GPU logits against the host logits -- and exits 0 when
 * every phase is within the tolerance given on the command line (argv[4] for qwen35, argv[3] for tinyllm).
 * With ENGINE_FORWARD_HOST_ONLY set the second model is not attached either (no GPU needed): the patched engines,
 * unattached, must then give the host logits exactly.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "eif_engine_cuda.h"

static uint32_t g_seed = 12345u;
static float frand(float scale) {
    g_seed = g_seed * 1664525u + 1013904223u;
    return scale * ((float)(g_seed >> 8) / 8388608.0f - 1.0f);
}

static double rel_l2(const float *a, const float *b, int n) {
    double num = 0, den = 0;
    for (int i = 0; i < n; i++) {
        const double d = (double)a[i] - b[i];
        num += d * d;
        den += (double)b[i] * b[i];
    }
    return sqrt(num / (den > 1e-30 ? den : 1e-30));
}

/* ---------------------------------------------------------------------------------------------------------------
 * A Qwen3.5 GGUF (the public GGUF v3 container, the tensor names the engine's loader looks up, fp32 tensors)
 * ------------------------------------------------------------------------------------------------------------- */

enum { QL = 24, QDIM = 128, QHID = 256, QNH = 4, QNKV = 2, QHD = 256, QNV = 4, QKD = 128, QVD = 128, QCK = 4,
       QVOC = 64, QCTX = 320 };

typedef struct {
    char name[64];
    uint64_t rows, cols;
    float *data;
} gt_t;

static gt_t g_t[400];
static int g_nt;

static float *tensor(uint64_t rows, uint64_t cols, float scale, float bias, const char *fmt, int l) {
    gt_t *t = &g_t[g_nt++];
    snprintf(t->name, sizeof t->name, fmt, l);
    t->rows = rows;
    t->cols = cols;
    t->data = (float *)malloc(rows * cols * sizeof(float));
    for (uint64_t i = 0; i < rows * cols; i++) t->data[i] = bias + frand(scale);
    return t->data;
}

static void put_u32(FILE *f, uint32_t v) { fwrite(&v, 4, 1, f); }
static void put_u64(FILE *f, uint64_t v) { fwrite(&v, 8, 1, f); }
static void put_str(FILE *f, const char *s) {
    put_u64(f, strlen(s));
    fwrite(s, 1, strlen(s), f);
}
static void put_kv_u32(FILE *f, const char *k, uint32_t v) {
    put_str(f, k);
    put_u32(f, 4); /* GGUF uint32 */
    put_u32(f, v);
}

static int write_qwen35_gguf(const char *path) {
    g_nt = 0;
    tensor(QVOC, QDIM, 0.6f, 0.f, "token_embd.weight", 0);
    tensor(1, QDIM, 0.1f, 1.f, "output_norm.weight", 0);
    for (int l = 0; l < QL; l++) {
        const int full = (l + 1) % 4 == 0; /* Qwen3.5 layout: full attention every 4th layer */
        tensor(1, QDIM, 0.1f, 1.f, "blk.%d.attn_norm.weight", l);
        tensor(1, QDIM, 0.1f, 1.f, "blk.%d.post_attention_norm.weight", l);
        tensor(QHID, QDIM, 0.15f, 0.f, "blk.%d.ffn_up.weight", l);
        tensor(QHID, QDIM, 0.15f, 0.f, "blk.%d.ffn_gate.weight", l);
        tensor(QDIM, QHID, 0.1f, 0.f, "blk.%d.ffn_down.weight", l);
        if (!full) {
            const int conv = 2 * QNV * QKD + QNV * QVD;
            tensor(conv, QDIM, 0.3f, 0.f, "blk.%d.attn_qkv.weight", l);
            tensor(QNV * QVD, QDIM, 0.3f, 0.f, "blk.%d.attn_gate.weight", l);
            tensor(QDIM, QNV * QVD, 0.1f, 0.f, "blk.%d.ssm_out.weight", l);
            tensor(QNV, QDIM, 0.3f, 0.f, "blk.%d.ssm_beta.weight", l);
            tensor(QNV, QDIM, 0.3f, 0.f, "blk.%d.ssm_alpha.weight", l);
            tensor(conv, QCK, 0.5f, 0.f, "blk.%d.ssm_conv1d.weight", l);
            tensor(1, QNV, 0.5f, 0.f, "blk.%d.ssm_dt.bias", l);
            tensor(1, QNV, 0.5f, -1.5f, "blk.%d.ssm_a", l); /* negative: A_log = log(-ssm_a) */
            tensor(1, QVD, 0.1f, 1.f, "blk.%d.ssm_norm.weight", l);
        } else {
            tensor(QNH * QHD * 2, QDIM, 0.3f, 0.f, "blk.%d.attn_q.weight", l);
            tensor(QNKV * QHD, QDIM, 0.3f, 0.f, "blk.%d.attn_k.weight", l);
            tensor(QNKV * QHD, QDIM, 0.3f, 0.f, "blk.%d.attn_v.weight", l);
            tensor(QDIM, QNH * QHD, 0.1f, 0.f, "blk.%d.attn_output.weight", l);
            tensor(1, QHD, 0.1f, 1.f, "blk.%d.attn_q_norm.weight", l);
            tensor(1, QHD, 0.1f, 1.f, "blk.%d.attn_k_norm.weight", l);
        }
    }
    FILE *f = fopen(path, "wb");
    if (!f) return -1;
    put_u32(f, 0x46554747u); /* "GGUF" */
    put_u32(f, 3);
    put_u64(f, (uint64_t)g_nt);
    put_u64(f, 15);
    put_str(f, "general.architecture");
    put_u32(f, 8); /* string */
    put_str(f, "qwen35");
    put_kv_u32(f, "qwen35.block_count", QL);
    put_kv_u32(f, "qwen35.embedding_length", QDIM);
    put_kv_u32(f, "qwen35.feed_forward_length", QHID);
    put_kv_u32(f, "qwen35.attention.head_count", QNH);
    put_kv_u32(f, "qwen35.attention.head_count_kv", QNKV);
    put_kv_u32(f, "qwen35.attention.key_length", QHD);
    put_kv_u32(f, "qwen35.context_length", QCTX);
    put_kv_u32(f, "qwen35.ssm.conv_kernel", QCK);
    put_kv_u32(f, "qwen35.ssm.state_size", QKD);
    put_kv_u32(f, "qwen35.ssm.group_count", QNV);
    put_kv_u32(f, "qwen35.ssm.time_step_rank", QNV);
    put_kv_u32(f, "qwen35.ssm.inner_size", QNV * QVD);
    put_kv_u32(f, "qwen35.full_attention_interval", 4);
    put_str(f, "qwen35.attention.layer_norm_rms_epsilon");
    put_u32(f, 6); /* float32 */
    const float eps = 1e-6f;
    fwrite(&eps, 4, 1, f);
    uint64_t off = 0;
    for (int i = 0; i < g_nt; i++) {
        put_str(f, g_t[i].name);
        const int two = g_t[i].rows > 1;
        put_u32(f, two ? 2 : 1);
        put_u64(f, g_t[i].cols);
        if (two) put_u64(f, g_t[i].rows);
        put_u32(f, 0); /* F32 */
        put_u64(f, off);
        off += (g_t[i].rows * g_t[i].cols * 4 + 31) & ~(uint64_t)31;
    }
    for (long p = ftell(f); p % 32; p++) fputc(0, f);
    for (int i = 0; i < g_nt; i++) {
        const size_t n = g_t[i].rows * g_t[i].cols * 4, pad = ((n + 31) & ~(size_t)31) - n;
        fwrite(g_t[i].data, 1, n, f);
        for (size_t p = 0; p < pad; p++) fputc(0, f);
        free(g_t[i].data);
    }
    fclose(f);
    return 0;
}

static int load_qwen35(qwen35_t *m, const char *path, void **state) {
    qwen35_config_t probe;
    memset(&probe, 0, sizeof probe);
    probe.dim = QDIM;
    probe.hidden_dim = QHID;
    probe.n_layers = QL;
    probe.n_heads = QNH;
    probe.n_kv_heads = QNKV;
    probe.head_dim = QHD;
    probe.vocab_size = QVOC;
    probe.max_seq_len = QCTX;
    probe.n_delta = 18;
    probe.n_full = 6;
    probe.lin_n_k_heads = QNV;
    probe.lin_k_head_dim = QKD;
    probe.lin_n_v_heads = QNV;
    probe.lin_v_head_dim = QVD;
    probe.conv_k_size = QCK;
    const size_t sz = qwen35_state_size(&probe) + 4096;
    *state = malloc(sz);
    return *state ? qwen35_load(m, path, *state, sz) : -1;
}

static int run_qwen35(const char *kv, const char *mode, double tol) {
    const char *path = "engine_forward_qwen35.gguf";
    if (write_qwen35_gguf(path) != 0) return 2;
    qwen35_t host, gpu;
    void *s1 = NULL, *s2 = NULL;
    if (load_qwen35(&host, path, &s1) != 0 || load_qwen35(&gpu, path, &s2) != 0) {
        fprintf(stderr, "qwen35_load failed\n");
        remove(path);
        return 2;
    }
    remove(path);
    const eif_cuda_dtype_t dt = strcmp(kv, "bf16") == 0 ? EIF_CUDA_BF16 : EIF_CUDA_F32;
    /* mode: "tokenwise" | "chunked", with "-proj" the projections (INT4 linears, the INT8 head) on the GPU too */
    const int pm = strncmp(mode, "chunked", 7) == 0 ? EIF_ENGINE_PREFILL_CHUNKED : EIF_ENGINE_PREFILL_TOKENWISE;
    const int proj = strstr(mode, "-proj") != NULL;
    int rc = getenv("ENGINE_FORWARD_HOST_ONLY") ? 0 : eif_q35_cuda_attach(&gpu, 0, dt, pm);
    if (rc == 0 && proj && !getenv("ENGINE_FORWARD_HOST_ONLY")) rc = eif_q35_cuda_set_projections(&gpu, 1);
    if (rc != 0) {
        fprintf(stderr, "attach failed: %d %s\n", rc, eif_q35_cuda_error(&gpu));
        return 2;
    }
    int toks[300];
    for (int i = 0; i < 300; i++) toks[i] = (int)((i * 37 + 11) % QVOC);
    double worst = 0;
    int ok = 1;
    /* prefill: a 64-token chunk and a 100-token continuation (two chunks inside the engine), then decode steps */
    const int chunks[2][2] = {{0, 64}, {64, 100}};
    for (int c = 0; c < 2; c++) {
        const float *lh = qwen35_prefill(&host, toks + chunks[c][0], chunks[c][1], chunks[c][0], true);
        static float keep[QVOC];
        if (!lh) return 2;
        memcpy(keep, lh, sizeof keep);
        const float *lg = qwen35_prefill(&gpu, toks + chunks[c][0], chunks[c][1], chunks[c][0], true);
        if (!lg) {
            fprintf(stderr, "GPU prefill failed: %s\n", eif_q35_cuda_error(&gpu));
            return 3;
        }
        const double e = rel_l2(lg, keep, QVOC);
        printf("qwen35 %s %s prefill chunk %d (%d tokens at %d): logits rel-L2 %.3e\n", kv, mode, c, chunks[c][1],
               chunks[c][0], e);
        ok &= e <= tol;
    }
    for (int p = 164; p < 200; p++) {
        static float keep[QVOC];
        const float *lh = qwen35_forward(&host, toks[p], p);
        if (!lh) return 2;
        memcpy(keep, lh, sizeof keep);
        const float *lg = qwen35_forward(&gpu, toks[p], p);
        if (!lg) {
            fprintf(stderr, "GPU forward failed at %d: %s\n", p, eif_q35_cuda_error(&gpu));
            return 3;
        }
        const double e = rel_l2(lg, keep, QVOC);
        worst = e > worst ? e : worst;
    }
    printf("qwen35 %s %s decode steps 164..199: worst logits rel-L2 %.3e\n", kv, mode, worst);
    ok &= worst <= tol;
    /* reset: both start over and agree again */
    qwen35_reset(&host);
    qwen35_reset(&gpu);
    static float keep0[QVOC];
    const float *l0 = qwen35_forward(&host, toks[5], 0);
    memcpy(keep0, l0, sizeof keep0);
    const float *l1 = qwen35_forward(&gpu, toks[5], 0);
    const double e0 = l1 ? rel_l2(l1, keep0, QVOC) : 1.0;
    printf("qwen35 %s %s after qwen35_reset: logits rel-L2 %.3e\n", kv, mode, e0);
    ok &= e0 <= tol;
    qwen35_free(&gpu); /* detaches */
    qwen35_free(&host);
    free(s1);
    free(s2);
    return ok ? 0 : 1;
}

/* ---------------------------------------------------------------------------------------------------------------
 * tinyllm: an fp32 model with random weights (Qwen2.5-0.5B attention heads: 14 q / 2 kv, head_dim 64)
 * ------------------------------------------------------------------------------------------------------------- */

enum { TDIM = 896, THID = 256, TNH = 14, TNKV = 2, THD = 64, TVOC = 96, TSEQ = 320 };

typedef struct {
    tinyllm_t llm;
    void *pool;
} tl_model_t;

static float *g_tw[16];

static void tl_weights_make(int n_layers) {
    const int q = TNH * THD, kvd = TNKV * THD;
    const size_t sizes[] = {(size_t)TVOC * TDIM, (size_t)n_layers * TDIM, (size_t)n_layers * TDIM, TDIM,
                            (size_t)n_layers * q * TDIM, (size_t)n_layers * kvd * TDIM, (size_t)n_layers * kvd * TDIM,
                            (size_t)n_layers * TDIM * q, (size_t)n_layers * THID * TDIM,
                            (size_t)n_layers * TDIM * THID, (size_t)n_layers * THID * TDIM,
                            (size_t)n_layers * q, (size_t)n_layers * kvd, (size_t)n_layers * kvd};
    const float scales[] = {0.5f, 0.1f, 0.1f, 0.1f, 0.06f, 0.06f, 0.06f, 0.03f, 0.05f, 0.05f, 0.05f, 0.5f, 0.5f, 0.5f};
    const float bias[] = {0, 1, 1, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = 0; i < 14; i++) {
        g_tw[i] = (float *)malloc(sizes[i] * sizeof(float));
        for (size_t j = 0; j < sizes[i]; j++) g_tw[i][j] = bias[i] + frand(scales[i]);
    }
}

static int tl_model_make(tl_model_t *t, int n_layers, int kv_type) {
    tinyllm_config_t cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.dim = TDIM;
    cfg.hidden_dim = THID;
    cfg.n_layers = n_layers;
    cfg.n_heads = TNH;
    cfg.n_kv_heads = TNKV;
    cfg.vocab_size = TVOC;
    cfg.seq_len = TSEQ;
    cfg.qtype = TINYLLM_QTYPE_FP32;
    cfg.head_dim = THD;
    cfg.rope_theta = 1000000.0f; /* Qwen2 */
    cfg.kv_type = kv_type;
    const size_t sz = tinyllm_memory_size(&cfg);
    t->pool = calloc(1, sz);
    if (!t->pool || tinyllm_init(&t->llm, &cfg, t->pool, sz) != 0) return -1;
    tinyllm_weights_t *w = &t->llm.weights;
    w->token_embedding = g_tw[0];
    w->rms_att_weight = g_tw[1];
    w->rms_ffn_weight = g_tw[2];
    w->rms_final_weight = g_tw[3];
    w->wq = g_tw[4];
    w->wk = g_tw[5];
    w->wv = g_tw[6];
    w->wo = g_tw[7];
    w->w1 = g_tw[8];
    w->w2 = g_tw[9];
    w->w3 = g_tw[10];
    w->bq = g_tw[11];
    w->bk = g_tw[12];
    w->bv = g_tw[13];
    return 0;
}

static int run_tinyllm(const char *kv, double tol) {
    const int kv_type = strcmp(kv, "int8") == 0;
    /* one layer with an INT8 cache: the reference writes each fp32 row into the buffer its INT8 rows alias
     * (src/eif_tinyllm.c:137-138, 417-418), which with more layers overwrites rows of later layers */
    const int n_layers = kv_type ? 1 : 3;
    tl_weights_make(n_layers);
    tl_model_t host, gpu;
    if (tl_model_make(&host, n_layers, kv_type) || tl_model_make(&gpu, n_layers, kv_type)) return 2;
    const eif_cuda_dtype_t dt = strcmp(kv, "bf16") == 0 ? EIF_CUDA_BF16 : EIF_CUDA_F32;
    const int rc = getenv("ENGINE_FORWARD_HOST_ONLY") ? 0 : eif_tl_cuda_attach(&gpu.llm, 0, dt);
    if (rc != 0) {
        fprintf(stderr, "attach failed: %d %s\n", rc, eif_tl_cuda_error(&gpu.llm));
        return 2;
    }
    float *emb = (float *)malloc(sizeof(float) * 300 * TDIM);
    for (int i = 0; i < 300 * TDIM; i++) emb[i] = frand(1.0f);
    static float keep[TVOC];
    int ok = 1;
    const int chunks[2][2] = {{0, 100}, {100, 70}};
    for (int c = 0; c < 2; c++) {
        const float *lh = tinyllm_forward_batch_embeddings(&host.llm, emb + (size_t)chunks[c][0] * TDIM, chunks[c][1],
                                                           chunks[c][0], true);
        if (!lh) return 2;
        memcpy(keep, lh, sizeof keep);
        const float *lg = tinyllm_forward_batch_embeddings(&gpu.llm, emb + (size_t)chunks[c][0] * TDIM, chunks[c][1],
                                                           chunks[c][0], true);
        if (!lg) {
            fprintf(stderr, "GPU prefill failed: %s\n", eif_tl_cuda_error(&gpu.llm));
            return 3;
        }
        const double e = rel_l2(lg, keep, TVOC);
        printf("tinyllm %s prefill chunk %d (%d tokens at %d): logits rel-L2 %.3e\n", kv, c, chunks[c][1],
               chunks[c][0], e);
        ok &= e <= tol;
    }
    double worst = 0;
    for (int p = 170; p < 230; p++) {
        const float *lh = tinyllm_forward_embedding(&host.llm, emb + (size_t)p * TDIM, p);
        if (!lh) return 2;
        memcpy(keep, lh, sizeof keep);
        const float *lg = tinyllm_forward_embedding(&gpu.llm, emb + (size_t)p * TDIM, p);
        if (!lg) {
            fprintf(stderr, "GPU forward failed at %d: %s\n", p, eif_tl_cuda_error(&gpu.llm));
            return 3;
        }
        const double e = rel_l2(lg, keep, TVOC);
        worst = e > worst ? e : worst;
    }
    printf("tinyllm %s decode steps 170..229: worst logits rel-L2 %.3e\n", kv, worst);
    ok &= worst <= tol;
    tinyllm_free(&gpu.llm);
    tinyllm_free(&host.llm);
    free(gpu.pool);
    free(host.pool);
    free(emb);
    for (int i = 0; i < 14; i++) free(g_tw[i]);
    return ok ? 0 : 1;
}

int main(int argc, char **argv) {
    if (argc >= 5 && strcmp(argv[1], "qwen35") == 0) return run_qwen35(argv[2], argv[3], atof(argv[4]));
    if (argc >= 4 && strcmp(argv[1], "tinyllm") == 0) return run_tinyllm(argv[2], atof(argv[3]));
    fprintf(stderr, "usage: %s qwen35 <f32|bf16> <tokenwise|chunked> <tol> | tinyllm <f32|bf16|int8> <tol>\n",
            argv[0]);
    return 2;
}
