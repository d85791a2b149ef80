/*
 * oracle.c -- CPU restatement ("port") of the bitllm.c token-mixing hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libeif_cuda.so, the Python host mirror)
 * links, loads or calls this file.  It is the checker the parity tests, the smoke check and the
 * CPU-baseline leg of bench.py compare the CUDA kernels against.
 *
 * Every function restates the arithmetic of one reference function, in the reference's loop
 * order and in fp32, so that results agree with the reference to fp32 rounding.  The restatement
 * is pinned against the reference itself: oracle/ref_shim.c compiles the reference's own
 * src/eif_qwen35.c into oracle/_ref/, tests/golden/gen_golden.py records its outputs on seeded
 * inputs, and tests/test_oracle.py checks this file against those fixtures.
 *
 * Reference paths are relative to the tevfik/bitllm.c project root.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_EXPORT __attribute__((visibility("default")))

static inline float orc_silu(float x) { return x / (1.0f + expf(-x)); }        /* src/eif_qwen35.c:40 */
static inline float orc_softplus(float x) { return logf(1.0f + expf(x)); }     /* src/eif_qwen35.c:41 */
static inline float orc_sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }  /* src/eif_qwen35.c:589,775 */

/* Per-head L2 normalisation, eps 1e-12 inside the square root (src/eif_qwen35.c:59-64). */
static void orc_l2norm(float *x, int n)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss + 1e-12f);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* ------------------------------------------------------------------------------------------------
 * Gated DeltaNet
 * ---------------------------------------------------------------------------------------------- */

/*
 * Delta rule for one sequence and one token, all heads (src/eif_qwen35.c:594-639).
 *   S    [H][dk][dv]  fp32, updated in place (row i = key dim, dv contiguous; src/eif_qwen35.c:602)
 *   q,k  [H][dk]      q is multiplied by q_scale first (the reference scales q by 1/sqrt(dk) at :580-584)
 *   v,o  [H][dv]
 *   beta [H], g [H]   decay = expf(g) (src/eif_qwen35.c:607)
 * Order of the reference: decay S, retrieve e = S^T k from the decayed S, rank-1 update, o = S^T q.
 */
ORC_EXPORT void orc_deltanet_rule(float *S, const float *q, const float *k, const float *v, const float *beta,
                                  const float *g, float q_scale, float *o, int H, int dk, int dv)
{
    float *e = (float *)malloc(sizeof(float) * (size_t)dv);
    float *qs = (float *)malloc(sizeof(float) * (size_t)dk);
    for (int h = 0; h < H; h++) {
        float *Sh = S + (size_t)h * dk * dv;
        const float *kh = k + (size_t)h * dk;
        const float *vh = v + (size_t)h * dv;
        float *oh = o + (size_t)h * dv;
        for (int i = 0; i < dk; i++) qs[i] = q[(size_t)h * dk + i] * q_scale;
        const float decay = expf(g[h]);
        const float bh = beta[h];
        for (int i = 0; i < dk; i++)
            for (int j = 0; j < dv; j++) Sh[(size_t)i * dv + j] *= decay;
        for (int j = 0; j < dv; j++) {
            float acc = 0.0f;
            for (int i = 0; i < dk; i++) acc += Sh[(size_t)i * dv + j] * kh[i];
            e[j] = acc;
        }
        for (int i = 0; i < dk; i++) {
            const float ki = bh * kh[i];
            for (int j = 0; j < dv; j++) Sh[(size_t)i * dv + j] += ki * (vh[j] - e[j]);
        }
        for (int j = 0; j < dv; j++) {
            float acc = 0.0f;
            for (int i = 0; i < dk; i++) acc += Sh[(size_t)i * dv + j] * qs[i];
            oh[j] = acc;
        }
    }
    free(e);
    free(qs);
}

/*
 * The whole DeltaNet mixer of one token of one sequence after the input projections
 * (deltanet_core, src/eif_qwen35.c:546-656), with n_k_heads == n_v_heads == H as the reference
 * indexes q/k by the v-head (src/eif_qwen35.c:601-605).
 *   qkv_raw [2*H*dk + H*dv]   consumed (conv + SiLU in place)
 *   z [H*dv], b_raw [H], a_raw [H]
 *   conv_state [conv_dim][conv_k], conv_w [conv_dim][conv_k]
 *   S [H][dk][dv]; dt_bias, A_log [H]; norm_w [dv]
 *   out [H*dv]  gated-RMSNorm output (input of out_proj)
 */
ORC_EXPORT void orc_deltanet_core(float *qkv_raw, const float *z, const float *b_raw, const float *a_raw,
                                  float *conv_state, float *S, const float *conv_w, const float *dt_bias,
                                  const float *A_log, const float *norm_w, float *out, int H, int dk, int dv,
                                  int conv_k)
{
    const int key_dim = H * dk, val_dim = H * dv, conv_dim = 2 * key_dim + val_dim;
    /* causal conv1d over the sliding window + SiLU (src/eif_qwen35.c:560-572) */
    for (int c = 0; c < conv_dim; c++) {
        float *row = conv_state + (size_t)c * conv_k;
        for (int i = 0; i < conv_k - 1; i++) row[i] = row[i + 1];
        row[conv_k - 1] = qkv_raw[c];
        float acc = 0.0f;
        for (int i = 0; i < conv_k; i++) acc += row[i] * conv_w[(size_t)c * conv_k + i];
        qkv_raw[c] = orc_silu(acc);
    }
    float *q = qkv_raw, *k = qkv_raw + key_dim, *v = qkv_raw + 2 * key_dim;
    /* q/k L2 norm per head; q scaled by 1/sqrt(dk) (src/eif_qwen35.c:579-585) */
    const float q_scale = 1.0f / sqrtf((float)dk);
    for (int h = 0; h < H; h++) {
        orc_l2norm(q + (size_t)h * dk, dk);
        for (int i = 0; i < dk; i++) q[(size_t)h * dk + i] *= q_scale;
    }
    for (int h = 0; h < H; h++) orc_l2norm(k + (size_t)h * dk, dk);
    /* beta = sigmoid(b); g = -exp(A_log) * softplus(a + dt_bias) (src/eif_qwen35.c:587-592, a_exp from :1362) */
    float *beta = (float *)calloc((size_t)H, sizeof(float));
    float *g = (float *)calloc((size_t)H, sizeof(float));
    for (int h = 0; h < H; h++) {
        beta[h] = 1.0f / (1.0f + expf(-b_raw[h]));
        const float A = expf(A_log[h]);
        g[h] = -A * orc_softplus(a_raw[h] + dt_bias[h]);
    }
    /* q is already scaled: the rule runs with q_scale = 1 */
    orc_deltanet_rule(S, q, k, v, beta, g, 1.0f, out, H, dk, dv);
    /* gated RMSNorm: o * rsqrt(mean(o^2) + 1e-6) * norm_w * silu(z) (src/eif_qwen35.c:642-653) */
    for (int h = 0; h < H; h++) {
        float *oh = out + (size_t)h * dv;
        const float *zh = z + (size_t)h * dv;
        float ss = 0.0f;
        for (int i = 0; i < dv; i++) ss += oh[i] * oh[i];
        const float rms = 1.0f / sqrtf(ss / dv + 1e-6f);
        for (int i = 0; i < dv; i++) oh[i] = oh[i] * rms * norm_w[i] * orc_silu(zh[i]);
    }
    free(beta);
    free(g);
}

/* ------------------------------------------------------------------------------------------------
 * GQA attention over the KV cache
 * ---------------------------------------------------------------------------------------------- */

/*
 * Decode attention of one query token over cache rows [0, pos] (fullatt_attend's GQA core,
 * src/eif_qwen35.c:741-771, and the tinyllm fp32 loop, src/eif_tinyllm.c:557-656):
 *   q        [nh*hd]                  rotated query
 *   k_cache  [>= pos+1][nkv*hd]       row t at t*kv_dim + kv_h*hd, kv_h = h / (nh/nkv)
 *   scale    score multiplier (1/sqrt(hd) in both engines)
 *   gate     [nh*hd] or NULL          output *= sigmoid(gate) (src/eif_qwen35.c:773-777)
 *   out      [nh*hd]
 * softmax: max-subtract, expf, divide by the sum (src/eif_qwen35.c:51-57).
 */
ORC_EXPORT void orc_attend_decode(const float *q, const float *k_cache, const float *v_cache, int pos, int nh,
                                  int nkv, int hd, float scale, const float *gate, float *out)
{
    const int kv_dim = nkv * hd, group = nh / nkv, n = pos + 1;
    float *att = (float *)malloc(sizeof(float) * (size_t)n);
    for (int h = 0; h < nh; h++) {
        const float *qh = q + (size_t)h * hd;
        const int kvh = h / group;
        for (int t = 0; t < n; t++) {
            const float *kt = k_cache + (size_t)t * kv_dim + (size_t)kvh * hd;
            float s = 0.0f;
            for (int i = 0; i < hd; i++) s += qh[i] * kt[i];
            att[t] = s * scale;
        }
        float mx = att[0];
        for (int t = 1; t < n; t++) if (att[t] > mx) mx = att[t];
        float sum = 0.0f;
        for (int t = 0; t < n; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
        for (int t = 0; t < n; t++) att[t] /= sum;
        float *oh = out + (size_t)h * hd;
        for (int i = 0; i < hd; i++) oh[i] = 0.0f;
        for (int t = 0; t < n; t++) {
            const float *vt = v_cache + (size_t)t * kv_dim + (size_t)kvh * hd;
            const float a = att[t];
            for (int i = 0; i < hd; i++) oh[i] += a * vt[i];
        }
    }
    free(att);
    if (gate)
        for (int i = 0; i < nh * hd; i++) out[i] *= orc_sigmoid(gate[i]);
}

/*
 * tinyllm INT8 KV cache write of one row (src/eif_tinyllm.c:509-553): per kv head, amax over the head's
 * hd values; scale = amax / 127 and inv = 127 / amax (both with amax := 1 when amax < 1e-12);
 * code = (long)(x * inv + (x >= 0 ? 0.5 : -0.5)) clamped to [-128, 127].
 *   x       [nkv*hd]   the rotated k (or v) row
 *   codes   [nkv*hd]   scales [nkv]
 * The reference is compiled with -O3 -mfma -ffast-math (CMakeLists.txt:19).  Under those flags its
 * compiler evaluates amax / 127.0f as amax * (1.0f / 127.0f) and contracts x * inv + 0.5 into one fma;
 * both are written out here so that this restatement gives the compiled reference's bits whatever flags
 * it is itself built with (pinned by tests/golden/tinyllm_int8_kv.npz).
 */
ORC_EXPORT void orc_kv_quantize(const float *x, int nkv, int hd, int8_t *codes, float *scales)
{
    for (int h = 0; h < nkv; h++) {
        const float *xh = x + (size_t)h * hd;
        float amax = 0.0f;
        for (int j = 0; j < hd; j++) {
            const float a = fabsf(xh[j]);
            if (a > amax) amax = a;
        }
        const int tiny = amax < 1e-12f;
        scales[h] = tiny ? 1.0f : amax * (1.0f / 127.0f);
        const float inv = 127.0f / (tiny ? 1.0f : amax);
        for (int j = 0; j < hd; j++) {
            long qv = (long)fmaf(xh[j], inv, xh[j] >= 0.0f ? 0.5f : -0.5f);
            if (qv > 127) qv = 127;
            else if (qv < -128) qv = -128;
            codes[(size_t)h * hd + j] = (int8_t)qv;
        }
    }
}

/*
 * tinyllm decode attention over an INT8 cache (src/eif_tinyllm.c:557-571, 615-625), rows [0, pos]:
 *   score_t = (sum_i q_i * code_k[t][i]) * k_scale[t] * scale
 *   softmax (src/eif_tinyllm.c:334-352: max-subtract, expf, times 1/sum)
 *   out_i   = sum_t (att_t * v_scale[t]) * code_v[t][i]
 *   k_codes / v_codes [>= pos+1][nkv*hd], k_scale / v_scale [>= pos+1][nkv]
 */
ORC_EXPORT void orc_attend_decode_i8(const float *q, const int8_t *k_codes, const float *k_scale,
                                     const int8_t *v_codes, const float *v_scale, int pos, int nh, int nkv, int hd,
                                     float scale, float *out)
{
    const int kv_dim = nkv * hd, group = nh / nkv, n = pos + 1;
    float *att = (float *)malloc(sizeof(float) * (size_t)n);
    for (int h = 0; h < nh; h++) {
        const float *qh = q + (size_t)h * hd;
        const int kvh = h / group;
        for (int t = 0; t < n; t++) {
            const int8_t *kt = k_codes + (size_t)t * kv_dim + (size_t)kvh * hd;
            float s = 0.0f;
            for (int i = 0; i < hd; i++) s += qh[i] * (float)kt[i];
            att[t] = (s * k_scale[(size_t)t * nkv + kvh]) * scale;
        }
        float mx = att[0];
        for (int t = 1; t < n; t++) if (att[t] > mx) mx = att[t];
        float sum = 0.0f;
        for (int t = 0; t < n; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
        const float inv_sum = 1.0f / sum;
        for (int t = 0; t < n; t++) att[t] *= inv_sum;
        float *oh = out + (size_t)h * hd;
        for (int i = 0; i < hd; i++) oh[i] = 0.0f;
        for (int t = 0; t < n; t++) {
            const int8_t *vt = v_codes + (size_t)t * kv_dim + (size_t)kvh * hd;
            const float a = att[t] * v_scale[(size_t)t * nkv + kvh];
            for (int i = 0; i < hd; i++) oh[i] += a * (float)vt[i];
        }
    }
    free(att);
}

/*
 * SubLN before o_proj (src/eif_qwen35.c:779-789): mode 2 = rsqrt(mean+1e-6) * sub_norm,
 * mode 1 = rsqrt only (!plain_linear, no sub_norm), mode 0 = copy.  In place over [n].
 */
ORC_EXPORT void orc_subln(float *x, const float *sub_norm, int mode, int n)
{
    if (mode == 0) return;
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float inv = 1.0f / sqrtf(ss / n + 1e-6f);
    for (int i = 0; i < n; i++) x[i] = x[i] * inv * (mode == 2 ? sub_norm[i] : 1.0f);
}

/*
 * Causal prefill attention (tinyllm_forward_batch_embeddings, src/eif_tinyllm.c:1158-1268):
 * token i of the chunk sits at position start_pos + i and sees cache rows t <= start_pos + i.
 *   q   [n_tok][nh*hd]     rotated queries
 *   out [n_tok][nh*hd]
 * softmax multiplies by 1/sum (src/eif_tinyllm.c:334-352).
 */
ORC_EXPORT void orc_attend_prefill(const float *q, const float *k_cache, const float *v_cache, int n_tok,
                                   int start_pos, int nh, int nkv, int hd, float scale, float *out)
{
    const int kv_dim = nkv * hd, group = nh / nkv, q_dim = nh * hd;
    float *att = (float *)malloc(sizeof(float) * (size_t)(start_pos + n_tok));
    for (int i = 0; i < n_tok; i++) {
        const int pos = start_pos + i;
        for (int h = 0; h < nh; h++) {
            const float *qh = q + (size_t)i * q_dim + (size_t)h * hd;
            const int kvh = h / group;
            for (int t = 0; t <= pos; t++) {
                const float *kt = k_cache + (size_t)t * kv_dim + (size_t)kvh * hd;
                float s = 0.0f;
                for (int d = 0; d < hd; d++) s += qh[d] * kt[d];
                att[t] = s * scale;
            }
            float mx = att[0];
            for (int t = 1; t <= pos; t++) if (att[t] > mx) mx = att[t];
            float sum = 0.0f;
            for (int t = 0; t <= pos; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
            const float inv = 1.0f / sum;
            for (int t = 0; t <= pos; t++) att[t] *= inv;
            float *oh = out + (size_t)i * q_dim + (size_t)h * hd;
            for (int d = 0; d < hd; d++) oh[d] = 0.0f;
            for (int t = 0; t <= pos; t++) {
                const float *vt = v_cache + (size_t)t * kv_dim + (size_t)kvh * hd;
                const float a = att[t];
                for (int d = 0; d < hd; d++) oh[d] += a * vt[d];
            }
        }
    }
    free(att);
}

/* ------------------------------------------------------------------------------------------------
 * RoPE and Qwen3.5 attention prep
 * ---------------------------------------------------------------------------------------------- */

/*
 * tinyllm RoPE tables for one position (src/eif_tinyllm.c:395-405):
 * freq_j = 1 / powf(theta, 2j/hd), angle = pos * freq_j, j < hd/2.
 */
ORC_EXPORT void orc_rope_table(int pos, int hd, float theta, float *cos_out, float *sin_out)
{
    for (int j = 0; j < hd / 2; j++) {
        /* the reference's expression as written; this file is compiled with the reference's own flags
         * (oracle/Makefile), so the compiler rewrites it the same way (under -ffast-math the result equals
         * powf(theta, -e) from libm, which is what the device tables use; pinned by tests/golden/tinyllm_*) */
        const float freq = 1.0f / powf(theta, (float)(2 * j) / (float)hd);
        const float val = (float)pos * freq;
        cos_out[j] = cosf(val);
        sin_out[j] = sinf(val);
    }
}

/*
 * Rotate n_heads heads of x [n_heads][hd] in place with the tables of orc_rope_table
 * (src/eif_tinyllm.c:482-507): NeoX half-split pairs (j, j+hd/2) when interleaved == 0 (Qwen2),
 * adjacent pairs (2j, 2j+1) when interleaved != 0 (llama-style GGUF).
 */
ORC_EXPORT void orc_rope_apply(float *x, int n_heads, int hd, const float *c, const float *s, int interleaved)
{
    const int half = hd / 2;
    for (int h = 0; h < n_heads; h++) {
        float *xh = x + (size_t)h * hd;
        for (int j = 0; j < half; j++) {
            const int ia = interleaved ? 2 * j : j;
            const int ib = interleaved ? 2 * j + 1 : j + half;
            const float x0 = xh[ia], x1 = xh[ib];
            /* x0 c - x1 s, x1 c + x0 s with the first product fused, as the reference's -mfma build contracts
             * them (bit-identical to its rotated rows, tests/golden/tinyllm_*.npz) */
            xh[ia] = fmaf(x0, c[j], -(x1 * s[j]));
            xh[ib] = fmaf(x1, c[j], x0 * s[j]);
        }
    }
}

/*
 * Qwen3.5 partial RoPE (src/eif_qwen35.c:502-535): the first n_rot = hd/4 dims of each head are
 * rotated as half-split pairs (i, i+n_rot/2) with theta = 1e7.
 */
ORC_EXPORT void orc_rope_partial(float *x, int pos, int n_heads, int hd)
{
    const int n_rot = (int)(hd * 0.25f), half = n_rot / 2;
    for (int i = 0; i < half; i++) {
        const float inv = 1.0f / powf(10000000.0f, 2.0f * i / (float)n_rot);
        const float theta = pos * inv, c = cosf(theta), s = sinf(theta);
        for (int h = 0; h < n_heads; h++) {
            float *xh = x + (size_t)h * hd;
            const float x0 = xh[i], x1 = xh[i + half];
            xh[i] = x0 * c - x1 * s;
            xh[i + half] = x0 * s + x1 * c;
        }
    }
}

/*
 * fullatt_prep (src/eif_qwen35.c:699-737): split interleaved [q | gate] heads, RMSNorm q and k per
 * head with q_norm / k_norm (eps 1e-6), partial RoPE on q and k, write k and v into cache row pos.
 *   qg [nh][2*hd]; k [nkv*hd] (modified in place like the reference's k_buf); v [nkv*hd]
 *   q_out, gate_out [nh*hd]; k_cache/v_cache [max_seq][nkv*hd]
 */
ORC_EXPORT void orc_fullatt_prep(const float *qg, float *k, const float *v, float *q_out, float *gate_out,
                                 const float *q_norm, const float *k_norm, float *k_cache, float *v_cache, int pos,
                                 int nh, int nkv, int hd)
{
    const int kv_dim = nkv * hd;
    for (int h = 0; h < nh; h++) {
        memcpy(q_out + (size_t)h * hd, qg + (size_t)h * 2 * hd, sizeof(float) * (size_t)hd);
        memcpy(gate_out + (size_t)h * hd, qg + (size_t)h * 2 * hd + hd, sizeof(float) * (size_t)hd);
    }
    for (int h = 0; h < nh; h++) {
        float *qh = q_out + (size_t)h * hd;
        float ss = 0.0f;
        for (int i = 0; i < hd; i++) ss += qh[i] * qh[i];
        const float inv = 1.0f / sqrtf(ss / hd + 1e-6f);
        for (int i = 0; i < hd; i++) qh[i] = qh[i] * inv * q_norm[i];
    }
    for (int h = 0; h < nkv; h++) {
        float *kh = k + (size_t)h * hd;
        float ss = 0.0f;
        for (int i = 0; i < hd; i++) ss += kh[i] * kh[i];
        const float inv = 1.0f / sqrtf(ss / hd + 1e-6f);
        for (int i = 0; i < hd; i++) kh[i] = kh[i] * inv * k_norm[i];
    }
    orc_rope_partial(q_out, pos, nh, hd);
    orc_rope_partial(k, pos, nkv, hd);
    memcpy(k_cache + (size_t)pos * kv_dim, k, sizeof(float) * (size_t)kv_dim);
    memcpy(v_cache + (size_t)pos * kv_dim, v, sizeof(float) * (size_t)kv_dim);
}

/* bf16 round-to-nearest-even of an fp32 array, widened back to fp32 (input generation for the bf16 paths). */
ORC_EXPORT void orc_round_bf16(float *x, size_t n)
{
    for (size_t i = 0; i < n; i++) {
        uint32_t u;
        memcpy(&u, &x[i], 4);
        if ((u & 0x7f800000u) != 0x7f800000u) u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
        else u &= 0xffff0000u;
        memcpy(&x[i], &u, 4);
    }
}

/* ------------------------------------------------------------------------------------------------
 * Projections
 * ---------------------------------------------------------------------------------------------- */

/* Weight i of a packed row in the engine's formats (quant type base: 0 fp32, 1 INT4, 2 2-bit ternary,
 * 3 dense ternary; 4 is the INT8 LM head):
 *   INT4   byte i/2, even column in the high nibble, value - 8              (src/eif_qwen35.c:335-343)
 *   2-bit  byte i/4, bits 2(i mod 4); code 1 = +1, 2 = -1, else 0           (src/eif_quantize_bitnet.c:52-64, 876-880)
 *   dense  byte i/5, base-3 digit i mod 5 (least significant first); 1 = +1, 2 = -1 (src/eif_qwen35.c:78-92)
 *   INT8   signed byte                                                      (src/eif_qwen35.c:384-420) */
static float orc_weight(const uint8_t *row, int i, int base)
{
    switch (base) {
    case 0: { float w; memcpy(&w, row + 4 * (size_t)i, 4); return w; }
    case 1: { const uint8_t b = row[i >> 1]; return (float)(((i & 1) ? (b & 0x0F) : (b >> 4)) - 8); }
    case 2: { const unsigned c = (row[i >> 2] >> (2 * (i & 3))) & 3u; return c == 1u ? 1.0f : (c == 2u ? -1.0f : 0.0f); }
    case 3: {
        unsigned b = row[i / 5];
        for (int p = 0; p < i % 5; p++) b /= 3u;
        const unsigned d = b % 3u;
        return d == 1u ? 1.0f : (d == 2u ? -1.0f : 0.0f);
    }
    default: return (float)(int8_t)row[i];
    }
}

static size_t orc_row_bytes(int cols, int base)  /* row_bytes, src/eif_qwen35.c:110-116 (+ INT8) */
{
    switch (base) {
    case 0: return (size_t)cols * 4;
    case 1: return (size_t)(cols + 1) / 2;
    case 2: return (size_t)(cols + 3) / 4;
    case 3: return (size_t)(cols + 4) / 5;
    default: return (size_t)cols;
    }
}

/*
 * out[t][rows] = W x[t] for n tokens: linear_gemv (src/eif_qwen35.c:422-443) per token, each kernel's scalar
 * form -- one fp32 sum a row in column order, then the row scale (fp32: none, f32_gemv :355-382); grouped
 * 2-bit ternary (quant_type >> 8 = group > 0) sums each group of columns and adds block_sum * scale
 * (eif_matmul_bitnet_block_f32, src/eif_quantize_bitnet.c:1376-1417).
 */
ORC_EXPORT void orc_linear(float *out, const uint8_t *W, const float *sc, const float *x, int n, int rows, int cols,
                           int quant_type)
{
    const int base = quant_type & 0xff, group = quant_type >> 8;
    const size_t rb = orc_row_bytes(cols, base);
    for (int t = 0; t < n; t++) {
        const float *xt = x + (size_t)t * cols;
        for (int r = 0; r < rows; r++) {
            const uint8_t *row = W + (size_t)r * rb;
            float acc = 0.0f;
            if (base == 2 && group > 0) {
                const int nb = (cols + group - 1) / group;
                for (int b = 0; b < nb; b++) {
                    float bs = 0.0f;
                    for (int c = b * group; c < cols && c < (b + 1) * group; c++) bs += orc_weight(row, c, base) * xt[c];
                    acc += bs * sc[(size_t)r * nb + b];
                }
            } else {
                for (int c = 0; c < cols; c++) acc += orc_weight(row, c, base) * xt[c];
                if (base != 0) acc *= sc[r];
            }
            out[(size_t)t * rows + r] = acc;
        }
    }
}
