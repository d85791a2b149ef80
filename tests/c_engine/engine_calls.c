/*
 * engine_calls.c -- the calls a C99 engine makes through include/eif_cuda.h, checked against plain C loops.
 *
 * The tinyllm decode step (src/eif_tinyllm.c:395-405 RoPE tables, :480-506 rotation, :509-549 INT8 cache
 * write, :551-656 attention) over an fp32 and an INT8 cache, as two calls and as one (eif_cuda_decode_step), and the DeltaNet delta rule (src/eif_qwen35.c:594-639),
 * run token by token through the host-pointer entry points; the reference loops below restate the same
 * arithmetic in C (RoPE tables in the form the reference's -ffast-math build evaluates, powf(theta, -e)).
 * Exit status 0 when every check passes (or when no CUDA device is present), 1 otherwise.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "eif_cuda.h"

#define NH 14
#define NKV 2
#define HD 64
#define T 48
#define DH 4   /* DeltaNet heads */
#define DK 64
#define DV 64

static uint32_t rng_state = 12345u;
static float rnd(void) { /* uniform in (-1, 1) from a 32-bit LCG */
    rng_state = rng_state * 1664525u + 1013904223u;
    return (float)((int32_t)rng_state) / 2147483648.0f;
}

static double rel_l2(const float *a, const float *b, int n) {
    double num = 0, den = 0;
    for (int i = 0; i < n; i++) {
        num += ((double)a[i] - b[i]) * ((double)a[i] - b[i]);
        den += (double)b[i] * b[i];
    }
    return den > 0 ? sqrt(num / den) : sqrt(num);
}

static void rope(float *x, int n_heads, int pos, float theta) {
    for (int h = 0; h < n_heads; h++)
        for (int j = 0; j < HD / 2; j++) {
            const float freq = powf(theta, -((float)(2 * j) / (float)HD));
            const float val = (float)pos * freq, c = cosf(val), s = sinf(val);
            float *xh = x + h * HD;
            const float x0 = xh[j], x1 = xh[j + HD / 2];
            xh[j] = fmaf(x0, c, -(x1 * s));
            xh[j + HD / 2] = fmaf(x1, c, x0 * s);
        }
}

static void quantize(const float *x, int8_t *codes, float *scales) {
    for (int h = 0; h < NKV; h++) {
        float amax = 0.0f;
        for (int j = 0; j < HD; j++) amax = fabsf(x[h * HD + j]) > amax ? fabsf(x[h * HD + j]) : amax;
        const int tiny = amax < 1e-12f;
        scales[h] = tiny ? 1.0f : amax * (1.0f / 127.0f);
        const float inv = 127.0f / (tiny ? 1.0f : amax);
        for (int j = 0; j < HD; j++) {
            const float v = x[h * HD + j];
            long qv = (long)fmaf(v, inv, v >= 0.0f ? 0.5f : -0.5f);
            codes[h * HD + j] = (int8_t)(qv > 127 ? 127 : qv < -128 ? -128 : qv);
        }
    }
}

/* tinyllm attention of one token over rows [0, pos]; row t of K / V dequantised as code * scale when ks. */
static void attend(const float *q, const float *kc, const float *vc, const int8_t *k8, const int8_t *v8,
                   const float *ks, const float *vs, int pos, float *out) {
    float att[T];
    for (int h = 0; h < NH; h++) {
        const int kvh = h / (NH / NKV);
        for (int t = 0; t <= pos; t++) {
            float s = 0.0f;
            for (int i = 0; i < HD; i++) {
                const int o = t * NKV * HD + kvh * HD + i;
                s += q[h * HD + i] * (k8 ? (float)k8[o] : kc[o]);
            }
            att[t] = (k8 ? s * ks[t * NKV + kvh] : s) * (1.0f / sqrtf((float)HD));
        }
        float mx = att[0], sum = 0.0f;
        for (int t = 1; t <= pos; t++) mx = att[t] > mx ? att[t] : mx;
        for (int t = 0; t <= pos; t++) { att[t] = expf(att[t] - mx); sum += att[t]; }
        for (int i = 0; i < HD; i++) out[h * HD + i] = 0.0f;
        for (int t = 0; t <= pos; t++) {
            const float a = att[t] / sum * (v8 ? vs[t * NKV + kvh] : 1.0f);
            for (int i = 0; i < HD; i++) {
                const int o = t * NKV * HD + kvh * HD + i;
                out[h * HD + i] += a * (v8 ? (float)v8[o] : vc[o]);
            }
        }
    }
}

static int fail_status(eif_cuda_ctx_t *ctx, const char *what, eif_status_t st) {
    fprintf(stderr, "%s: status %d (%s)\n", what, (int)st, eif_cuda_last_error(ctx));
    return 1;
}

/* one_call: the step as eif_cuda_decode_step (RoPE, row write, attention in one call) instead of
 * eif_cuda_rope_append + eif_cuda_attend_decode */
static int tinyllm_decode(eif_cuda_ctx_t *ctx, eif_cuda_dtype_t dtype, int one_call) {
    eif_cuda_kv_t *kv = NULL;
    eif_status_t st = eif_cuda_kv_alloc(ctx, 1, 1, T, NKV, HD, dtype, &kv);
    if (st != EIF_STATUS_OK) return fail_status(ctx, "kv_alloc", st);
    const float theta = 1e6f;
    if ((st = eif_cuda_kv_set_rope(ctx, kv, theta, 0)) != EIF_STATUS_OK) return fail_status(ctx, "kv_set_rope", st);
    static float kc[T * NKV * HD], vc[T * NKV * HD], ks[T * NKV], vs[T * NKV];
    static int8_t k8[T * NKV * HD], v8[T * NKV * HD];
    float q[NH * HD], k[NKV * HD], v[NKV * HD], qr[NH * HD], out[NH * HD], ref[NH * HD];
    double worst = 0.0;
    int code_mismatch = 0;
    for (int pos = 0; pos < T - 4; pos++) {
        for (int i = 0; i < NH * HD; i++) q[i] = 2.0f * rnd();
        for (int i = 0; i < NKV * HD; i++) { k[i] = 2.0f * rnd(); v[i] = 2.0f * rnd(); }
        /* the engine: RoPE + cache write of the new row, then the head loop */
        if (one_call) {
            if ((st = eif_cuda_decode_step(ctx, kv, 0, q, k, v, &pos, NH, 1.0f / sqrtf((float)HD), out)) != EIF_STATUS_OK)
                return fail_status(ctx, "decode_step", st);
        } else {
            if ((st = eif_cuda_rope_append(ctx, kv, 0, q, k, v, &pos, NH, qr)) != EIF_STATUS_OK)
                return fail_status(ctx, "rope_append", st);
            if ((st = eif_cuda_attend_decode(ctx, kv, 0, qr, &pos, NH, 1.0f / sqrtf((float)HD), NULL,
                                             EIF_CUDA_SUBLN_NONE, NULL, out)) != EIF_STATUS_OK)
                return fail_status(ctx, "attend_decode", st);
        }
        /* the reference loops */
        float qh[NH * HD], kh[NKV * HD];
        memcpy(qh, q, sizeof qh);
        memcpy(kh, k, sizeof kh);
        rope(qh, NH, pos, theta);
        rope(kh, NKV, pos, theta);
        if (one_call) memcpy(qr, qh, sizeof qh); /* q stays on the device: compare the reference with itself */
        memcpy(kc + pos * NKV * HD, kh, sizeof kh);
        memcpy(vc + pos * NKV * HD, v, sizeof v);
        if (dtype == EIF_CUDA_INT8) {
            quantize(kh, k8 + pos * NKV * HD, ks + pos * NKV);
            quantize(v, v8 + pos * NKV * HD, vs + pos * NKV);
            int8_t dk[NKV * HD], dv[NKV * HD];
            float dks[NKV], dvs[NKV];
            if ((st = eif_cuda_kv_download_int8(ctx, kv, 0, 0, pos, 1, dk, dv, dks, dvs)) != EIF_STATUS_OK)
                return fail_status(ctx, "kv_download_int8", st);
            code_mismatch += memcmp(dk, k8 + pos * NKV * HD, sizeof dk) != 0 || memcmp(dv, v8 + pos * NKV * HD, sizeof dv) != 0 ||
                             memcmp(dks, ks + pos * NKV, sizeof dks) != 0 || memcmp(dvs, vs + pos * NKV, sizeof dvs) != 0;
            attend(qh, NULL, NULL, k8, v8, ks, vs, pos, ref);
        } else {
            attend(qh, kc, vc, NULL, NULL, NULL, NULL, pos, ref);
        }
        const double e = rel_l2(out, ref, NH * HD);
        worst = e > worst ? e : worst;
        const double eq = rel_l2(qr, qh, NH * HD);
        worst = eq > worst ? eq : worst;
    }
    eif_cuda_kv_free(kv);
    printf("tinyllm decode, %s cache, %s: worst rel-L2 %.2e, rows with code / scale mismatches %d\n",
           dtype == EIF_CUDA_INT8 ? "INT8" : "fp32", one_call ? "eif_cuda_decode_step" : "rope_append + attend_decode",
           worst, code_mismatch);
    return worst <= 1e-5 && code_mismatch == 0 ? 0 : 1;
}

static int deltanet_rule(eif_cuda_ctx_t *ctx) {
    eif_cuda_delta_t *dn = NULL;
    eif_status_t st = eif_cuda_delta_alloc(ctx, 1, 1, DH, DK, DV, 0, &dn);
    if (st != EIF_STATUS_OK) return fail_status(ctx, "delta_alloc", st);
    static float S[DH * DK * DV];
    memset(S, 0, sizeof S);
    const float q_scale = 1.0f / sqrtf((float)DK);
    double worst = 0.0;
    for (int step = 0; step < 12; step++) {
        float q[DH * DK], k[DH * DK], v[DH * DV], beta[DH], g[DH], o[DH * DV], ref[DH * DV];
        for (int h = 0; h < DH; h++) {
            float nq = 0.0f, nk = 0.0f;
            for (int i = 0; i < DK; i++) {
                q[h * DK + i] = rnd();
                k[h * DK + i] = rnd();
                nq += q[h * DK + i] * q[h * DK + i];
                nk += k[h * DK + i] * k[h * DK + i];
            }
            for (int i = 0; i < DK; i++) { q[h * DK + i] /= sqrtf(nq); k[h * DK + i] /= sqrtf(nk); }
            for (int j = 0; j < DV; j++) v[h * DV + j] = rnd();
            beta[h] = 0.5f + 0.4f * rnd();
            g[h] = -0.3f + 0.2f * rnd();
        }
        if ((st = eif_cuda_deltanet_step(ctx, dn, 0, q, k, v, beta, g, q_scale, o)) != EIF_STATUS_OK)
            return fail_status(ctx, "deltanet_step", st);
        for (int h = 0; h < DH; h++) { /* decay, retrieve from the decayed state, update, output */
            float *Sh = S + h * DK * DV;
            const float decay = expf(g[h]);
            for (int i = 0; i < DK * DV; i++) Sh[i] *= decay;
            for (int j = 0; j < DV; j++) {
                float e = 0.0f;
                for (int i = 0; i < DK; i++) e += Sh[i * DV + j] * k[h * DK + i];
                const float d = v[h * DV + j] - e;
                for (int i = 0; i < DK; i++) Sh[i * DV + j] += beta[h] * k[h * DK + i] * d;
            }
            for (int j = 0; j < DV; j++) {
                float acc = 0.0f;
                for (int i = 0; i < DK; i++) acc += Sh[i * DV + j] * q[h * DK + i] * q_scale;
                ref[h * DV + j] = acc;
            }
        }
        const double e = rel_l2(o, ref, DH * DV);
        worst = e > worst ? e : worst;
    }
    eif_cuda_delta_free(dn);
    printf("DeltaNet rule: worst rel-L2 %.2e over 12 steps\n", worst);
    return worst <= 1e-5 ? 0 : 1;
}

int main(void) {
    if (eif_cuda_device_count() == 0) {
        printf("no CUDA device: nothing to run\n");
        return 0;
    }
    eif_cuda_ctx_t *ctx = NULL;
    eif_status_t st = eif_cuda_init(&ctx, 0);
    if (st != EIF_STATUS_OK) {
        fprintf(stderr, "eif_cuda_init: status %d\n", (int)st);
        return 1;
    }
    int bad = 0;
    bad |= tinyllm_decode(ctx, EIF_CUDA_F32, 0);
    bad |= tinyllm_decode(ctx, EIF_CUDA_INT8, 0);
    bad |= tinyllm_decode(ctx, EIF_CUDA_F32, 1);
    bad |= tinyllm_decode(ctx, EIF_CUDA_INT8, 1);
    bad |= deltanet_rule(ctx);
    eif_cuda_free(ctx);
    printf(bad ? "FAILED\n" : "OK\n");
    return bad;
}
