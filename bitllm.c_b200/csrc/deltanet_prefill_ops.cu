// deltanet_prefill_ops.cu -- the parts of deltanet_core (src/eif_qwen35.c:546-656) around the delta rule,
// for a whole prefill chunk of n_tok tokens per sequence, so that prefill_chunk's per-token loop
// (src/eif_qwen35.c:1104-1106) becomes: pre ops -> chunked rule (deltanet_chunked.cu) -> post ops.
//
// dn_prefill_pre_kernel  one CTA per (token, sequence), one warp per head: the causal conv1d over the
//     conv_k-long window of each of the head's q / k / v channels (:560-572; the window reaches back into
//     the layer's conv state for the chunk's first conv_k - 1 tokens), SiLU, the L2 norms of q and k
//     (eps 1e-12 inside the root) with q scaled by 1/sqrt(d_k) (:579-585), and the gates
//     beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) (:587-592).  q / k / v leave as bf16, the
//     operands of the chunked rule; the gates stay fp32.
// dn_conv_state_kernel   one thread per (sequence, channel): the window after the chunk = its last conv_k
//     inputs (older ones from the previous window when n_tok < conv_k), what the per-token shifts of
//     :561-569 leave behind.
// dn_prefill_post_kernel one CTA per (token, sequence), one warp per head: the gated RMSNorm
//     o * rsqrt(mean(o^2) + 1e-6) * norm_w * silu(z) of the rule's fp32 output (:642-653).
// The arithmetic of each value follows deltanet_core_kernel (mixer_fused.cu), the per-token path.
#include <math.h>

#include "internal.h"
#include "common.cuh"

namespace {

constexpr int kMaxPerLane = 8;  // d_k, d_v <= 256

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

__global__ void __launch_bounds__(256) dn_prefill_pre_kernel(const DeltaPrefillArgs a) {
    const int t = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int H = a.H, dk = a.dk, dv = a.dv, ck = a.conv_k, n = a.n_tok;
    const int key_dim = H * dk, conv_dim = 2 * key_dim + H * dv;
    const size_t tok = (size_t)b * n + t;
    // causal conv1d over the window x_{t-ck+1} .. x_t of channel c, then SiLU
    auto conv_silu = [&](int c) -> float {
        const float *w = a.conv_w + (size_t)c * ck;
        const float *win = a.conv + ((size_t)b * conv_dim + c) * ck;  // x_{-ck} .. x_{-1}
        float acc = 0.f;
        for (int j = 0; j < ck; ++j) {
            const int tt = t - (ck - 1) + j;
            const float x = tt >= 0 ? a.qkv[((size_t)b * n + tt) * conv_dim + c] : win[ck + tt];
            acc += x * w[j];
        }
        return silu_f(acc);
    };
    const float q_scale = 1.0f / sqrtf((float)dk);
    const int nq = dk / 32, nv = dv / 32;
    for (int h = warp; h < H; h += nw) {
        float qv[kMaxPerLane], kv[kMaxPerLane];
        float sq = 0.f, sk = 0.f;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; ++m) {
            if (m < nq) {
                const int i = lane + 32 * m;
                qv[m] = conv_silu(h * dk + i);
                kv[m] = conv_silu(key_dim + h * dk + i);
                sq += qv[m] * qv[m];
                sk += kv[m] * kv[m];
            }
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const float iq = 1.0f / sqrtf(sq + 1e-12f), ik = 1.0f / sqrtf(sk + 1e-12f);
        const size_t th = tok * H + h;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; ++m) {
            if (m < nq) {
                const int i = lane + 32 * m;
                a.q[th * dk + i] = __float2bfloat16_rn(qv[m] * iq * q_scale);
                a.k[th * dk + i] = __float2bfloat16_rn(kv[m] * ik);
            }
            if (m < nv) {
                const int i = lane + 32 * m;
                a.v[th * dv + i] = __float2bfloat16_rn(conv_silu(2 * key_dim + h * dv + i));
            }
        }
        if (lane == 0) {
            a.beta[th] = 1.0f / (1.0f + expf(-a.b_raw[th]));
            const float x = a.a_raw[th] + a.dt_bias[h];
            a.g[th] = -a.a_exp[h] * logf(1.0f + expf(x));
        }
    }
}

__global__ void __launch_bounds__(256) dn_conv_state_kernel(const DeltaPrefillArgs a) {
    const int conv_dim = 2 * a.H * a.dk + a.H * a.dv, ck = a.conv_k, n = a.n_tok;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)a.B * conv_dim) return;
    const size_t b = idx / conv_dim, c = idx % conv_dim;
    float *row = a.conv + idx * ck;
    // in increasing j: an entry taken from the old window (index n + j) has not been overwritten yet
    for (int j = 0; j < ck; ++j) {
        const int tt = n - ck + j;
        row[j] = tt >= 0 ? a.qkv[(b * n + tt) * conv_dim + c] : row[ck + tt];
    }
}

__global__ void __launch_bounds__(256) dn_prefill_post_kernel(const DeltaPrefillArgs a) {
    const int t = blockIdx.x, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int H = a.H, dv = a.dv, nv = dv / 32;
    const size_t tok = (size_t)b * a.n_tok + t;
    for (int h = warp; h < H; h += nw) {
        const float *o = a.o + (tok * H + h) * dv;
        float ov[kMaxPerLane], ss = 0.f;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; ++m)
            if (m < nv) {
                ov[m] = o[lane + 32 * m];
                ss += ov[m] * ov[m];
            }
        ss = warp_sum(ss);
        const float rms = 1.0f / sqrtf(ss / dv + 1e-6f);
        const float *z = a.z + tok * H * dv + (size_t)h * dv;
        float *out = a.out + tok * H * dv + (size_t)h * dv;
#pragma unroll
        for (int m = 0; m < kMaxPerLane; ++m)
            if (m < nv) {
                const int i = lane + 32 * m;
                out[i] = ov[m] * rms * a.norm_w[i] * silu_f(z[i]);
            }
    }
}

}  // namespace

cudaError_t launch_deltanet_prefill_pre(cudaStream_t st, const DeltaPrefillArgs &a) {
    if (a.dk % 32 || a.dv % 32 || a.dk > 32 * kMaxPerLane || a.dv > 32 * kMaxPerLane) return cudaErrorInvalidValue;
    const int threads = 32 * (a.H < 8 ? a.H : 8);
    dn_prefill_pre_kernel<<<dim3(a.n_tok, a.B), threads, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t n = (size_t)a.B * (2 * a.H * a.dk + a.H * a.dv);
    dn_conv_state_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(a);  // after the pre kernel read the window
    return cudaGetLastError();
}

cudaError_t launch_deltanet_prefill_post(cudaStream_t st, const DeltaPrefillArgs &a) {
    if (a.dv % 32 || a.dv > 32 * kMaxPerLane) return cudaErrorInvalidValue;
    const int threads = 32 * (a.H < 8 ? a.H : 8);
    dn_prefill_post_kernel<<<dim3(a.n_tok, a.B), threads, 0, st>>>(a);
    return cudaGetLastError();
}
