// deltanet.cu -- Gated DeltaNet recurrent step on B200.
//
// Reference: the per-head delta rule of deltanet_core, src/eif_qwen35.c:594-639 (bitllm.c):
//     S <- exp(g) S;   e = S^T k;   S <- S + beta k (v - e)^T;   o = S^T q
// with S [d_k][d_v] row-major (d_v contiguous).  The reference walks S four times per head; here S
// makes exactly one trip HBM -> registers -> HBM per step.
//
// Decomposition.  The two reductions (S^T k and S^T q) run over the ROWS i of S, independently for
// every column j, so a head's columns split across CTAs with no communication: a CTA owns COLS
// columns and all d_k rows of one (sequence, head).  Inside the CTA a thread owns a float4 of
// columns in NP rows, held in registers for the whole step:
//   1. issue all NP streaming loads of the S tile (ld.global.cs: S is touched once per step);
//   2. scale by exp(g), partial e over the thread's rows, reduce over rows (shuffles, then smem);
//   3. rank-1 update in registers, streaming store of the new tile;
//   4. partial o over the rows of the NEW S, same reduction, write o.
// The update uses the retrieved e from the decayed S, as the reference does (:611-631).
#include "internal.h"
#include "common.cuh"

namespace {

template <int DK, int DV, int COLS, int THREADS>
__global__ void __launch_bounds__(THREADS) delta_rule_kernel(float *__restrict__ S, const float *__restrict__ q,
                                                             const float *__restrict__ k,
                                                             const float *__restrict__ v,
                                                             const float *__restrict__ beta,
                                                             const float *__restrict__ g, float q_scale,
                                                             float *__restrict__ o, int H) {
    constexpr int LPR = COLS / 4;       // threads covering one row segment (float4 each)
    constexpr int RP = THREADS / LPR;   // rows covered per pass
    constexpr int NP = DK / RP;         // passes (float4 registers per thread)
    constexpr int NW = THREADS / 32;
    static_assert(COLS % 4 == 0 && LPR <= 32 && 32 % LPR == 0, "column split");
    static_assert(DK % RP == 0 && DV % COLS == 0, "tile shape");

    const int cb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lc = tid % LPR;
    const int rg = tid / LPR;
    const size_t bh = (size_t)b * H + h;
    const int col0 = cb * COLS + lc * 4;

    __shared__ float sk[DK];
    __shared__ float sq[DK];
    __shared__ float4 red[NW][LPR];

    float *Sh = S + bh * DK * DV;

    float4 s[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p)
        s[p] = __ldcs(reinterpret_cast<const float4 *>(Sh + (size_t)(rg + p * RP) * DV + col0));

    for (int i = tid; i < DK; i += THREADS) {
        sk[i] = k[bh * DK + i];
        sq[i] = q[bh * DK + i] * q_scale;
    }
    const float decay = expf(g[bh]);
    const float bet = beta[bh];
    const float4 vv = *reinterpret_cast<const float4 *>(v + bh * DV + col0);
    __syncthreads();

    // column reduction over all rows of the CTA: lanes that share lc, then warps through smem
    auto colsum = [&](float4 x) -> float4 {
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) x = f4_add(x, f4_shfl_xor(x, off));
        if (lane < LPR) red[warp][lc] = x;
        __syncthreads();
        float4 t = red[0][lc];
#pragma unroll
        for (int w = 1; w < NW; ++w) t = f4_add(t, red[w][lc]);
        __syncthreads();
        return t;
    };

    // 1-2: decay and retrieve
    float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const float ki = sk[rg + p * RP];
        s[p].x *= decay; s[p].y *= decay; s[p].z *= decay; s[p].w *= decay;
        e.x += s[p].x * ki; e.y += s[p].y * ki; e.z += s[p].z * ki; e.w += s[p].w * ki;
    }
    e = colsum(e);
    const float4 dlt = make_float4(vv.x - e.x, vv.y - e.y, vv.z - e.z, vv.w - e.w);

    // 3-4: update, store, output from the updated state
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int i = rg + p * RP;
        const float ki = bet * sk[i];
        s[p].x += ki * dlt.x; s[p].y += ki * dlt.y; s[p].z += ki * dlt.z; s[p].w += ki * dlt.w;
        __stcs(reinterpret_cast<float4 *>(Sh + (size_t)i * DV + col0), s[p]);
        const float qi = sq[i];
        acc.x += s[p].x * qi; acc.y += s[p].y * qi; acc.z += s[p].z * qi; acc.w += s[p].w * qi;
    }
    acc = colsum(acc);
    if (tid < LPR) *reinterpret_cast<float4 *>(o + bh * DV + col0) = acc;
}

template <int DK, int DV, int COLS, int THREADS>
cudaError_t launch_rule_t(cudaStream_t st, float *S, const float *q, const float *k, const float *v,
                          const float *beta, const float *g, float q_scale, float *o, int B, int H) {
    dim3 grid(DV / COLS, H, B);
    delta_rule_kernel<DK, DV, COLS, THREADS><<<grid, THREADS, 0, st>>>(S, q, k, v, beta, g, q_scale, o, H);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_delta_rule(cudaStream_t st, float *S, const float *q, const float *k, const float *v,
                              const float *beta, const float *g, float q_scale, float *o, int B, int H, int dk,
                              int dv, int sm_count, bool *supported) {
    (void)sm_count;
    *supported = true;
    if (dk == 128 && dv == 128) return launch_rule_t<128, 128, 32, 128>(st, S, q, k, v, beta, g, q_scale, o, B, H);
    if (dk == 64 && dv == 64) return launch_rule_t<64, 64, 32, 128>(st, S, q, k, v, beta, g, q_scale, o, B, H);
    if (dk == 128 && dv == 64) return launch_rule_t<128, 64, 32, 128>(st, S, q, k, v, beta, g, q_scale, o, B, H);
    if (dk == 64 && dv == 128) return launch_rule_t<64, 128, 32, 128>(st, S, q, k, v, beta, g, q_scale, o, B, H);
    if (dk == 256 && dv == 256) return launch_rule_t<256, 256, 32, 256>(st, S, q, k, v, beta, g, q_scale, o, B, H);
    *supported = false;
    return cudaSuccess;
}
