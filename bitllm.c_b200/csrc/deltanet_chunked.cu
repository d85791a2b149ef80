// deltanet_chunked.cu -- Gated DeltaNet prefill in the chunked WY / UT form.
//
// Reference: the engine runs its prefill token by token (prefill_chunk calls deltanet_core per token,
// src/eif_qwen35.c:1104-1106), i.e. the recurrence of src/eif_qwen35.c:594-639:
//     S_i = a_i S_{i-1} + b_i k_i (v_i - a_i S_{i-1}^T k_i)^T,   o_i = S_i^T (q_scale q_i),   a_i = e^{g_i}
// Chunked restatement (64 tokens, G_i = within-chunk inclusive cumsum of g, S0 = state at chunk start):
//     u_i = b_i (v_i - a_i S_{i-1}^T k_i)  satisfies  (I + A) U = diag(b) V - diag(b e^G) K S0,
//     A_ij = b_i e^{G_i - G_j} k_i.k_j (j < i),  T = (I + A)^-1,  W = T diag(b e^G) K,  U' = T diag(b) V
//     U = U' - W S0
//     O = q_scale [ diag(e^G) Q S0 + (e^{G_i - G_j} Q K^T)_{j <= i} U ]
//     S_C = e^{G_C} S0 + (diag(e^{G_C - G}) K)^T U
// which is algebraically the token-by-token recurrence (the same decay-first order).
//
// Decomposition: one CTA per (sequence, head, 64-column slice of d_v): the columns of S evolve
// independently (column j of u depends on column j of S only), so slices need no communication.
// The CTA walks the chunks in order with the fp32 state held in registers (mma accumulator layout) by
// warps 0-3; bf16 copies of S feed the products that read it.  TMA brings the next chunk's q / k / v
// tiles (128-byte swizzle, no multicast) while the current chunk is processed.  The chunk GEMMs run on
// the tensor cores (mma.m16n8k16, bf16 in, fp32 accumulate); T comes from a blocked forward
// substitution in fp32 (16 x 16 diagonal blocks per warp, then three block levels).
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int C = 64;        // chunk length
constexpr int DK = 128;      // key head dim
constexpr int DS = 64;       // value columns per CTA
constexpr int kThreads = 256;
constexpr int FP = 68;       // fp32 row pitch (floats) of the 64 x 64 scratch matrices

// bf16 matrices are stored in 128-byte-swizzled boxes of 64 columns: [box][row][8 x 16 B]
__device__ __forceinline__ uint32_t sw(int rows, int row, int col) {
    return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

// smem layout (bytes)
constexpr int STG_Q = 0, STG_K = C * DK * 2, STG_V = 2 * C * DK * 2, STG_BYTES = 2 * C * DK * 2 + C * DS * 2;
constexpr int OFF_STG = 0;                                   // two stages
constexpr int OFF_KKF = 2 * STG_BYTES;                       // fp32 [64][FP]: K K^T, then A
constexpr int OFF_QKF = OFF_KKF + C * FP * 4;                // fp32 [64][FP]: Q K^T, then T
constexpr int OFF_TB = OFF_QKF + C * FP * 4;                 // bf16 64 x 64: T
constexpr int OFF_QKM = OFF_TB + C * C * 2;                  // bf16 64 x 64: q_scale e^{G_i-G_j} Q K^T (j <= i)
constexpr int OFF_X = OFF_QKM + C * C * 2;                   // bf16 64 x 192: [b e^G K | b V]
constexpr int OFF_KT = OFF_X + C * (DK + DS) * 2;            // bf16 64 x 128: e^{G_C - G} K
constexpr int OFF_W = OFF_KT + C * DK * 2;                   // bf16 64 x 128: W
constexpr int OFF_U = OFF_W + C * DK * 2;                    // bf16 64 x 64: U
constexpr int OFF_SB = OFF_U + C * DS * 2;                   // bf16 128 x 64: S (bf16 copy)
constexpr int OFF_VEC = OFF_SB + DK * DS * 2;                // fp32: G[64], beta[64], eG[64], eGC[64]
constexpr int OFF_BAR = OFF_VEC + 4 * C * 4;
constexpr int kSmem = OFF_BAR + 64 + 1024;

struct ChunkArgs {
    const __nv_bfloat16 *q, *k, *v;  // (for reference only; tiles come through the tensor maps)
    const float *beta, *g;           // [B][T][H]
    __nv_bfloat16 *o;                // [B][T][H][dv]
    float *S;                        // layer state [B][H][DK][dv]
    int B, T, H, dv;
    float q_scale;
    unsigned *dev_err;
};

__global__ void __launch_bounds__(kThreads, 1)
    deltanet_chunked_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const ChunkArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sb = smem_u32(sm);
    float *KKf = reinterpret_cast<float *>(sm + OFF_KKF);
    float *QKf = reinterpret_cast<float *>(sm + OFF_QKF);
    float *Gv = reinterpret_cast<float *>(sm + OFF_VEC), *Bv = Gv + C, *eG = Gv + 2 * C, *eGC = Gv + 3 * C;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);

    const int slice = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int mi = lane >> 3, r8 = lane & 7;
    const int n_chunks = (p.T + C - 1) / C;
    const size_t bh = (size_t)b * p.H + h;

    if (tid == 0) {
        mbar_init(smem_u32(bars), 1);
        mbar_init(smem_u32(bars + 1), 1);
        fence_barrier_init();
    }

    // ---- initial state: warps 0-3 hold S rows [32w, 32w+32) x 64 columns in accumulator layout
    float S[2][8][4];
    float *Sg = p.S + bh * DK * p.dv + slice * DS;
    if (warp < 4) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int row = warp * 32 + mt * 16 + g8, col = nt * 8 + 2 * t4;
                S[mt][nt][0] = Sg[(size_t)row * p.dv + col];
                S[mt][nt][1] = Sg[(size_t)row * p.dv + col + 1];
                S[mt][nt][2] = Sg[(size_t)(row + 8) * p.dv + col];
                S[mt][nt][3] = Sg[(size_t)(row + 8) * p.dv + col + 1];
                *reinterpret_cast<uint32_t *>(sm + OFF_SB + sw(DK, row, col)) = pack_bf16x2(S[mt][nt][0], S[mt][nt][1]);
                *reinterpret_cast<uint32_t *>(sm + OFF_SB + sw(DK, row + 8, col)) =
                    pack_bf16x2(S[mt][nt][2], S[mt][nt][3]);
            }
    }
    __syncthreads();

    auto issue = [&](int c) {  // TMA for chunk c into stage c & 1 (thread 0)
        const int s = c & 1;
        const uint32_t bar = smem_u32(bars + s), base = sb + OFF_STG + s * STG_BYTES;
        const int row = b * p.T + c * C;
        mbar_arrive_expect_tx(bar, STG_BYTES);
        for (int d = 0; d < 2; ++d) {
            tma_load_3d(base + STG_Q + d * C * 128, &tmQ, d * 64, h, row, bar);
            tma_load_3d(base + STG_K + d * C * 128, &tmK, d * 64, h, row, bar);
        }
        tma_load_3d(base + STG_V, &tmV, slice * DS, h, row, bar);
    };
    if (tid == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        issue(0);
    }

    float Up[8][4];  // U' tiles of warps 0-3 (rows 16w..16w+15, all 64 columns)
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
        const int s = c & 1;
        const int t0 = c * C;
        const uint32_t stg = sb + OFF_STG + s * STG_BYTES;
        uint8_t *stgp = sm + OFF_STG + s * STG_BYTES;
        if (tid == 0 && c + 1 < n_chunks) {
            fence_proxy_async_smem();
            issue(c + 1);
        }
        // ---- P0: beta, g (zero past T: such tokens leave S untouched), cumulative log decay
        if (tid < C) {
            const bool valid = t0 + tid < p.T;
            const size_t ix = ((size_t)b * p.T + t0 + tid) * p.H + h;
            Bv[tid] = valid ? p.beta[ix] : 0.f;
            Gv[tid] = valid ? p.g[ix] : 0.f;
        }
        __syncthreads();
        if (warp == 0) {
            float x0 = Gv[2 * lane], x1 = Gv[2 * lane + 1];
            x1 += x0;
            float run = x1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, run, o);
                if (lane >= o) run += y;
            }
            const float excl = run - x1;
            Gv[2 * lane] = excl + x0;
            Gv[2 * lane + 1] = run;
        }
        ok = mbar_wait(smem_u32(bars + s), (c >> 1) & 1, p.dev_err);
        if (!__syncthreads_and(ok)) {  // CTA-uniform: every thread leaves the loop together
            ok = false;
            break;
        }
        if (tid < C) {
            eG[tid] = expf(Gv[tid]);
            eGC[tid] = expf(Gv[C - 1] - Gv[tid]);
        }

        // ---- P1: K K^T (warps 0-3) and Q K^T (warps 4-7): m-tile = warp & 3, 8 n-tiles, 8 k-steps
        {
            const int mt = warp & 3;
            const uint32_t abase = stg + (warp < 4 ? STG_K : STG_Q), kbase = stg + STG_K;
            float acc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < DK / 16; ++ks) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(abase + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kbase + sw(C, np * 16 + (mi >> 1) * 8 + r8, ks * 16 + (mi & 1) * 8), b0, b1, b2, b3);
                    mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            }
            float *dst = warp < 4 ? KKf : QKf;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int row = mt * 16 + g8, col = nt * 8 + 2 * t4;
                dst[row * FP + col] = acc[nt][0];
                dst[row * FP + col + 1] = acc[nt][1];
                dst[(row + 8) * FP + col] = acc[nt][2];
                dst[(row + 8) * FP + col + 1] = acc[nt][3];
            }
        }
        __syncthreads();

        // ---- P2: A (in KKf), masked decayed Q K^T (bf16), X = [b e^G K | b V], Kt = e^{G_C - G} K
        for (int e = tid; e < C * C; e += kThreads) {
            const int i = e >> 6, j = e & 63;
            const float dec = j <= i ? expf(Gv[i] - Gv[j]) : 0.f;
            KKf[i * FP + j] = j < i ? Bv[i] * dec * KKf[i * FP + j] : 0.f;
            const float qk = j <= i ? p.q_scale * dec * QKf[i * FP + j] : 0.f;
            *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_QKM + sw(C, i, j)) = __float2bfloat16_rn(qk);
        }
        for (int e = tid; e < C * (DK / 8); e += kThreads) {  // 16-byte units of K rows
            const int j = e >> 4, u = e & 15;
            const uint4 kv = *reinterpret_cast<const uint4 *>(stgp + STG_K + sw(C, j, u * 8));
            const float fx = Bv[j] * eG[j], fk = eGC[j];
            uint32_t w[4] = {kv.x, kv.y, kv.z, kv.w}, xo[4], ko[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float lo = bf16lo_to_f32(w[q]), hi = bf16hi_to_f32(w[q]);
                xo[q] = pack_bf16x2(lo * fx, hi * fx);
                ko[q] = pack_bf16x2(lo * fk, hi * fk);
            }
            *reinterpret_cast<uint4 *>(sm + OFF_X + sw(C, j, u * 8)) = make_uint4(xo[0], xo[1], xo[2], xo[3]);
            *reinterpret_cast<uint4 *>(sm + OFF_KT + sw(C, j, u * 8)) = make_uint4(ko[0], ko[1], ko[2], ko[3]);
        }
        for (int e = tid; e < C * (DS / 8); e += kThreads) {  // 16-byte units of the V slice
            const int j = e >> 3, u = e & 7;
            const uint4 vv = *reinterpret_cast<const uint4 *>(stgp + STG_V + sw(C, j, u * 8));
            const float fb = Bv[j];
            uint32_t w[4] = {vv.x, vv.y, vv.z, vv.w}, xo[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) xo[q] = pack_bf16x2(bf16lo_to_f32(w[q]) * fb, bf16hi_to_f32(w[q]) * fb);
            *reinterpret_cast<uint4 *>(sm + OFF_X + sw(C, j, DK + u * 8)) = make_uint4(xo[0], xo[1], xo[2], xo[3]);
        }
        __syncthreads();

        // ---- T = (I + A)^-1 in fp32 (into QKf): diagonal 16 x 16 blocks by forward substitution
        float *Tf = QKf;
        if (warp < 4 && lane < 16) {
            const int o = warp * 16, cidx = lane;  // block offset, column of the block
            float col[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                float acc = r == cidx ? 1.f : 0.f;
#pragma unroll
                for (int m = 0; m < 16; ++m)
                    if (m < r) acc -= KKf[(o + r) * FP + o + m] * col[m];
                col[r] = r < cidx ? 0.f : acc;
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) Tf[(o + r) * FP + o + cidx] = col[r];
        } else if (warp >= 4) {
            // zero the strictly upper blocks (used as scratch below, then as zeros of T)
            for (int e = tid - 128; e < C * C; e += 128) {
                const int i = e >> 6, j = e & 63;
                if ((j >> 4) > (i >> 4)) Tf[i * FP + j] = 0.f;
            }
        }
        __syncthreads();
        // off-diagonal blocks by level: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ; R kept in block (J, I)
        for (int lvl = 1; lvl <= 3; ++lvl) {
            const int nblk = 4 - lvl;
            for (int e = tid; e < nblk * 256; e += kThreads) {
                const int J = e >> 8, I = J + lvl, rr = (e >> 4) & 15, cc = e & 15;
                float acc = 0.f;
                for (int K = J; K < I; ++K)
#pragma unroll
                    for (int m = 0; m < 16; ++m) acc += KKf[(I * 16 + rr) * FP + K * 16 + m] * Tf[(K * 16 + m) * FP + J * 16 + cc];
                Tf[(J * 16 + rr) * FP + I * 16 + cc] = acc;  // R_IJ stored transposed-position (upper)
            }
            __syncthreads();
            for (int e = tid; e < nblk * 256; e += kThreads) {
                const int J = e >> 8, I = J + lvl, rr = (e >> 4) & 15, cc = e & 15;
                float acc = 0.f;
#pragma unroll
                for (int m = 0; m < 16; ++m) acc -= Tf[(I * 16 + rr) * FP + I * 16 + m] * Tf[(J * 16 + m) * FP + I * 16 + cc];
                Tf[(I * 16 + rr) * FP + J * 16 + cc] = acc;
            }
            __syncthreads();
        }
        for (int e = tid; e < C * C; e += kThreads) {
            const int i = e >> 6, j = e & 63;
            *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_TB + sw(C, i, j)) = __float2bfloat16_rn(j <= i ? Tf[i * FP + j] : 0.f);
        }
        __syncthreads();

        // ---- P3: [W | U'] = T X.  warps 0-3: m-tile w, W cols 0-63 and U' cols 0-63; warps 4-7: W cols 64-127
        {
            const int mt = warp & 3;
            const int wc0 = warp < 4 ? 0 : 64;
            float wacc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                wacc[nt][0] = wacc[nt][1] = wacc[nt][2] = wacc[nt][3] = 0.f;
                Up[nt][0] = Up[nt][1] = Up[nt][2] = Up[nt][3] = 0.f;
            }
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(sb + OFF_TB + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(sb + OFF_X + sw(C, ks * 16 + (mi & 1) * 8 + r8, wc0 + np * 16 + (mi >> 1) * 8), b0, b1, b2,
                              b3);
                    mma_bf16_16816(wacc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(wacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                    if (warp < 4) {
                        ldsm_x4_t(sb + OFF_X + sw(C, ks * 16 + (mi & 1) * 8 + r8, DK + np * 16 + (mi >> 1) * 8), b0,
                                  b1, b2, b3);
                        mma_bf16_16816(Up[2 * np], a0, a1, a2, a3, b0, b1);
                        mma_bf16_16816(Up[2 * np + 1], a0, a1, a2, a3, b2, b3);
                    }
                }
            }
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int row = mt * 16 + g8, col = wc0 + nt * 8 + 2 * t4;
                *reinterpret_cast<uint32_t *>(sm + OFF_W + sw(C, row, col)) = pack_bf16x2(wacc[nt][0], wacc[nt][1]);
                *reinterpret_cast<uint32_t *>(sm + OFF_W + sw(C, row + 8, col)) = pack_bf16x2(wacc[nt][2], wacc[nt][3]);
            }
        }
        __syncthreads();

        // ---- P4: warps 0-3: U = U' - W S (m-tile w) -> bf16; warps 4-7: Q S (m-tile w-4), kept in registers
        float qs[8][4];
        {
            const int mt = warp & 3;
            const uint32_t abase = warp < 4 ? sb + OFF_W : stg + STG_Q;
            float acc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < DK / 16; ++ks) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(abase + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(sb + OFF_SB + sw(DK, ks * 16 + (mi & 1) * 8 + r8, np * 16 + (mi >> 1) * 8), b0, b1, b2, b3);
                    mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            }
            if (warp < 4) {
#pragma unroll
                for (int nt = 0; nt < 8; ++nt) {
                    const int row = mt * 16 + g8, col = nt * 8 + 2 * t4;
                    *reinterpret_cast<uint32_t *>(sm + OFF_U + sw(C, row, col)) =
                        pack_bf16x2(Up[nt][0] - acc[nt][0], Up[nt][1] - acc[nt][1]);
                    *reinterpret_cast<uint32_t *>(sm + OFF_U + sw(C, row + 8, col)) =
                        pack_bf16x2(Up[nt][2] - acc[nt][2], Up[nt][3] - acc[nt][3]);
                }
            } else {
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int q = 0; q < 4; ++q) qs[nt][q] = acc[nt][q];
            }
        }
        __syncthreads();

        // ---- P5: warps 4-7: O = q_scale e^G Q S + QKm U -> bf16 out; warps 0-3: S = e^{G_C} S + Kt^T U
        if (warp >= 4) {
            const int mt = warp & 3;
            float acc[8][4];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(sb + OFF_QKM + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(sb + OFF_U + sw(C, ks * 16 + (mi & 1) * 8 + r8, np * 16 + (mi >> 1) * 8), b0, b1, b2, b3);
                    mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            }
            const int r0 = mt * 16 + g8;
            const float f0 = p.q_scale * eG[r0], f1 = p.q_scale * eG[r0 + 8];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int col = slice * DS + nt * 8 + 2 * t4;
                if (t0 + r0 < p.T)
                    *reinterpret_cast<uint32_t *>(p.o + (((size_t)b * p.T + t0 + r0) * p.H + h) * p.dv + col) =
                        pack_bf16x2(acc[nt][0] + f0 * qs[nt][0], acc[nt][1] + f0 * qs[nt][1]);
                if (t0 + r0 + 8 < p.T)
                    *reinterpret_cast<uint32_t *>(p.o + (((size_t)b * p.T + t0 + r0 + 8) * p.H + h) * p.dv + col) =
                        pack_bf16x2(acc[nt][2] + f1 * qs[nt][2], acc[nt][3] + f1 * qs[nt][3]);
            }
        } else {
            const float dC = expf(Gv[C - 1]);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                    for (int q = 0; q < 4; ++q) S[mt][nt][q] *= dC;
#pragma unroll
            for (int ks = 0; ks < C / 16; ++ks) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    // A = Kt^T rows (key dims) 32w + 16mt .. +16, k = tokens 16ks .. +16 (transposed load)
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(sb + OFF_KT + sw(C, ks * 16 + (mi >> 1) * 8 + r8, warp * 32 + mt * 16 + (mi & 1) * 8), a0,
                              a1, a2, a3);
#pragma unroll
                    for (int np = 0; np < 4; ++np) {
                        uint32_t b0, b1, b2, b3;
                        ldsm_x4_t(sb + OFF_U + sw(C, ks * 16 + (mi & 1) * 8 + r8, np * 16 + (mi >> 1) * 8), b0, b1, b2,
                                  b3);
                        mma_bf16_16816(S[mt][2 * np], a0, a1, a2, a3, b0, b1);
                        mma_bf16_16816(S[mt][2 * np + 1], a0, a1, a2, a3, b2, b3);
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 8; ++nt) {
                    const int row = warp * 32 + mt * 16 + g8, col = nt * 8 + 2 * t4;
                    *reinterpret_cast<uint32_t *>(sm + OFF_SB + sw(DK, row, col)) = pack_bf16x2(S[mt][nt][0], S[mt][nt][1]);
                    *reinterpret_cast<uint32_t *>(sm + OFF_SB + sw(DK, row + 8, col)) =
                        pack_bf16x2(S[mt][nt][2], S[mt][nt][3]);
                }
        }
        __syncthreads();
    }

    // ---- final state back to the layer's S
    if (ok && warp < 4) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                const int row = warp * 32 + mt * 16 + g8, col = nt * 8 + 2 * t4;
                Sg[(size_t)row * p.dv + col] = S[mt][nt][0];
                Sg[(size_t)row * p.dv + col + 1] = S[mt][nt][1];
                Sg[(size_t)(row + 8) * p.dv + col] = S[mt][nt][2];
                Sg[(size_t)(row + 8) * p.dv + col + 1] = S[mt][nt][3];
            }
    }
}

}  // namespace

bool deltanet_chunked_supported(int dk, int dv) { return dk == DK && dv % DS == 0 && dv <= 256; }

cudaError_t launch_deltanet_chunked(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                    const CUtensorMap &tv, const float *beta, const float *g, __nv_bfloat16 *o,
                                    float *S, int B, int T, int H, int dv, float q_scale, unsigned *dev_err) {
    ChunkArgs p{nullptr, nullptr, nullptr, beta, g, o, S, B, T, H, dv, q_scale, dev_err};
    cudaError_t e = cudaFuncSetAttribute(deltanet_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    dim3 grid(dv / DS, H, B);
    deltanet_chunked_kernel<<<grid, kThreads, kSmem, st>>>(tq, tk, tv, p);
    return cudaGetLastError();
}
