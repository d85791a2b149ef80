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
// Two kernels:
//   chunk_solve_kernel   one CTA per (sequence, head, chunk), all in parallel: K K^T on the tensor cores,
//                        A, then T = (I + A)^-1 in fp32 by blocked forward substitution (16 x 16 diagonal
//                        blocks per warp, three block levels); T is written as bf16 [64 x 64] per chunk.
//   deltanet_chunked_kernel  one CTA per (sequence, head, 64-column slice of d_v): the columns of S
//                        evolve independently (column j of u depends on column j of S only), so slices
//                        need no communication.  It walks the chunks in order with the fp32 state in
//                        registers (mma accumulator layout, warps 0-3); TMA brings the next chunk's q / k
//                        / v / T tiles (128-byte swizzle, no multicast) during the current one; every
//                        product runs on the tensor cores (mma.m16n8k16, bf16 in, fp32 accumulate).
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int C = 64;    // chunk length
constexpr int DK = 128;  // key head dim
constexpr int DS = 64;   // value columns per CTA of the state kernel
constexpr int FP = 68;   // fp32 row pitch (floats) of the 64 x 64 scratch matrices

// bf16 matrices are stored in 128-byte-swizzled boxes of 64 columns: [box][row][8 x 16 B]
__device__ __forceinline__ uint32_t sw(int rows, int row, int col) {
    return (uint32_t)((col >> 6) * rows * 128 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

// Loads beta and g of a chunk (zero past T: such tokens leave S untouched) and forms G = inclusive
// cumsum of g; tid < 64 loads, warp 0 scans.  Ends with the data in smem after a __syncthreads.
__device__ __forceinline__ void load_chunk_gates(const float *beta, const float *g, int b, int h, int H, int T,
                                                 int t0, float *Gv, float *Bv) {
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < C) {
        const bool valid = t0 + tid < T;
        const size_t ix = ((size_t)b * T + t0 + tid) * H + h;
        Bv[tid] = valid ? beta[ix] : 0.f;
        Gv[tid] = valid ? g[ix] : 0.f;
    }
    __syncthreads();
    if (tid < 32) {
        const float x0 = Gv[2 * lane], x1 = Gv[2 * lane + 1] + x0;
        float run = x1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, run, o);
            if (lane >= o) run += y;
        }
        Gv[2 * lane] = run - x1 + x0;
        Gv[2 * lane + 1] = run;
    }
}

// ==================================================================================================
// Kernel A: T = (I + A)^-1 of every chunk
// ==================================================================================================
constexpr int kSolveThreads = 128;
constexpr int SOL_K = 0;                      // bf16 64 x 128 K tile (TMA)
constexpr int SOL_A = C * DK * 2;             // fp32 [64][FP] A
constexpr int SOL_T = SOL_A + C * FP * 4;     // fp32 [64][FP] T
constexpr int SOL_VEC = SOL_T + C * FP * 4;   // G[64], beta[64]
constexpr int SOL_BAR = SOL_VEC + 2 * C * 4;
constexpr int kSolveSmem = SOL_BAR + 16 + 1024;

__global__ void __launch_bounds__(kSolveThreads) chunk_solve_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                    const float *__restrict__ beta,
                                                                    const float *__restrict__ g,
                                                                    __nv_bfloat16 *__restrict__ Tout, int T, int H,
                                                                    unsigned *dev_err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sb = smem_u32(sm);
    float *Af = reinterpret_cast<float *>(sm + SOL_A), *Tf = reinterpret_cast<float *>(sm + SOL_T);
    float *Gv = reinterpret_cast<float *>(sm + SOL_VEC), *Bv = Gv + C;
    const uint32_t bar = smem_u32(sm + SOL_BAR);
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z, n_chunks = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int mi = lane >> 3, r8 = lane & 7;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, C * DK * 2);
        for (int d = 0; d < 2; ++d) tma_load_3d(sb + SOL_K + d * C * 128, &tmK, d * 64, h, b * T + c * C, bar);
    }
    load_chunk_gates(beta, g, b, h, H, T, c * C, Gv, Bv);
    const bool ok = mbar_wait(bar, 0, dev_err);
    if (!__syncthreads_and(ok)) return;

    // K K^T: warp w owns rows 16w..16w+15; A_ij = b_i e^{G_i - G_j} k_i.k_j for j < i
    {
        float acc[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < DK / 16; ++ks) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(sb + SOL_K + sw(C, warp * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(sb + SOL_K + sw(C, np * 16 + (mi >> 1) * 8 + r8, ks * 16 + (mi & 1) * 8), b0, b1, b2, b3);
                mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
            }
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int i = warp * 16 + g8 + (q >> 1) * 8, j = nt * 8 + 2 * t4 + (q & 1);
                Af[i * FP + j] = j < i ? Bv[i] * expf(Gv[i] - Gv[j]) * acc[nt][q] : 0.f;
            }
    }
    __syncthreads();

    // diagonal 16 x 16 blocks (lanes 0-15 of each warp: one column each); lanes 16-31 zero the upper blocks
    if (lane < 16) {
        const int o = warp * 16, cidx = lane;
        float col[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float acc = r == cidx ? 1.f : 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m)
                if (m < r) acc -= Af[(o + r) * FP + o + m] * col[m];
            col[r] = r < cidx ? 0.f : acc;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) Tf[(o + r) * FP + o + cidx] = col[r];
    } else {
        for (int e = warp * 16 + lane - 16; e < C * C; e += 64) {
            const int i = e >> 6, j = e & 63;
            if ((j >> 4) > (i >> 4)) Tf[i * FP + j] = 0.f;
        }
    }
    __syncthreads();
    // off-diagonal blocks by level: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ; R_IJ kept in block (J, I)
    for (int lvl = 1; lvl <= 3; ++lvl) {
        const int nblk = 4 - lvl;
        for (int e = tid; e < nblk * 256; e += kSolveThreads) {
            const int J = e >> 8, I = J + lvl, rr = (e >> 4) & 15, cc = e & 15;
            float acc = 0.f;
            for (int K = J; K < I; ++K)
#pragma unroll
                for (int m = 0; m < 16; ++m) acc += Af[(I * 16 + rr) * FP + K * 16 + m] * Tf[(K * 16 + m) * FP + J * 16 + cc];
            Tf[(J * 16 + rr) * FP + I * 16 + cc] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nblk * 256; e += kSolveThreads) {
            const int J = e >> 8, I = J + lvl, rr = (e >> 4) & 15, cc = e & 15;
            float acc = 0.f;
#pragma unroll
            for (int m = 0; m < 16; ++m) acc -= Tf[(I * 16 + rr) * FP + I * 16 + m] * Tf[(J * 16 + m) * FP + I * 16 + cc];
            Tf[(I * 16 + rr) * FP + J * 16 + cc] = acc;
        }
        __syncthreads();
    }
    // T (lower, upper zeroed) -> bf16 rows of 64 for the state kernel's TMA
    __nv_bfloat16 *dst = Tout + (((size_t)b * H + h) * n_chunks + c) * C * C;
    for (int e = tid; e < C * C / 8; e += kSolveThreads) {
        const int i = e >> 3, j0 = (e & 7) * 8;
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int j = j0 + 2 * q;
            w[q] = pack_bf16x2(j <= i ? Tf[i * FP + j] : 0.f, j + 1 <= i ? Tf[i * FP + j + 1] : 0.f);
        }
        *reinterpret_cast<uint4 *>(dst + i * C + j0) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ==================================================================================================
// Kernel B: the chunk products and the state recurrence
// ==================================================================================================
constexpr int kThreads = 256;
// stage: Q (2 boxes), K (2 boxes), V slice (1 box), T (1 box)
constexpr int STG_Q = 0, STG_K = C * DK * 2, STG_V = 2 * C * DK * 2, STG_T = STG_V + C * DS * 2,
              STG_BYTES = STG_T + C * C * 2;
constexpr int OFF_STG = 0;                                   // two stages
constexpr int OFF_QKM = 2 * STG_BYTES;                       // bf16 64 x 64: q_scale e^{G_i-G_j} Q K^T (j <= i)
constexpr int OFF_X = OFF_QKM + C * C * 2;                   // bf16 64 x 192: [b e^G K | b V]
constexpr int OFF_KT = OFF_X + C * (DK + DS) * 2;            // bf16 64 x 128: e^{G_C - G} K
constexpr int OFF_W = OFF_KT + C * DK * 2;                   // bf16 64 x 128: W
constexpr int OFF_U = OFF_W + C * DK * 2;                    // bf16 64 x 64: U
constexpr int OFF_SB = OFF_U + C * DS * 2;                   // bf16 128 x 64: S (bf16 copy)
constexpr int OFF_VEC = OFF_SB + DK * DS * 2;                // fp32: G[64], beta[64], eG[64], eGC[64]
constexpr int OFF_BAR = OFF_VEC + 4 * C * 4;
constexpr int kSmem = OFF_BAR + 64 + 1024;

struct ChunkArgs {
    const float *beta, *g;  // [B][T][H]
    __nv_bfloat16 *o;       // [B][T][H][dv]
    float *S;               // layer state [B][H][DK][dv]
    int B, T, H, dv, n_chunks;
    float q_scale;
    unsigned *dev_err;
};

__global__ void __launch_bounds__(kThreads, 1)
    deltanet_chunked_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                            const ChunkArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sb = smem_u32(sm);
    float *Gv = reinterpret_cast<float *>(sm + OFF_VEC), *Bv = Gv + C, *eG = Gv + 2 * C, *eGC = Gv + 3 * C;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);

    const int slice = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int mi = lane >> 3, r8 = lane & 7;
    const int n_chunks = p.n_chunks;
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
        tma_load_3d(base + STG_T, &tmT, 0, 0, (int)(bh * n_chunks + c) * C, bar);
    };
    if (tid == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmT);
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
        // ---- P0: beta, g, cumulative log decay
        load_chunk_gates(p.beta, p.g, b, h, p.H, p.T, t0, Gv, Bv);
        ok = mbar_wait(smem_u32(bars + s), (c >> 1) & 1, p.dev_err);
        if (!__syncthreads_and(ok)) {  // CTA-uniform: every thread leaves the loop together
            ok = false;
            break;
        }
        if (tid < C) {
            eG[tid] = expf(Gv[tid]);
            eGC[tid] = expf(Gv[C - 1] - Gv[tid]);
        }

        // ---- P1: Q K^T -> q_scale e^{G_i - G_j} (j <= i) as bf16; warp w: rows 16(w&3).., columns 32(w>>2)..
        {
            const int mt = warp & 3, n0 = (warp >> 2) * 32;
            float acc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
            for (int ks = 0; ks < DK / 16; ++ks) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(stg + STG_Q + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(stg + STG_K + sw(C, n0 + np * 16 + (mi >> 1) * 8 + r8, ks * 16 + (mi & 1) * 8), b0, b1, b2,
                            b3);
                    mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int i = mt * 16 + g8 + hr * 8, j = n0 + nt * 8 + 2 * t4;
                    const float v0 = j <= i ? p.q_scale * expf(Gv[i] - Gv[j]) * acc[nt][2 * hr] : 0.f;
                    const float v1 = j + 1 <= i ? p.q_scale * expf(Gv[i] - Gv[j + 1]) * acc[nt][2 * hr + 1] : 0.f;
                    *reinterpret_cast<uint32_t *>(sm + OFF_QKM + sw(C, i, j)) = pack_bf16x2(v0, v1);
                }
        }
        __syncthreads();  // eG / eGC ready

        // ---- P2: X = [b e^G K | b V], Kt = e^{G_C - G} K (bf16, swizzled)
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

        // ---- P3: [W | U'] = T X.  warps 0-3: m-tile w, W cols 0-63 and U'; warps 4-7: W cols 64-127
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
                ldsm_x4(stg + STG_T + sw(C, mt * 16 + (mi & 1) * 8 + r8, ks * 16 + (mi >> 1) * 8), a0, a1, a2, a3);
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

size_t deltanet_chunked_workspace(int B, int T, int H) {
    return (size_t)B * H * ((T + C - 1) / C) * C * C * 2;
}

cudaError_t launch_deltanet_chunked(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                    const CUtensorMap &tv, const CUtensorMap &tt, void *t_ws, const float *beta,
                                    const float *g, __nv_bfloat16 *o, float *S, int B, int T, int H, int dv,
                                    float q_scale, unsigned *dev_err, int *n_launches) {
    *n_launches = 0;
    const int n_chunks = (T + C - 1) / C;
    cudaError_t e = cudaFuncSetAttribute(chunk_solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSolveSmem);
    if (e != cudaSuccess) return e;
    chunk_solve_kernel<<<dim3(n_chunks, H, B), kSolveThreads, kSolveSmem, st>>>(
        tk, beta, g, static_cast<__nv_bfloat16 *>(t_ws), T, H, dev_err);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*n_launches;
    ChunkArgs p{beta, g, o, S, B, T, H, dv, n_chunks, q_scale, dev_err};
    e = cudaFuncSetAttribute(deltanet_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    deltanet_chunked_kernel<<<dim3(dv / DS, H, B), kThreads, kSmem, st>>>(tq, tk, tv, tt, p);
    e = cudaGetLastError();
    if (e == cudaSuccess) ++*n_launches;
    return e;
}
