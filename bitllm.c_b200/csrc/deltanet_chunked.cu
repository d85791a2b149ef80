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
//                        A, then T = (I + A)^-1 in fp32 by forward substitution (one column of T per
//                        thread, in registers); writes T diag(-b e^G) and T diag(b) as bf16 [64 x 64]
//                        each, and G, per chunk.
//   deltanet_chunked_kernel  one CTA per (sequence, head, 64-column slice of d_v): the columns of S
//                        evolve independently (column j of u depends on column j of S only), so slices
//                        need no communication.  Every chunk product runs on tcgen05 (fp32 accumulators
//                        in tensor memory; bf16 operands in shared memory, except the A operands of the
//                        state chain's products, which the prep warps write into tensor memory); the fp32
//                        state stays in registers; TMA brings q / k / v / T two chunks ahead (128-byte
//                        swizzle, no multicast).  Warp roles are described above the kernel.
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
constexpr float kLog2e = 1.4426950408889634f;
constexpr int SOL_K = 0;                      // bf16 64 x 128 K tile (TMA); later fp32 [64][64] T
constexpr int SOL_A = C * DK * 2;             // fp32 [64][FP] A
constexpr int SOL_VEC = SOL_A + C * FP * 4;   // G[64], beta[64], -beta e^G [64]
constexpr int SOL_BAR = SOL_VEC + 3 * C * 4;
constexpr int kSolveSmem = SOL_BAR + 16 + 1024;  // ~35 KB: six CTAs per SM

// Outputs per (sequence, head, chunk): Tout [128][64] bf16 = T diag(-b e^G) ; T diag(b) (the A operands
// of W and U' in the state kernel, with the minus sign of U = U' - W S folded in) and Gout [64] fp32 = G.
__global__ void __launch_bounds__(kSolveThreads, 5) chunk_solve_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                    const float *__restrict__ beta,
                                                                    const float *__restrict__ g,
                                                                    __nv_bfloat16 *__restrict__ Tout,
                                                                    float *__restrict__ Gout, int T, int H,
                                                                    unsigned *dev_err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = smem_align1024(smem_raw);
    const uint32_t sb = smem_u32(sm);
    float *Af = reinterpret_cast<float *>(sm + SOL_A), *Tf = reinterpret_cast<float *>(sm + SOL_K);
    float *Gv = reinterpret_cast<float *>(sm + SOL_VEC), *Bv = Gv + C, *Xv = Gv + 2 * C;
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
    if (tid < C) Xv[tid] = -Bv[tid] * expf(Gv[tid]);  // read after the solve's barriers

    // K K^T: warp w owns rows 16w..16w+15 and needs the columns j < 16 (w + 1) only (16-column groups
    // np <= w); A_ij = b_i e^{G_i - G_j} k_i.k_j for j < i, 0 elsewhere, kept as its transpose
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
                if (np > warp) break;  // warp-uniform
                uint32_t b0, b1, b2, b3;
                ldsm_x4(sb + SOL_K + sw(C, np * 16 + (mi >> 1) * 8 + r8, ks * 16 + (mi & 1) * 8), b0, b1, b2, b3);
                mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
                mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
            }
        }
        const int i0 = warp * 16 + g8;
        const float gi0 = Gv[i0] * kLog2e, gi1 = Gv[i0 + 8] * kLog2e, bi0 = Bv[i0], bi1 = Bv[i0 + 8];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int j = nt * 8 + 2 * t4;
            const float2 gj = *reinterpret_cast<const float2 *>(Gv + j);
            const float gj0 = gj.x * kLog2e, gj1 = gj.y * kLog2e;
            // e^{G_i - G_j} <= 1 on the SFU (ex2.approx, relative error ~2^-22); stored transposed, Af[j][i] = A_ij
            Af[j * FP + i0] = j < i0 ? bi0 * fast_exp2(gi0 - gj0) * acc[nt][0] : 0.f;
            Af[(j + 1) * FP + i0] = j + 1 < i0 ? bi0 * fast_exp2(gi0 - gj1) * acc[nt][1] : 0.f;
            Af[j * FP + i0 + 8] = j < i0 + 8 ? bi1 * fast_exp2(gi1 - gj0) * acc[nt][2] : 0.f;
            Af[(j + 1) * FP + i0 + 8] = j + 1 < i0 + 8 ? bi1 * fast_exp2(gi1 - gj1) * acc[nt][3] : 0.f;
        }
    }
    __syncthreads();  // A complete; the K tile is dead from here on (its space holds T)

    // T = (I + A)^-1 by right-looking forward substitution in fp32, one column c of T per thread of warps 0-1:
    // u = e_c in registers; at step r, t_r = u_r is final and every later row takes its share,
    // u_i -= A_ir t_r (i > r), from float4 broadcasts of row r of A^T.  No reduction or shuffle per step: the
    // dependency chain is one FMA a step.  Warp w's columns are >= 32 w, so its first 32 w steps are skipped
    // (exactly zero); rows above the diagonal come out exactly 0.
    if (warp < 2) {
        const int c = tid, r0 = 32 * warp;
        float u[C];
#pragma unroll
        for (int i = 0; i < C; ++i) u[i] = i == c ? 1.f : 0.f;
#pragma unroll
        for (int r = 0; r < C - 1; ++r) {
            if (r < r0) continue;  // warp-uniform
            const float t = u[r];
            const unsigned long long nt2 = f2_pack(-t, -t);
            const float *arow = Af + r * FP;  // A^T row r: A_ir for i = 0 .. 63
#pragma unroll
            for (int g = (r + 1) / 4; g < C / 4; ++g) {
                const float4 a4 = *reinterpret_cast<const float4 *>(arow + 4 * g);
                if (4 * g > r) {  // a whole group: two packed FMAs (fma.rn.f32x2, the same rounding as fmaf)
                    f2_unpack(ffma2(f2_pack(a4.x, a4.y), nt2, f2_pack(u[4 * g], u[4 * g + 1])), u[4 * g], u[4 * g + 1]);
                    f2_unpack(ffma2(f2_pack(a4.z, a4.w), nt2, f2_pack(u[4 * g + 2], u[4 * g + 3])), u[4 * g + 2],
                              u[4 * g + 3]);
                } else {
                    if (4 * g + 1 > r) u[4 * g + 1] = fmaf(a4.y, -t, u[4 * g + 1]);
                    if (4 * g + 2 > r) u[4 * g + 2] = fmaf(a4.z, -t, u[4 * g + 2]);
                    u[4 * g + 3] = fmaf(a4.w, -t, u[4 * g + 3]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < C; ++i) Tf[i * C + c] = u[i];
    }
    __syncthreads();
    // T diag(-b e^G) ; T diag(b) (T lower triangular) -> bf16 rows of 64 for the state kernel's TMA; G
    const size_t chunk_ix = ((size_t)b * H + h) * n_chunks + c;
    __nv_bfloat16 *dst = Tout + chunk_ix * 2 * C * C;
    for (int e = tid; e < C * C / 8; e += kSolveThreads) {  // T is exactly 0 above the diagonal
        const int i = e >> 3, j0 = (e & 7) * 8;
        const float4 ta = *reinterpret_cast<const float4 *>(Tf + i * C + j0);
        const float4 tb = *reinterpret_cast<const float4 *>(Tf + i * C + j0 + 4);
        const float4 xa = *reinterpret_cast<const float4 *>(Xv + j0), xb = *reinterpret_cast<const float4 *>(Xv + j0 + 4);
        const float4 ba = *reinterpret_cast<const float4 *>(Bv + j0), bb = *reinterpret_cast<const float4 *>(Bv + j0 + 4);
        const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
        uint32_t w1[4], w2[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            w1[q] = pack_bf16x2(tv[2 * q] * xv[2 * q], tv[2 * q + 1] * xv[2 * q + 1]);
            w2[q] = pack_bf16x2(tv[2 * q] * bv[2 * q], tv[2 * q + 1] * bv[2 * q + 1]);
        }
        *reinterpret_cast<uint4 *>(dst + i * C + j0) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
        *reinterpret_cast<uint4 *>(dst + C * C + i * C + j0) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
    }
    if (tid < C) Gout[chunk_ix * C + tid] = Gv[tid];
}

// ==================================================================================================
// Kernel B: the chunk products on tcgen05 and the state recurrence
// ==================================================================================================
// Products of chunk c (M = 128 TMEM lanes, fp32 accumulators; "lanes 0-63" are the chunk's tokens in the
// upper half, "lanes 64-127" in the lower half).  Slot s = c & 1 of TMEM holds 192 columns:
//   Dp[:, 0:128]   = [T2 ; T1] K            lanes 64-127: -W (prep MMA; lanes 0-63 dead)
//   Dp[:, 128:192] = [0 ; T2] V             lanes 64-127: U'
//   A1 = Dp[:, 0:64] as bf16 pairs          lanes 0-63: Q~ (prep warps 4-5), lanes 64-127: -W (prep warps 6-7,
//                                           converted in place)
//   A2 = Dp[:, 64:96] as bf16 pairs         lanes 0-63: QKm (prep warps 4-5); lanes 64-127 dead
//   Dp[:, 128:192] += A1 S                  lanes 0-63: Q~ S, lanes 64-127: U = U' - W S    (tensor-memory A)
//   Ds  = Kt^T U                            S_next = e^{G_C} S + Ds
//   Dp[:, 128:192] += A2 U                  lanes 0-63: O (lanes 64-127 are dead by then)  (tensor-memory A)
//   Dq  = [Q ; *] K^T                       lanes 0-63: Q K^T (prep)
// with T1 = T diag(-b e^G), T2 = T diag(b) (from chunk_solve_kernel), Q~ = q_scale e^G Q,
// Kt = e^{G_C - G} K and QKm = q_scale e^{G_i - G_j} Q K^T (j <= i); "*" rows only reach dead lanes.
// The chain's A operands never touch shared memory: the tensor cores read them from TMEM, and shared memory
// carries only the B operands (S, U), the TMA stages and Kt -- the kernel is bound by shared-memory traffic
// and the chain's round trips, so this is what sets its speed.
// Roles (352 threads):
//   warps 0-3  state: thread r owns row r of the fp32 state slice (64 columns, registers) and TMEM lane r;
//              all four form the next S (bf16 copy for the MMA); warps 2-3 turn U (lanes 64-127) into the bf16
//              B operand; warps 0-1 store O (lanes 0-63).
//   warps 4-7  prep, ahead of the state by up to two chunks: warps 4-5 (lanes 0-63) QKm from Dq and Q~ from the
//              TMA stage into A1 / A2; warps 6-7 (lanes 64-127) -W into A1, Kt into its shared buffer (two).
//   warp 8     MMA issuer of the state chain; owns the TMEM allocation.
//   warp 9     MMA issuer of the prep products (Dq, Dp).
//   warp 10    TMA producer (two stages); its lanes also copy the chunk's G into the stage.
// Every wait is a bounded mbarrier wait; the prep warps agree on aborting through a barrier reduction.
constexpr int kThreads = 352;
// one stage: [Q box0 | K box0 | Q box1 | K box1] 32 KB, V 8 KB, zeros 8 KB, T2 8 KB, T1 8 KB, G 256 B
// ([0 ; T2] and [T2 ; T1] are the A operands of U' and -W: 128 rows from one start)
constexpr int SL_V = 32768, SL_Z = 40960, SL_T2 = 49152, SL_T1 = 57344, SL_G = 65536, SLOT = 66560;
constexpr int STAGE_TX = 57344;               // bytes TMA brings per stage
constexpr int OFF_KT = 2 * SLOT;              // Kt of chunks c & 1 = 0 / 1, 2 boxes each
constexpr int OFF_SB = OFF_KT + 32768;        // S slice, bf16 [128 key rows][64 columns]
constexpr int OFF_U = OFF_SB + 16384;         // U, bf16 [64 tokens][64 columns]
constexpr int OFF_VEC = OFF_U + 8192;         // bf16x2 pairs q_scale e^G, e^{G_C - G}; fp32 e^{g} [64 each]; e^{G_C} ring [4]
constexpr int OFF_BAR = OFF_VEC + 1024;
constexpr int kSmem = OFF_BAR + 256 + 1024;
constexpr int TM_DS = 384, TM_DQ = 448, kTmemCols = 512;  // Dp of slot s at columns 192 s

enum {
    B_FULL = 0,      // [2] stage landed (TMA tx + G copied)
    B_EMPTY = 2,     // [2] stage consumed (prep MMAs + 128 prep threads)
    B_QDONE = 4,     // Dq ready
    B_DQFREE = 5,    // Dq read (warps 4-5)
    B_PDONE = 6,     // [2] Dp of the slot ready; the slot's A1 / A2 and Kt buffer free to write
    B_DPFREE = 8,    // [2] O of the slot read (warps 0-1)
    B_PREP = 10,     // [2] A1, A2, Kt and the gates of the chunk written (prep)
    B_M1 = 12,       // S product done: U in TMEM
    B_UREADY = 13,   // U written (warps 2-3)
    B_DS = 14,       // Ds done; U's first reader done
    B_ODONE = 15,    // [2] O of the slot done
    B_SREADY = 17,   // next S written (state)
    B_COUNT = 18
};

struct ChunkArgs {
    const float *G;         // [B][H][n_chunks][64] cumulative log decays (chunk_solve_kernel)
    __nv_bfloat16 *o;       // [B][T][H][dv] bf16, unless o_f32 is set
    float *o_f32;           // [B][T][H][dv] fp32 output, or null
    float *S;               // layer state [B][H][DK][dv]
    int B, T, H, dv, n_chunks;
    float q_scale;
    unsigned *dev_err;
};

__device__ __forceinline__ uint32_t swz(int row, int u) { return (uint32_t)(row * 128 + ((u ^ (row & 7)) << 4)); }

// 8 bf16 times a bf16 scale given as a duplicated pair
__device__ __forceinline__ uint4 scale8(uint4 v, uint32_t f2) {
    return make_uint4(bf16x2_mul(v.x, f2), bf16x2_mul(v.y, f2), bf16x2_mul(v.z, f2), bf16x2_mul(v.w, f2));
}

// 64 fp32 values -> one 128-byte swizzled bf16 row (times `f`)
__device__ __forceinline__ void store_row64(uint8_t *box, int row, const float *v, float f) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
        *reinterpret_cast<uint4 *>(box + swz(row, u)) =
            make_uint4(pack_bf16x2(v[8 * u] * f, v[8 * u + 1] * f), pack_bf16x2(v[8 * u + 2] * f, v[8 * u + 3] * f),
                       pack_bf16x2(v[8 * u + 4] * f, v[8 * u + 5] * f), pack_bf16x2(v[8 * u + 6] * f, v[8 * u + 7] * f));
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(v));
    tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(v + 32));
}

__global__ void __launch_bounds__(kThreads, 1)
    deltanet_chunked_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                            const ChunkArgs p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *sm = smem_align1024(smem_raw);
    const uint32_t sb = smem_u32(sm);
    uint32_t *fq2 = reinterpret_cast<uint32_t *>(sm + OFF_VEC), *fk2 = fq2 + C;
    float *decv = reinterpret_cast<float *>(fq2 + 2 * C), *dCv = decv + C;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + B_COUNT);

    const int slice = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_chunks = p.n_chunks;
    const size_t bh = (size_t)b * p.H + h;

    if (tid == 0) {
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(B_FULL + s), 2);
            mbar_init(bar(B_EMPTY + s), 1 + 128);
            mbar_init(bar(B_DPFREE + s), 64);
            mbar_init(bar(B_PREP + s), 128);
        }
        mbar_init(bar(B_QDONE), 1);
        mbar_init(bar(B_DQFREE), 64);
        mbar_init(bar(B_PDONE), 1);
        mbar_init(bar(B_PDONE + 1), 1);
        mbar_init(bar(B_M1), 1);
        mbar_init(bar(B_UREADY), 64);
        mbar_init(bar(B_DS), 1);
        mbar_init(bar(B_ODONE), 1);
        mbar_init(bar(B_ODONE + 1), 1);
        mbar_init(bar(B_SREADY), 128);
        fence_barrier_init();
    }
    // zero rows 0-63 of the [0 ; T2] operand of both stages (TMA never writes them)
    for (int e = tid; e < 2 * 512; e += kThreads)
        reinterpret_cast<uint4 *>(sm + (e >> 9) * SLOT + SL_Z)[e & 511] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    if (warp == 8) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4) {
        // ------------------------------------------------------------------ state
        const int r = tid;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float S[64];
        float *Sg = p.S + (bh * DK + r) * p.dv + slice * DS;
#pragma unroll
        for (int j = 0; j < 64; j += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(Sg + j);
            S[j] = v.x;
            S[j + 1] = v.y;
            S[j + 2] = v.z;
            S[j + 3] = v.w;
        }
        store_row64(sm + OFF_SB, r, S, 1.f);
        fence_proxy_async_smem();
        mbar_arrive(bar(B_SREADY));
        bool ok = true;
        for (int c = 0; c < n_chunks; ++c) {
            const int slot = c & 1;
            const uint32_t dcol = tmem + lane_off + slot * 192 + 128;
            if (!mbar_wait(bar(B_PREP + slot), (c >> 1) & 1, p.dev_err)) { ok = false; break; }
            const float dC = dCv[c & 3];
            if (warp >= 2) {  // U (lanes 64-127) -> the bf16 B operand of Ds and O
                if (!mbar_wait(bar(B_M1), c & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
                float u[64];
                tmem_ld64(dcol, u);
                tmem_wait_ld();
                store_row64(sm + OFF_U, r - 64, u, 1.f);
                fence_proxy_async_smem();
                tc_fence_before();
                mbar_arrive(bar(B_UREADY));
            }
            if (!mbar_wait(bar(B_DS), c & 1, p.dev_err)) { ok = false; break; }
            tc_fence_after();
            {
                float d[64];
                tmem_ld64(tmem + lane_off + TM_DS, d);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 64; ++j) S[j] = fmaf(dC, S[j], d[j]);
            }
            store_row64(sm + OFF_SB, r, S, 1.f);
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(B_SREADY));
            if (warp < 2) {  // O (lanes 0-63)
                if (!mbar_wait(bar(B_ODONE + slot), (c >> 1) & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
                float o[64];
                tmem_ld64(dcol, o);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(bar(B_DPFREE + slot));
                const int t = c * C + r;
                if (t < p.T) {
                    const size_t orow = (((size_t)b * p.T + t) * p.H + h) * p.dv + slice * DS;
                    store_scaled32(p.o + orow, p.o_f32 ? p.o_f32 + orow : nullptr, *reinterpret_cast<float(*)[32]>(o),
                                   1.f);
                    store_scaled32(p.o + orow + 32, p.o_f32 ? p.o_f32 + orow + 32 : nullptr,
                                   *reinterpret_cast<float(*)[32]>(o + 32), 1.f);
                }
            }
        }
        if (ok) {
#pragma unroll
            for (int j = 0; j < 64; j += 4) *reinterpret_cast<float4 *>(Sg + j) = make_float4(S[j], S[j + 1], S[j + 2], S[j + 3]);
        }
    } else if (warp < 8) {
        // ------------------------------------------------------------------ prep
        const int pt = tid - 128, pw = warp - 4;
        const uint32_t lane_off = (uint32_t)(pw * 32) << 16;
        for (int c = 0; c < n_chunks; ++c) {
            const int s = c & 1;
            uint8_t *stg = sm + s * SLOT;
            const float *Gst = reinterpret_cast<const float *>(stg + SL_G);
            bool ok = mbar_wait(bar(B_FULL + s), (c >> 1) & 1, p.dev_err);
            if (pt < C) {  // per-token scales as duplicated bf16 pairs, per-token decays e^{g}, and e^{G_C}
                const float G = ok ? Gst[pt] : 0.f, GC = ok ? Gst[C - 1] : 0.f;
                const float Gp = ok && pt > 0 ? Gst[pt - 1] : 0.f;
                const uint32_t q1 = pack_bf16x2(p.q_scale * expf(G), 0.f) & 0xffffu;
                const uint32_t k1 = pack_bf16x2(expf(GC - G), 0.f) & 0xffffu;
                fq2[pt] = q1 | (q1 << 16);
                fk2[pt] = k1 | (k1 << 16);
                decv[pt] = expf(G - Gp);
                if (pt == 0) dCv[c & 3] = expf(GC);
            }
            named_bar_sync(1, 128);
            const uint32_t a1 = tmem + lane_off + s * 192;  // A1 = slot columns 0-63, A2 = 64-95
            if (pw < 2) {
                const int i = pt;
                // QKm row i from Dq
                if (ok) ok = mbar_wait(bar(B_QDONE), c & 1, p.dev_err);
                float a[64];
                if (ok) {
                    tc_fence_after();
                    tmem_ld64(tmem + lane_off + TM_DQ, a);
                    tmem_wait_ld();
                }
                tc_fence_before();
                mbar_arrive(bar(B_DQFREE));
                uint32_t qk[32];
                {
                    const int jmax = pw * 32 + 31;
                    float e = p.q_scale;
#pragma unroll
                    for (int u = 7; u >= 0; --u) {
                        if (8 * u > jmax) {
#pragma unroll
                            for (int q = 0; q < 8; ++q) a[8 * u + q] = 0.f;
                            continue;
                        }
                        const float4 d0 = reinterpret_cast<const float4 *>(decv)[2 * u];
                        const float4 d1 = reinterpret_cast<const float4 *>(decv)[2 * u + 1];
                        const float d[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
                        for (int q = 7; q >= 0; --q) {
                            const int j = 8 * u + q;
                            const bool in = j <= i;
                            a[j] = in ? e * a[j] : 0.f;
                            e = in ? e * d[q] : e;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 32; ++q) qk[q] = pack_bf16x2(a[2 * q], a[2 * q + 1]);
                }
                if (ok) ok = mbar_wait(bar(B_PDONE + s), (c >> 1) & 1, p.dev_err);
                if (ok) {
                    tc_fence_after();
                    tmem_st32u(a1 + 64, qk);
                    // Q~ row i = q_scale e^{G_i} Q row i (bf16 products) from the stage's two Q boxes, one box
                    // (32 columns of pairs) at a time
                    const uint32_t f2 = fq2[i];
#pragma unroll
                    for (int bx = 0; bx < 2; ++bx) {
                        uint32_t qt[32];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const uint4 v = scale8(*reinterpret_cast<const uint4 *>(stg + bx * 16384 + swz(i, u)), f2);
                            qt[4 * u] = v.x;
                            qt[4 * u + 1] = v.y;
                            qt[4 * u + 2] = v.z;
                            qt[4 * u + 3] = v.w;
                        }
                        tmem_st32u(a1 + 32 * bx, qt);
                    }
                }
                mbar_arrive(bar(B_EMPTY + s));  // last read of the stage by this thread
            } else {
                // thread q handles 16-byte unit q & 7 of rows (q >> 3) + 8 m (m < 8) of both 64-column boxes:
                // the swizzled offset is a per-thread constant plus 1024 m
                const int q = pt - 64, j0 = q >> 3;
                const uint32_t off0 = swz(j0, q & 7);
                uint4 t[16];
#pragma unroll
                for (int n = 0; n < 16; ++n)  // Kt = e^{G_C - G} K
                    t[n] = *reinterpret_cast<const uint4 *>(stg + (n >> 3) * 16384 + 8192 + off0 + (n & 7) * 1024);
#pragma unroll
                for (int n = 0; n < 16; ++n) t[n] = scale8(t[n], fk2[j0 + 8 * (n & 7)]);
                mbar_arrive(bar(B_EMPTY + s));
                // the slot's Dp has landed, and with it the Kt buffer of chunk c - 2 is free (its O product
                // completed before the O read that let the prep issuer fill this slot)
                if (ok) ok = mbar_wait(bar(B_PDONE + s), (c >> 1) & 1, p.dev_err);
                if (ok) {
#pragma unroll
                    for (int n = 0; n < 16; ++n)
                        *reinterpret_cast<uint4 *>(sm + OFF_KT + s * 16384 + (n >> 3) * 8192 + off0 + (n & 7) * 1024) =
                            t[n];
                    // -W (lanes 64-127, fp32 columns 0-127) -> bf16 pairs in columns 0-63, in place: each half is
                    // read completely before its pairs overwrite the columns it came from
                    tc_fence_after();
#pragma unroll 1
                    for (int hh = 0; hh < 2; ++hh) {
                        float w[64];
                        tmem_ld64(a1 + 64 * hh, w);
                        tmem_wait_ld();
                        uint32_t wp[32];
#pragma unroll
                        for (int k2 = 0; k2 < 32; ++k2) wp[k2] = pack_bf16x2(w[2 * k2], w[2 * k2 + 1]);
                        tmem_st32u(a1 + 32 * hh, wp);
                    }
                }
            }
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(B_PREP + s));
            if (!named_bar_and(1, 128, ok)) break;  // uniform: the scale vectors are rewritten next chunk
        }
    } else if (warp == 8) {
        // ------------------------------------------------------------------ state-chain MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_kmn = umma_idesc_bf16(128, 64, false, true);
            constexpr uint32_t id_mnmn = umma_idesc_bf16(128, 64, true, true);
            int last_bar = -1;
            uint32_t last_par = 0;
            for (int c = 0; c < n_chunks; ++c) {
                const int slot = c & 1;
                const uint32_t dcol = tmem + slot * 192 + 128, a1 = tmem + slot * 192;
                if (!mbar_wait(bar(B_SREADY), c & 1, p.dev_err)) break;
                if (!mbar_wait(bar(B_PREP + slot), (c >> 1) & 1, p.dev_err)) break;
                tc_fence_after();
                // [Q~ ; -W] S: A from tensor memory (8 columns of bf16 pairs per K step of 16)
#pragma unroll
                for (int ks = 0; ks < 8; ++ks)
                    umma_bf16_ts(dcol, a1 + ks * 8, umma_desc_sw128(sb + OFF_SB + ks * 2048, 8192, 1024), id_kmn, 1);
                umma_commit(bar(B_M1));
                last_bar = B_M1;
                last_par = c & 1;
                if (!mbar_wait(bar(B_UREADY), c & 1, p.dev_err)) break;
                tc_fence_after();
                // Ds = Kt^T U first (the state chain waits for it), then O += QKm U
                const uint32_t kt = sb + OFF_KT + slot * 16384;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + TM_DS, umma_desc_sw128(kt + kk * 2048, 8192, 1024),
                                 umma_desc_sw128(sb + OFF_U + kk * 2048, 8192, 1024), id_mnmn, kk > 0);
                umma_commit(bar(B_DS));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ts(dcol, a1 + 64 + kk * 8, umma_desc_sw128(sb + OFF_U + kk * 2048, 8192, 1024), id_kmn, 1);
                umma_commit(bar(B_ODONE + slot));
                last_bar = B_ODONE + slot;
                last_par = (c >> 1) & 1;
            }
            if (last_bar >= 0) mbar_wait(bar(last_bar), last_par, p.dev_err);  // own MMAs drained
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------ prep MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_q = umma_idesc_bf16(128, 64, false, false);
            constexpr uint32_t id_w = umma_idesc_bf16(128, 128, false, true);
            constexpr uint32_t id_u = umma_idesc_bf16(128, 64, false, true);
            int last_bar = -1;
            uint32_t last_par = 0;
            for (int c = 0; c < n_chunks; ++c) {
                const int s = c & 1;
                const uint32_t stg = sb + s * SLOT;
                if (!mbar_wait(bar(B_FULL + s), (c >> 1) & 1, p.dev_err)) break;
                if (c >= 1 && !mbar_wait(bar(B_DQFREE), (c - 1) & 1, p.dev_err)) break;
                tc_fence_after();
#pragma unroll
                for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_bf16_ss(tmem + TM_DQ, umma_desc_sw128(stg + kb * 16384 + kk * 32, 16, 1024),
                                     umma_desc_sw128(stg + kb * 16384 + 8192 + kk * 32, 16, 1024), id_q, kb | kk);
                umma_commit(bar(B_QDONE));
                last_bar = B_QDONE;
                last_par = c & 1;
                if (c >= 2 && !mbar_wait(bar(B_DPFREE + s), ((c - 2) >> 1) & 1, p.dev_err)) break;
                tc_fence_after();
                // -W = T1 K into lanes 64-127 (A = [T2 ; T1]; B = K key-major: two 64-column groups 16 KB apart)
                // and U' = T2 V into lanes 64-127 (A = [0 ; T2])
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + s * 192, umma_desc_sw128(stg + SL_T2 + kk * 32, 16, 1024),
                                 umma_desc_sw128(stg + 8192 + kk * 2048, 16384, 1024), id_w, kk > 0);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_bf16_ss(tmem + s * 192 + 128, umma_desc_sw128(stg + SL_Z + kk * 32, 16, 1024),
                                 umma_desc_sw128(stg + SL_V + kk * 2048, 8192, 1024), id_u, kk > 0);
                umma_commit(bar(B_PDONE + s));
                umma_commit(bar(B_EMPTY + s));
                last_bar = B_PDONE + s;
                last_par = (c >> 1) & 1;
            }
            if (last_bar >= 0) mbar_wait(bar(last_bar), last_par, p.dev_err);  // own MMAs drained
        }
    } else {
        // ------------------------------------------------------------------ TMA producer (+ G copy)
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            prefetch_tmap(&tmT);
        }
        int issued = 0;
        for (int c = 0; c < n_chunks; ++c) {
            const int s = c & 1;
            const bool free_ok = c < 2 || mbar_wait(bar(B_EMPTY + s), ((c - 2) >> 1) & 1, p.dev_err);
            if (!__all_sync(0xffffffffu, free_ok)) break;
            const uint32_t stg = sb + s * SLOT, full = bar(B_FULL + s);
            const size_t chunk_ix = bh * n_chunks + c;
            if (lane == 0) {
                const int row = b * p.T + c * C;
                mbar_arrive_expect_tx(full, STAGE_TX);
#pragma unroll
                for (int d = 0; d < 2; ++d) {
                    tma_load_3d(stg + d * 16384, &tmQ, d * 64, h, row, full);
                    tma_load_3d(stg + d * 16384 + 8192, &tmK, d * 64, h, row, full);
                }
                tma_load_3d(stg + SL_V, &tmV, slice * DS, h, row, full);
                tma_load_3d(stg + SL_T1, &tmT, 0, 0, (int)chunk_ix * 2 * C, full);
                tma_load_3d(stg + SL_T2, &tmT, 0, 0, (int)chunk_ix * 2 * C + C, full);
            }
            reinterpret_cast<float2 *>(sm + s * SLOT + SL_G)[lane] =
                __ldg(reinterpret_cast<const float2 *>(p.G + chunk_ix * C) + lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(full);
            issued = c + 1;
        }
        // every issued load has landed before the CTA may exit (bounded)
        if (lane == 0)
            for (int c = max(0, issued - 2); c < issued; ++c) mbar_wait(bar(B_FULL + (c & 1)), (c >> 1) & 1, p.dev_err);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

bool deltanet_chunked_supported(int dk, int dv) { return dk == DK && dv % DS == 0 && dv <= 256; }

size_t deltanet_chunked_tmat_bytes(int B, int T, int H) { return (size_t)B * H * ((T + C - 1) / C) * 2 * C * C * 2; }

size_t deltanet_chunked_workspace(int B, int T, int H) {
    return deltanet_chunked_tmat_bytes(B, T, H) + (size_t)B * H * ((T + C - 1) / C) * C * 4;
}

cudaError_t launch_deltanet_chunked(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                    const CUtensorMap &tv, const CUtensorMap &tt, void *t_ws, const float *beta,
                                    const float *g, __nv_bfloat16 *o, float *o_f32, float *S, int B, int T, int H,
                                    int dv, float q_scale, unsigned *dev_err, int *n_launches) {
    *n_launches = 0;
    const int n_chunks = (T + C - 1) / C;
    cudaError_t e = cudaFuncSetAttribute(chunk_solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSolveSmem);
    if (e != cudaSuccess) return e;
    float *Gws = reinterpret_cast<float *>(static_cast<char *>(t_ws) + deltanet_chunked_tmat_bytes(B, T, H));
    chunk_solve_kernel<<<dim3(n_chunks, H, B), kSolveThreads, kSolveSmem, st>>>(
        tk, beta, g, static_cast<__nv_bfloat16 *>(t_ws), Gws, T, H, dev_err);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ++*n_launches;
    ChunkArgs p{Gws, o, o_f32, S, B, T, H, dv, n_chunks, q_scale, dev_err};
    e = cudaFuncSetAttribute(deltanet_chunked_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    deltanet_chunked_kernel<<<dim3(dv / DS, H, B), kThreads, kSmem, st>>>(tq, tk, tv, tt, p);
    e = cudaGetLastError();
    if (e == cudaSuccess) ++*n_launches;
    return e;
}
