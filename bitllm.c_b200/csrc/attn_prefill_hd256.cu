// attn_prefill_hd256.cu -- causal GQA prefill attention for head_dim 256 (Qwen3.5 full attention) on the
// B200 5th-generation tensor cores.
//
// Reference: Qwen3.5's prefill_chunk runs fullatt_attend once per token (src/eif_qwen35.c:1122-1133; the
// attention core at :741-771): token i of the chunk, at position start_pos + i, attends to cache rows
// 0 .. start_pos + i; softmax(scale * q.k) . v per query head with kv head = h / (Hq / Hkv).
//
// Why a kernel of its own: at head_dim 256 the two-query-tile design of attn_prefill_tc.cu would need
// 2 x 256 TMEM columns for the O accumulators alone, plus S.  Here one CTA = one 128-row query tile of
// one (sequence, query head), key tiles of 64 keys, and S double-buffered in TMEM so that the tensor
// cores compute S(j+1) = Q K_{j+1}^T while the softmax warps work on S(j).  6 warps:
//   warp 4      TMA producer: Q once (four 64-dim boxes), then K and V tiles of 64 keys (four boxes each)
//               into double-buffered 128-byte-swizzled rings (no multicast);
//   warp 5      MMA issuer, one thread: S(j) = Q K_j^T into S[j & 1] (A, B from smem), then
//               O += P(j-1) V_{j-1} with P read from TMEM (TS form) and V from smem;
//   warps 0-3   softmax, thread r = query row r = TMEM lane r: tile max with the causal mask, the running
//               max kept while a tile stays within 2^8 of it (O is rescaled in TMEM only when a row's max
//               really moves, and only by the warps that have such a row), p = 2^(scale*s - m) written as
//               bf16 pairs over the first 32 columns of S[j & 1]; at the end O / l -> bf16 -> global.
// TMEM: S0 [0, 64), S1 [64, 128), O [128, 384).
// Work order: the longest causal rows first.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int BM = 128, BN = 64, HD = 256;
constexpr int kThreads = 192;
constexpr int QBOX = BM * 128;   // 16 KB: 64 dims of the 128 query rows
constexpr int KBOX = BN * 128;   // 8 KB: 64 dims of the 64 keys
constexpr int KVTILE = 4 * KBOX;  // 32 KB
constexpr int OFF_Q = 0, OFF_K = 4 * QBOX, OFF_V = OFF_K + 2 * KVTILE, OFF_BAR = OFF_V + 2 * KVTILE;
constexpr int kSmem = OFF_BAR + 256 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t TM_O = 128;
constexpr float kRescaleLog2 = 8.0f;

enum {
    BAR_Q = 0,
    BAR_KFULL = 1,   // [2]
    BAR_KEMPTY = 3,  // [2]
    BAR_VFULL = 5,   // [2]
    BAR_VEMPTY = 7,  // [2]
    BAR_SFULL = 9,   // [2] S buffer holds S(j)
    BAR_PFULL = 11,  // [2] S buffer holds P(j) (4 softmax warps)
    BAR_PEMPTY = 13, // PV(j) done (one phase per key tile)
    BAR_COUNT = 14
};

struct Params {
    int B, n_tok, start_pos, Hq, G, max_seq, n_tiles;
    float scale_log2;
    __nv_bfloat16 *out;  // bf16 output, unless out_f32 is set
    float *out_f32;
    unsigned *dev_err;
};

template <bool MASK>
__device__ __forceinline__ void tile_max32(const float (&x)[32], float scale, int lim, float &mt) {
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float v0 = x[i] * scale, v1 = x[i + 1] * scale;
        if (MASK) {
            if (i > lim) v0 = -INFINITY;
            if (i + 1 > lim) v1 = -INFINITY;
        }
        mt = fmax3(mt, v0, v1);
    }
}

template <bool MASK>
__device__ __forceinline__ void tile_exp32(const float (&x)[32], float scale, float m_use, int lim,
                                           unsigned long long &sum2, uint32_t *pk) {
    const unsigned long long sc2 = f2_pack(scale, scale), nm2 = f2_pack(-m_use, -m_use);
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
        float v0, v1;
        f2_unpack(ffma2(f2_pack(x[i], x[i + 1]), sc2, nm2), v0, v1);
        if (MASK) {
            if (i > lim) v0 = -INFINITY;
            if (i + 1 > lim) v1 = -INFINITY;
        }
        const float e0 = fast_exp2(v0), e1 = fast_exp2(v1);
        sum2 = fadd2(sum2, f2_pack(e0, e1));
        pk[i / 2] = pack_bf16x2(e0, e1);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_hd256_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + BAR_COUNT + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per_tile = p.B * p.Hq;
    const int tile = p.n_tiles - 1 - (int)blockIdx.x / per_tile;  // heaviest first
    const int rem = (int)blockIdx.x % per_tile;
    const int b = rem / p.Hq, h = rem - b * p.Hq, kvh = h / p.G;
    const int q0 = tile * BM;
    const int rows = min(BM, p.n_tok - q0);
    const int nkv = (p.start_pos + q0 + rows - 1) / BN + 1;
    const int kv_end = p.start_pos + p.n_tok;  // rows at or past this were not written by this prefill

    if (threadIdx.x == 0) {
        mbar_init(bar(BAR_Q), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(BAR_KFULL + s), 1);
            mbar_init(bar(BAR_KEMPTY + s), 1);
            mbar_init(bar(BAR_VFULL + s), 1);
            mbar_init(bar(BAR_VEMPTY + s), 1);
            mbar_init(bar(BAR_SFULL + s), 1);
            mbar_init(bar(BAR_PFULL + s), 4);
        }
        mbar_init(bar(BAR_PEMPTY), 1);
        fence_barrier_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_arrive_expect_tx(bar(BAR_Q), 4 * QBOX);
            for (int d = 0; d < 4; ++d)
                tma_load_3d(sbase + OFF_Q + d * QBOX, &tmQ, d * 64, h, b * p.n_tok + q0, bar(BAR_Q));
            for (int j = 0; j < nkv; ++j) {
                const int s = j & 1;
                const uint32_t par = ((j >> 1) & 1) ^ 1;
                const int row = b * p.max_seq + j * BN;
                if (!mbar_wait(bar(BAR_KEMPTY + s), par, p.dev_err)) break;
                mbar_arrive_expect_tx(bar(BAR_KFULL + s), KVTILE);
                for (int d = 0; d < 4; ++d)
                    tma_load_3d(sbase + OFF_K + s * KVTILE + d * KBOX, &tmK, d * 64, kvh, row, bar(BAR_KFULL + s));
                if (!mbar_wait(bar(BAR_VEMPTY + s), par, p.dev_err)) break;
                mbar_arrive_expect_tx(bar(BAR_VFULL + s), KVTILE);
                for (int d = 0; d < 4; ++d)
                    tma_load_3d(sbase + OFF_V + s * KVTILE + d * KBOX, &tmV, d * 64, kvh, row, bar(BAR_VFULL + s));
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_qk = umma_idesc_bf16(BM, BN, false, false);
        constexpr uint32_t idesc_pv = umma_idesc_bf16(BM, HD, false, true);
        bool ok = mbar_wait(bar(BAR_Q), 0, p.dev_err);
        for (int j = 0; ok && j <= nkv; ++j) {
            if (j < nkv) {
                // S(j) = Q K_j^T into S[j & 1] (P(j-2) there was consumed by PV(j-2), issued earlier)
                const int s = j & 1;
                if (!mbar_wait(bar(BAR_KFULL + s), (j >> 1) & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t kb = sbase + OFF_K + s * KVTILE;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_bf16_ss(tmem + s * BN,
                                     umma_desc_sw128(sbase + OFF_Q + (kk >> 2) * QBOX + (kk & 3) * 32, 16, 1024),
                                     umma_desc_sw128(kb + (kk >> 2) * KBOX + (kk & 3) * 32, 16, 1024), idesc_qk, kk > 0);
                    umma_commit(bar(BAR_SFULL + s));
                    umma_commit(bar(BAR_KEMPTY + s));
                }
                __syncwarp();
            }
            if (j >= 1) {
                const int jj = j - 1, sv = jj & 1;
                if (!mbar_wait(bar(BAR_VFULL + sv), (jj >> 1) & 1, p.dev_err)) { ok = false; break; }
                const int first_bad = kv_end - jj * BN;  // keys of tile jj at or past kv_end
                if (first_bad < BN) {
                    // their p is 0, but 0 * (a non-finite stale row) would be NaN: zero those V rows
                    for (int r = max(first_bad, 0); r < BN; ++r)
                        for (int d = 0; d < 4; ++d)
                            if (lane < 8)
                                reinterpret_cast<uint4 *>(smem + OFF_V + sv * KVTILE + d * KBOX + r * 128)[lane] =
                                    make_uint4(0, 0, 0, 0);
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                if (!mbar_wait(bar(BAR_PFULL + sv), (jj >> 1) & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t vb = sbase + OFF_V + sv * KVTILE;
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)
                        umma_bf16_ts(tmem + TM_O, tmem + sv * BN + kk * 8, umma_desc_sw128(vb + kk * 2048, KBOX, 1024),
                                     idesc_pv, (jj > 0 || kk > 0));
                    umma_commit(bar(BAR_PEMPTY));
                    umma_commit(bar(BAR_VEMPTY + sv));
                }
                __syncwarp();
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warps 0-3
        const int r = threadIdx.x;  // query row of the tile == TMEM lane
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const uint32_t o_col = tmem + lane_base + TM_O;
        const int qpos = p.start_pos + q0 + r;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            const int s = j & 1;
            const uint32_t s_col = tmem + lane_base + s * BN;
            if (!mbar_wait(bar(BAR_SFULL + s), (j >> 1) & 1, p.dev_err)) { ok = false; break; }
            tc_fence_after();
            const int kbase = j * BN;
            const bool diag = kbase + BN - 1 > p.start_pos + q0;
            const int lim = qpos - kbase;  // columns past lim are masked on diagonal tiles
            float x[32], y[32];
            tmem_ld32(s_col, x);
            tmem_ld32(s_col + 32, y);
            tmem_wait_ld();
            float mt = -INFINITY;
            if (diag) {
                tile_max32<true>(x, p.scale_log2, lim, mt);
                tile_max32<true>(y, p.scale_log2, lim - 32, mt);
            } else {
                tile_max32<false>(x, p.scale_log2, 0, mt);
                tile_max32<false>(y, p.scale_log2, 0, mt);
            }
            const bool grow = m == -INFINITY ? mt > -INFINITY : mt > m + kRescaleLog2;
            const float m_new = grow ? mt : m;
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float corr = grow ? fast_exp2(m - m_use) : 1.f;
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                // PV(j-1) must be complete before O is rescaled
                if (!mbar_wait(bar(BAR_PEMPTY), (j - 1) & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    float o[32];
                    tmem_ld32(o_col + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= corr;
                    tmem_st32(o_col + c * 32, o);
                }
                tmem_wait_st();
            }
            unsigned long long sum2 = 0;
            uint32_t pk[32];
            if (diag) {
                tile_exp32<true>(x, p.scale_log2, m_use, lim, sum2, pk);
                tile_exp32<true>(y, p.scale_log2, m_use, lim - 32, sum2, pk + 16);
            } else {
                tile_exp32<false>(x, p.scale_log2, m_use, 0, sum2, pk);
                tile_exp32<false>(y, p.scale_log2, m_use, 0, sum2, pk + 16);
            }
            tmem_st32u(s_col, pk);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_PFULL + s));
            float s0, s1;
            f2_unpack(sum2, s0, s1);
            l = l * corr + (s0 + s1);
            m = m_new;
        }
        if (ok && mbar_wait(bar(BAR_PEMPTY), (nkv - 1) & 1, p.dev_err)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            const size_t orow = (((size_t)b * p.n_tok + q0 + r) * p.Hq + h) * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float o[32];
                tmem_ld32(o_col + c * 32, o);
                tmem_wait_ld();
                if (r < rows)
                    store_scaled32(p.out + orow + c * 32, p.out_f32 ? p.out_f32 + orow + c * 32 : nullptr, o, inv);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

cudaError_t launch_attend_prefill_hd256(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                        const CUtensorMap &tv, int B, int n_tok, int start_pos, int Hq, int Hkv,
                                        int max_seq, float scale, __nv_bfloat16 *out, float *out_f32,
                                        unsigned *dev_err) {
    Params p;
    p.B = B;
    p.n_tok = n_tok;
    p.start_pos = start_pos;
    p.Hq = Hq;
    p.G = Hq / Hkv;
    p.max_seq = max_seq;
    p.n_tiles = (n_tok + BM - 1) / BM;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.out_f32 = out_f32;
    p.dev_err = dev_err;
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_hd256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    attn_prefill_hd256_kernel<<<(unsigned)(p.n_tiles * B * Hq), kThreads, kSmem, st>>>(tq, tk, tv, p);
    return cudaGetLastError();
}
