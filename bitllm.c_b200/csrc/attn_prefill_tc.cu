// attn_prefill_tc.cu -- causal GQA prefill attention on B200 5th-generation tensor cores.
//
// Reference: the batched prefill attention of tinyllm_forward_batch_embeddings
// (src/eif_tinyllm.c:1158-1268) and Qwen3.5's per-token fullatt_attend in prefill_chunk
// (src/eif_qwen35.c:1122-1133): token i of the chunk sits at position start_pos + i and attends to
// cache rows 0 .. start_pos + i; softmax(scale * q.k) . v per query head, kv head = h / (Hq/Hkv).
//
// One CTA = 128 query rows of one (sequence, query head); 6 warps, warp-specialised:
//   warp 4      TMA producer: the Q tile once, then K and V tiles of 128 keys into double-buffered
//               128-byte-swizzled smem rings (no multicast);
//   warp 5      MMA issuer: S_j = Q K_j^T into a double-buffered TMEM S (tcgen05.mma kind::f16,
//               M = N = 128, bf16 in, fp32 accumulate), then O += P_{j-1} V_{j-1} into TMEM O, each
//               completion signalled with tcgen05.commit on an mbarrier;
//   warps 0-3   softmax: thread r owns query row r; reads its S row with tcgen05.ld, applies the
//               causal mask on diagonal tiles, online softmax in base 2, rescales its O row in TMEM
//               when the running max moves, writes P (bf16) into swizzled smem as the A operand of
//               the next MMA; finally O / l -> bf16 -> global.
// Work order: the longest causal rows first (q tile index descending), so the tail is short tiles.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int kPThreads = 192;
constexpr int TILE = BM * HD * 2;  // 32 KB: one Q, P, K or V tile (two 64-column swizzled boxes)
constexpr int OFF_Q = 0, OFF_P = TILE, OFF_K = 2 * TILE, OFF_V = 4 * TILE, OFF_BAR = 6 * TILE;
constexpr int kPSmem = OFF_BAR + 256 + 1024;
constexpr uint32_t kTmemCols = 512;  // S0 [0,128) S1 [128,256) O [256,384)

struct PrefillParams {
    int B, n_tok, start_pos, Hq, Hkv, G, max_seq, n_qt;
    float scale_log2;
    __nv_bfloat16 *out;
    unsigned *dev_err;
};

__global__ void __launch_bounds__(kPThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t sQ = sbase + OFF_Q, sP = sbase + OFF_P;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    // barrier slots
    const uint32_t q_full = smem_u32(bars + 0);
    const uint32_t k_full0 = smem_u32(bars + 1), k_empty0 = smem_u32(bars + 3);
    const uint32_t v_full0 = smem_u32(bars + 5), v_empty0 = smem_u32(bars + 7);
    const uint32_t s_full0 = smem_u32(bars + 9), s_free0 = smem_u32(bars + 11);
    const uint32_t p_full = smem_u32(bars + 13), p_empty = smem_u32(bars + 14);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per_tile = p.B * p.Hq;
    const int qt = p.n_qt - 1 - (int)blockIdx.x / per_tile;
    const int rem = (int)blockIdx.x % per_tile;
    const int b = rem / p.Hq, h = rem - b * p.Hq, kvh = h / p.G;
    const int q0 = qt * BM;
    const int rows = min(BM, p.n_tok - q0);
    const int q_last_pos = p.start_pos + q0 + rows - 1;
    const int nkv = q_last_pos / BN + 1;
    const int kv_end = p.start_pos + p.n_tok;  // rows at or past this were not written by this prefill

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(k_full0 + 8 * s, 1);
            mbar_init(k_empty0 + 8 * s, 1);
            mbar_init(v_full0 + 8 * s, 1);
            mbar_init(v_empty0 + 8 * s, 1);
            mbar_init(s_full0 + 8 * s, 1);
            mbar_init(s_free0 + 8 * s, 4);
        }
        mbar_init(p_full, 4);
        mbar_init(p_empty, 1);
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
            mbar_arrive_expect_tx(q_full, TILE);
            for (int d = 0; d < 2; ++d) tma_load_3d(sQ + d * (TILE / 2), &tmQ, d * 64, h, b * p.n_tok + q0, q_full);
            for (int j = 0; j < nkv; ++j) {
                const int s = j & 1;
                const uint32_t par = ((j >> 1) & 1) ^ 1;
                const int row = b * p.max_seq + j * BN;
                const uint32_t kdst = sbase + OFF_K + s * TILE, vdst = sbase + OFF_V + s * TILE;
                if (!mbar_wait(k_empty0 + 8 * s, par, p.dev_err)) break;
                mbar_arrive_expect_tx(k_full0 + 8 * s, TILE);
                for (int d = 0; d < 2; ++d)
                    for (int hf = 0; hf < 2; ++hf)
                        tma_load_3d(kdst + d * (TILE / 2) + hf * (TILE / 4), &tmK, d * 64, kvh, row + hf * 64,
                                    k_full0 + 8 * s);
                if (!mbar_wait(v_empty0 + 8 * s, par, p.dev_err)) break;
                mbar_arrive_expect_tx(v_full0 + 8 * s, TILE);
                for (int d = 0; d < 2; ++d)
                    for (int hf = 0; hf < 2; ++hf)
                        tma_load_3d(vdst + d * (TILE / 2) + hf * (TILE / 4), &tmV, d * 64, kvh, row + hf * 64,
                                    v_full0 + 8 * s);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_qk = umma_idesc_bf16(BM, BN, false, false);
        constexpr uint32_t idesc_pv = umma_idesc_bf16(BM, HD, false, true);
        bool ok = mbar_wait(q_full, 0, p.dev_err);
        for (int j = 0; ok && j <= nkv; ++j) {
            if (j < nkv) {
                const int s = j & 1;
                const uint32_t u = (j >> 1) & 1;
                if (!mbar_wait(k_full0 + 8 * s, u, p.dev_err) || !mbar_wait(s_free0 + 8 * s, u ^ 1, p.dev_err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t kb = sbase + OFF_K + s * TILE;
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk) {
                        const uint32_t off = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
                        umma_bf16_ss(tmem + s * BN, umma_desc_sw128(sQ + off, 16, 1024),
                                     umma_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0);
                    }
                    umma_commit(s_full0 + 8 * s);
                    umma_commit(k_empty0 + 8 * s);
                }
                __syncwarp();
            }
            if (j >= 1) {
                const int jj = j - 1, s = jj & 1;
                const uint32_t u = (jj >> 1) & 1;
                if (!mbar_wait(p_full, jj & 1, p.dev_err) || !mbar_wait(v_full0 + 8 * s, u, p.dev_err)) {
                    ok = false;
                    break;
                }
                const uint32_t vb = sbase + OFF_V + s * TILE;
                const int first_bad = kv_end - jj * BN;  // keys of this tile at or past kv_end
                if (first_bad < BN) {
                    // their p is 0, but 0 * (a non-finite stale row) would be NaN: zero those V rows
                    for (int r = max(first_bad, 0); r < BN; ++r)
                        for (int d = 0; d < 2; ++d) {
                            uint4 *dst = reinterpret_cast<uint4 *>(smem + OFF_V + s * TILE + d * (TILE / 2) + r * 128);
                            if (lane < 8) dst[lane] = make_uint4(0, 0, 0, 0);
                        }
                    fence_proxy_async_smem();
                    __syncwarp();
                }
                tc_fence_after();
                if (lane == 0) {
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk) {
                        const uint32_t aoff = (kk >> 2) * (TILE / 2) + (kk & 3) * 32;
                        umma_bf16_ss(tmem + 2 * BN, umma_desc_sw128(sP + aoff, 16, 1024),
                                     umma_desc_sw128(vb + kk * 2048, TILE / 2, 1024), idesc_pv, (jj > 0 || kk > 0));
                    }
                    umma_commit(v_empty0 + 8 * s);
                    umma_commit(p_empty);
                }
                __syncwarp();
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warps 0-3
        const int r = threadIdx.x;  // query row of this thread == TMEM lane
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        const int qpos = p.start_pos + q0 + r;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            const int s = j & 1;
            if (!mbar_wait(s_full0 + 8 * s, (j >> 1) & 1, p.dev_err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float x[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                float t[32];
                tmem_ld32(tmem + lane_base + s * BN + c * 32, t);
#pragma unroll
                for (int i = 0; i < 32; ++i) x[c * 32 + i] = t[i];
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free0 + 8 * s);

            const int kbase = j * BN;
            const bool diag = kbase + BN - 1 > p.start_pos + q0;  // some key of the tile is past some row
            float mt = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                float v = x[c] * p.scale_log2;
                if (diag && kbase + c > qpos) v = -INFINITY;
                x[c] = v;
                mt = fmaxf(mt, v);
            }
            const float m_new = fmaxf(m, mt);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float corr = fast_exp2(m - m_use);
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
                x[c] = fast_exp2(x[c] - m_use);
                sum += x[c];
            }
            if (j > 0) {
                if (!mbar_wait(p_empty, (j - 1) & 1, p.dev_err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
                    for (int c = 0; c < HD / 32; ++c) {
                        float o[32];
                        tmem_ld32(tmem + lane_base + 2 * BN + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= corr;
                        tmem_st32(tmem + lane_base + 2 * BN + c * 32, o);
                    }
                    tmem_wait_st();
                }
            }
            // P row -> smem, K-major 128-byte swizzle (the A operand layout of the PV MMA)
#pragma unroll
            for (int uu = 0; uu < BN / 8; ++uu) {
                const int chunk = uu >> 3, ui = uu & 7;
                uint4 w;
                w.x = pack_bf16x2(x[uu * 8 + 0], x[uu * 8 + 1]);
                w.y = pack_bf16x2(x[uu * 8 + 2], x[uu * 8 + 3]);
                w.z = pack_bf16x2(x[uu * 8 + 4], x[uu * 8 + 5]);
                w.w = pack_bf16x2(x[uu * 8 + 6], x[uu * 8 + 7]);
                *reinterpret_cast<uint4 *>(smem + OFF_P + chunk * (TILE / 2) + r * 128 + ((ui ^ (r & 7)) << 4)) = w;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            l = l * corr + sum;
            m = m_new;
        }
        if (ok && mbar_wait(p_empty, (nkv - 1) & 1, p.dev_err)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            __nv_bfloat16 *orow = p.out + (((size_t)b * p.n_tok + q0 + r) * p.Hq + h) * HD;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                float o[32];
                tmem_ld32(tmem + lane_base + 2 * BN + c * 32, o);
                tmem_wait_ld();
                if (r < rows) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 w;
                        w.x = pack_bf16x2(o[q4 * 8 + 0] * inv, o[q4 * 8 + 1] * inv);
                        w.y = pack_bf16x2(o[q4 * 8 + 2] * inv, o[q4 * 8 + 3] * inv);
                        w.z = pack_bf16x2(o[q4 * 8 + 4] * inv, o[q4 * 8 + 5] * inv);
                        w.w = pack_bf16x2(o[q4 * 8 + 6] * inv, o[q4 * 8 + 7] * inv);
                        *reinterpret_cast<uint4 *>(orow + c * 32 + q4 * 8) = w;
                    }
                }
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

bool prefill_tc_supported(int D) { return D == HD; }

cudaError_t launch_attend_prefill_tc(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                     const CUtensorMap &tv, int B, int n_tok, int start_pos, int Hq, int Hkv,
                                     int max_seq, float scale, __nv_bfloat16 *out, unsigned *dev_err) {
    PrefillParams p;
    p.B = B;
    p.n_tok = n_tok;
    p.start_pos = start_pos;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.max_seq = max_seq;
    p.n_qt = (n_tok + BM - 1) / BM;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.dev_err = dev_err;
    cudaError_t e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    if (e != cudaSuccess) return e;
    const unsigned grid = (unsigned)(p.n_qt * B * Hq);
    attn_prefill_tc_kernel<<<grid, kPThreads, kPSmem, st>>>(tq, tk, tv, p);
    return cudaGetLastError();
}
