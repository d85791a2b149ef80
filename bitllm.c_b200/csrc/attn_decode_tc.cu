// attn_decode_tc.cu -- split-K GQA decode attention for a bf16 KV cache on B200.
//
// Same contract as the SIMT kernel of attn_decode.cu (fullatt_attend's head loop,
// src/eif_qwen35.c:741-771; tinyllm decode, src/eif_tinyllm.c:555-656): every (sequence, kv head,
// key chunk) item leaves unnormalised partials (m, l, o[G][D]) -- one per consumer warp, over the warp's
// 16 keys of its group's tiles -- that attn_decode_combine merges with the other chunks'.
//
// Structure (persistent, one CTA per SM; NG groups of 4 consumer warps + 1 producer warp, NG = 2 at
// head_dim 64 / 128 and 1 at 256):
//   last warp  producer: one lane streams K and V tiles of 64 keys x D through an NS-stage ring with
//           3-D TMA tile loads (128-byte swizzle, no multicast) completing on "full" mbarriers;
//   consumer groups take the tiles round-robin; each warp of a group takes 16 keys of its tiles.
//           S^T = K Q^T and O^T += V^T P^T run on the tensor cores (mma.m16n8k16, bf16 in, fp32
//           accumulate), fed by ldmatrix from the swizzled tiles; online softmax in base 2 with warp
//           shuffles; the tile is released through an "empty" mbarrier (four arrivals, its group's).
// Each K/V byte crosses HBM once and serves all G query heads of its kv head.
//
// Exactness: the query (pre-scaled by scale*log2 e) and the probabilities are split into two
// bf16 terms, x = hi + lo (hi = bf16(x), lo = bf16(x - hi), ~16 significant bits); hi and lo ride
// in the 8 MMA columns (4 heads x {hi, lo}) and are summed after the product.  K and V are exact
// bf16, products are exact in fp32, so results match fp32 arithmetic on the bf16 cache to ~1e-6.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int KT = 64;              // keys per tile
constexpr int kConsumers = 4;       // consumer warps of a group, 16 keys of a tile each
constexpr int kSmemLimit = 227 * 1024;

// NG groups of four consumer warps take the tiles round-robin (two warps per SM sub-partition hide each
// other's MMA / shuffle latencies at head_dim 64 / 128; head_dim 256 has the registers for one group)
template <int D, int NB, int NG>
struct TcCfg {
    static constexpr int CW = kConsumers * NG;       // consumer warps
    static constexpr int THREADS = 32 * (CW + 1);
    static constexpr int HS = 4 * NB;                 // head slots (G <= HS)
    static constexpr int BOX = 64 * 128;              // one 64-key x 64-dim swizzled box, bytes
    static constexpr int TILE = (D / 64) * BOX;       // K (or V) tile bytes
    static constexpr int STAGE = 2 * TILE;
    static constexpr int QSLOT = HS * D * 4;          // the query rows of an item (G heads)
    static constexpr int EXTRA = CW * 16 * HS * 4     // P transpose
                                 + 2 * QSLOT          // two query slots
                                 + 64 * 8             // barriers
                                 + 1024;              // alignment slack
    static constexpr int FIT = ((kSmemLimit - EXTRA) / STAGE) > 8 ? 8 : ((kSmemLimit - EXTRA) / STAGE);
    // a multiple of the groups: a stage is always consumed by the same group, so a barrier's phase parity
    // cannot alias between two groups' uses (their TMA copies may land out of order)
    static constexpr int NS = FIT / NG * NG;
    static constexpr int SMEM = NS * STAGE + EXTRA;
    static_assert(NS >= 2, "pipeline needs two stages");
};

constexpr int tc_groups(int D) { return D <= 128 ? 2 : 1; }

struct TcParams {
    const float *q;
    const int *pos;
    const int *row_seq;  // nullptr, or the cache sequence of each query row (prefill rows)
    int max_seq, max_len, Hkv, G, Hq;
    int nchunk, chunk_keys, n_items;
    float qscale;  // scale * log2(e)
    float *part_o;
    float2 *part_ml;
    unsigned *dev_err;
};

struct ItemInfo {
    int b, cb, kvh, t_begin, t_end, ntiles;  // b: query row, cb: its cache sequence
};

__device__ __forceinline__ ItemInfo item_info(const TcParams &p, int item, bool report) {
    ItemInfo it;
    const int unit = item / p.nchunk, c = item - unit * p.nchunk;
    it.b = unit / p.Hkv;
    it.kvh = unit - it.b * p.Hkv;
    it.cb = p.row_seq ? p.row_seq[it.b] : it.b;
    int pp = p.pos[it.b];
    if (pp < 0 || pp >= p.max_len) {  // max_len = the caller's bound + 1, never above max_seq
        if (report) atomicOr(p.dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
        pp = -1;
    }
    it.t_begin = c * p.chunk_keys;
    it.t_end = min(pp + 1, it.t_begin + p.chunk_keys);
    it.ntiles = it.t_end > it.t_begin ? (it.t_end - it.t_begin + KT - 1) / KT : 0;
    return it;
}

template <int D, int NB, int NG>
__global__ void __launch_bounds__(TcCfg<D, NB, NG>::THREADS, 1)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const TcParams p) {
    using C = TcCfg<D, NB, NG>;
    constexpr int NS = C::NS, HS = C::HS, MT = D / 16;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    float *pbuf = reinterpret_cast<float *>(smem + NS * C::STAGE);  // [4][16][HS]
    float *qbuf = pbuf + C::CW * 16 * HS;                           // [2][G][D] query rows of an item
    uint64_t *bars = reinterpret_cast<uint64_t *>(qbuf + 2 * HS * D);
    // bars: full[NS], empty[NS], qfull[2], qempty[2]
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NS);
    const uint32_t qfull0 = smem_u32(bars + 2 * NS), qempty0 = smem_u32(bars + 2 * NS + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kConsumers);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(qfull0 + 8 * s, 1);
            mbar_init(qempty0 + 8 * s, C::CW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    griddep_wait();  // a no-op unless launched as a programmatic dependent (these kernels are ordinary launches)
    griddep_launch_dependents();  // the chunk combine may launch now; it waits for this grid's results

    if (warp == C::CW) {
        // ------------------------------------------------------------------ producer
        // one lane: per item a bulk copy of its query rows into one of two slots (the consumers never wait on
        // a global load between items), then the item's K / V tiles
        if (lane != 0) return;
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        const uint32_t qbytes = (uint32_t)(p.G * D * 4);
        uint32_t it = 0, qn = 0;
        for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++qn) {
            const ItemInfo inf = item_info(p, item, false);
            const uint32_t qs = qn & 1;  // slot use qn >> 1 waits for the consumers' release of the previous use
            if (!mbar_wait(qempty0 + 8 * qs, ((qn >> 1) & 1) ^ 1, p.dev_err)) return;
            mbar_arrive_expect_tx(qfull0 + 8 * qs, qbytes);
            bulk_load(smem_u32(qbuf + qs * HS * D), p.q + ((size_t)inf.b * p.Hq + (size_t)inf.kvh * p.G) * D, qbytes,
                      qfull0 + 8 * qs);
            for (int i = 0; i < inf.ntiles; ++i, ++it) {
                const uint32_t s = it % NS, ph = (it / NS) & 1;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1, p.dev_err)) return;
                const uint32_t fb = full0 + 8 * s;
                mbar_arrive_expect_tx(fb, C::STAGE);
                const int row = inf.cb * p.max_seq + inf.t_begin + i * KT;
                const uint32_t kdst = smem_u32(smem + s * C::STAGE), vdst = kdst + C::TILE;
#pragma unroll
                for (int j = 0; j < D / 64; ++j) {
                    tma_load_3d(kdst + j * C::BOX, &tmK, j * 64, inf.kvh, row, fb);
                    tma_load_3d(vdst + j * C::BOX, &tmV, j * 64, inf.kvh, row, fb);
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const int grp = warp / kConsumers, sl = warp % kConsumers;  // group, 16-key slice of the tile
    float *pw = pbuf + warp * 16 * HS;
    uint32_t it = 0, item_no = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++item_no) {
        const ItemInfo inf = item_info(p, item, warp == 0 && lane == 0);

        // Q^T fragments: column g of the 8 is head (g & 3) of the block, hi part for g < 4, lo for g >= 4
        const uint32_t qs = item_no & 1;
        if (!mbar_wait(qfull0 + 8 * qs, (item_no >> 1) & 1, p.dev_err)) return;
        uint32_t qf[NB][MT][2];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const int j = nb * 4 + (g & 3);
            const bool on = j < p.G;
            const float *qh = qbuf + qs * HS * D + (on ? j : 0) * D;
#pragma unroll
            for (int kc = 0; kc < MT; ++kc) {
                float v[4];
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {  // dims (2t, 2t+1) and (2t+8, 2t+9) of the 16-dim chunk
                    const float2 q2 = *reinterpret_cast<const float2 *>(qh + kc * 16 + 2 * t + 8 * e2);
                    float hi, lo;
                    split_bf16(on ? q2.x * p.qscale : 0.f, hi, lo);
                    v[2 * e2] = g < 4 ? hi : lo;
                    split_bf16(on ? q2.y * p.qscale : 0.f, hi, lo);
                    v[2 * e2 + 1] = g < 4 ? hi : lo;
                }
                qf[nb][kc][0] = pack_bf16x2(v[0], v[1]);
                qf[nb][kc][1] = pack_bf16x2(v[2], v[3]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(qempty0 + 8 * qs);

        float oacc[NB][MT][4];
        float m_run[NB][2], l_run[NB][2];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) oacc[nb][mt][0] = oacc[nb][mt][1] = oacc[nb][mt][2] = oacc[nb][mt][3] = 0.f;
            m_run[nb][0] = m_run[nb][1] = -INFINITY;
            l_run[nb][0] = l_run[nb][1] = 0.f;
        }

        for (int i = 0; i < inf.ntiles; ++i, ++it) {
            if ((int)(it % NG) != grp) continue;  // another group's tile
            const uint32_t s = it % NS, ph = (it / NS) & 1;
            if (!mbar_wait(full0 + 8 * s, ph, p.dev_err)) return;
            const uint32_t kbase = smem_u32(smem + s * C::STAGE), vbase = kbase + C::TILE;
            const int key0 = inf.t_begin + i * KT + sl * 16;  // first key of this warp
            const int nvalid = inf.t_end - key0;                // keys of the warp below t_end (may be <= 0)

            // ---- S^T = K Q^T over the head dim (two accumulator chains)
            float sa[NB][4], sb[NB][4];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) sa[nb][0] = sa[nb][1] = sa[nb][2] = sa[nb][3] = sb[nb][0] = sb[nb][1] =
                sb[nb][2] = sb[nb][3] = 0.f;
            {
                const int mi = lane >> 3, r = lane & 7;
                const int key = sl * 16 + (mi & 1) * 8 + r;
                const uint32_t rowaddr = kbase + key * 128;
#pragma unroll
                for (int kc = 0; kc < MT; ++kc) {
                    const int chunk = (kc & 3) * 2 + (mi >> 1);
                    const uint32_t addr = rowaddr + (kc >> 2) * C::BOX + ((chunk ^ (key & 7)) << 4);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(addr, a0, a1, a2, a3);
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
                        if (kc & 1)
                            mma_bf16_16816(sb[nb], a0, a1, a2, a3, qf[nb][kc][0], qf[nb][kc][1]);
                        else
                            mma_bf16_16816(sa[nb], a0, a1, a2, a3, qf[nb][kc][0], qf[nb][kc][1]);
                    }
                }
            }

            // ---- online softmax (base 2); lanes t and t^2 hold the hi / lo columns of the same heads
            const bool v0 = g < nvalid, v1 = g + 8 < nvalid;
            bool rescale = false;
            float pr[NB][4];
            float corr[NB][2];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float s0 = sa[nb][e] + sb[nb][e], s1 = sa[nb][2 + e] + sb[nb][2 + e];
                    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
                    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
                    s0 = v0 ? s0 : -INFINITY;
                    s1 = v1 ? s1 : -INFINITY;
                    float mx = fmaxf(s0, s1);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float m_new = fmaxf(m_run[nb][e], mx);
                    const float m_use = m_new == -INFINITY ? 0.f : m_new;
                    const float c = fast_exp2(m_run[nb][e] - m_use);
                    const float p0 = fast_exp2(s0 - m_use), p1 = fast_exp2(s1 - m_use);
                    l_run[nb][e] = l_run[nb][e] * c + p0 + p1;
                    m_run[nb][e] = m_new;
                    corr[nb][e] = c;
                    rescale |= c != 1.f;
                    pr[nb][e] = p0;
                    pr[nb][2 + e] = p1;
                }
            }
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        oacc[nb][mt][0] *= corr[nb][0];
                        oacc[nb][mt][1] *= corr[nb][1];
                        oacc[nb][mt][2] *= corr[nb][0];
                        oacc[nb][mt][3] *= corr[nb][1];
                    }
            }

            // ---- P^T fragments through a small per-warp transpose buffer [16 keys][HS]
            if (t < 2) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    pw[g * HS + nb * 4 + 2 * t] = pr[nb][0];
                    pw[g * HS + nb * 4 + 2 * t + 1] = pr[nb][1];
                    pw[(g + 8) * HS + nb * 4 + 2 * t] = pr[nb][2];
                    pw[(g + 8) * HS + nb * 4 + 2 * t + 1] = pr[nb][3];
                }
            }
            __syncwarp();
            uint32_t pf[NB][2];
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const int col = nb * 4 + (g & 3);
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = 2 * t + (e & 1) + (e >> 1) * 8;
                    float hi, lo;
                    split_bf16(pw[key * HS + col], hi, lo);
                    v[e] = g < 4 ? hi : lo;
                }
                pf[nb][0] = pack_bf16x2(v[0], v[1]);
                pf[nb][1] = pack_bf16x2(v[2], v[3]);
            }
            __syncwarp();

            // ---- keys past t_end: their p is 0; zero their V rows so stale non-finite cache rows cannot
            //      turn 0 * v into NaN (only the last tile of a chunk can hold such keys)
            if (nvalid < 16) {
                for (int r = max(nvalid, 0); r < 16; ++r) {
                    const int key = sl * 16 + r;
                    for (int j = lane; j < (D / 64) * 8; j += 32) {
                        uint4 *dst = reinterpret_cast<uint4 *>(smem + s * C::STAGE + C::TILE + (j >> 3) * C::BOX +
                                                                key * 128 + (j & 7) * 16);
                        *dst = make_uint4(0, 0, 0, 0);
                    }
                }
                __syncwarp();
            }

            // ---- O^T += V^T P^T over this warp's 16 keys
            {
                const int mi = lane >> 3, r = lane & 7;
                const int key = sl * 16 + (mi >> 1) * 8 + r;
                const uint32_t rowaddr = vbase + key * 128;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const int dchunk = mt * 2 + (mi & 1);  // 16-byte chunk of 8 dims
                    const uint32_t addr = rowaddr + (dchunk >> 3) * C::BOX + (((dchunk & 7) ^ (key & 7)) << 4);
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(addr, a0, a1, a2, a3);
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) mma_bf16_16816(oacc[nb][mt], a0, a1, a2, a3, pf[nb][0], pf[nb][1]);
                }
            }
            if (nvalid < 16) fence_proxy_async_smem();  // generic writes above precede the next TMA write
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * s);
        }

        // ---- item epilogue: reduce l over the 8 key lanes, add the lo columns onto hi, and write this warp's
        // partial (m in natural-log units, l, o) as partial 4 * item + warp: the combine weighs the four warps'
        // partials like chunks, so the warps never wait for one another
        const size_t pbase = ((size_t)item * C::CW + warp) * p.G;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float l = l_run[nb][e];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                const int h = nb * 4 + 2 * t + e;
                if (g == 0 && t < 2 && h < p.G) {
                    const float m = m_run[nb][e];
                    p.part_ml[pbase + h] = make_float2(m == -INFINITY ? -INFINITY : m * 0.69314718055994531f, l);
                }
            }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    float o = oacc[nb][mt][r];
                    o += __shfl_xor_sync(0xffffffffu, o, 2);
                    const int h = nb * 4 + 2 * t + (r & 1);
                    if (t < 2 && h < p.G) p.part_o[(pbase + h) * D + mt * 16 + g + (r >> 1) * 8] = o;
                }
    }
}

template <int D, int NB>
cudaError_t launch_tc_t(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv, const TcParams &p,
                        int sm_count) {
    constexpr int NG = tc_groups(D);
    using C = TcCfg<D, NB, NG>;
    cudaError_t e = cudaFuncSetAttribute(attn_decode_tc_kernel<D, NB, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM);
    if (e != cudaSuccess) return e;
    const int grid = p.n_items < sm_count ? p.n_items : sm_count;
    attn_decode_tc_kernel<D, NB, NG><<<grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);  // not a programmatic dependent (see launch_attend_decode)
    return cudaGetLastError();
}

}  // namespace

bool decode_tc_supported(int D, int G) { return (D == 64 || D == 128 || D == 256) && G >= 1 && G <= 8; }

int decode_tc_partials(int D) { return kConsumers * tc_groups(D); }

cudaError_t launch_attend_decode_tc(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                    const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                    float2 *part_ml, int sm_count) {
    TcParams p;
    p.q = a.q;
    p.pos = a.pos;
    p.row_seq = a.row_seq;
    p.max_seq = a.max_seq;
    p.max_len = a.max_len;
    p.Hkv = a.Hkv;
    p.G = a.Hq / a.Hkv;
    p.Hq = a.Hq;
    p.nchunk = nchunk;
    p.chunk_keys = chunk_keys;
    p.n_items = a.B * a.Hkv * nchunk;
    p.qscale = a.scale * 1.4426950408889634f;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.dev_err = a.dev_err;
    const int NB = p.G > 4 ? 2 : 1;
    switch (a.D * 10 + NB) {
        case 641: return launch_tc_t<64, 1>(st, tk, tv, p, sm_count);
        case 642: return launch_tc_t<64, 2>(st, tk, tv, p, sm_count);
        case 1281: return launch_tc_t<128, 1>(st, tk, tv, p, sm_count);
        case 1282: return launch_tc_t<128, 2>(st, tk, tv, p, sm_count);
        case 2561: return launch_tc_t<256, 1>(st, tk, tv, p, sm_count);
        case 2562: return launch_tc_t<256, 2>(st, tk, tv, p, sm_count);
        default: return cudaErrorInvalidValue;
    }
}
