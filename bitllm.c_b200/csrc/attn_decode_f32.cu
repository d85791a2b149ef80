// attn_decode_f32.cu -- split-K GQA decode attention over an fp32 KV cache, fed by TMA, exact fp32 math.
//
// The reference's own cache type (qwen35_attn_state_t, include/eif_qwen35.h:204-208; tinyllm's
// key_cache / value_cache, src/eif_tinyllm.c:131-134).  Same contract as the other decode kernels: every
// (sequence, kv head, key chunk) item leaves an unnormalised partial (m, l, o[G][D]) that
// attn_decode_combine merges (gate and SubLN included); the arithmetic is fullatt_attend's head loop
// (src/eif_qwen35.c:741-771) and tinyllm's (src/eif_tinyllm.c:557-656) in fp32 FMAs, the online softmax in
// base 2 (the query is pre-scaled by scale * log2 e).
//
// Structure (persistent, one CTA per SM, NW + 1 warps):
//   last warp, producer: one lane streams K and V tiles of 32 keys x D through an NS-stage ring with 3-D TMA
//           tile loads (boxes of 32 keys x 32 floats = 128-byte rows, 128-byte swizzle, no multicast);
//   warps 0 .. NW-1 consumers, one tile each, round-robin over the item's tiles:
//     scores   lane = key: float4 rows of K from the swizzled tile (the swizzle spreads the 32 lanes' rows
//              over all banks), the query's float4s broadcast from the warp's copy in shared memory;
//     softmax  per head across the warp's 32 keys with shuffles;
//     P V      lane = head dims (D / 32 each): the probabilities broadcast from a per-warp buffer, the V rows
//              from the swizzled tile; keys past pos are skipped, so stale rows are never read.
// The SIMT kernel of attn_decode.cu reads K and V straight from global memory with one dependent load per
// key in P V; this one keeps NS 32-key tiles in flight per SM (12 at head_dim 64, 4 at 128), with 4
// consumer warps (more warps would take the shared memory the deeper ring needs).
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int kSmemLimit = 227 * 1024;
constexpr int HS = 8;           // head slots (G <= 8)

// Ring depth NS is a multiple of the NW consumer warps that take tiles round-robin, so the consecutive uses
// of a stage within an item go to the same warp: a warp never polls a stage whose previous use belongs to
// another warp and may not have landed yet (a parity wait cannot tell use k from use k-2, and TMA copies
// complete out of order).  Items are separated by the merge barrier.
template <int D>
struct F32Cfg {
    // keys per tile (one consumer warp): 32, or 16 at head_dim 256, where a 32-key stage (64 KB) would leave
    // room for too few stages; there the two half-warps take the two halves of every key's dims
    static constexpr int KT = D == 256 ? 16 : 32;
    static constexpr int NW = 4;                     // consumer warps
    static constexpr int THREADS = 32 * (NW + 1);
    static constexpr int BOX = KT * 128;              // KT keys x 32 floats, 128-byte swizzle
    static constexpr int TILE = (D / 32) * BOX;       // K (or V) tile bytes
    static constexpr int STAGE = 2 * TILE;
    static constexpr int EXTRA = 2 * HS * D * 4       // two query slots (an item's rows, bulk-copied)
                                 + NW * HS * D * 4    // per-warp scaled query copies
                                 + NW * 32 * HS * 4   // per-warp probabilities
                                 + NW * HS * D * 4    // merge buffer o
                                 + 2 * NW * HS * 4    // merge m, l
                                 + 64 * 8             // barriers
                                 + 1024;              // alignment slack
    static constexpr int NS_FIT = (kSmemLimit - EXTRA) / STAGE;
    static constexpr int NS = (NS_FIT > 16 ? 16 : NS_FIT) / NW * NW;
    static constexpr int SMEM = NS * STAGE + EXTRA;
    static_assert(NS >= NW && NS % NW == 0, "ring depth a multiple of the consumer warps");
};

struct F32Params {
    const float *q;
    const int *pos;
    const int *row_seq;  // nullptr, or the cache sequence of each query row (prefill rows)
    int max_seq, max_len, Hkv, Hq;
    int nchunk, chunk_keys, n_items;
    float qscale;  // scale * log2(e)
    float *part_o;
    float2 *part_ml;
    unsigned *dev_err;
};

struct ItemInfo {
    int b, cb, kvh, t_begin, t_end, ntiles;  // b: query row, cb: its cache sequence
};

__device__ __forceinline__ ItemInfo item_info(const F32Params &p, int item, bool report, int KT) {
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

__device__ __forceinline__ float4 lds128(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds64(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}

// Byte offset of floats [4c, 4c+4) of row `key` in one KT-key x 32-float box (128-byte swizzle: the 16-byte
// chunk index XOR the row index mod 8).
__device__ __forceinline__ uint32_t box_off(int key, int c) { return key * 128 + ((c ^ (key & 7)) << 4); }

template <int D, int G>
__global__ void __launch_bounds__(F32Cfg<D>::THREADS, 1)
    attn_decode_f32_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const F32Params p) {
    using C = F32Cfg<D>;
    constexpr int NS = C::NS, DL = D / 32, NW = C::NW, KT = C::KT;
    static_assert(DL == 2 || DL == 4 || DL == 8, "head_dim 64, 128 or 256");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    float *qbuf = reinterpret_cast<float *>(smem + NS * C::STAGE);  // [2][G][D] query rows of an item
    float *sq = qbuf + 2 * HS * D;                                   // [NW][HS][D]
    float *pw = sq + NW * HS * D;                                    // [NW][KT][HS]
    float *ow = pw + NW * KT * HS;                                 // [NW][HS][D]
    float *mw = ow + NW * HS * D;                                  // [NW][HS]
    float *lw = mw + NW * HS;                                      // [NW][HS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(lw + NW * HS);
    // bars: full[NS], empty[NS], merged, drained, qfull[2], qempty[2]
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NS);
    const uint32_t merged = smem_u32(bars + 2 * NS), drained = smem_u32(bars + 2 * NS + 1);
    const uint32_t qfull0 = smem_u32(bars + 2 * NS + 2), qempty0 = smem_u32(bars + 2 * NS + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);  // the one warp that takes the tile
        }
        mbar_init(merged, NW);
        mbar_init(drained, NW);
        for (int s = 0; s < 2; ++s) {
            mbar_init(qfull0 + 8 * s, 1);
            mbar_init(qempty0 + 8 * s, NW);
        }
        fence_barrier_init();
    }
    __syncthreads();
    griddep_wait();  // a no-op unless launched as a programmatic dependent (these kernels are ordinary launches)
    griddep_launch_dependents();  // the chunk combine may launch now; it waits for this grid's results

    if (warp == NW) {
        // ------------------------------------------------------------------ producer
        // one lane: per item a bulk copy of its query rows into one of two slots (the consumers never wait on
        // a global load between items), then the item's K / V tiles
        if (lane != 0) return;
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        constexpr uint32_t qbytes = (uint32_t)(G * D * 4);
        uint32_t it = 0, qn = 0;
        for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++qn) {
            const ItemInfo inf = item_info(p, item, false, KT);
            const uint32_t qs = qn & 1;  // slot use qn >> 1 waits for the consumers' release of the previous use
            if (!mbar_wait(qempty0 + 8 * qs, ((qn >> 1) & 1) ^ 1, p.dev_err)) return;
            mbar_arrive_expect_tx(qfull0 + 8 * qs, qbytes);
            bulk_load(smem_u32(qbuf + qs * HS * D), p.q + ((size_t)inf.b * p.Hq + (size_t)inf.kvh * G) * D, qbytes,
                      qfull0 + 8 * qs);
            for (int i = 0; i < inf.ntiles; ++i, ++it) {
                const uint32_t s = it % NS, ph = (it / NS) & 1;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1, p.dev_err)) return;
                const uint32_t fb = full0 + 8 * s;
                mbar_arrive_expect_tx(fb, C::STAGE);
                const int row = inf.cb * p.max_seq + inf.t_begin + i * KT;
                const uint32_t kdst = smem_u32(smem + s * C::STAGE), vdst = kdst + C::TILE;
#pragma unroll
                for (int j = 0; j < D / 32; ++j) {
                    tma_load_3d(kdst + j * C::BOX, &tmK, j * 32, inf.kvh, row, fb);
                    tma_load_3d(vdst + j * C::BOX, &tmV, j * 32, inf.kvh, row, fb);
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    float *sqw = sq + warp * HS * D;
    float *pww = pw + warp * KT * HS;
    const uint32_t sqw_a = smem_u32(sqw), pww_a = smem_u32(pww);
    uint32_t it_base = 0, item_no = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++item_no) {
        const ItemInfo inf = item_info(p, item, warp == 0 && lane == 0, KT);
        const uint32_t qs = item_no & 1;
        if (!mbar_wait(qfull0 + 8 * qs, (item_no >> 1) & 1, p.dev_err)) return;
        const float *qh = qbuf + qs * HS * D;
        for (int i = lane; i < G * D; i += 32) sqw[i] = qh[i] * p.qscale;  // the G heads' rows, [h][D]
        __syncwarp();
        if (lane == 0) mbar_arrive(qempty0 + 8 * qs);

        float m[G], l[G], acc[G][DL];
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m[h] = -INFINITY;
            l[h] = 0.f;
#pragma unroll
            for (int e = 0; e < DL; ++e) acc[h][e] = 0.f;
        }

        for (int i = warp; i < inf.ntiles; i += NW) {
            const uint32_t it = it_base + i;
            const uint32_t s = it % NS, ph = (it / NS) & 1;
            const int t0 = inf.t_begin + i * KT;
            const int nvalid = min(KT, inf.t_end - t0);  // >= 1
            if (!mbar_wait(full0 + 8 * s, ph, p.dev_err)) return;
            const uint32_t kbase = smem_u32(smem + s * C::STAGE), vbase = kbase + C::TILE;

            // ---- scores: lane = key (KT 32); at KT 16 lane = key + 16 * half, each half over D / 2 dims
            constexpr int JB = KT == 32 ? D / 32 : D / 64;  // boxes per lane
            const int key = lane & (KT - 1), jb0 = KT == 32 ? 0 : (lane >> 4) * JB;
            float sc[G];
#pragma unroll
            for (int h = 0; h < G; ++h) sc[h] = 0.f;
#pragma unroll
            for (int j = 0; j < JB; ++j) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float4 k4 = lds128(kbase + (jb0 + j) * C::BOX + box_off(key, c));
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const float4 q4 = lds128(sqw_a + (h * D + (jb0 + j) * 32 + c * 4) * 4);
                        sc[h] = fmaf(q4.x, k4.x, sc[h]);
                        sc[h] = fmaf(q4.y, k4.y, sc[h]);
                        sc[h] = fmaf(q4.z, k4.z, sc[h]);
                        sc[h] = fmaf(q4.w, k4.w, sc[h]);
                    }
                }
            }
            if constexpr (KT == 16) {
#pragma unroll
                for (int h = 0; h < G; ++h) sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], 16);
            }

            // ---- online softmax (base 2) per head over the tile's keys (at KT 16 both halves hold each key)
            const bool valid = key < nvalid;
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float x = valid ? sc[h] : -INFINITY;
                const float m_new = fmaxf(m[h], warp_max(x));
                const float m_use = m_new == -INFINITY ? 0.f : m_new;
                const float corr = fast_exp2(m[h] - m_use);
                const float pr = valid ? fast_exp2(x - m_use) : 0.f;
                l[h] = l[h] * corr + warp_sum(lane < KT ? pr : 0.f);
                m[h] = m_new;
#pragma unroll
                for (int e = 0; e < DL; ++e) acc[h][e] *= corr;
                if (lane < KT) pww[lane * HS + h] = pr;
            }
            __syncwarp();

            // ---- P V: lane = dims [lane*DL, lane*DL + DL); keys past t_end are not read
            auto pv_key = [&](int r) {
                float pr[HS];
                const float4 pa = lds128(pww_a + r * HS * 4);
                pr[0] = pa.x; pr[1] = pa.y; pr[2] = pa.z; pr[3] = pa.w;
                if constexpr (G > 4) {
                    const float4 pb = lds128(pww_a + (r * HS + 4) * 4);
                    pr[4] = pb.x; pr[5] = pb.y; pr[6] = pb.z; pr[7] = pb.w;
                }
                float v[DL];
                if constexpr (DL == 2) {
                    const float2 v2 = lds64(vbase + (lane >> 4) * C::BOX + box_off(r, (lane & 15) >> 1) + (lane & 1) * 8);
                    v[0] = v2.x; v[1] = v2.y;
                } else if constexpr (DL == 8) {
                    const uint32_t vb = vbase + (lane >> 2) * C::BOX;
                    const float4 v0 = lds128(vb + box_off(r, (lane & 3) * 2));
                    const float4 v1 = lds128(vb + box_off(r, (lane & 3) * 2 + 1));
                    v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
                    v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
                } else {
                    const float4 v4 = lds128(vbase + (lane >> 3) * C::BOX + box_off(r, lane & 7));
                    v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
                }
#pragma unroll
                for (int h = 0; h < G; ++h)
#pragma unroll
                    for (int e = 0; e < DL; ++e) acc[h][e] = fmaf(pr[h], v[e], acc[h][e]);
            };
            if (nvalid == KT) {
#pragma unroll 8
                for (int r = 0; r < KT; ++r) pv_key(r);
            } else {
                for (int r = 0; r < nvalid; ++r) pv_key(r);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * s);
        }
        it_base += inf.ntiles;

        // ---- item epilogue: merge the NW warps' (m, l, o)
        if (item_no > 0 && !mbar_wait(drained, (item_no - 1) & 1, p.dev_err)) return;
        float *oww = ow + warp * HS * D;
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
            for (int e = 0; e < DL; ++e) oww[h * D + lane * DL + e] = acc[h][e];
        if (lane == 0) {
#pragma unroll
            for (int h = 0; h < G; ++h) {
                mw[warp * HS + h] = m[h];
                lw[warp * HS + h] = l[h];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(merged);
        if (!mbar_wait(merged, item_no & 1, p.dev_err)) return;
        const size_t pbase = (size_t)item * G;
        for (int idx = threadIdx.x; idx < G * D; idx += 32 * NW) {
            const int h = idx / D, d = idx - h * D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < NW; ++w) M = fmaxf(M, mw[w * HS + h]);
            float O = 0.f, L = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    const float f = fast_exp2(mw[w * HS + h] - M);
                    O += ow[(w * HS + h) * D + d] * f;
                    L += lw[w * HS + h] * f;
                }
            }
            p.part_o[(pbase + h) * D + d] = O;
            if (d == 0) p.part_ml[pbase + h] = make_float2(M == -INFINITY ? -INFINITY : M * 0.69314718055994531f, L);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(drained);
    }
}

template <int D, int G>
cudaError_t launch_f32_t(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv, const F32Params &p,
                         int sm_count) {
    using C = F32Cfg<D>;
    cudaError_t e =
        cudaFuncSetAttribute(attn_decode_f32_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    const int grid = p.n_items < sm_count ? p.n_items : sm_count;
    attn_decode_f32_kernel<D, G><<<grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);  // not a programmatic dependent (see launch_attend_decode)
    return cudaGetLastError();
}

template <int D>
cudaError_t dispatch_g(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv, const F32Params &p, int G,
                       int sm_count) {
    switch (G) {
        case 1: return launch_f32_t<D, 1>(st, tk, tv, p, sm_count);
        case 2: return launch_f32_t<D, 2>(st, tk, tv, p, sm_count);
        case 3: return launch_f32_t<D, 3>(st, tk, tv, p, sm_count);
        case 4: return launch_f32_t<D, 4>(st, tk, tv, p, sm_count);
        case 5: return launch_f32_t<D, 5>(st, tk, tv, p, sm_count);
        case 6: return launch_f32_t<D, 6>(st, tk, tv, p, sm_count);
        case 7: return launch_f32_t<D, 7>(st, tk, tv, p, sm_count);
        case 8: return launch_f32_t<D, 8>(st, tk, tv, p, sm_count);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool decode_f32_supported(int D, int G) { return (D == 64 || D == 128 || D == 256) && G >= 1 && G <= 8; }

cudaError_t launch_attend_decode_f32(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                     const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                     float2 *part_ml, int sm_count) {
    F32Params p;
    p.q = a.q;
    p.pos = a.pos;
    p.row_seq = a.row_seq;
    p.max_seq = a.max_seq;
    p.max_len = a.max_len;
    p.Hkv = a.Hkv;
    p.Hq = a.Hq;
    p.nchunk = nchunk;
    p.chunk_keys = chunk_keys;
    p.n_items = a.B * a.Hkv * nchunk;
    p.qscale = a.scale * 1.4426950408889634f;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.dev_err = a.dev_err;
    const int G = a.Hq / a.Hkv;
    if (a.D == 64) return dispatch_g<64>(st, tk, tv, p, G, sm_count);
    if (a.D == 128) return dispatch_g<128>(st, tk, tv, p, G, sm_count);
    if (a.D == 256) return dispatch_g<256>(st, tk, tv, p, G, sm_count);
    return cudaErrorInvalidValue;
}
