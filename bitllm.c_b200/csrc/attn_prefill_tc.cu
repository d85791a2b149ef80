// attn_prefill_tc.cu -- causal GQA prefill attention on B200 5th-generation tensor cores.
//
// Reference: the batched prefill attention of tinyllm_forward_batch_embeddings
// (src/eif_tinyllm.c:1158-1268) and Qwen3.5's per-token fullatt_attend in prefill_chunk
// (src/eif_qwen35.c:1122-1133): token i of the chunk sits at position start_pos + i and attends to
// cache rows 0 .. start_pos + i; softmax(scale * q.k) . v per query head, kv head = h / (Hq/Hkv).
//
// One CTA = two 128-row query tiles (A, B) of one (sequence, query head) sharing every K / V tile;
// 10 warps, warp-specialised:
//   warp 8      TMA producer: both Q tiles once, then K and V tiles of 128 keys into double-buffered
//               128-byte-swizzled smem rings (no multicast);
//   warp 9      MMA issuer, one thread, per key tile j and query tile t in turn:
//                 O_t += P_t(j-1) V_{j-1}   tcgen05.mma, A = P from TMEM, B = V from smem
//                 S_t(j) = Q_t K_j^T        tcgen05.mma, A and B from smem
//               (M = N = 128, bf16 in, fp32 accumulate in TMEM), completions signalled to mbarriers
//               with tcgen05.commit.  tcgen05.mma ops execute in issue order, so S_t(j) may overwrite
//               the TMEM columns that held P_t(j-1);
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: thread r owns query row r.  The row
//               keeps a reference max while a tile's max stays within 2^8 of it (every p <= 256: the
//               same result, and O is rescaled in TMEM only when the max really moves), so one pass over
//               S (tcgen05.ld) computes p = 2^(scale*s - m_ref) with packed f32x2 arithmetic (a third of
//               the exponentials by a polynomial on the FMA pipe) while it takes the causally masked tile
//               max; P stays in registers until the max is known and is then written as bf16 pairs into
//               the first 64 columns of its own S buffer with tcgen05.st.  A warp with a row whose max
//               moved redoes the pass from S (still in TMEM); the first tile takes the max first.  At the
//               end O / l -> bf16 -> global.
// The two tiles ping-pong: while one warpgroup runs its softmax the tensor cores run the other
// tile's PV and S.  P never touches shared memory, so each PV product reads only V from smem.
// Instantiated for head_dim 64 and 128 (one or two 64-column boxes per tile).
// TMEM: S_A (and P_A) [0,128), S_B (P_B) [128,256), O_A [256, 256 + HD), O_B [256 + HD, 256 + 2 HD).
// Persistent: one CTA per SM takes work items (two query tiles of one (sequence, head)) in rounds, the
// longest causal rows first and alternate rounds walked backwards; the next item's Q load and first
// products overlap the current item's last softmax, PV and output.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int BM = 128, BN = 128;
constexpr int BOX = BM * 128;  // 16 KB: one 64-column swizzled box of a 128-row Q, K or V tile
constexpr int kPThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;

// Shared-memory plan of the HD (64 or 128) instantiation: Q_A, Q_B | K[2] | V[2], HD / 64 boxes per tile.
template <int HD>
struct PrefillLayout {
    static constexpr int NBOX = HD / 64;
    static constexpr int TILE = NBOX * BOX;
    static constexpr int OFF_Q = 0, OFF_K = 2 * TILE, OFF_V = 4 * TILE, OFF_BAR = 6 * TILE;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
};

struct PrefillParams {
    int B, n_tok, start_pos, Hq, Hkv, G, max_seq, n_pairs;
    float scale_log2;
    __nv_bfloat16 *out;  // bf16 output, unless out_f32 is set
    float *out_f32;
    unsigned *dev_err;
};

// Tile max of scale * s over 32 columns of one row (columns past `lim` masked when MASK).
template <bool MASK>
__device__ __forceinline__ void chunk_max(const float (&x)[32], float scale, int lim, float &mt) {
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

// 2^x for a pair on the FMA and integer pipes instead of the SFU (the exponentials of a 128 x 128 score tile
// take as long on the SFU as the tile's MMAs on the tensor cores).  x = k + f with k = rint(x), by adding
// 1.5 * 2^23 (whose low mantissa bits then hold k), f in [-1/2, 1/2]; 2^f by a degree-3 polynomial whose
// coefficients were fitted for this kernel by iteratively reweighted least squares on the relative error
// over [-1/2, 1/2] (maximum relative error 7.6e-5, below 2^-9, the precision of the bf16 P it feeds); 2^k
// enters as k << 23 added to the polynomial's bits (the rounding constant's bits vanish in that shift).
// x is clamped at -125 so that the exponent stays normal (2^-125 stands in for 0; masked entries do not
// come here).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &y0, float &y1) {
    constexpr float kRound = 12582912.f;  // 1.5 * 2^23
    constexpr float c0 = 0.99992824f, c1 = 0.69326097f, c2 = 0.24260852f, c3 = 0.055170499f;
    const unsigned long long x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
    const unsigned long long t = fadd2(x, f2_pack(kRound, kRound));
    const unsigned long long k = fadd2(t, f2_pack(-kRound, -kRound));
    const unsigned long long f = ffma2(k, f2_pack(-1.f, -1.f), x);
    unsigned long long p = ffma2(f2_pack(c3, c3), f, f2_pack(c2, c2));
    p = ffma2(p, f, f2_pack(c1, c1));
    p = ffma2(p, f, f2_pack(c0, c0));
    float p0, p1, t0, t1;
    f2_unpack(p, p0, p1);
    f2_unpack(t, t0, t1);
    y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
    y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// p = 2^(scale * s - m_use) over 32 columns: packed running sum, bf16 pairs into pk[16].  Unmasked tiles
// take one pair in three through exp2_poly2, the rest through the SFU.
template <bool MASK>
__device__ __forceinline__ void chunk_exp(const float (&x)[32], float scale, float m_use, int lim,
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
        float e0, e1;
        if (!MASK && (i / 2) % 3 == 2) {
            exp2_poly2(v0, v1, e0, e1);
        } else {
            e0 = fast_exp2(v0);
            e1 = fast_exp2(v1);
        }
        sum2 = fadd2(sum2, f2_pack(e0, e1));
        pk[i / 2] = pack_bf16x2(e0, e1);
    }
}

// barrier slots (each 8 bytes) in the barrier area
enum {
    BAR_Q = 0,
    BAR_KFULL = 1,   // 2 stages
    BAR_KEMPTY = 3,  // 2
    BAR_VFULL = 5,   // 2
    BAR_VEMPTY = 7,  // 2
    BAR_SFULL = 9,   // per tile (A, B)
    BAR_PFULL = 11,  // per tile
    BAR_PEMPTY = 13, // per tile: PV of that tile done
    BAR_QFREE = 15,  // every S MMA of the item done: the Q tiles may be replaced by the next item's
    BAR_OFREE = 16,  // per tile: the softmax warps have read O of the item (the next item may overwrite it)
    BAR_COUNT = 18
};

// One work item = two 128-row query tiles (A, B) of one (sequence, query head).
struct PItem {
    int b, h, kvh, q0[2], rows[2], nkv[2], nkv_all;
};

__device__ __forceinline__ PItem make_item(const PrefillParams &p, int w) {
    PItem it;
    const int per_pair = p.B * p.Hq;
    const int pair = p.n_pairs - 1 - w / per_pair;  // heaviest first
    const int rem = w % per_pair;
    it.b = rem / p.Hq;
    it.h = rem - it.b * p.Hq;
    it.kvh = it.h / p.G;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        it.q0[t] = (2 * pair + t) * BM;
        it.rows[t] = max(0, min(BM, p.n_tok - it.q0[t]));
        it.nkv[t] = it.rows[t] > 0 ? (p.start_pos + it.q0[t] + it.rows[t] - 1) / BN + 1 : 0;
    }
    it.nkv_all = max(it.nkv[0], it.nkv[1]);
    return it;
}

// The k-th item of this CTA: rounds of gridDim.x items, alternate rounds walked backwards (heavy items
// first and the per-CTA totals balanced); -1 past the last item.
__device__ __forceinline__ int item_of(int k, int n_items) {
    const int G = gridDim.x;
    const int w = k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
    return w < n_items ? w : -1;
}

template <int HD>
__global__ void __launch_bounds__(kPThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const PrefillParams p) {
    using L = PrefillLayout<HD>;
    constexpr int TILE = L::TILE, NBOX = L::NBOX, OFF_Q = L::OFF_Q, OFF_K = L::OFF_K, OFF_V = L::OFF_V,
                  OFF_BAR = L::OFF_BAR;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    const uint32_t sbase = smem_u32(smem);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + BAR_COUNT + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_items = p.n_pairs * p.B * p.Hq;
    const int kv_end = p.start_pos + p.n_tok;  // rows at or past this were not written by this prefill

    if (threadIdx.x == 0) {
        mbar_init(bar(BAR_Q), 1);
        mbar_init(bar(BAR_QFREE), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(BAR_KFULL + s), 1);
            mbar_init(bar(BAR_KEMPTY + s), 1);
            mbar_init(bar(BAR_VFULL + s), 1);
            mbar_init(bar(BAR_VEMPTY + s), 1);
            mbar_init(bar(BAR_SFULL + s), 1);
            mbar_init(bar(BAR_PFULL + s), 4);
            mbar_init(bar(BAR_PEMPTY + s), 1);
            mbar_init(bar(BAR_OFREE + s), 4);
        }
        fence_barrier_init();
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Persistent: every role walks the same item sequence (item_of) and keeps running counts, so the
    // barrier phases continue from one item to the next; the producer loads the next item's Q as soon as
    // the last S MMA of the current one is done (QFREE), and the first PV of a tile waits until the softmax
    // warps have read the previous item's O out of TMEM (OFREE).
    if (warp == 8) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            uint32_t kv_it = 0;  // K / V tiles issued so far (ring slot kv_it & 1)
            int item_no = 0;
            bool ok = true;
            for (int k = 0; ok; ++k) {
                const int w = item_of(k, n_items);
                if (w < 0) break;
                const PItem it = make_item(p, w);
                if (item_no > 0 && !mbar_wait(bar(BAR_QFREE), (item_no - 1) & 1, p.dev_err)) break;
                const int nq = it.rows[1] > 0 ? 2 : 1;
                mbar_arrive_expect_tx(bar(BAR_Q), nq * TILE);
                for (int t = 0; t < nq; ++t)
                    for (int d = 0; d < NBOX; ++d)
                        tma_load_3d(sbase + OFF_Q + t * TILE + d * BOX, &tmQ, d * 64, it.h, it.b * p.n_tok + it.q0[t],
                                    bar(BAR_Q));
                for (int j = 0; j < it.nkv_all; ++j, ++kv_it) {
                    const int s = kv_it & 1;
                    const uint32_t par = ((kv_it >> 1) & 1) ^ 1;
                    const int row = it.b * p.max_seq + j * BN;
                    if (!mbar_wait(bar(BAR_KEMPTY + s), par, p.dev_err)) { ok = false; break; }
                    mbar_arrive_expect_tx(bar(BAR_KFULL + s), TILE);
                    const uint32_t kdst = sbase + OFF_K + s * TILE, vdst = sbase + OFF_V + s * TILE;
                    for (int d = 0; d < NBOX; ++d)
                        for (int hf = 0; hf < 2; ++hf)
                            tma_load_3d(kdst + d * BOX + hf * (BOX / 2), &tmK, d * 64, it.kvh, row + hf * 64,
                                        bar(BAR_KFULL + s));
                    if (!mbar_wait(bar(BAR_VEMPTY + s), par, p.dev_err)) { ok = false; break; }
                    mbar_arrive_expect_tx(bar(BAR_VFULL + s), TILE);
                    for (int d = 0; d < NBOX; ++d)
                        for (int hf = 0; hf < 2; ++hf)
                            tma_load_3d(vdst + d * BOX + hf * (BOX / 2), &tmV, d * 64, it.kvh, row + hf * 64,
                                        bar(BAR_VFULL + s));
                }
                ++item_no;
            }
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc_qk = umma_idesc_bf16(BM, BN, false, false);
        constexpr uint32_t idesc_pv = umma_idesc_bf16(BM, HD, false, true);
        uint32_t kv_base = 0;                     // K / V tiles of the previous items
        uint32_t pv_cnt[2] = {0, 0};              // PV products issued per tile (= P tiles consumed)
        uint32_t ep_cnt[2] = {0, 0};              // earlier items with work for the tile (its O read-outs)
        int item_no = 0;
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int w = item_of(k, n_items);
            if (w < 0) break;
            const PItem it = make_item(p, w);
            if (!mbar_wait(bar(BAR_Q), item_no & 1, p.dev_err)) break;
            for (int j = 0; ok && j <= it.nkv_all; ++j) {
                const int jj = j - 1;
                const uint32_t kj = kv_base + j, kjj = kv_base + jj;
                const int s = kj & 1, sv = kjj & 1;
                if (j >= 1) {
                    if (!mbar_wait(bar(BAR_VFULL + sv), (kjj >> 1) & 1, p.dev_err)) { ok = false; break; }
                    const int first_bad = kv_end - jj * BN;  // keys of tile jj at or past kv_end
                    if (first_bad < BN) {
                        // their p is 0, but 0 * (a non-finite stale row) would be NaN: zero those V rows
                        for (int r = max(first_bad, 0); r < BN; ++r)
                            for (int d = 0; d < NBOX; ++d)
                                if (lane < 8)
                                    reinterpret_cast<uint4 *>(smem + OFF_V + sv * TILE + d * BOX + r * 128)[lane] =
                                        make_uint4(0, 0, 0, 0);
                        fence_proxy_async_smem();
                        __syncwarp();
                    }
                }
                if (j < it.nkv_all && !mbar_wait(bar(BAR_KFULL + s), (kj >> 1) & 1, p.dev_err)) { ok = false; break; }
                for (int t = 0; t < 2; ++t) {
                    if (j >= 1 && jj < it.nkv[t]) {
                        // O_t += P_t(jj) V_jj once the softmax has written P_t(jj) into TMEM; the item's first
                        // product overwrites O_t, so the previous item's O_t must have been read out
                        if (jj == 0 && ep_cnt[t] > 0 &&
                            !mbar_wait(bar(BAR_OFREE + t), (ep_cnt[t] - 1) & 1, p.dev_err)) { ok = false; break; }
                        if (!mbar_wait(bar(BAR_PFULL + t), pv_cnt[t] & 1, p.dev_err)) { ok = false; break; }
                        tc_fence_after();
                        if (lane == 0) {
                            const uint32_t vb = sbase + OFF_V + sv * TILE;
#pragma unroll
                            for (int kk = 0; kk < BN / 16; ++kk)
                                umma_bf16_ts(tmem + 2 * BN + t * HD, tmem + t * BN + kk * 8,
                                             umma_desc_sw128(vb + kk * 2048, BOX, 1024), idesc_pv, (jj > 0 || kk > 0));
                            umma_commit(bar(BAR_PEMPTY + t));
                        }
                        __syncwarp();
                        ++pv_cnt[t];
                    }
                    if (j < it.nkv[t]) {
                        // S_t(j) = Q_t K_j^T (issued after PV_t(j-1), which read the same TMEM columns)
                        if (lane == 0) {
                            const uint32_t qb = sbase + OFF_Q + t * TILE, kb = sbase + OFF_K + s * TILE;
#pragma unroll
                            for (int kk = 0; kk < HD / 16; ++kk) {
                                const uint32_t off = (kk >> 2) * BOX + (kk & 3) * 32;
                                umma_bf16_ss(tmem + t * BN, umma_desc_sw128(qb + off, 16, 1024),
                                             umma_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0);
                            }
                            umma_commit(bar(BAR_SFULL + t));
                        }
                        __syncwarp();
                    }
                }
                if (!ok) break;
                if (lane == 0) {
                    if (j < it.nkv_all) umma_commit(bar(BAR_KEMPTY + s));
                    if (j >= 1) umma_commit(bar(BAR_VEMPTY + sv));
                    if (j == it.nkv_all - 1) umma_commit(bar(BAR_QFREE));  // the item's last S products
                }
                __syncwarp();
            }
            kv_base += it.nkv_all;
            for (int t = 0; t < 2; ++t)
                if (it.nkv[t] > 0) ++ep_cnt[t];
            ++item_no;
        }
    } else {
        // ------------------------------------------------------------------ softmax warps (tile A: 0-3, B: 4-7)
        const int t = warp >> 2;
        const int r = threadIdx.x & 127;  // query row of the tile == TMEM lane
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_col = tmem + lane_base + t * BN, o_col = tmem + lane_base + 2 * BN + t * HD;
        uint32_t s_cnt = 0, pv_base = 0;  // S tiles and PV products of this tile so far
        bool ok = true;
        for (int k = 0; ok; ++k) {
            const int w = item_of(k, n_items);
            if (w < 0) break;
            const PItem it = make_item(p, w);
            if (it.nkv[t] == 0) continue;
            const int qpos = p.start_pos + it.q0[t] + r;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < it.nkv[t]; ++j) {
                if (!mbar_wait(bar(BAR_SFULL + t), (s_cnt++) & 1, p.dev_err)) { ok = false; break; }
                tc_fence_after();
                const int kbase = j * BN;
                const bool diag = kbase + BN - 1 > p.start_pos + it.q0[t];
                const int lim = qpos - kbase;  // diagonal tiles: columns past lim are masked
                // One pass over S: the tile max of scale * s and p = 2^(scale*s - m_ref) against the row's
                // reference max, P held in registers.  The first tile has no reference (m = -inf) and takes the
                // max first; later tiles redo the pass (S is still in TMEM) only where a row's max moved more
                // than 2^8 above its reference.
                float mt = -INFINITY;
                if (j == 0) {
#pragma unroll
                    for (int c = 0; c < BN / 32; c += 2) {
                        float x[32], y[32];
                        tmem_ld32(s_col + c * 32, x);
                        tmem_ld32(s_col + c * 32 + 32, y);
                        tmem_wait_ld();
                        if (diag) {
                            chunk_max<true>(x, p.scale_log2, lim - c * 32, mt);
                            chunk_max<true>(y, p.scale_log2, lim - c * 32 - 32, mt);
                        } else {
                            chunk_max<false>(x, p.scale_log2, 0, mt);
                            chunk_max<false>(y, p.scale_log2, 0, mt);
                        }
                    }
                }
                const float m_ref = j == 0 ? (mt == -INFINITY ? 0.f : mt) : m;
                uint32_t pk[BN / 2];
                unsigned long long sum2 = 0;
                auto exp_pass = [&](float m_use, bool track) {
                    sum2 = 0;
#pragma unroll
                    for (int c = 0; c < BN / 32; c += 2) {
                        float x[32], y[32];
                        tmem_ld32(s_col + c * 32, x);
                        tmem_ld32(s_col + c * 32 + 32, y);
                        tmem_wait_ld();
                        if (diag) {
                            if (track) {
                                chunk_max<true>(x, p.scale_log2, lim - c * 32, mt);
                                chunk_max<true>(y, p.scale_log2, lim - c * 32 - 32, mt);
                            }
                            chunk_exp<true>(x, p.scale_log2, m_use, lim - c * 32, sum2, pk + c * 16);
                            chunk_exp<true>(y, p.scale_log2, m_use, lim - c * 32 - 32, sum2, pk + c * 16 + 16);
                        } else {
                            if (track) {
                                chunk_max<false>(x, p.scale_log2, 0, mt);
                                chunk_max<false>(y, p.scale_log2, 0, mt);
                            }
                            chunk_exp<false>(x, p.scale_log2, m_use, 0, sum2, pk + c * 16);
                            chunk_exp<false>(y, p.scale_log2, m_use, 0, sum2, pk + c * 16 + 16);
                        }
                    }
                };
                exp_pass(m_ref, j > 0);
                // the row keeps its reference max while the tile max stays within 2^8 of it; the first
                // unmasked tile of a row always moves it (m = -inf)
                const bool grow = m == -INFINITY ? mt > -INFINITY : mt > m + kRescaleLog2;
                const float m_new = grow ? mt : m;
                const float m_use = m_new == -INFINITY ? 0.f : m_new;
                const float corr = grow ? fast_exp2(m - m_use) : 1.f;
                if (j > 0) {
                    // PV_t(j-1) has finished (it precedes S_t(j) in the tensor pipe); O may be rescaled
                    if (!mbar_wait(bar(BAR_PEMPTY + t), (pv_base + j - 1) & 1, p.dev_err)) { ok = false; break; }
                    tc_fence_after();
                    if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                        for (int c = 0; c < HD / 32; ++c) {
                            float o[32];
                            tmem_ld32(o_col + c * 32, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i) o[i] *= corr;
                            tmem_st32(o_col + c * 32, o);
                        }
                        tmem_wait_st();
                        exp_pass(m_use, false);  // P against the new max (tcgen05.ld is warp-wide: all rows redo)
                    }
                }
                // P as bf16 pairs into TMEM columns [0, 64) of S (the S values there were read above)
                tmem_st32u(s_col, *reinterpret_cast<uint32_t(*)[32]>(pk));
                tmem_st32u(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(pk + 32));
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(BAR_PFULL + t));
                float s0, s1;
                f2_unpack(sum2, s0, s1);
                l = l * corr + (s0 + s1);
                m = m_new;
            }
            if (!ok) break;
            if (!mbar_wait(bar(BAR_PEMPTY + t), (pv_base + it.nkv[t] - 1) & 1, p.dev_err)) break;
            pv_base += it.nkv[t];
            tc_fence_after();
            const float inv = 1.0f / l;
            const size_t orow = (((size_t)it.b * p.n_tok + it.q0[t] + r) * p.Hq + it.h) * HD;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                float o[32];
                tmem_ld32(o_col + c * 32, o);
                tmem_wait_ld();
                if (r < it.rows[t])
                    store_scaled32(p.out + orow + c * 32, p.out_f32 ? p.out_f32 + orow + c * 32 : nullptr, o, inv);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(BAR_OFREE + t));  // O_t may be overwritten by the next item
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

bool prefill_tc_supported(int D) { return D == 64 || D == 128 || D == 256; }

cudaError_t launch_attend_prefill_tc(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                     const CUtensorMap &tv, int B, int n_tok, int start_pos, int Hq, int Hkv,
                                     int max_seq, int D, float scale, __nv_bfloat16 *out, float *out_f32,
                                     unsigned *dev_err) {
    PrefillParams p;
    p.B = B;
    p.n_tok = n_tok;
    p.start_pos = start_pos;
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.G = Hq / Hkv;
    p.max_seq = max_seq;
    p.n_pairs = (n_tok + 2 * BM - 1) / (2 * BM);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.out_f32 = out_f32;
    p.dev_err = dev_err;
    // persistent: one CTA per SM walks the items (pairs of query tiles) in rounds
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int n_items = p.n_pairs * B * Hq;
    const unsigned grid = (unsigned)(n_items < sms ? n_items : sms);
    auto run = [&](auto kernel, int smem) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        kernel<<<grid, kPThreads, smem, st>>>(tq, tk, tv, p);
        return cudaGetLastError();
    };
    if (D == 64) return run(attn_prefill_tc_kernel<64>, PrefillLayout<64>::SMEM);
    if (D == 128) return run(attn_prefill_tc_kernel<128>, PrefillLayout<128>::SMEM);
    if (D == 256)
        return launch_attend_prefill_hd256(st, tq, tk, tv, B, n_tok, start_pos, Hq, Hkv, max_seq, scale, out, out_f32,
                                           dev_err);
    return cudaErrorInvalidValue;
}
