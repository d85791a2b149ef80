// attn_decode_i8.cu -- split-K GQA decode attention over tinyllm's INT8 KV cache on B200 tensor cores.
//
// Same contract as the other decode kernels (attn_decode.cu, attn_decode_tc.cu): every (sequence, kv head,
// key chunk) item leaves an unnormalised partial (m, l, o[G][D]) that attn_decode_combine merges.  The
// arithmetic is tinyllm's INT8 branch (src/eif_tinyllm.c:563-571, 618-625): score_t = (q . code_k[t]) *
// k_scale[t] * scale, softmax, o = sum_t (p_t * v_scale[t]) * code_v[t].
//
// Structure (persistent, one CTA per SM, 4 NG + 1 warps):
//   last warp, producer: one lane streams K and V tiles of 64 keys x D int8 codes through an NS-stage ring
//           with 3-D TMA tile loads (boxes of 64 keys x 128 bytes with the 128-byte swizzle at head_dim >= 128,
//           64 keys x 64 bytes with the 64-byte swizzle at head_dim 64; no multicast) and copies
//           the tile's 64 K and 64 V scales (aligned 256-byte runs of the head-major scale rows) into the
//           same stage with bulk asynchronous copies on the same "full" mbarrier;
//   warps 0 .. NW-1 consumers in NG groups of KG = 64 / KPW warps that take tiles round-robin: at head_dim 64
//           eight groups of two, each warp 32 keys of a tile (two 16-key halves, independent work for the
//           scheduler); at 128 two groups and at 256 one group of four, 16 keys a warp (as the registers
//           allow).  Per 16 keys:
//     S = Q K^T   in exact integer arithmetic (mma.m16n8k32 on 8-bit operands, int32 accumulators): the
//                 query of each head, scaled by a power of two so that its largest |q| lies in [2^21, 2^22),
//                 is rounded to integers and split into bytes q = hi * 2^16 + mid * 2^8 + lo; one u8 x s8
//                 MMA takes mid (rows 0-7 = the G <= 8 heads) and lo (rows 8-15), one s8 x s8 MMA takes hi;
//                 B = the K codes exactly as ldmatrix delivers them from the int8 tile viewed as 16-bit pairs
//                 (key g, dims 4t .. 4t+3 = the MMA's k slots 4t .. 4t+3): no widening of K at all;
//     softmax     online in base 2; the S accumulator of a thread (head g, keys 2t, 2t+1, 2t+8, 2t+9) is
//                 already the A-fragment layout of P, so no transpose;
//     O += P V    A = p * v_scale (f16 high / low rows as for q); B = the V codes from ldmatrix.trans of
//                 the 16-bit view, which gives each thread two keys of two adjacent dims: the even dims
//                 and the odd dims of a 16-dim chunk form two n-tiles.
// Exactness: the score sums are exact integers (the query quantised to 22 bits of its head's largest
// element), combined with one rounding; in P V codes are exact in f16, products are exact in the fp32
// accumulator and p * v_scale is split as hi + lo (22 significant bits) after scaling by a power of two that
// keeps the largest v_scale seen times 2^k below 2^14 (adapted tile by tile, never raised, so no f16 part
// overflows whatever the values' magnitude); the scalings are undone exactly.  Results match fp32 arithmetic
// on the codes to ~1e-7.
#include <cuda_fp16.h>
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int KT = 64;          // keys per tile
constexpr int kSmemLimit = 227 * 1024;
constexpr int HS = 8;           // head slots: MMA rows g (high part) and g + 8 (low part)

// NG consumer groups take alternate tiles (more tiles in flight per SM where the registers allow).
// KH kv heads a stage: 2 ("pair" mode, head_dim 64 with an even kv-head count) puts both halves of every 128-byte
// cache row in one stage, so a tile streams whole rows (a stage of one head's 64-byte halves leaves the other
// halves of the same DRAM pages to another CTA later, which caps the stream near 0.57 of the copy peak); the
// consumer groups then split by head.
template <int D, int NG, int KH, int KPW>
struct I8Cfg {
    static constexpr int KG = KT / KPW;               // consumer warps per group: KPW keys of a tile each
    static constexpr int NW = KG * NG;                // consumer warps
    static constexpr int TG = NG / KH;                // tiles in flight (consumer groups per tile: KH)
    static constexpr int THREADS = 32 * (NW + 1);
    static constexpr int BW = D >= 128 ? 128 : 64;    // box width in code bytes (= dims); the swizzle span
    static constexpr int BOX = 64 * BW;               // 64 keys x BW code bytes
    static constexpr int TILE = (D / BW) * BOX;       // K (or V) tile bytes of one head
    static constexpr int STAGE = 2 * KH * TILE;       // [K head 0 .. KH-1][V head 0 .. KH-1]
    static constexpr int SCALES = 2 * KH * KT * 4;    // per stage: [head][K, V][64 keys] scales
    static constexpr int QSLOT = KH * HS * D * 4;     // the query rows of an item (KH x G heads)
    static constexpr int EXTRA = 2 * QSLOT                    // two query slots
                                 + NW * HS * D * 4            // merge buffer o
                                 + 2 * NW * HS * 4            // merge m, l
                                 + 64 * 8                     // barriers
                                 + 1024;                      // alignment slack
    static constexpr int NS_FIT = (kSmemLimit - EXTRA) / (STAGE + SCALES);
    // a multiple of NG: consecutive uses of a stage within an item go to the same group, which has consumed
    // the previous use itself before it polls the next (a parity wait cannot tell use k from use k-2, and
    // TMA copies complete out of order)
    static constexpr int NS = (NS_FIT > 16 ? 16 : NS_FIT) / TG * TG;
    static constexpr int SMEM = NS * (STAGE + SCALES) + EXTRA;
    static_assert(NS >= 2 && NS % TG == 0, "ring depth a multiple of the tiles in flight");
    static_assert(NG % KH == 0, "consumer groups a multiple of the heads a stage");
};

struct I8Params {
    const float *q;
    const float *ks, *vs;  // [B][Hkv][sstride] scales
    const int *pos;
    const int *row_seq;  // nullptr, or the cache sequence of each query row (prefill rows)
    int max_seq, max_len, Hkv, G, Hq, sstride;
    int nchunk, chunk_keys, n_items;
    float qscale;  // scale * log2(e)
    float *part_o;
    float2 *part_ml;
    unsigned *dev_err;
};

struct ItemInfo {
    int b, cb, kvh, c, t_begin, t_end, ntiles;  // b: query row, cb: its cache sequence, kvh: first kv head, c: chunk
};

// item = ((row * (Hkv / KH)) + head group) * nchunk + chunk
template <int KH>
__device__ __forceinline__ ItemInfo item_info(const I8Params &p, int item, bool report) {
    ItemInfo it;
    const int unit = item / p.nchunk, c = item - unit * p.nchunk, hg = p.Hkv / KH;
    it.b = unit / hg;
    it.kvh = (unit - it.b * hg) * KH;
    it.c = c;
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

// Two of the four codes of `u` (= packed int8 ^ 0x80808080, i.e. x + 128 per byte) as an exact f16 pair:
// byte_perm places each byte under 0x64 (f16 0x64uu = 1024 + u), then 1152 = 1024 + 128 is subtracted.
__device__ __forceinline__ uint32_t codes_f16x2(uint32_t u, uint32_t sel) {
    const uint32_t h = __byte_perm(u, 0x64646464u, sel);
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
    return r;
}
constexpr uint32_t kSelB02 = 0x5240, kSelB13 = 0x5341;  // bytes (0, 2) / (1, 3)

// (x0, x1) = hi + lo with hi = f16(x), lo = f16(x - hi); x0 in the low halves.
__device__ __forceinline__ void split_f16x2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Byte b of each of x0 .. x3, packed in that order (the 4 k-slots of one 8-bit MMA fragment register).
__device__ __forceinline__ uint32_t byte_column(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3, uint32_t b) {
    const uint32_t sel = b | ((b + 4) << 4);
    return __byte_perm(__byte_perm(x0, x1, sel), __byte_perm(x2, x3, sel), 0x5410);
}

// D = A(16x32, row) * B(32x8, col) + D in exact integer arithmetic: A unsigned bytes (u8) or signed (s8), B the
// signed int8 codes.
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory address of the 16-byte chunk `chunk` (16 dims) of row `key` in a tile of boxes of 64 keys x
// BW bytes: the TMA 128-byte swizzle XORs the chunk index with the row index mod 8 (BW 128), the 64-byte
// swizzle bits 4-5 of the offset with bits 7-8 (BW 64).
template <int BW>
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int key, int chunk) {
    if constexpr (BW == 128)
        return base + (chunk >> 3) * 8192 + key * 128 + (((chunk & 7) ^ (key & 7)) << 4);
    else
        return base + (chunk >> 2) * 4096 + key * 64 + (((chunk & 3) ^ ((key >> 1) & 3)) << 4);
}

template <int D, int NG, int KH, int KPW>
__global__ void __launch_bounds__(I8Cfg<D, NG, KH, KPW>::THREADS, 1)
    attn_decode_i8_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const I8Params p) {
    using C = I8Cfg<D, NG, KH, KPW>;
    constexpr int kGroup = C::KG, NH = KPW / 16;  // warps per group; 16-key halves a warp takes per tile
    constexpr int TG = C::TG;
    constexpr int NS = C::NS, KS = D / 16, NT = D / 8, NW = C::NW;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_align1024(smem_raw);
    float *sbuf = reinterpret_cast<float *>(smem + NS * C::STAGE);  // [NS][KH][2][64] K, V scales per stage
    float *qbuf = sbuf + NS * KH * 2 * KT;                          // [2][KH * G][D] query rows of an item
    float *ow = qbuf + 2 * KH * HS * D;                             // [NW][HS][D]
    float *mw = ow + NW * HS * D;                                   // [NW][HS]
    float *lw = mw + NW * HS;                                       // [NW][HS]
    uint64_t *bars = reinterpret_cast<uint64_t *>(lw + NW * HS);
    // bars: full[NS], empty[NS], merged, drained, qfull[2], qempty[2]
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NS);
    const uint32_t merged = smem_u32(bars + 2 * NS), drained = smem_u32(bars + 2 * NS + 1);
    const uint32_t qfull0 = smem_u32(bars + 2 * NS + 2), qempty0 = smem_u32(bars + 2 * NS + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, kGroup * KH);  // the warps of the KH groups that take the tile
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
        // one lane: per item a bulk copy of its query rows into one of two slots, so the consumers never wait
        // on a global load between items; per tile the TMA loads of the K / V codes and two bulk copies of
        // their 64 K / V scales (256-byte runs of the head-major scale rows; keys past t_end come along and
        // are masked)
        if (lane != 0) return;
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        const uint32_t qbytes = (uint32_t)(KH * p.G * D * 4);
        uint32_t it = 0, qn = 0;
        for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++qn) {
            const ItemInfo inf = item_info<KH>(p, item, false);
            const uint32_t qs = qn & 1;  // slot use qn >> 1 waits for the consumers' release of the previous use
            if (!mbar_wait(qempty0 + 8 * qs, ((qn >> 1) & 1) ^ 1, p.dev_err)) return;
            mbar_arrive_expect_tx(qfull0 + 8 * qs, qbytes);
            bulk_load(smem_u32(qbuf + qs * KH * HS * D), p.q + ((size_t)inf.b * p.Hq + (size_t)inf.kvh * p.G) * D,
                      qbytes, qfull0 + 8 * qs);
            for (int i = 0; i < inf.ntiles; ++i, ++it) {
                const uint32_t s = it % NS, ph = (it / NS) & 1;
                if (!mbar_wait(empty0 + 8 * s, ph ^ 1, p.dev_err)) return;
                const uint32_t fb = full0 + 8 * s;
                const int t0 = inf.t_begin + i * KT;
                const int row = inf.cb * p.max_seq + t0;
                mbar_arrive_expect_tx(fb, C::STAGE + C::SCALES);
                const uint32_t kdst = smem_u32(smem + s * C::STAGE), vdst = kdst + KH * C::TILE;
#pragma unroll
                for (int h = 0; h < KH; ++h) {
#pragma unroll
                    for (int j = 0; j < D / C::BW; ++j) {
                        tma_load_3d(kdst + h * C::TILE + j * C::BOX, &tmK, j * C::BW, inf.kvh + h, row, fb);
                        tma_load_3d(vdst + h * C::TILE + j * C::BOX, &tmV, j * C::BW, inf.kvh + h, row, fb);
                    }
                    const size_t srow = ((size_t)inf.cb * p.Hkv + inf.kvh + h) * p.sstride + t0;
                    const uint32_t sdst = smem_u32(sbuf + (s * KH + h) * 2 * KT);
                    bulk_load(sdst, p.ks + srow, KT * 4, fb);
                    bulk_load(sdst + KT * 4, p.vs + srow, KT * 4, fb);
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    const int g = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, mr = lane & 7;               // ldmatrix: matrix / row this lane addresses
    const int grp = warp / kGroup, wk = (warp % kGroup) * KPW;  // group; first tile row of this warp's keys
    const int tg = grp / KH, hh = grp - tg * KH;                 // the group's tile slot and head within the stage
    const int my_key = wk + (mi & 1) * 8 + mr;             // tile row (key) of this lane's ldmatrix rows
    uint32_t it_base = 0, item_no = 0;
    for (int item = blockIdx.x; item < p.n_items; item += gridDim.x, ++item_no) {
        const ItemInfo inf = item_info<KH>(p, item, warp == 0 && lane == 0);

        // ---- query fragments: head g of the kv group, dims (4t .. 4t+3) of every 16-dim chunk (the k slots
        //      4t .. 4t+3 of the 8-bit MMA's A fragment)
        const bool on = g < p.G;
        const uint32_t qs = item_no & 1;
        if (!mbar_wait(qfull0 + 8 * qs, (item_no >> 1) & 1, p.dev_err)) return;
        const float *qh = qbuf + qs * KH * HS * D + (hh * p.G + (on ? g : 0)) * D;
        float qv[KS][4];
        float amax = 0.f;
#pragma unroll
        for (int kc = 0; kc < KS; ++kc) {
            const float4 q4 = *reinterpret_cast<const float4 *>(qh + kc * 16 + 4 * t);
            qv[kc][0] = on ? q4.x * p.qscale : 0.f;
            qv[kc][1] = on ? q4.y * p.qscale : 0.f;
            qv[kc][2] = on ? q4.z * p.qscale : 0.f;
            qv[kc][3] = on ? q4.w * p.qscale : 0.f;
            amax = fmax3(amax, fmaxf(fabsf(qv[kc][0]), fabsf(qv[kc][1])), fmaxf(fabsf(qv[kc][2]), fabsf(qv[kc][3])));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(qempty0 + 8 * qs);
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        int e2 = 0;
        if (amax > 0.f && isfinite(amax)) {
            int ex;
            frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
            e2 = max(-126, min(126, 22 - ex));
        }
        // the head's q as integers of at most 22 bits (its largest |q| scaled into [2^21, 2^22)), split into
        // bytes q = hi * 2^16 + mid * 2^8 + lo: mid and lo unsigned, hi (|hi| <= 64) signed
        const float qmul = __int_as_float((127 + e2) << 23), qdiv = __int_as_float((127 - e2) << 23);
        uint32_t qlo[KS], qmid[KS], qhi[KS];
#pragma unroll
        for (int kc = 0; kc < KS; ++kc) {
            const uint32_t x0 = (uint32_t)__float2int_rn(qv[kc][0] * qmul), x1 = (uint32_t)__float2int_rn(qv[kc][1] * qmul);
            const uint32_t x2 = (uint32_t)__float2int_rn(qv[kc][2] * qmul), x3 = (uint32_t)__float2int_rn(qv[kc][3] * qmul);
            qlo[kc] = byte_column(x0, x1, x2, x3, 0);
            qmid[kc] = byte_column(x0, x1, x2, x3, 1);
            qhi[kc] = byte_column(x0, x1, x2, x3, 2);
        }

        float oacc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
        float m_run = -INFINITY, l_run = 0.f;
        // p * v_scale enters the f16 P operand multiplied by pmul (a power of two, uniform over the warp): p <= 1,
        // so the largest v_scale seen times pmul below 2^14 keeps every f16 part finite; pmul is set from the
        // first tile and only ever lowered (the accumulators are rescaled with it, exactly), whatever the
        // magnitude of the values
        float pmul = 0.f;

        for (int i = tg; i < inf.ntiles; i += TG) {  // this group's tiles of the item (its head of each)
            const uint32_t it = it_base + i;
            const uint32_t s = it % NS, ph = (it / NS) & 1;
            const int key0 = inf.t_begin + i * KT + wk;         // first key of this warp
            const int nvalid = inf.t_end - key0;                // keys of the warp below t_end (may be <= 0)
            if (!mbar_wait(full0 + 8 * s, ph, p.dev_err)) return;
            const float *scs = sbuf + (s * KH + hh) * 2 * KT + wk;  // this warp's keys: K scales, V scales at +64
            const uint32_t kbase = smem_u32(smem + s * C::STAGE) + hh * C::TILE, vbase = kbase + KH * C::TILE;

            // ---- S = Q K^T in integers, per 16-key half h: n-tiles of keys 0-7 and 8-15 of the half; the K codes
            //      from ldmatrix are the B fragments as they are (key g, dims 4t .. 4t+3 of a 16-dim chunk).  A u8
            //      MMA takes mid (rows g) and lo (rows g + 8), an s8 MMA hi (rows g); sums of 256 products stay in
            //      int32.  A half's sums become scores before the next half starts (fewer live registers).
            //      Online softmax (base 2) for head g over keys 16h + (2t, 2t+1, 8+2t, 9+2t); the score of a key
            //      is hi * 2^16 + (mid * 2^8 + lo) (the bracket exact in int32), rounded once in the FMA.
            float sv[4 * NH], vsc[4 * NH];
            float mx = -INFINITY;
#pragma unroll
            for (int hf = 0; hf < NH; ++hf) {
                int aml[2][4], ah[2][4];
#pragma unroll
                for (int n = 0; n < 2; ++n)
                    aml[n][0] = aml[n][1] = aml[n][2] = aml[n][3] = ah[n][0] = ah[n][1] = ah[n][2] = ah[n][3] = 0;
#pragma unroll
                for (int kp = 0; kp < KS / 2; ++kp) {
                    uint32_t r0, r1, r2, r3;  // (keys 0-7 | 8-15 of the half) x (chunk 2kp | 2kp+1)
                    ldsm_x4(tile_addr<C::BW>(kbase, my_key + 16 * hf, 2 * kp + (mi >> 1)), r0, r1, r2, r3);
                    const int c0 = 2 * kp, c1 = 2 * kp + 1;
                    mma_u8s8_16832(aml[0], qmid[c0], qlo[c0], qmid[c1], qlo[c1], r0, r2);
                    mma_u8s8_16832(aml[1], qmid[c0], qlo[c0], qmid[c1], qlo[c1], r1, r3);
                    mma_s8s8_16832(ah[0], qhi[c0], 0u, qhi[c1], 0u, r0, r2);
                    mma_s8s8_16832(ah[1], qhi[c0], 0u, qhi[c1], 0u, r1, r3);
                }
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {  // keys past t_end: masked (their scale slots hold stale values)
                    const int e = 4 * hf + q4, n = q4 >> 1, j = q4 & 1;
                    const int kk = 16 * hf + 8 * n + 2 * t + j;
                    const bool ok = kk < nvalid;
                    const float raw = fmaf((float)ah[n][j], 65536.f, (float)(aml[n][j] * 256 + aml[n][2 + j]));
                    vsc[e] = ok ? scs[KT + kk] : 0.f;
                    sv[e] = ok ? (raw * qdiv) * scs[kk] : -INFINITY;
                    mx = fmaxf(mx, sv[e]);
                }
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            // this lane's largest V scale: p <= 1, so p * v_scale * pmul stays below 2^14 (f16 parts finite) while
            // vmx * pmul < 2^14; checked in the rescale vote below
            float vmx = 0.f;
#pragma unroll
            for (int e = 0; e < 4 * NH; ++e) vmx = fmaxf(vmx, vsc[e]);
            const bool need = vmx * pmul >= 16384.f || (pmul == 0.f && vmx > 0.f);
            const float m_new = fmaxf(m_run, mx);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float corr = fast_exp2(m_run - m_use);
            float pe[4 * NH], psum = 0.f;
#pragma unroll
            for (int e = 0; e < 4 * NH; ++e) {
                pe[e] = fast_exp2(sv[e] - m_use);
                psum += pe[e];
            }
            l_run = l_run * corr + psum;
            m_run = m_new;
            if (__any_sync(0xffffffffu, corr != 1.f || need)) {  // a new running max, or a new P scale
                float ocorr = corr;
                if (__any_sync(0xffffffffu, need)) {  // rare: the warp's keys (lanes t) agree on pmul
                    float w = vmx;
                    w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, 1));
                    w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, 2));
                    if (w * pmul >= 16384.f || pmul == 0.f) {
                        int ex;
                        frexpf(w, &ex);  // w in [2^(ex-1), 2^ex): w * np in [2^13, 2^14)
                        const float np = __int_as_float((127 + max(-126, min(126, 14 - ex))) << 23);
                        if (pmul != 0.f) ocorr *= np / pmul;  // a power of two: exact
                        pmul = np;
                    }
                }
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    oacc[n][0] *= ocorr;
                    oacc[n][1] *= ocorr;
                    oacc[n][2] *= ocorr;
                    oacc[n][3] *= ocorr;
                }
            }

            // ---- O += P V per half: rows g (hi) / g+8 (lo) of P, k slots = the half's keys (2t, 2t+1) and
            //      (8+2t, 9+2t); ldmatrix.trans of (keys 0-7 | 8-15) x (chunk 2cp | 2cp+1); even / odd dims of a
            //      chunk are n-tiles 2c and 2c+1
#pragma unroll
            for (int hf = 0; hf < NH; ++hf) {
                uint32_t pa0, pa1, pa2, pa3;
                split_f16x2(pe[4 * hf] * vsc[4 * hf] * pmul, pe[4 * hf + 1] * vsc[4 * hf + 1] * pmul, pa0, pa1);
                split_f16x2(pe[4 * hf + 2] * vsc[4 * hf + 2] * pmul, pe[4 * hf + 3] * vsc[4 * hf + 3] * pmul, pa2, pa3);
#pragma unroll
                for (int cp = 0; cp < D / 32; ++cp) {
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4_t(tile_addr<C::BW>(vbase, my_key + 16 * hf, 2 * cp + (mi >> 1)), r0, r1, r2, r3);
                    r0 ^= 0x80808080u;
                    r1 ^= 0x80808080u;
                    r2 ^= 0x80808080u;
                    r3 ^= 0x80808080u;
                    mma_f16_16816(oacc[4 * cp + 0], pa0, pa1, pa2, pa3, codes_f16x2(r0, kSelB02), codes_f16x2(r1, kSelB02));
                    mma_f16_16816(oacc[4 * cp + 1], pa0, pa1, pa2, pa3, codes_f16x2(r0, kSelB13), codes_f16x2(r1, kSelB13));
                    mma_f16_16816(oacc[4 * cp + 2], pa0, pa1, pa2, pa3, codes_f16x2(r2, kSelB02), codes_f16x2(r3, kSelB02));
                    mma_f16_16816(oacc[4 * cp + 3], pa0, pa1, pa2, pa3, codes_f16x2(r2, kSelB13), codes_f16x2(r3, kSelB13));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * s);
        }

        it_base += inf.ntiles;

        // ---- item epilogue: l over the 4 lanes of a head, hi + lo rows, merge the NW warps
        float l = l_run;
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        // the previous item's merge must be finished reading ow before it is overwritten
        if (item_no > 0 && !mbar_wait(drained, (item_no - 1) & 1, p.dev_err)) return;
        if (on) {
            float *oh = ow + (warp * HS + g) * D;
            const float unscale = __int_as_float(max(0, 254 - ((__float_as_int(pmul) >> 23) & 0xff)) << 23);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
                const int d = (n >> 1) * 16 + 4 * t + (n & 1);  // n-tile n, column 2t -> dim d; 2t+1 -> d + 2
                oh[d] = (oacc[n][0] + oacc[n][2]) * unscale;
                oh[d + 2] = (oacc[n][1] + oacc[n][3]) * unscale;
            }
            if (t == 0) {
                mw[warp * HS + g] = m_run;
                lw[warp * HS + g] = l;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(merged);
        if (!mbar_wait(merged, item_no & 1, p.dev_err)) return;
        // per kv head h2 of the stage: merge the warps of its groups (w = (tile slot * KH + h2) * 4 + k) into the
        // partial of (row, kv head, chunk)
        for (int idx = threadIdx.x; idx < KH * p.G * D; idx += 32 * NW) {
            const int h2 = idx / (p.G * D), hd = idx - h2 * p.G * D, h = hd / D, d = hd - h * D;
            const size_t pbase = (((size_t)inf.b * p.Hkv + inf.kvh + h2) * p.nchunk + inf.c) * p.G;
            float M = -INFINITY;
#pragma unroll
            for (int t2 = 0; t2 < TG; ++t2)
#pragma unroll
                for (int k = 0; k < kGroup; ++k) M = fmaxf(M, mw[((t2 * KH + h2) * kGroup + k) * HS + h]);
            float O = 0.f, L = 0.f;
            if (M != -INFINITY) {
#pragma unroll
                for (int t2 = 0; t2 < TG; ++t2)
#pragma unroll
                    for (int k = 0; k < kGroup; ++k) {
                        const int w = (t2 * KH + h2) * kGroup + k;
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

template <int D, int NG, int KH, int KPW>
cudaError_t launch_i8_t(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv, I8Params p, int sm_count) {
    using C = I8Cfg<D, NG, KH, KPW>;
    cudaError_t e =
        cudaFuncSetAttribute(attn_decode_i8_kernel<D, NG, KH, KPW>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    p.n_items /= KH;  // items of KH kv heads each
    const int grid = p.n_items < sm_count ? p.n_items : sm_count;
    attn_decode_i8_kernel<D, NG, KH, KPW><<<grid, C::THREADS, C::SMEM, st>>>(tk, tv, p);  // not a programmatic dependent (see launch_attend_decode)
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attend_decode_i8(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                    const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                    float2 *part_ml, int sm_count) {
    I8Params p;
    p.q = a.q;
    p.ks = a.k_scale;
    p.vs = a.v_scale;
    p.sstride = a.scale_stride;
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
    switch (a.D) {
        case 64:  // four groups; with an even kv-head count both heads of a 128-byte cache row a stage
            return decode_i8_heads_per_item(64, p.Hkv) == 2 ? launch_i8_t<64, 8, 2, 32>(st, tk, tv, p, sm_count)
                                                             : launch_i8_t<64, 8, 1, 32>(st, tk, tv, p, sm_count);
        case 128: return launch_i8_t<128, 2, 1, 16>(st, tk, tv, p, sm_count);
        case 256: return launch_i8_t<256, 1, 1, 16>(st, tk, tv, p, sm_count);  // 249 registers: one group
        default: return cudaErrorInvalidValue;
    }
}
