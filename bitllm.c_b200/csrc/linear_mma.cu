// linear_mma.cu -- the integer-weight projections (INT8 head, INT4, 2-bit ternary with a scale a row) on the
// tensor cores: out[t] = W x[t] for n tokens, with the same results as fp32 arithmetic to ~1e-7.
//
// Reference: linear_gemv / linear_gemm / int8_gemv (src/eif_qwen35.c:384-443, 1033-1063) and the BitNet
// kernel eif_matmul_bitnet_f32 (src/eif_quantize_bitnet.c:834-889); formats as in linear.cu.
//
// Exactness: weights are small integers (|w| <= 128), exact in f16.  Each token's x is scaled by a power of two
// so that its largest |x| lies in [2^13, 2^14) and split as hi = f16(x), lo = f16(x - hi) (22 significant bits);
// the products w * hi and w * lo are exact in the fp32 accumulator of mma.m16n8k16, and the scaling is undone
// exactly after the sum.
//
// Structure: 8 warps a CTA, split as RG row tiles x KS column slices (RG * KS = 8; KS > 1 spreads short, wide
// matrices over more warps, the slices' sums meeting in shared memory).  A warp owns 16 rows (MMA rows g and
// g + 8 of lane (g, t)) and streams them in blocks of 64 bytes a row: lane t of a row quad loads 16 bytes of rows
// g and g + 8 (4-byte words w), so a warp instruction moves 8 rows x 64 contiguous bytes.  The lane's words are
// decoded straight into A fragments: an integer field k in the low byte under 0x64 is the f16 1024 + k (one
// byte permute for two weights), one f16x2 subtract removes the bias.  Because the reduction order is free,
// each k16 step takes the four weights a lane decodes together (slots 2t, 2t+1, 2t+8, 2t+9), and x is staged in
// shared memory in that order (per word, the format's decode order), one f16 plane for hi and one for lo:
//   INT8   word = 4 columns, one step;        pairs (0, 1) (2, 3);          bias 1152 (codes ^ 0x80)
//   INT4   word = 8 columns, two steps;       pairs (0, 2) (4, 6) | (1, 3) (5, 7) (high / low nibbles); bias 1032
//   2-bit  word = 16 columns, four steps;     k = 1 + bit0 - bit1 for all fields at once, field q of each byte
//          masked in place: step q has pairs (q, 4+q) (8+q, 12+q) as 1024 + 4^q k, bias 1024 + 4^q, so the
//          weights carry 4^q; the staged x of that step's columns is scaled by 4^-q (exact) to match.
// Row pitch of the staged x: each lane's 16-byte range of columns is followed by 4 empty f16 slots and a token
// row is padded to 32 (mod 128) bytes, so the B-fragment loads (8 tokens x 4 lanes x 8 bytes) hit 32 distinct
// banks.  Launched as a programmatic dependent (the first weights are fetched before griddepcontrol.wait).
#include <cuda_fp16.h>

#include "internal.h"
#include "common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kPad = 4;  // empty f16 slots after each lane range
constexpr int kStages = 4;  // weight ring depth a warp (1 KB a stage: 16 rows x 64 bytes)
constexpr size_t kSmemCap = 200 * 1024;

__host__ __device__ constexpr int mma_cpw(int wt) {
    return wt == EIF_CUDA_W_INT8 ? 4 : wt == EIF_CUDA_W_INT4 ? 8 : 16;
}


__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
// 16-byte asynchronous global -> shared copy, L2 only (the weights are streamed once)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bytes (lo, hi) of `v` under 0x64 as an f16 pair, minus the bias pair
__device__ __forceinline__ uint32_t pair_f16(uint32_t v, uint32_t sel, uint32_t bias2) {
    const uint32_t h = __byte_perm(v, 0x64646464u, sel);
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(bias2));
    return r;
}
constexpr uint32_t kSel01 = 0x5140, kSel23 = 0x5342;  // bytes (0, 1) / (2, 3) of v, each under a 0x64 byte

// Position (f16 slot) of column c within a staged token row: lane range c / CPL, then the word, then the
// format's decode order within the word.
template <int WT>
__device__ __forceinline__ int xpos(int c) {
    constexpr int CPW = mma_cpw(WT), CPL = 4 * CPW;
    const int tr = c / CPL, o = c - tr * CPL, wi = o / CPW, cw = o - wi * CPW;
    int pw;
    if constexpr (WT == EIF_CUDA_W_INT8)
        pw = cw;
    else if constexpr (WT == EIF_CUDA_W_INT4)
        pw = (cw & 1) * 4 + (cw >> 1);  // order 0 2 4 6 1 3 5 7
    else
        pw = (cw & 3) * 4 + (cw >> 2);  // order 0 4 8 12 1 5 9 13 ...: step q = cw & 3
    return tr * (CPL + kPad) + wi * CPW + pw;
}

// the power of two column c's staged x carries (2-bit: 4^-q of its step)
template <int WT>
__device__ __forceinline__ float xstep_scale(int c) {
    if constexpr (WT == EIF_CUDA_W_TERNARY2) {
        const int q = c & 3;  // the field within its byte = the step within its word
        return __int_as_float((127 - 2 * q) << 23);
    } else {
        return 1.f;
    }
}

// column (0..15) of a 16-column unit that decode position 4k + i of the unit holds (units start on 16 columns)
template <int WT>
__host__ __device__ constexpr int group_col(int k, int i) {
    return WT == EIF_CUDA_W_INT8 ? 4 * k + i : WT == EIF_CUDA_W_INT4 ? 8 * (k >> 1) + (k & 1) + 2 * i : k + 4 * i;
}

struct MmaArgs {
    const uint8_t *W;
    const float *scales;  // a scale a row
    const float *x;       // [n][cols]
    float *out;           // [n][rows]
    int rows, cols, n, n_blocks, ks, pitch;  // n_blocks: 64-byte blocks a padded row; pitch: f16 a token row
    size_t stride;
};

template <int WT, int NT>
__global__ void __launch_bounds__(kThreads, 1) linear_mma_kernel(const MmaArgs a) {
    constexpr int CPW = mma_cpw(WT), CPL = 4 * CPW, SPW = CPW / 4, TOK = 8 * NT;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    // [kWarps][kStages][2][32][16 B] weight ring | x hi [TOK][pitch] | x lo | 2^-e2 [TOK] | 2^e2 [TOK] | sums
    uint8_t *ring = smem + (size_t)warp * kStages * 1024;
    __half *xh = reinterpret_cast<__half *>(smem + (size_t)kWarps * kStages * 1024);
    __half *xl = xh + (size_t)TOK * a.pitch;
    float *xinv = reinterpret_cast<float *>(xl + (size_t)TOK * a.pitch);
    float *xmul = xinv + TOK;
    float *red = xmul + TOK;  // [kWarps][NT * 4][32]
    const int KS = a.ks, RG = kWarps / KS, rg = warp / KS, ks = warp - rg * KS;
    const int n_rt = (a.rows + 15) / 16;
    // balanced slices, none empty (KS <= n_blocks): every slice's warp meets its row group at each tile's end
    const int b_begin = ks * a.n_blocks / KS, nb = (ks + 1) * a.n_blocks / KS - b_begin;
    const int rt0 = blockIdx.x * RG + rg, rt_stride = gridDim.x * RG;
    // the warp's work items j = (row tile rt0 + (j / nb) * rt_stride, block b_begin + j % nb)
    const int n_items = rt0 < n_rt ? (n_rt - rt0 + rt_stride - 1) / rt_stride * nb : 0;
    const uint32_t ring_s = smem_addr(ring) + lane * 16;

    // item j's 16 bytes of rows g and g + 8 into ring slot j % kStages (one commit group per item, empty past the end)
    auto issue = [&](int j) {
        if (j < n_items) {
            const int rt = rt0 + (j / nb) * rt_stride, b = b_begin + j % nb;
            const size_t off = (size_t)b * 64 + (size_t)t * 16;
            const int ra = min(rt * 16 + g, a.rows - 1), rb = min(rt * 16 + g + 8, a.rows - 1);
            const uint32_t dst = ring_s + (j % kStages) * 1024;
            cp_async16(dst, a.W + (size_t)ra * a.stride + off);
            cp_async16(dst + 512, a.W + (size_t)rb * a.stride + off);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < kStages - 1; ++j) issue(j);  // weights do not depend on the previous kernel
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();  // after the wait: a dependent that starts early finds every earlier grid complete

    uint32_t *tmax = reinterpret_cast<uint32_t *>(red);  // per-token largest |x| (bits), before the sums use red
    const int n_cols = a.n_blocks * 4 * CPL;  // columns of the padded rows (those past `cols` stage as zeros)
    for (int t0 = 0; t0 < a.n; t0 += TOK) {
        if (t0 > 0) {
            __syncthreads();  // the previous pass's readers of x are done
#pragma unroll
            for (int j = 0; j < kStages - 1; ++j) issue(j);
        }
        // ---- stage the token tile over all threads (16-column units of float4 loads where rows allow; else 8
        //      elements in flight a thread, its (token, column) pairs advancing by kThreads columns with no
        //      divisions): (1) every token's largest |x| (a warp max, one
        //      shared atomicMax on the bits, which order non-negative floats), (2) x * 2^e2 (the largest in
        //      [2^13, 2^14)) split into hi / lo at its decode-order position; padded columns stage as zeros (they
        //      meet zero weights); tokens past n are not staged (their MMA columns are never written out)
        const int nv = min(TOK, a.n - t0);
        // vectorised staging where every token row starts on 16 bytes and holds whole 16-column units
        const bool vec = a.cols % 16 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
        const int g16 = a.cols / 16;
        if (threadIdx.x < TOK) tmax[threadIdx.x] = 0u;
        __syncthreads();
        if (vec) {  // 16 columns a unit: four float4 loads
            const int units = nv * g16;
            for (int u0 = threadIdx.x; __any_sync(0xffffffffu, u0 < units); u0 += kThreads) {
                const int tk = u0 < units ? u0 / g16 : -1;
                float m = 0.f;
                if (tk >= 0) {
                    const float4 *src = reinterpret_cast<const float4 *>(a.x + (size_t)(t0 + tk) * a.cols + (u0 - tk * g16) * 16);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float4 f = __ldg(src + k);
                        m = fmaxf(m, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
                    }
                }
                const int tk0 = __shfl_sync(0xffffffffu, tk, 0), tk31 = __shfl_sync(0xffffffffu, tk, 31);
                if (tk0 == tk31) {
                    const uint32_t mm = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
                    if (lane == 0 && tk0 >= 0 && mm) atomicMax(&tmax[tk0], mm);
                } else if (tk >= 0 && m > 0.f) {
                    atomicMax(&tmax[tk], __float_as_uint(m));
                }
            }
        } else {
            int tk = 0, c = threadIdx.x;
            while (c >= a.cols && tk < nv) c -= a.cols, ++tk;
            // every lane runs the loop while any lane has elements left (the shuffles need the whole warp)
            while (__any_sync(0xffffffffu, tk < nv)) {
                float v[8];
                int tk8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    tk8[u] = tk;
                    v[u] = tk < nv ? fabsf(__ldg(a.x + (size_t)(t0 + tk) * a.cols + c)) : 0.f;
                    c += kThreads;
                    while (c >= a.cols && tk < nv) c -= a.cols, ++tk;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {  // one atomic a warp where its lanes share a token
                    const int tkv = tk8[u] < nv ? tk8[u] : -1;
                    const int tk0 = __shfl_sync(0xffffffffu, tkv, 0), tk31 = __shfl_sync(0xffffffffu, tkv, 31);
                    if (tk0 == tk31) {
                        if (tk0 >= 0) {
                            const uint32_t m = __reduce_max_sync(0xffffffffu, __float_as_uint(v[u]));
                            if (lane == 0 && m) atomicMax(&tmax[tk0], m);
                        }
                    } else if (tkv >= 0 && v[u] > 0.f) {
                        atomicMax(&tmax[tkv], __float_as_uint(v[u]));
                    }
                }
            }
        }
        __syncthreads();
        if (threadIdx.x < TOK) {
            const float amax = __uint_as_float(tmax[threadIdx.x]);
            int e2 = 0;
            if (amax > 0.f && isfinite(amax)) {
                int ex;
                frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
                e2 = max(-126, min(126, 14 - ex));
            }
            xinv[threadIdx.x] = __int_as_float((127 - e2) << 23);
            xmul[threadIdx.x] = __int_as_float((127 + e2) << 23);
        }
        __syncthreads();
        if (vec) {  // a unit: 16 columns, staged as four 8-byte chunks of the decode order
            const int units = nv * (n_cols / 16);
            for (int u = threadIdx.x; u < units; u += kThreads) {
                const int tk = u / (n_cols / 16), c = (u - tk * (n_cols / 16)) * 16;
                float v[16];
                if (c < a.cols) {
                    const float4 *src = reinterpret_cast<const float4 *>(a.x + (size_t)(t0 + tk) * a.cols + c);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float4 f = __ldg(src + k);
                        v[4 * k] = f.x, v[4 * k + 1] = f.y, v[4 * k + 2] = f.z, v[4 * k + 3] = f.w;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 16; ++k) v[k] = 0.f;
                }
                const float mul = xmul[tk];
                const size_t base = (size_t)tk * a.pitch + xpos<WT>(c);
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // chunk k: the four columns decode position base + 4k holds
                    float y[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) y[i] = v[group_col<WT>(k, i)] * mul * xstep_scale<WT>(group_col<WT>(k, i));
                    const __half2 h01 = __floats2half2_rn(y[0], y[1]), h23 = __floats2half2_rn(y[2], y[3]);
                    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                    const __half2 l01 = __floats2half2_rn(y[0] - f01.x, y[1] - f01.y);
                    const __half2 l23 = __floats2half2_rn(y[2] - f23.x, y[3] - f23.y);
                    *reinterpret_cast<uint2 *>(xh + base + 4 * k) =
                        make_uint2(*reinterpret_cast<const uint32_t *>(&h01), *reinterpret_cast<const uint32_t *>(&h23));
                    *reinterpret_cast<uint2 *>(xl + base + 4 * k) =
                        make_uint2(*reinterpret_cast<const uint32_t *>(&l01), *reinterpret_cast<const uint32_t *>(&l23));
                }
            }
        } else {
            int tk = 0, c = threadIdx.x;
            while (c >= n_cols && tk < nv) c -= n_cols, ++tk;
            while (tk < nv) {
                float v[8];
                int tk8[8], c8[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    tk8[u] = tk;
                    c8[u] = c;
                    v[u] = (tk < nv && c < a.cols) ? __ldg(a.x + (size_t)(t0 + tk) * a.cols + c) : 0.f;
                    c += kThreads;
                    while (c >= n_cols && tk < nv) c -= n_cols, ++tk;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (tk8[u] >= nv) break;
                    const float x = v[u] * xmul[tk8[u]] * xstep_scale<WT>(c8[u]);  // exact: powers of two
                    const __half h = __float2half_rn(x);
                    const size_t p = (size_t)tk8[u] * a.pitch + xpos<WT>(c8[u]);
                    xh[p] = h;
                    xl[p] = __float2half_rn(x - __half2float(h));
                }
            }
        }
        __syncthreads();
        // ---- the warp's items: item j + kStages - 1 is issued, item j waited for and computed
        constexpr int AC = NT == 1 ? 2 : 1;  // independent accumulator sets (with hi / lo: 2 AC NT MMA chains)
        float accs[AC][2][NT][4];
        for (int j = 0; j < n_items; ++j) {
            const int jr = j / nb, b = b_begin + (j - jr * nb), rt = rt0 + jr * rt_stride;
            if (b == b_begin) {
#pragma unroll
                for (int s2 = 0; s2 < AC; ++s2)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int e = 0; e < 4; ++e) accs[s2][h][nt][e] = 0.f;
            }
            issue(j + kStages - 1);
            cp_async_wait<kStages - 1>();  // this thread's copies of item j have landed
            const uint32_t slot = ring_s + (j % kStages) * 1024;
            const uint4 c0 = lds128(slot), c1 = lds128(slot + 512);
            const uint32_t wa[4] = {c0.x, c0.y, c0.z, c0.w}, wb[4] = {c1.x, c1.y, c1.z, c1.w};
            const int rbase = (4 * b + t) * (CPL + kPad);
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
                uint32_t fa[4], fb[4];  // per step: the word prepared so that bytes (0,1) / (2,3) are its pairs
                if constexpr (WT == EIF_CUDA_W_INT8) {
                    fa[0] = wa[wi] ^ 0x80808080u;
                    fb[0] = wb[wi] ^ 0x80808080u;
                } else if constexpr (WT == EIF_CUDA_W_INT4) {
                    fa[0] = (wa[wi] >> 4) & 0x0F0F0F0Fu;  // even columns
                    fa[1] = wa[wi] & 0x0F0F0F0Fu;         // odd columns
                    fb[0] = (wb[wi] >> 4) & 0x0F0F0F0Fu;
                    fb[1] = wb[wi] & 0x0F0F0F0Fu;
                } else {
                    const uint32_t ka = wa[wi] + 0x55555555u - 3u * ((wa[wi] >> 1) & 0x55555555u);
                    const uint32_t kb = wb[wi] + 0x55555555u - 3u * ((wb[wi] >> 1) & 0x55555555u);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        fa[q] = ka & (0x03030303u << (2 * q));
                        fb[q] = kb & (0x03030303u << (2 * q));
                    }
                }
#pragma unroll
                for (int ss = 0; ss < SPW; ++ss) {
                    uint32_t bias2;
                    if constexpr (WT == EIF_CUDA_W_INT8)
                        bias2 = 0x64806480u;  // 1152
                    else if constexpr (WT == EIF_CUDA_W_INT4)
                        bias2 = 0x64086408u;  // 1032
                    else
                        bias2 = ss == 0 ? 0x64016401u : ss == 1 ? 0x64046404u : ss == 2 ? 0x64106410u : 0x64406440u;
                    const uint32_t a0 = pair_f16(fa[ss], kSel01, bias2), a2 = pair_f16(fa[ss], kSel23, bias2);
                    const uint32_t a1 = pair_f16(fb[ss], kSel01, bias2), a3 = pair_f16(fb[ss], kSel23, bias2);
                    const int pos = rbase + wi * CPW + 4 * ss;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const size_t ro = (size_t)(nt * 8 + g) * a.pitch + pos;
                        const uint2 bh = *reinterpret_cast<const uint2 *>(xh + ro);
                        const uint2 bl = *reinterpret_cast<const uint2 *>(xl + ro);
                        mma_16816(accs[wi % AC][0][nt], a0, a1, a2, a3, bh.x, bh.y);
                        mma_16816(accs[wi % AC][1][nt], a0, a1, a2, a3, bl.x, bl.y);
                    }
                }
            }
            if (b != b_begin + nb - 1) continue;
            // ---- the row tile's last block: sum the chains; the KS slices' sums meet in shared memory
            float acc[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float v = 0.f;
#pragma unroll
                    for (int s2 = 0; s2 < AC; ++s2) v += accs[s2][0][nt][e] + accs[s2][1][nt][e];
                    acc[nt][e] = v;
                }
            if (KS > 1) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) red[((size_t)warp * NT * 4 + nt * 4 + e) * 32 + lane] = acc[nt][e];
                asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(32 * KS) : "memory");
                if (ks == 0) {
                    for (int k2 = 1; k2 < KS; ++k2)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                acc[nt][e] += red[((size_t)(warp + k2) * NT * 4 + nt * 4 + e) * 32 + lane];
                }
            }
            if (ks == 0) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int row = rt * 16 + g + (e >> 1) * 8, tk = nt * 8 + 2 * t + (e & 1), tok = t0 + tk;
                        if (row < a.rows && tok < a.n)
                            a.out[(size_t)tok * a.rows + row] = (acc[nt][e] * xinv[tk]) * __ldg(a.scales + row);
                    }
            }
            if (KS > 1) asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(32 * KS) : "memory");
        }
        cp_async_wait<0>();  // no copy of this pass outstanding
    }
}

// f16 slots of a staged token row: lane ranges of CPL columns + kPad, padded to 32 (mod 128) bytes
int mma_pitch(int wt, int n_blocks) {
    const int slots = n_blocks * 4 * (4 * mma_cpw(wt) + kPad);
    return ((2 * slots + 127) / 128 * 128 + 32) / 2;
}

size_t mma_smem(int pitch, int NT) {
    return (size_t)kWarps * kStages * 1024 + (size_t)2 * 8 * NT * pitch * 2 + 2 * 8 * NT * 4 +
           (size_t)kWarps * NT * 4 * 32 * 4;
}

template <int WT, int NT>
cudaError_t go(cudaStream_t st, MmaArgs a, size_t smem, int sm_count) {
    auto kernel = linear_mma_kernel<WT, NT>;
    static unsigned long long raised = 0;  // devices on which the dynamic shared-memory limit is at the cap
    int dev = 0;
    if (smem > 48 * 1024 && (cudaGetDevice(&dev) != cudaSuccess || dev >= 64 || !(raised >> dev & 1ull))) {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
        if (e != cudaSuccess) return e;
        if (dev < 64) raised |= 1ull << dev;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    // column slices: enough warps to fill the GPU twice over where the rows alone do not
    const int n_rt = (a.rows + 15) / 16;
    int ks = 1;
    while (ks < kWarps && n_rt * ks < 2 * kWarps * sm_count && a.n_blocks >= 2 * ks) ks *= 2;
    a.ks = ks;
    const int rg = kWarps / ks;
    int grid = (n_rt + rg - 1) / rg;
    if (grid > per_sm * sm_count) grid = per_sm * sm_count;
    return launch_pdl(kernel, dim3(grid), dim3(kThreads), smem, st, a);
}

template <int WT>
cudaError_t go_nt(cudaStream_t st, const MmaArgs &a, int NT, int sm_count) {
    const size_t smem = mma_smem(a.pitch, NT);
    switch (NT) {
        case 4: return go<WT, 4>(st, a, smem, sm_count);
        case 2: return go<WT, 2>(st, a, smem, sm_count);
        default: return go<WT, 1>(st, a, smem, sm_count);
    }
}

}  // namespace

bool linear_mma_supported(const eif_cuda_linear &lin) {
    const bool fmt = lin.wtype == EIF_CUDA_W_INT8 || lin.wtype == EIF_CUDA_W_INT4 ||
                     (lin.wtype == EIF_CUDA_W_TERNARY2 && lin.group == 0);
    return fmt && lin.stride % 64 == 0 && mma_smem(mma_pitch(lin.wtype, (int)(lin.stride / 64)), 1) <= kSmemCap;
}

cudaError_t launch_linear_mma(cudaStream_t st, const eif_cuda_linear &lin, const float *x, int n, float *out,
                              int sm_count) {
    MmaArgs a{lin.W, lin.scales, x, out, lin.rows, lin.cols, n, (int)(lin.stride / 64), 1, 0, lin.stride};
    a.pitch = mma_pitch(lin.wtype, a.n_blocks);
    int NT = n > 16 ? 4 : n > 8 ? 2 : 1;
    while (NT > 1 && mma_smem(a.pitch, NT) > kSmemCap) NT >>= 1;
    switch (lin.wtype) {
        case EIF_CUDA_W_INT8: return go_nt<EIF_CUDA_W_INT8>(st, a, NT, sm_count);
        case EIF_CUDA_W_INT4: return go_nt<EIF_CUDA_W_INT4>(st, a, NT, sm_count);
        default: return go_nt<EIF_CUDA_W_TERNARY2>(st, a, NT, sm_count);
    }
}
