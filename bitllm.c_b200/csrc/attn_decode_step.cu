// attn_decode_step.cu -- a whole tinyllm decode step of one layer for small batches, in one launch.
//
// Reference: the per-token attention block of tinyllm_forward_embedding_ex -- RoPE of the new q and k with
// the per-position tables (src/eif_tinyllm.c:395-405, rotation :480-507), the new k / v row written into
// the cache at pos (:415-418), then the head loop over rows [0, pos] (:555-656: scores q.k_t * scale,
// softmax, o = sum_t p_t v_t).  It is rope_append_kernel followed by the split-K decode and its combine,
// with the same arithmetic, for the batches where launch latency rather than HBM sets the step time.
//
// One cluster of NC CTAs per (sequence b, kv head): every CTA rotates the G query heads of the group into
// shared memory and takes one chunk of the key range, whose K and V rows it brings into shared memory with
// bulk copies issued at the start (one round trip, rows padded by 16 bytes so that lanes reading one column
// of consecutive rows hit different banks); the CTA whose chunk holds pos rotates k, writes the new K / V
// row to the cache and places its own copy of that row in the chunk (no CTA reads a row this launch writes).
// The chunk's keys are spread over the four warps.  Each CTA merges its warps into a partial
// (m, l, o[G][D]) in shared memory; after a cluster barrier every CTA combines a slice of the G x D outputs
// from all NC partials through distributed shared memory, and a second barrier keeps the partials alive
// until the last peer has read them.
// fp32 and bf16 caches, head_dim 64 / 128, G <= 8.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

constexpr int kStepThreads = 128;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepStageBytes = 100 * 1024;  // shared memory for a CTA's staged K / V rows

template <typename KT>
__device__ __forceinline__ KT to_cache(float x);
template <>
__device__ __forceinline__ float to_cache<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_cache<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Shared-memory row stride of a staged K / V row: the row plus 16 bytes.
template <typename KT, int D>
constexpr int step_row_bytes() { return D * (int)sizeof(KT) + 16; }

template <typename KT, int D, int G>
__global__ void __launch_bounds__(kStepThreads) attn_decode_step_kernel(const DecodeStepArgs a) {
    constexpr int DL = D / 32, HALF = D / 2;
    constexpr int KV_VEC = 16 / (int)sizeof(KT);
    constexpr int RB = step_row_bytes<KT, D>(), RS = RB / (int)sizeof(KT);  // row stride, bytes / elements
    static_assert(DL == 2 || DL == 4, "head_dim 64 / 128");
    const int nc = a.nc, rank = (int)cluster_ctarank();
    const int kvh = blockIdx.x / nc, b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int Hq = a.Hkv * G;

    __shared__ float sq[G][D];
    __shared__ __align__(16) KT krow[D], vrow[D];  // the new row, as stored in the cache
    __shared__ float wm[kStepWarps][G], wl[kStepWarps][G];
    __shared__ float wacc[kStepWarps][G][D];  // warp partials; the CTA partial is merged into wacc[0]
    __shared__ float pm[G], pl[G];
    __shared__ __align__(8) uint64_t rows_bar;
    extern __shared__ __align__(16) uint8_t kvs[];  // the chunk's K rows, then its V rows (stride RB)

    int p = a.pos[b];
    // pos past the bound the launch was sized for (max_pos of the _dev call) is refused like one outside
    // the cache: the staged chunk would not fit
    const bool pos_ok = p >= 0 && p < a.max_seq && (p + nc) / nc <= a.chunk_cap;
    if (!pos_ok) {
        if (threadIdx.x == 0 && rank == 0 && kvh == 0) atomicOr(a.dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
        p = -1;  // no keys, no row written: the output is zeros
    }
    const int L = p + 1, chunk = (L + nc - 1) / nc;
    const int t_begin = min(L, rank * chunk), t_end = min(L, t_begin + chunk);
    const int n_rows = t_end - t_begin;  // at most a.chunk_cap
    const bool owner = pos_ok && t_begin <= p && p < t_end;
    const size_t row_stride = (size_t)a.Hkv * D;
    KT *Kb = static_cast<KT *>(a.Kc) + ((size_t)b * a.max_seq * a.Hkv + kvh) * D;
    KT *Vb = static_cast<KT *>(a.Vc) + ((size_t)b * a.max_seq * a.Hkv + kvh) * D;
    KT *ks = reinterpret_cast<KT *>(kvs), *vs = reinterpret_cast<KT *>(kvs + (size_t)a.chunk_cap * RB);

    // the chunk's rows (all but the new one) start towards shared memory
    const uint32_t rbar = smem_u32(&rows_bar);
    const int n_copy = n_rows - (owner ? 1 : 0);
    if (threadIdx.x == 0) {
        mbar_init(rbar, 1);
        fence_barrier_init();
        mbar_arrive_expect_tx(rbar, (uint32_t)(2 * n_copy * D * (int)sizeof(KT)));
    }
    __syncthreads();
    for (int r = threadIdx.x; r < 2 * n_rows; r += kStepThreads) {
        const int t = t_begin + (r >> 1);
        if (t == p) continue;
        const bool isv = r & 1;
        bulk_load(smem_u32(kvs) + (uint32_t)((isv ? a.chunk_cap : 0) + (t - t_begin)) * RB,
                  (isv ? Vb : Kb) + (size_t)t * row_stride, D * (uint32_t)sizeof(KT), rbar);
    }

    // rotated q of the group's heads, and (owner) the rotated k: the rotation of rope_append_kernel
    const float *cs = a.cos_t + (size_t)(pos_ok ? p : 0) * HALF;
    const float *sn = a.sin_t + (size_t)(pos_ok ? p : 0) * HALF;
    for (int it = threadIdx.x; it < (G + (owner ? 1 : 0)) * HALF; it += kStepThreads) {
        const int g = it / HALF, j = it - g * HALF;
        const bool isk = g == G;
        const float *src = isk ? a.k + ((size_t)b * a.Hkv + kvh) * D : a.q + ((size_t)b * Hq + kvh * G + g) * D;
        const int ia = a.interleaved ? 2 * j : j, ib = a.interleaved ? 2 * j + 1 : j + HALF;
        const float x0 = src[ia], x1 = src[ib], c = cs[j], s = sn[j];
        const float y0 = __fmaf_rn(x0, c, -__fmul_rn(x1, s)), y1 = __fmaf_rn(x1, c, __fmul_rn(x0, s));
        if (isk) {
            krow[ia] = to_cache<KT>(y0);
            krow[ib] = to_cache<KT>(y1);
        } else {
            sq[g][ia] = y0;
            sq[g][ib] = y1;
        }
    }
    if (owner)
        for (int d = threadIdx.x; d < D; d += kStepThreads) vrow[d] = to_cache<KT>(a.v[((size_t)b * a.Hkv + kvh) * D + d]);
    __syncthreads();
    if (owner)  // the new row: into the cache, and into its place in the staged chunk
        for (int d = threadIdx.x; d < D; d += kStepThreads) {
            Kb[(size_t)p * row_stride + d] = krow[d];
            Vb[(size_t)p * row_stride + d] = vrow[d];
            ks[(size_t)(p - t_begin) * RS + d] = krow[d];
            vs[(size_t)(p - t_begin) * RS + d] = vrow[d];
        }
    // a wait that gives up leaves the partial empty (the error word tells the host)
    const bool rows_ok = mbar_wait(rbar, 0, a.dev_err);
    __syncthreads();

    float m[G], l[G], acc[G][DL];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[h][i] = 0.f;
    }
    // warp w takes keys [w0, w1) of the chunk, in blocks of 32 (lane = key for the scores)
    const int per_warp = (n_rows + kStepWarps - 1) / kStepWarps;
    const int w0 = rows_ok ? warp * per_warp : 0, w1 = rows_ok ? min(n_rows, w0 + per_warp) : 0;
    for (int t0 = w0; t0 < w1; t0 += 32) {
        const int t = t0 + lane;
        const bool valid = t < w1;
        float s[G];
#pragma unroll
        for (int h = 0; h < G; ++h) s[h] = 0.f;
        if (valid) {
            const KT *kr = ks + (size_t)t * RS;
#pragma unroll 4
            for (int d = 0; d < D; d += KV_VEC) {
                float kv[KV_VEC];
                KvLoad<KT, KV_VEC>::load(kr + d, kv);
#pragma unroll
                for (int h = 0; h < G; ++h) {
#pragma unroll
                    for (int j = 0; j < KV_VEC; ++j) s[h] += sq[h][d + j] * kv[j];
                }
            }
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
            const float sc = valid ? s[h] * a.scale : -INFINITY;
            const float m_new = fmaxf(m[h], warp_max(sc));
            const float corr = expf(m[h] - m_new);
            const float pr = valid ? expf(sc - m_new) : 0.f;
            l[h] = l[h] * corr + warp_sum(pr);
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[h][i] *= corr;
            m[h] = m_new;
            s[h] = pr;
        }
        const int nvalid = min(32, w1 - t0);
        for (int j = 0; j < nvalid; ++j) {
            const KT *vr = vs + (size_t)(t0 + j) * RS + lane * DL;
            float vv[DL];
            KvLoad<KT, DL>::load(vr, vv);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float pj = __shfl_sync(0xffffffffu, s[h], j);
#pragma unroll
                for (int i = 0; i < DL; ++i) acc[h][i] += pj * vv[i];
            }
        }
    }

    // the CTA's partial: its warps merged into wacc[0] (each element read and written by one thread)
#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (lane == 0) {
            wm[warp][h] = m[h];
            wl[warp][h] = l[h];
        }
#pragma unroll
        for (int i = 0; i < DL; ++i) wacc[warp][h][lane * DL + i] = acc[h][i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += kStepThreads) {
        const int h = i / D, d = i - h * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kStepWarps; ++w) M = fmaxf(M, wm[w][h]);
        float O = 0.f, Ls = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kStepWarps; ++w) {
                const float f = expf(wm[w][h] - M);
                O += wacc[w][h][d] * f;
                Ls += wl[w][h] * f;
            }
        }
        wacc[0][h][d] = O;
        if (d == 0) {
            pm[h] = M;
            pl[h] = Ls;
        }
    }

    // the cluster's partials -> this CTA's slice of the G x D outputs
    cluster_sync_all();
    const int per = (G * D + nc - 1) / nc;
    const uint32_t pm_a = smem_u32(pm), pl_a = smem_u32(pl), po_a = smem_u32(&wacc[0][0][0]);
    for (int i = rank * per + threadIdx.x; i < min(G * D, (rank + 1) * per); i += kStepThreads) {
        const int h = i / D;
        float M = -INFINITY;
        for (int r = 0; r < nc; ++r) M = fmaxf(M, ld_shared_cluster_f32(mapa_shared(pm_a + 4 * h, r)));
        float O = 0.f, Ls = 0.f;
        if (M != -INFINITY)
            for (int r = 0; r < nc; ++r) {
                const float f = expf(ld_shared_cluster_f32(mapa_shared(pm_a + 4 * h, r)) - M);
                O += ld_shared_cluster_f32(mapa_shared(po_a + 4 * i, r)) * f;
                Ls += ld_shared_cluster_f32(mapa_shared(pl_a + 4 * h, r)) * f;
            }
        a.out[((size_t)b * Hq + kvh * G) * D + i] = Ls > 0.f ? O / Ls : 0.f;
    }
    cluster_sync_all();  // peers may still read this CTA's partial until here
}

template <typename KT, int D>
cudaError_t launch_g(cudaStream_t st, const DecodeStepArgs &a, int G) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nc * a.Hkv, a.B, 1);
    cfg.blockDim = dim3(kStepThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)2 * a.chunk_cap * step_row_bytes<KT, D>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.nc;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // the shared-memory opt-in is made once per kernel and device (for the whole staging budget), not per launch
    static bool opted[64][9] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
    auto go = [&](auto kernel) {
        if (dev < 0 || !opted[dev][G]) {
            const cudaError_t e =
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kStepStageBytes);
            if (e != cudaSuccess) return e;
            if (dev >= 0) opted[dev][G] = true;
        }
        return cudaLaunchKernelEx(&cfg, kernel, a);
    };
    switch (G) {
        case 1: return go(attn_decode_step_kernel<KT, D, 1>);
        case 2: return go(attn_decode_step_kernel<KT, D, 2>);
        case 3: return go(attn_decode_step_kernel<KT, D, 3>);
        case 4: return go(attn_decode_step_kernel<KT, D, 4>);
        case 5: return go(attn_decode_step_kernel<KT, D, 5>);
        case 6: return go(attn_decode_step_kernel<KT, D, 6>);
        case 7: return go(attn_decode_step_kernel<KT, D, 7>);
        case 8: return go(attn_decode_step_kernel<KT, D, 8>);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

int decode_step_chunks(eif_cuda_dtype_t dtype, int D, int G, int B, int Hkv, int max_len, int sm_count,
                       int *chunk_cap) {
    if (dtype != EIF_CUDA_F32 && dtype != EIF_CUDA_BF16) return 0;
    if ((D != 64 && D != 128) || G < 1 || G > 8 || max_len < 1) return 0;
    // a chunk's K and V rows must fit the shared-memory budget of the staged copy
    const int rb = D * (dtype == EIF_CUDA_F32 ? 4 : 2) + 16, cap = kStepStageBytes / (2 * rb);
    int nc = (max_len + 63) / 64;  // at least 64 keys a CTA
    if (nc > 8) nc = 8;            // the portable cluster size
    if ((max_len + nc - 1) / nc > cap) return 0;
    if ((long)B * Hkv * nc > 2L * sm_count) return 0;
    *chunk_cap = (max_len + nc - 1) / nc;
    return nc;
}

cudaError_t launch_attend_decode_step(cudaStream_t st, const DecodeStepArgs &a) {
    const int G = a.Hq / a.Hkv;
    if (a.dtype == EIF_CUDA_F32) return a.D == 64 ? launch_g<float, 64>(st, a, G) : launch_g<float, 128>(st, a, G);
    return a.D == 64 ? launch_g<__nv_bfloat16, 64>(st, a, G) : launch_g<__nv_bfloat16, 128>(st, a, G);
}
