// attn_decode.cu -- split-K GQA decode attention over the KV cache.
//
// Reference: the head loop of fullatt_attend (src/eif_qwen35.c:741-771) and the inline tinyllm
// decode attention (src/eif_tinyllm.c:555-656): for every query head h (kv head h / (Hq/Hkv)),
// scores s_t = scale * q.k_t for t <= pos, softmax, o = sum_t p_t v_t; then the Qwen3.5 epilogue
// o *= sigmoid(gate) and SubLN (src/eif_qwen35.c:773-789).
//
// Work split: one unit = (sequence b, kv head); the unit's key range [0, pos[b]] is cut into
// `nchunk` chunks, one CTA per (chunk, unit).  A CTA serves ALL G = Hq/Hkv query heads of its kv
// head, so every K/V byte is read from HBM once.  Each CTA leaves an unnormalised partial
// (running max m, sum l, o[G][D]) in scratch; attn_decode_combine merges the chunks of a sequence
// with a log-sum-exp rescale, applies the gate and the SubLN of the whole row and writes out.
//
// This file holds the split choice, the combine and the SIMT kernel (fp32, bf16 or INT8 cache, fp32
// arithmetic, K / V read straight from global memory): lanes own keys for the scores and own head-dim
// slices for P.V.  The TMA-fed kernels take the common shapes (attn_decode_tc.cu: bf16, attn_decode_i8.cu:
// INT8, attn_decode_f32.cu: fp32 at head_dim 64 / 128); the SIMT kernel serves the rest (fp32 at head_dim
// 256, BITLLM_DECODE_SIMT=1).  Its INT8 branch is tinyllm kv_type 1 (src/eif_tinyllm.c:563-571, 618-625):
// score = (q . codes) * k_scale * scale, and the key's probability times its v_scale weights the V codes;
// codes widen to fp32 exactly (i8x4_to_f32).
#include <math.h>

#include "internal.h"
#include "common.cuh"

namespace {

constexpr int kDecodeThreads = 128;
constexpr int kDecodeWarps = kDecodeThreads / 32;

template <typename KT, int D, int G>
__global__ void __launch_bounds__(kDecodeThreads) attn_decode_simt_kernel(
    const KT *__restrict__ Kc, const KT *__restrict__ Vc, const float *__restrict__ q, const int *__restrict__ pos,
    int max_seq, int max_len, int Hkv, int chunk, int nchunk, float scale, float *__restrict__ part_o,
    float2 *__restrict__ part_ml, unsigned *__restrict__ dev_err, const float *__restrict__ k_scale,
    const float *__restrict__ v_scale, int sstride, const int *__restrict__ row_seq) {
    griddep_wait();  // a no-op unless launched as a programmatic dependent (these kernels are ordinary launches)
    griddep_launch_dependents();  // the chunk combine may launch now; it waits for this grid's results
    constexpr int DL = D / 32;  // head-dim elements per lane in P.V
    static_assert(D % 32 == 0 && (DL == 2 || DL == 4 || DL == 8), "head_dim 64/128/256");
    constexpr bool kI8 = sizeof(KT) == 1;  // INT8 cache: codes, one K and one V scale per (row, kv head)
    constexpr int KV_VEC = 16 / (int)sizeof(KT);  // elements per 16-byte K load

    const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int Hq = Hkv * G;

    __shared__ float sq[G][D];
    __shared__ float wm[kDecodeWarps][G], wl[kDecodeWarps][G];
    __shared__ float wacc[kDecodeWarps][G][D];

    int p = pos[b];
    if (p < 0 || p >= max_len) {  // max_len = the caller's bound + 1, never above max_seq
        if (threadIdx.x == 0 && c == 0 && kvh == 0) atomicOr(dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
        p = -1;  // no keys: the partial is empty and the combine writes zeros
    }
    const int L = p + 1;
    const int t_begin = c * chunk;
    const int t_end = min(L, t_begin + chunk);

    for (int i = threadIdx.x; i < G * D; i += kDecodeThreads)
        sq[i / D][i % D] = q[(size_t)b * Hq * D + (size_t)kvh * G * D + i];
    __syncthreads();

    float m[G], l[G], acc[G][DL];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int i = 0; i < DL; ++i) acc[h][i] = 0.f;
    }

    const size_t row_stride = (size_t)Hkv * D;
    const int cb = row_seq ? row_seq[b] : b;  // the cache sequence of query row b
    const KT *Kb = Kc + ((size_t)cb * max_seq * Hkv + kvh) * D;
    const KT *Vb = Vc + ((size_t)cb * max_seq * Hkv + kvh) * D;

    for (int t0 = t_begin + warp * 32; t0 < t_end; t0 += kDecodeWarps * 32) {
        const int t = t0 + lane;
        const bool valid = t < t_end;
        float s[G];
#pragma unroll
        for (int h = 0; h < G; ++h) s[h] = 0.f;
        float ksc = 1.f, vsc = 1.f;
        if constexpr (kI8) {
            if (valid) {
                const size_t si = ((size_t)cb * Hkv + kvh) * sstride + t;
                ksc = k_scale[si];
                vsc = v_scale[si];
            }
        }
        if (valid) {
            const KT *kr = Kb + (size_t)t * row_stride;
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
            // INT8: (q . codes * k_scale) * scale, the reference's order (src/eif_tinyllm.c:571)
            const float sc = valid ? (kI8 ? (s[h] * ksc) * scale : s[h] * scale) : -INFINITY;
            const float m_new = fmaxf(m[h], warp_max(sc));
            const float corr = expf(m[h] - m_new);  // 0 on the first block (m = -inf)
            const float pr = valid ? expf(sc - m_new) : 0.f;
            l[h] = l[h] * corr + warp_sum(pr);
#pragma unroll
            for (int i = 0; i < DL; ++i) acc[h][i] *= corr;
            m[h] = m_new;
            s[h] = kI8 ? pr * vsc : pr;  // INT8: p * v_scale weights the codes (src/eif_tinyllm.c:622-625)
        }
        const int nvalid = min(32, t_end - t0);
        const KT *vrow = Vb + (size_t)t0 * row_stride + lane * DL;
        if (nvalid == 32) {
            // a full block: a constant trip count, unrolled so that eight rows' loads are in flight together
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                float vv[DL];
                KvLoad<KT, DL>::load(vrow + (size_t)j * row_stride, vv);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float pj = __shfl_sync(0xffffffffu, s[h], j);
#pragma unroll
                    for (int i = 0; i < DL; ++i) acc[h][i] += pj * vv[i];
                }
            }
        } else {
            for (int j = 0; j < nvalid; ++j) {
                float vv[DL];
                KvLoad<KT, DL>::load(vrow + (size_t)j * row_stride, vv);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float pj = __shfl_sync(0xffffffffu, s[h], j);
#pragma unroll
                    for (int i = 0; i < DL; ++i) acc[h][i] += pj * vv[i];
                }
            }
        }
    }

    // merge the warps of the CTA
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
    const size_t unit = (size_t)b * Hkv + kvh;
    for (int i = threadIdx.x; i < G * D; i += kDecodeThreads) {
        const int h = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, wm[w][h]);
        float O = 0.f, Ls = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kDecodeWarps; ++w) {
                const float f = expf(wm[w][h] - M);
                O += wacc[w][h][d] * f;
                Ls += wl[w][h] * f;
            }
        }
        part_o[((unit * nchunk + c) * G + h) * D + d] = O;
        if (d == 0) part_ml[(unit * nchunk + c) * G + h] = make_float2(M, Ls);
    }
}

// One CTA per sequence: merge the chunk partials of every head, gate, SubLN over the whole row.
__global__ void __launch_bounds__(256) attn_decode_combine_kernel(
    const float *__restrict__ part_o, const float2 *__restrict__ part_ml, int Hq, int Hkv, int D, int nchunk,
    const float *__restrict__ gate, int subln, const float *__restrict__ sub_norm, float *__restrict__ out) {
    // launched as a programmatic dependent of the decode kernel: resident early, it waits here for that grid's
    // partials (and, through it, for the gate written before it)
    griddep_wait();
    extern __shared__ float smem[];
    const int b = blockIdx.x;
    const int G = Hq / Hkv;
    const int row = Hq * D;
    float *w = smem;             // [Hq][nchunk] chunk weights e^{m_c - M} / L
    float *rowbuf = smem + Hq * nchunk;  // [Hq*D]
    __shared__ float red[32];

    // chunk weights: one warp per head, lanes over the chunks
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int hc = threadIdx.x >> 5; hc < Hq; hc += nw) {
        const int kvh = hc / G, g = hc % G;
        const float2 *ml = part_ml + ((size_t)b * Hkv + kvh) * nchunk * G + g;  // chunk c at ml[c * G]
        float M = -INFINITY;
        for (int c = lane; c < nchunk; c += 32) M = fmaxf(M, ml[(size_t)c * G].x);
        M = warp_max(M);
        float Ls = 0.f;
        if (M != -INFINITY)
            for (int c = lane; c < nchunk; c += 32) {
                const float2 v = ml[(size_t)c * G];
                Ls += v.y * expf(v.x - M);
            }
        Ls = warp_sum(Ls);
        for (int c = lane; c < nchunk; c += 32)
            w[hc * nchunk + c] = (M == -INFINITY || Ls == 0.f) ? 0.f : expf(ml[(size_t)c * G].x - M) / Ls;
    }
    __syncthreads();

    // weighted sum over the chunks, kCombineRun row elements per thread at once and kChunkRun chunks of them
    // loaded before they are added (in chunk order): 32 independent loads in flight, so a split into many
    // chunks (small batches) is not a chain of round trips to L2
    constexpr int kCombineRun = 8, kChunkRun = 4;
    float ss = 0.f;
    for (int i0 = threadIdx.x; i0 < row; i0 += kCombineRun * blockDim.x) {
        const float *po[kCombineRun];
        const float *wh[kCombineRun];
        float o[kCombineRun];
#pragma unroll
        for (int k = 0; k < kCombineRun; ++k) {
            const int i = min(i0 + k * (int)blockDim.x, row - 1);  // clamped lanes compute a copy, not stored
            const int h = i / D, d = i % D;
            const int kvh = h / G, g = h % G;
            po[k] = part_o + (((size_t)b * Hkv + kvh) * nchunk * G + g) * D + d;
            wh[k] = w + h * nchunk;
            o[k] = 0.f;
        }
        int c = 0;
        for (; c + kChunkRun <= nchunk; c += kChunkRun) {
            float v[kChunkRun][kCombineRun];
#pragma unroll
            for (int u = 0; u < kChunkRun; ++u)
#pragma unroll
                for (int k = 0; k < kCombineRun; ++k) v[u][k] = po[k][(size_t)(c + u) * G * D];
#pragma unroll
            for (int u = 0; u < kChunkRun; ++u)
#pragma unroll
                for (int k = 0; k < kCombineRun; ++k) o[k] += v[u][k] * wh[k][c + u];
        }
        for (; c < nchunk; ++c)
#pragma unroll
            for (int k = 0; k < kCombineRun; ++k) o[k] += po[k][(size_t)c * G * D] * wh[k][c];
#pragma unroll
        for (int k = 0; k < kCombineRun; ++k) {
            const int i = i0 + k * (int)blockDim.x;
            if (i >= row) break;
            float v = o[k];
            if (gate) v *= 1.0f / (1.0f + expf(-gate[(size_t)b * row + i]));
            rowbuf[i] = v;
            ss += v * v;
        }
    }
    if (subln != EIF_CUDA_SUBLN_NONE) {
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        if (threadIdx.x < 32) {
            float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
            t = warp_sum(t);
            if (threadIdx.x == 0) red[0] = t;
        }
        __syncthreads();
        const float inv = 1.0f / sqrtf(red[0] / row + 1e-6f);
        for (int i = threadIdx.x; i < row; i += blockDim.x) {
            float o = rowbuf[i] * inv;
            if (subln == EIF_CUDA_SUBLN_WEIGHT) o *= sub_norm[i];
            out[(size_t)b * row + i] = o;
        }
    } else {
        for (int i = threadIdx.x; i < row; i += blockDim.x) out[(size_t)b * row + i] = rowbuf[i];
    }
}

struct Split {
    int nchunk, chunk;
    bool tc;
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Partials each item leaves: the bf16 tensor-core kernel writes one per consumer warp (its warps need no
// merge in shared memory, and the combine weighs them like chunks); the other kernels one per item.
int item_partials(const DecodeArgs &a, bool tc) { return tc && a.dtype == EIF_CUDA_BF16 ? decode_tc_partials(a.D) : 1; }

// Scratch bytes of the chunk partials: o [units][nchunk * ip][G][D] and (m, l) [units][nchunk * ip][G].
size_t partials_bytes(const DecodeArgs &a, int nchunk, int ip = 1) {
    const size_t units = (size_t)a.B * a.Hkv;
    const size_t G = (size_t)(a.Hq / a.Hkv);
    const size_t n = (size_t)nchunk * ip;
    return align256(units * n * G * a.D * sizeof(float)) + align256(units * n * G * sizeof(float2));
}

// The TMA-fed persistent kernels: bf16 / INT8 caches on the tensor cores, fp32 caches in fp32 FMAs.
bool use_tc(const DecodeArgs &a) {
    if (!a.tmk || !a.tmv || a.force_simt) return false;
    // the kernels stage each item's query rows with a bulk copy (16-byte aligned source)
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) != 0) return false;
    if (a.dtype == EIF_CUDA_F32) return decode_f32_supported(a.D, a.Hq / a.Hkv);
    return decode_tc_supported(a.D, a.Hq / a.Hkv);
}

// Tensor-core path: persistent CTAs (one per SM) take items round-robin, so pick the chunk count that
// minimises the busiest CTA's tiles plus the partials it writes and the combine reads back.
Split choose_split_tc(const DecodeArgs &a, int sm_count) {
    // an item is (row, kh kv heads, chunk): the INT8 kernel takes both heads of a 128-byte row at head_dim 64
    const int kh = a.dtype == EIF_CUDA_INT8 ? decode_i8_heads_per_item(a.D, a.Hkv) : 1;
    const long units = (long)a.B * a.Hkv / kh;
    const long tpu = (a.max_len + 63) / 64;  // 64-key tiles per unit
    // K + V bytes of a 64-key tile of the unit's kh heads (INT8: codes plus the two scales of every key)
    const double tile_bytes = kh * (a.dtype == EIF_CUDA_INT8 ? 64.0 * (a.D * 2 + 8)
                                                              : 64.0 * a.D * 2 * (a.dtype == EIF_CUDA_F32 ? 4 : 2));
    // Cost of a split, in bytes streamed by the busiest CTA (items go round-robin over the persistent
    // CTAs): its tiles plus a fixed cost per item.  The bf16 kernel at head_dim 256 (three 64 KB stages
    // per CTA) was measured elastic: a CTA with more items than the others streams up to half again its
    // fair share of HBM while they idle, so the whole job's bytes per SM bound it first, and an
    // item (q load, merge of the four warps, its share of the combine) costs about 64 KB of streaming;
    // the others were measured best at the most even split, with the partial's bytes as the item cost.
    const bool elastic = a.dtype == EIF_CUDA_BF16 && a.D >= 256;
    const double item_bytes = elastic ? 65536.0 : 2.0 * kh * (a.Hq / a.Hkv) * a.D * 4;
    const double fair = (double)units * tpu * tile_bytes / sm_count;
    int best = 1;
    double best_cost = 1e300;
    for (int nc = 1; nc <= 64 && nc <= tpu; ++nc) {
        const long ct = (tpu + nc - 1) / nc;
        const long ncu = (tpu + ct - 1) / ct;  // chunks actually used
        const long items = units * ncu;
        if (a.max_ws_bytes && ncu > 1 && partials_bytes(a, (int)ncu, item_partials(a, true)) > a.max_ws_bytes) break;
        const long per_cta = (items + sm_count - 1) / sm_count;
        const double busiest = per_cta * ct * tile_bytes;
        const double cost = (elastic ? fmax(fair, busiest / 1.5) : busiest) + per_cta * item_bytes;
        if (cost < best_cost * 0.999) {
            best_cost = cost;
            best = (int)ncu;
        }
    }
    const int chunk_tiles = (int)((tpu + best - 1) / best);
    return {best, chunk_tiles * 64, true};
}

Split choose_split(const DecodeArgs &a, int sm_count) {
    if (use_tc(a)) return choose_split_tc(a, sm_count);
    const int units = a.B * a.Hkv;
    const int L = a.max_len > 0 ? a.max_len : 1;
    // aim at >= 4 CTAs per SM, chunks of at least 64 keys
    int want = (4 * sm_count + units - 1) / units;
    int max_chunks = (L + 63) / 64;
    int nchunk = want < max_chunks ? want : max_chunks;
    if (nchunk < 1) nchunk = 1;
    if (a.max_ws_bytes)
        while (nchunk > 1 && partials_bytes(a, nchunk) > a.max_ws_bytes) --nchunk;
    int chunk = (L + nchunk - 1) / nchunk;
    nchunk = (L + chunk - 1) / chunk;
    return {nchunk, chunk, false};
}

template <typename KT, int D, int G>
cudaError_t launch_simt(cudaStream_t st, const DecodeArgs &a, const Split &sp, float *part_o, float2 *part_ml) {
    dim3 grid(sp.nchunk, a.Hkv, a.B);
    attn_decode_simt_kernel<KT, D, G><<<grid, kDecodeThreads, 0, st>>>(
        static_cast<const KT *>(a.K), static_cast<const KT *>(a.V), a.q, a.pos, a.max_seq, a.max_len, a.Hkv, sp.chunk,
        sp.nchunk, a.scale, part_o, part_ml, a.dev_err, a.k_scale, a.v_scale, a.scale_stride, a.row_seq);
    return cudaGetLastError();
}

template <typename KT, int D>
cudaError_t dispatch_g(cudaStream_t st, const DecodeArgs &a, const Split &sp, float *po, float2 *pml, bool *ok) {
    switch (a.Hq / a.Hkv) {
        case 1: return launch_simt<KT, D, 1>(st, a, sp, po, pml);
        case 2: return launch_simt<KT, D, 2>(st, a, sp, po, pml);
        case 3: return launch_simt<KT, D, 3>(st, a, sp, po, pml);
        case 4: return launch_simt<KT, D, 4>(st, a, sp, po, pml);
        case 5: return launch_simt<KT, D, 5>(st, a, sp, po, pml);
        case 6: return launch_simt<KT, D, 6>(st, a, sp, po, pml);
        case 7: return launch_simt<KT, D, 7>(st, a, sp, po, pml);
        case 8: return launch_simt<KT, D, 8>(st, a, sp, po, pml);
        default: *ok = false; return cudaSuccess;
    }
}

template <typename KT>
cudaError_t dispatch_d(cudaStream_t st, const DecodeArgs &a, const Split &sp, float *po, float2 *pml, bool *ok) {
    switch (a.D) {
        case 64: return dispatch_g<KT, 64>(st, a, sp, po, pml, ok);
        case 128: return dispatch_g<KT, 128>(st, a, sp, po, pml, ok);
        case 256: return dispatch_g<KT, 256>(st, a, sp, po, pml, ok);
        default: *ok = false; return cudaSuccess;
    }
}

}  // namespace

namespace {
__global__ void prefill_rows_kernel(int *row_seq, int *pos, int rows, int n_tok, int start_pos) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows) {
        row_seq[i] = i / n_tok;
        pos[i] = start_pos + i % n_tok;
    }
}
}  // namespace

cudaError_t launch_prefill_rows(cudaStream_t st, int *row_seq, int *pos, int batch, int n_tok, int start_pos) {
    const int rows = batch * n_tok;
    prefill_rows_kernel<<<(rows + 255) / 256, 256, 0, st>>>(row_seq, pos, rows, n_tok, start_pos);
    return cudaGetLastError();
}

size_t decode_workspace_bytes(const DecodeArgs &a, int sm_count) {
    const Split sp = choose_split(a, sm_count);
    return partials_bytes(a, sp.nchunk, item_partials(a, sp.tc));
}

void decode_plan(const DecodeArgs &a, int sm_count, int *nchunk, int *chunk_keys, size_t *ws_bytes) {
    const Split sp = choose_split(a, sm_count);
    *nchunk = sp.nchunk;
    *chunk_keys = sp.chunk;
    *ws_bytes = partials_bytes(a, sp.nchunk, item_partials(a, sp.tc));
}

// The decode kernels are ordinary launches: as programmatic dependents (starting while the kernel before them
// drains) the config-5 step measured 0.4-2.2 % slower at batch 256 and 1.4-2.5 % at batch 32 (A/B on two boxes).  Their
// griddepcontrol calls are no-ops then.  The chunk combine after them is a programmatic dependent.
cudaError_t launch_attend_decode(cudaStream_t st, const DecodeArgs &a, void *ws, size_t ws_bytes, int sm_count,
                                 bool *supported, int *n_launches) {
    *supported = true;
    *n_launches = 0;
    const Split sp = choose_split(a, sm_count);
    const size_t units = (size_t)a.B * a.Hkv;
    const int G = a.Hq / a.Hkv;
    const int n_part = sp.nchunk * item_partials(a, sp.tc);  // partials per unit, merged by the combine
    const size_t o_bytes = align256(units * n_part * G * a.D * sizeof(float));
    if (partials_bytes(a, sp.nchunk, item_partials(a, sp.tc)) > ws_bytes) return cudaErrorInvalidValue;
    float *part_o = static_cast<float *>(ws);
    float2 *part_ml = reinterpret_cast<float2 *>(static_cast<char *>(ws) + o_bytes);
    cudaError_t e;
    if (sp.tc && a.dtype == EIF_CUDA_F32)
        e = launch_attend_decode_f32(st, *a.tmk, *a.tmv, a, sp.nchunk, sp.chunk, part_o, part_ml, sm_count);
    else if (sp.tc && a.dtype == EIF_CUDA_INT8)
        e = launch_attend_decode_i8(st, *a.tmk, *a.tmv, a, sp.nchunk, sp.chunk, part_o, part_ml, sm_count);
    else if (sp.tc)
        e = launch_attend_decode_tc(st, *a.tmk, *a.tmv, a, sp.nchunk, sp.chunk, part_o, part_ml, sm_count);
    else if (a.dtype == EIF_CUDA_F32)
        e = dispatch_d<float>(st, a, sp, part_o, part_ml, supported);
    else if (a.dtype == EIF_CUDA_INT8)
        e = dispatch_d<int8_t>(st, a, sp, part_o, part_ml, supported);
    else
        e = dispatch_d<__nv_bfloat16>(st, a, sp, part_o, part_ml, supported);
    if (!*supported || e != cudaSuccess) return e;
    ++*n_launches;
    const size_t smem = ((size_t)a.Hq * n_part + (size_t)a.Hq * a.D) * sizeof(float);
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(attn_decode_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    e = launch_pdl(attn_decode_combine_kernel, dim3(a.B), dim3(256), smem, st, (const float *)part_o,
                   (const float2 *)part_ml, a.Hq, a.Hkv, a.D, n_part, a.gate, (int)a.subln, a.sub_norm, a.out);
    ++*n_launches;
    return e;
}
