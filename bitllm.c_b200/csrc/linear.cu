// linear.cu -- the engines' quantised projections on the GPU: out[t] = W x[t] for n tokens, fp32 arithmetic.
//
// Reference: linear_gemv (src/eif_qwen35.c:422-443) with its kernels -- fp32 (f32_gemv :355-382), signed INT4
// (int4_gemv :293-352), BitNet 2-bit ternary with a scale a row or a scale per group of columns
// (eif_matmul_bitnet_f32 / eif_matmul_bitnet_block_f32, src/eif_quantize_bitnet.c:834-889, 1356-1420), BitNet
// dense base-3 ternary (bitnet_gemv_dense, src/eif_qwen35.c:148-180) -- its batched twin linear_gemm (:1033-1063)
// and the INT8 LM head int8_gemv (:384-420).
//
// Device layout: the engine's packed rows, each padded with zero bytes to a multiple of 64, so that a warp reads
// a row as aligned 4-byte words, 128 contiguous bytes an instruction.  This kernel serves the formats the
// tensor-core kernel of linear_mma.cu does not: fp32 weights, grouped 2-bit scales and dense ternary.
//
// Kernel: one warp per group of R = 4 rows, lane l taking words l, l + 32, ... of the four rows (U words of each
// row a work item; the next item's words are in flight while the current one is computed).  Launched as a
// programmatic dependent: each CTA fetches its first weights before waiting for the previous kernel, so a chain of
// small projections overlaps one launch's tail with the next one's weight stream.  A tile of T tokens (1, 2, 4 or 8) sits in shared memory token-minor, [column][T] in
// planes of up to four tokens, with one empty slot after each word's columns: lane l's column c = w * CPW + i
// then lands in bank (w * (CPW + 1) + i) mod 32, distinct across the warp because CPW + 1 is odd.
// Each weight is decoded once per tile and meets the T tokens with T FMAs.  Decoding builds the float directly:
// an integer field k in the low byte of 0x4B000000 is the float 2^23 + k, and subtracting 2^23 + bias gives
// k - bias exactly (one byte permute and one FADD a weight):
//   INT8   k = byte ^ 0x80, bias 128;  INT4  k = nibble, bias 8;
//   2-bit  k = 1 + bit0 - bit1 (code 0 -> 0, 1 -> +1, 2 -> -1, 3 -> 0, as the reference's byte table), bias 1,
//          computed for all 16 fields of a word by one add-subtract and spread to bytes by four shift-ands;
//   dense  k = 1 + digit value, from a 256-entry shared table of a byte's five digits (2 bits each), bias 1.
// The 4 x T accumulators of a warp are summed across lanes by a transposed butterfly (R*T - 1 shuffles instead of
// 5 R T); the scale is applied as the reference applies it (per row after the sum, or per group inside it).
#include "internal.h"
#include "common.cuh"

namespace {

constexpr int kRows = 4;    // rows a warp
constexpr int kUnroll = 4;  // words of each row a lane has in flight
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr size_t kSmemCap = 200 * 1024;
constexpr int kDenseLut = 256 * 4;  // bytes of the dense-ternary digit table at the front of shared memory
#ifndef EIF_LINEAR_MMA_MIN_TOKENS
#define EIF_LINEAR_MMA_MIN_TOKENS 4
#endif
constexpr int kMmaMinTokens = EIF_LINEAR_MMA_MIN_TOKENS;  // tokens from which the tensor-core kernel runs

__host__ __device__ constexpr int cols_per_word(int wt) {
    return wt == EIF_CUDA_W_F32 ? 1
           : wt == EIF_CUDA_W_INT8 ? 4
           : wt == EIF_CUDA_W_INT4 ? 8
           : wt == EIF_CUDA_W_TERNARY2 ? 16
                                       : 20;  // dense ternary: five a byte
}

// shared-memory slots (one per column, plus one empty slot per word's columns) for a padded row of n_words words
__host__ __device__ constexpr int x_slots(int wt, int n_words) {
    return cols_per_word(wt) == 1 ? n_words : n_words * (cols_per_word(wt) + 1);
}

template <int CPW>
__device__ __forceinline__ int xslot(int c) {
    return CPW == 1 ? c : c + c / CPW;
}

// floats of the staged token tile, rounded to 16 bytes
__host__ __device__ constexpr int tile_floats(int wt, int n_words, int T) { return (x_slots(wt, n_words) * T + 3) / 4 * 4; }

// the tile, the dense table and the slices' sums ([kWarps][4 T] floats)
size_t tile_smem(int wt, int n_words, int T) {
    return (size_t)tile_floats(wt, n_words, T) * sizeof(float) + (wt == EIF_CUDA_W_TERNARY_DENSE ? kDenseLut : 0) +
           (size_t)kWarps * kRows * T * sizeof(float);
}

// tokens a tile: the largest of 8, 4, 2, 1 not above n whose tile fits in shared memory (0: none fits)
int pick_tile(int wt, int n_words, int n) {
    int T = n >= 8 ? 8 : n >= 4 ? 4 : n >= 2 ? 2 : 1;
    while (T > 1 && tile_smem(wt, n_words, T) > kSmemCap) T >>= 1;
    return tile_smem(wt, n_words, T) <= kSmemCap ? T : 0;
}

// the float of the integer field in byte j of `bytes`, minus the bias (bias_2p23 = 2^23 + bias)
__device__ __forceinline__ float field_float(uint32_t bytes, int j, float bias_2p23) {
    return __uint_as_float(__byte_perm(bytes, 0x4B000000u, 0x7440u + j)) - bias_2p23;
}

template <int T>
__device__ __forceinline__ void load_tile(const float *xs, int n_slots, int s, float (&x)[T]) {
    if constexpr (T == 1) {
        x[0] = xs[s];
    } else if constexpr (T == 2) {
        const float2 v = reinterpret_cast<const float2 *>(xs)[s];
        x[0] = v.x, x[1] = v.y;
    } else {
#pragma unroll
        for (int p = 0; p < T / 4; ++p) {
            const float4 v = reinterpret_cast<const float4 *>(xs)[(size_t)p * n_slots + s];
            x[4 * p] = v.x, x[4 * p + 1] = v.y, x[4 * p + 2] = v.z, x[4 * p + 3] = v.w;
        }
    }
}

template <int T>
__device__ __forceinline__ void store_tile(float *xs, int n_slots, int s, const float (&x)[T]) {
    if constexpr (T == 1) {
        xs[s] = x[0];
    } else if constexpr (T == 2) {
        reinterpret_cast<float2 *>(xs)[s] = make_float2(x[0], x[1]);
    } else {
#pragma unroll
        for (int p = 0; p < T / 4; ++p)
            reinterpret_cast<float4 *>(xs)[(size_t)p * n_slots + s] =
                make_float4(x[4 * p], x[4 * p + 1], x[4 * p + 2], x[4 * p + 3]);
    }
}

// A word of the format, prepared once, then weight i of it as a float.
template <int WT>
struct Word {
    uint32_t f[4];
    __device__ __forceinline__ void prepare(uint32_t w, const uint32_t *dlut) {
        if constexpr (WT == EIF_CUDA_W_F32) {
            f[0] = w;
        } else if constexpr (WT == EIF_CUDA_W_INT8) {
            f[0] = w ^ 0x80808080u;
        } else if constexpr (WT == EIF_CUDA_W_INT4) {
            f[0] = (w >> 4) & 0x0F0F0F0Fu;  // high nibbles: even columns
            f[1] = w & 0x0F0F0F0Fu;         // low nibbles: odd columns
        } else if constexpr (WT == EIF_CUDA_W_TERNARY2) {
            const uint32_t k = (w & 0x55555555u) + 0x55555555u - ((w >> 1) & 0x55555555u);  // fields 1 + b0 - b1
#pragma unroll
            for (int q = 0; q < 4; ++q) f[q] = (k >> (2 * q)) & 0x03030303u;  // byte j of f[q]: field 4j + q
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) f[j] = dlut[(w >> (8 * j)) & 0xffu];  // five 2-bit fields 1 + value
        }
    }
    __device__ __forceinline__ float operator()(int i) const {
        if constexpr (WT == EIF_CUDA_W_F32) {
            return __uint_as_float(f[0]);
        } else if constexpr (WT == EIF_CUDA_W_INT8) {
            return field_float(f[0], i, 8388736.f);
        } else if constexpr (WT == EIF_CUDA_W_INT4) {
            return field_float(f[i & 1], i >> 1, 8388616.f);
        } else if constexpr (WT == EIF_CUDA_W_TERNARY2) {
            return field_float(f[i & 3], i >> 2, 8388609.f);
        } else {
            return __uint_as_float(0x4B000000u | ((f[i / 5] >> (2 * (i % 5))) & 3u)) - 8388609.f;
        }
    }
};

// Sum K = 2^m values across the warp.  Afterwards each of the 32/K lanes l with l / (32/K) == idx holds the total
// of value idx: every butterfly step sends the half of the values the partner keeps.
template <int K>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[K], int lane) {
#pragma unroll
    for (int k = K, off = 16; k > 1; k >>= 1, off >>= 1) {
        const bool upper = lane & off;
#pragma unroll
        for (int i = 0; i < k / 2; ++i) {
            const float send = upper ? v[i] : v[i + k / 2];
            const float keep = upper ? v[i + k / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    float s = v[0];
#pragma unroll
    for (int off = 16 / K; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    return s;
}

struct LinArgs {
    const uint8_t *W;
    const float *scales;
    const float *x;  // [n][cols]
    float *out;      // [n][rows]
    int rows, cols, n, n_words;
    size_t stride;   // bytes between padded rows
    int group;       // grouped ternary: columns a scale (a multiple of 16), else 0
    int n_scales_row;
    int ks;          // column slices: the CTA's 8 warps are 8 / ks row-group lanes x ks slices of the words
};

template <int WT, int T, bool GROUPED>
__global__ void __launch_bounds__(kThreads, T == 1 ? 3 : 1) linear_kernel(const LinArgs a) {
    constexpr int CPW = cols_per_word(WT);
    constexpr int K = kRows * T;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *dlut = reinterpret_cast<uint32_t *>(smem);
    float *xs = reinterpret_cast<float *>(smem + (WT == EIF_CUDA_W_TERNARY_DENSE ? kDenseLut : 0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_groups = (a.rows + kRows - 1) / kRows;
    const int n_slots = x_slots(WT, a.n_words);
    const int n_cols = a.n_words * CPW;  // columns of the padded rows (those past `cols` meet zeros)
    // The CTA's warps: RG row-group lanes x KS column slices.  A warp's work items: (row group g, word block it)
    // for g = g0, g0 + gstride, ... and it over its slice's blocks of 32 * U words (the same count for every slice,
    // so the slices of a row group meet at its end together).  Item j + 1's weights are loaded while item j is
    // computed, across groups and tiles.
    const int KS = a.ks, RG = kWarps / KS, rg = warp / KS, ks = warp - rg * KS;
    const int wps = (a.n_words + KS - 1) / KS, w_begin = ks * wps, w_end = min(a.n_words, w_begin + wps);
    const int g0 = blockIdx.x * RG + rg, gstride = gridDim.x * RG;
    const int ipg = (wps + 32 * kUnroll - 1) / (32 * kUnroll);
    const int n_items = g0 < n_groups ? (n_groups - g0 + gstride - 1) / gstride * ipg : 0;
    auto load = [&](int j, uint32_t (&raw)[kUnroll][kRows]) {
        const int g = g0 + (j / ipg) * gstride, w0 = w_begin + lane + (j % ipg) * 32 * kUnroll;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const uint32_t *wr = reinterpret_cast<const uint32_t *>(a.W + (size_t)min(g * kRows + r, a.rows - 1) * a.stride);
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) raw[u][r] = (w0 + 32 * u < w_end) ? __ldg(wr + w0 + 32 * u) : 0u;
        }
    };
    float *red = xs + tile_floats(WT, a.n_words, T);  // [kWarps][K] the slices' sums
    uint32_t raw[kUnroll][kRows];
    if (n_items > 0) load(0, raw);  // the weights do not depend on the previous kernel: fetch before waiting
    griddep_wait();  // x is the previous kernel's output
    griddep_launch_dependents();  // after the wait: a dependent that starts early finds every earlier grid complete
    if constexpr (WT == EIF_CUDA_W_TERNARY_DENSE) {
        for (int b = threadIdx.x; b < 256; b += kThreads) {
            uint32_t e = 0, v = b;
#pragma unroll
            for (int p = 0; p < 5; ++p) {
                const uint32_t d = v % 3u;  // digit 1 -> +1, 2 -> -1, 0 -> 0; stored as 1 + value
                v /= 3u;
                e |= (d == 1u ? 2u : (d == 2u ? 0u : 1u)) << (2 * p);
            }
            dlut[b] = e;
        }
    }
    float acc[K];
    for (int t0 = 0; t0 < a.n; t0 += T) {
        __syncthreads();  // the previous tile's readers are done
        for (int c = threadIdx.x; c < n_cols; c += kThreads) {
            float v[T];
#pragma unroll
            for (int t = 0; t < T; ++t)
                v[t] = (c < a.cols && t0 + t < a.n) ? __ldg(a.x + (size_t)(t0 + t) * a.cols + c) : 0.f;
            store_tile<T>(xs, n_slots, xslot<CPW>(c), v);
        }
        __syncthreads();
        const bool more_tiles = t0 + T < a.n;
        for (int j = 0; j < n_items; ++j) {
            const int it = j % ipg, g = g0 + (j / ipg) * gstride, r0 = g * kRows;
            uint32_t nxt[kUnroll][kRows];
            if (j + 1 < n_items)
                load(j + 1, nxt);
            else if (more_tiles)
                load(0, nxt);
            if (it == 0) {
#pragma unroll
                for (int k = 0; k < K; ++k) acc[k] = 0.f;
            }
            const int w0 = w_begin + lane + it * 32 * kUnroll;
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int w = w0 + 32 * u;
                if (w >= w_end) break;
                Word<WT> wd[kRows];
#pragma unroll
                for (int r = 0; r < kRows; ++r) wd[r].prepare(raw[u][r], dlut);
                float part[K];
#pragma unroll
                for (int k = 0; k < K; ++k) part[k] = 0.f;
#pragma unroll
                for (int i = 0; i < CPW; ++i) {
                    float xv[T];
                    load_tile<T>(xs, n_slots, xslot<CPW>(w * CPW + i), xv);
#pragma unroll
                    for (int r = 0; r < kRows; ++r) {
                        const float wv = wd[r](i);
#pragma unroll
                        for (int t = 0; t < T; ++t) {
                            float &d = GROUPED ? part[r * T + t] : acc[r * T + t];
                            d = fmaf(wv, xv[t], d);
                        }
                    }
                }
                if constexpr (GROUPED) {  // the word's 16 columns share one group's scale
                    const int grp = (w * CPW) / a.group;
#pragma unroll
                    for (int r = 0; r < kRows; ++r) {
                        const float s = (r0 + r < a.rows && grp < a.n_scales_row)
                                            ? __ldg(a.scales + (size_t)(r0 + r) * a.n_scales_row + grp) : 0.f;
#pragma unroll
                        for (int t = 0; t < T; ++t) acc[r * T + t] = fmaf(s, part[r * T + t], acc[r * T + t]);
                    }
                }
            }
            if (it == ipg - 1) {
                float tot = warp_transpose_sum<K>(acc, lane);
                constexpr int per = 32 / K;  // lanes holding each total
                const int idx = lane / per;
                if (KS > 1) {  // the row group's slices meet in shared memory; slice 0 writes
                    if ((lane & (per - 1)) == 0) red[warp * K + idx] = tot;
                    asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(32 * KS) : "memory");
                    if (ks == 0)
                        for (int k2 = 1; k2 < KS; ++k2) tot += red[(warp + k2) * K + idx];
                }
                if (ks == 0 && (lane & (per - 1)) == 0) {
                    const int r = idx / T, t = idx % T, row = r0 + r;
                    if (row < a.rows && t0 + t < a.n) {
                        const float s = (WT == EIF_CUDA_W_F32 || GROUPED) ? 1.f : __ldg(a.scales + row);
                        a.out[(size_t)(t0 + t) * a.rows + row] = tot * s;
                    }
                }
                if (KS > 1) asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(32 * KS) : "memory");
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u)
#pragma unroll
                for (int r = 0; r < kRows; ++r) raw[u][r] = nxt[u][r];
        }
    }
}

template <int WT, int T, bool G>
cudaError_t go(cudaStream_t st, LinArgs a, size_t smem, int sm_count) {
    auto kernel = linear_kernel<WT, T, G>;
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
    // column slices: enough warps to fill the GPU twice over where the row groups alone do not, each slice
    // at least 32 words (a word a lane)
    const int n_groups = (a.rows + kRows - 1) / kRows;
    int ks = 1;
    while (ks < kWarps && n_groups * ks < 2 * kWarps * sm_count && a.n_words >= 32 * 2 * ks) ks *= 2;
    a.ks = ks;
    const int rg = kWarps / ks;
    int grid = (n_groups + rg - 1) / rg;
    if (grid > per_sm * sm_count) grid = per_sm * sm_count;
    // programmatic dependent launch: the CTAs may start while the previous kernel on the stream drains; each one
    // loads its first weights and then waits for that kernel's completion (griddepcontrol.wait) before reading x
    return launch_pdl(kernel, dim3(grid), dim3(kThreads), smem, st, a);
}

template <int WT, bool G>
cudaError_t go_t(cudaStream_t st, const LinArgs &a, int T, size_t smem, int sm_count) {
    switch (T) {
        case 8: return go<WT, 8, G>(st, a, smem, sm_count);
        case 4: return go<WT, 4, G>(st, a, smem, sm_count);
        case 2: return go<WT, 2, G>(st, a, smem, sm_count);
        default: return go<WT, 1, G>(st, a, smem, sm_count);
    }
}

}  // namespace

size_t linear_row_bytes(int wtype, int cols) {  // row_bytes, src/eif_qwen35.c:110-116 (INT8: a byte a weight)
    switch (wtype) {
        case EIF_CUDA_W_F32: return (size_t)cols * 4;
        case EIF_CUDA_W_INT8: return (size_t)cols;
        case EIF_CUDA_W_INT4: return (size_t)(cols + 1) / 2;
        case EIF_CUDA_W_TERNARY2: return (size_t)(cols + 3) / 4;
        default: return (size_t)(cols + 4) / 5;
    }
}

bool linear_fits(int wtype, size_t stride) { return pick_tile(wtype, (int)(stride / 4), 1) == 1; }

cudaError_t launch_linear(cudaStream_t st, const eif_cuda_linear &lin, const float *x, int n, float *out,
                          int sm_count) {
    // below kMmaMinTokens tokens the CUDA-core kernel, from there on the tensor cores (where the format allows)
    if (n >= kMmaMinTokens && linear_mma_supported(lin)) return launch_linear_mma(st, lin, x, n, out, sm_count);
    const LinArgs a{lin.W, lin.scales, x, out, lin.rows, lin.cols, n, (int)(lin.stride / 4), lin.stride,
                    lin.group, lin.n_scales_row, 1};
    const int T = pick_tile(lin.wtype, a.n_words, n);
    if (T == 0) return cudaErrorInvalidValue;
    const size_t smem = tile_smem(lin.wtype, a.n_words, T);
    switch (lin.wtype) {
        case EIF_CUDA_W_F32: return go_t<EIF_CUDA_W_F32, false>(st, a, T, smem, sm_count);
        case EIF_CUDA_W_INT4: return go_t<EIF_CUDA_W_INT4, false>(st, a, T, smem, sm_count);
        case EIF_CUDA_W_TERNARY2:
            return lin.group ? go_t<EIF_CUDA_W_TERNARY2, true>(st, a, T, smem, sm_count)
                             : go_t<EIF_CUDA_W_TERNARY2, false>(st, a, T, smem, sm_count);
        case EIF_CUDA_W_TERNARY_DENSE: return go_t<EIF_CUDA_W_TERNARY_DENSE, false>(st, a, T, smem, sm_count);
        default: return go_t<EIF_CUDA_W_INT8, false>(st, a, T, smem, sm_count);
    }
}
