// linear.cu -- the engines' quantised projections on the GPU: out[t] = W x[t] for n tokens, fp32 arithmetic.
//
// Reference: linear_gemv (src/eif_qwen35.c:422-443) with its kernels -- fp32 (f32_gemv :355-382), signed INT4
// (int4_gemv :293-352), BitNet 2-bit ternary with a scale a row or a scale per group of columns
// (eif_matmul_bitnet_f32 / eif_matmul_bitnet_block_f32, src/eif_quantize_bitnet.c:834-889, 1356-1420), BitNet
// dense base-3 ternary (bitnet_gemv_dense, src/eif_qwen35.c:148-180) -- its batched twin linear_gemm (:1033-1063)
// and the INT8 LM head int8_gemv (:384-420).
//
// Device layout: the engine's packed rows, each padded with zero bytes to a multiple of 16, so that a warp reads
// a row as aligned 4-byte words, 128 contiguous bytes an instruction.
//
// Kernel: one warp per group of R = 4 rows, lane l taking words l, l + 32, ... of the four rows (U words of each
// row in flight per lane).  A tile of T tokens (1, 2, 4 or 8) sits in shared memory token-minor, [column][T] in
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

namespace {

constexpr int kRows = 4;    // rows a warp
constexpr int kUnroll = 4;  // words of each row a lane has in flight
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr size_t kSmemCap = 200 * 1024;
constexpr int kDenseLut = 256 * 4;  // bytes of the dense-ternary digit table at the front of shared memory

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

size_t tile_smem(int wt, int n_words, int T) {
    return (size_t)x_slots(wt, n_words) * T * sizeof(float) + (wt == EIF_CUDA_W_TERNARY_DENSE ? kDenseLut : 0);
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
};

template <int WT, int T, bool GROUPED>
__global__ void __launch_bounds__(kThreads) linear_kernel(const LinArgs a) {
    constexpr int CPW = cols_per_word(WT);
    constexpr int K = kRows * T;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t *dlut = reinterpret_cast<uint32_t *>(smem);
    float *xs = reinterpret_cast<float *>(smem + (WT == EIF_CUDA_W_TERNARY_DENSE ? kDenseLut : 0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_groups = (a.rows + kRows - 1) / kRows;
    const int n_slots = x_slots(WT, a.n_words);
    const int n_cols = a.n_words * CPW;  // columns of the padded rows (those past `cols` meet zeros)
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
        for (int g = blockIdx.x * kWarps + warp; g < n_groups; g += gridDim.x * kWarps) {
            const int r0 = g * kRows;
            const uint32_t *wr[kRows];
#pragma unroll
            for (int r = 0; r < kRows; ++r)
                wr[r] = reinterpret_cast<const uint32_t *>(a.W + (size_t)min(r0 + r, a.rows - 1) * a.stride);
            float acc[K];
#pragma unroll
            for (int k = 0; k < K; ++k) acc[k] = 0.f;
            for (int w0 = lane; w0 < a.n_words; w0 += 32 * kUnroll) {
                uint32_t raw[kUnroll][kRows];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u)
#pragma unroll
                    for (int r = 0; r < kRows; ++r)
                        raw[u][r] = (w0 + 32 * u < a.n_words) ? __ldg(wr[r] + w0 + 32 * u) : 0u;
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int w = w0 + 32 * u;
                    if (w >= a.n_words) break;
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
            }
            const float tot = warp_transpose_sum<K>(acc, lane);
            constexpr int per = 32 / K;  // lanes holding each total
            if ((lane & (per - 1)) == 0) {
                const int idx = lane / per, r = idx / T, t = idx % T, row = r0 + r;
                if (row < a.rows && t0 + t < a.n) {
                    const float s = (WT == EIF_CUDA_W_F32 || GROUPED) ? 1.f : __ldg(a.scales + row);
                    a.out[(size_t)(t0 + t) * a.rows + row] = tot * s;
                }
            }
        }
    }
}

template <int WT, int T, bool G>
cudaError_t go(cudaStream_t st, const LinArgs &a, size_t smem, int sm_count) {
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
    const int n_groups = (a.rows + kRows - 1) / kRows;
    int grid = (n_groups + kWarps - 1) / kWarps;
    if (grid > per_sm * sm_count) grid = per_sm * sm_count;
    kernel<<<grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
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
    const LinArgs a{lin.W, lin.scales, x, out, lin.rows, lin.cols, n, (int)(lin.stride / 4), lin.stride,
                    lin.group, lin.n_scales_row};
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
