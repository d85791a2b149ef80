// kv.cu -- KV-cache row writes and dtype conversions.
//
// kv_append writes the new token's rotated k / v at row pos[b] of every sequence: the memcpy into
// the cache at src/eif_qwen35.c:734-736 and the direct cache writes of src/eif_tinyllm.c:417-418,
// for a whole batch in one launch.  A bf16 cache rounds to nearest even.  An INT8 cache (tinyllm kv_type 1)
// is written by kv_quantize_kernel: codes and a scale per (row, kv head) as at src/eif_tinyllm.c:509-553.
#include "internal.h"
#include "common.cuh"

namespace {

template <typename T>
EIF_DEV T from_f32(float x);
template <>
EIF_DEV float from_f32<float>(float x) { return x; }
template <>
EIF_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__global__ void kv_append_kernel(T *__restrict__ K, T *__restrict__ V, const int *__restrict__ pos,
                                 const float *__restrict__ k, const float *__restrict__ v, int max_seq, int kv_dim,
                                 unsigned *__restrict__ dev_err) {
    const int b = blockIdx.x;
    const int p = pos[b];
    if (p < 0 || p >= max_seq) {
        if (threadIdx.x == 0) atomicOr(dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
        return;
    }
    const size_t row = ((size_t)b * max_seq + p) * kv_dim;
    for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
        K[row + i] = from_f32<T>(k[(size_t)b * kv_dim + i]);
        V[row + i] = from_f32<T>(v[(size_t)b * kv_dim + i]);
    }
}

__global__ void f32_to_bf16_kernel(const float *__restrict__ s, __nv_bfloat16 *__restrict__ d, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __float2bfloat16_rn(s[i]);
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16 *__restrict__ s, float *__restrict__ d, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        d[i] = __bfloat162float(s[i]);
}

// INT8 cache write: one warp per (row, kv head, K or V), lane l holding values [l*VPL, l*VPL + VPL) of the
// head; quantize_head_warp makes the codes and the scale.
template <int VPL>
__global__ void __launch_bounds__(256) kv_quantize_kernel(int8_t *__restrict__ K, int8_t *__restrict__ V,
                                                          float *__restrict__ ks, float *__restrict__ vs,
                                                          const int *__restrict__ pos, int seq, int t0,
                                                          const float *__restrict__ k, const float *__restrict__ v,
                                                          int n_rows, int max_seq, int nkv, int sstride,
                                                          unsigned *__restrict__ dev_err) {
    constexpr int HD = 32 * VPL;
    const int lane = threadIdx.x & 31;
    const long item = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= 2L * n_rows * nkv) return;
    const bool is_v = item & 1;
    const long rh = item >> 1;
    const int r = (int)(rh / nkv), h = (int)(rh % nkv);
    int b = seq, t = t0 + r;
    if (pos) {
        b = r;
        t = pos[r];
        if (t < 0 || t >= max_seq) {
            if (lane == 0 && h == 0 && !is_v) atomicOr(dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
            return;
        }
    }
    const size_t drow = (size_t)b * max_seq + t;
    float x[VPL];
    const float *src = (is_v ? v : k) + ((size_t)r * nkv + h) * HD + lane * VPL;  // caller's rows: no alignment
#pragma unroll
    for (int i = 0; i < VPL; ++i) x[i] = src[i];
    quantize_head_warp<VPL>(x, (is_v ? V : K) + (drow * nkv + h) * HD,
                            (is_v ? vs : ks) + ((size_t)b * nkv + h) * sstride + t, lane);
}

__global__ void kv_dequantize_kernel(const int8_t *__restrict__ K, const float *__restrict__ ks, int seq, int t0,
                                     float *__restrict__ out, size_t n, int max_seq, int nkv, int hd, int sstride) {
    const size_t base = ((size_t)seq * max_seq + t0) * nkv * hd;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t rh = i / hd;  // (row, kv head) of element i, rows counted from t0
        const int r = (int)(rh / nkv), h = (int)(rh % nkv);
        out[i] = (float)K[base + i] * ks[((size_t)seq * nkv + h) * sstride + t0 + r];
    }
}

unsigned grid_for(size_t n) {
    size_t g = (n + 255) / 256;
    if (g > 148u * 16u) g = 148u * 16u;
    return g ? (unsigned)g : 1u;
}

}  // namespace

cudaError_t launch_kv_append(cudaStream_t st, void *K, void *V, eif_cuda_dtype_t dtype, const int *pos,
                             const float *k, const float *v, int B, int max_seq, int kv_dim, unsigned *dev_err) {
    const int threads = kv_dim >= 256 ? 256 : 128;
    if (dtype == EIF_CUDA_F32)
        kv_append_kernel<float><<<B, threads, 0, st>>>(static_cast<float *>(K), static_cast<float *>(V), pos, k, v,
                                                        max_seq, kv_dim, dev_err);
    else
        kv_append_kernel<__nv_bfloat16><<<B, threads, 0, st>>>(static_cast<__nv_bfloat16 *>(K),
                                                                static_cast<__nv_bfloat16 *>(V), pos, k, v, max_seq,
                                                                kv_dim, dev_err);
    return cudaGetLastError();
}

cudaError_t launch_f32_to_bf16(cudaStream_t st, const float *src, __nv_bfloat16 *dst, size_t n) {
    f32_to_bf16_kernel<<<grid_for(n), 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_bf16_to_f32(cudaStream_t st, const __nv_bfloat16 *src, float *dst, size_t n) {
    bf16_to_f32_kernel<<<grid_for(n), 256, 0, st>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_kv_quantize(cudaStream_t st, int8_t *K, int8_t *V, float *ks, float *vs, const int *pos,
                               int seq, int t0, const float *k, const float *v, int n_rows, int max_seq, int nkv,
                               int hd, int scale_stride, unsigned *dev_err) {
    const long warps = 2L * n_rows * nkv;
    const unsigned grid = (unsigned)((warps + 7) / 8);
    if (grid == 0) return cudaSuccess;
    switch (hd) {
        case 64:
            kv_quantize_kernel<2><<<grid, 256, 0, st>>>(K, V, ks, vs, pos, seq, t0, k, v, n_rows, max_seq, nkv,
                                                         scale_stride, dev_err);
            break;
        case 128:
            kv_quantize_kernel<4><<<grid, 256, 0, st>>>(K, V, ks, vs, pos, seq, t0, k, v, n_rows, max_seq, nkv,
                                                         scale_stride, dev_err);
            break;
        case 256:
            kv_quantize_kernel<8><<<grid, 256, 0, st>>>(K, V, ks, vs, pos, seq, t0, k, v, n_rows, max_seq, nkv,
                                                         scale_stride, dev_err);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_kv_dequantize(cudaStream_t st, const int8_t *K, const float *ks, int seq, int t0, float *out,
                                 int n_rows, int max_seq, int nkv, int hd, int scale_stride) {
    const size_t n = (size_t)n_rows * nkv * hd;
    if (n == 0) return cudaSuccess;
    kv_dequantize_kernel<<<grid_for(n), 256, 0, st>>>(K, ks, seq, t0, out, n, max_seq, nkv, hd, scale_stride);
    return cudaGetLastError();
}
