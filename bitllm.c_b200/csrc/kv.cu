// kv.cu -- KV-cache row writes and dtype conversions.
//
// kv_append writes the new token's rotated k / v at row pos[b] of every sequence: the memcpy into
// the cache at src/eif_qwen35.c:734-736 and the direct cache writes of src/eif_tinyllm.c:417-418,
// for a whole batch in one launch.  A bf16 cache rounds to nearest even.
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
