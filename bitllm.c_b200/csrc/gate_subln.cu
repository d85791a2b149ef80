// gate_subln.cu -- the output epilogue of Qwen3.5's full attention over whole rows
// (src/eif_qwen35.c:773-789): o *= sigmoid(gate) per element, then SubLN over the row's n_heads*head_dim
// values (o * rsqrt(mean(o^2) + 1e-6) [* sub_norm], or a copy for plain_linear).  It follows the prefill
// kernels, which then write the raw attention in fp32 (SubLN normalises each row to unit RMS, so a bf16
// rounding of o would show up at full size in the output); the decode path does the same arithmetic inside
// its chunk-combine kernel.  One CTA per row (token of a sequence); the row stays in shared memory between
// the sum of squares and the scaling.
#include <math.h>

#include "internal.h"
#include "common.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) gate_subln_kernel(const float *__restrict__ o,
                                                              const float *__restrict__ gate, int dim, int subln,
                                                              const float *__restrict__ sub_norm,
                                                              float *__restrict__ out) {
    extern __shared__ float rowbuf[];
    __shared__ float red[32];
    const size_t base = (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += kThreads) {
        float x = o[base + i];
        if (gate) x *= 1.0f / (1.0f + expf(-gate[base + i]));
        rowbuf[i] = x;
        ss += x * x;
    }
    if (subln == EIF_CUDA_SUBLN_NONE) {
        for (int i = threadIdx.x; i < dim; i += kThreads) out[base + i] = rowbuf[i];
        return;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf(red[0] / dim + 1e-6f);
    for (int i = threadIdx.x; i < dim; i += kThreads) {
        float x = rowbuf[i] * inv;
        if (subln == EIF_CUDA_SUBLN_WEIGHT) x *= sub_norm[i];
        out[base + i] = x;
    }
}

}  // namespace

cudaError_t launch_gate_subln(cudaStream_t st, const float *o, const float *gate, int rows, int dim, int subln,
                              const float *sub_norm, float *out) {
    const size_t smem = (size_t)dim * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(gate_subln_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
    }
    gate_subln_kernel<<<rows, kThreads, smem, st>>>(o, gate, dim, subln, sub_norm, out);
    return cudaGetLastError();
}
