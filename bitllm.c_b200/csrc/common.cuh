// common.cuh -- small device helpers shared by the kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define EIF_DEV __device__ __forceinline__

EIF_DEV float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

EIF_DEV float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}

EIF_DEV float4 f4_add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }

EIF_DEV float4 f4_shfl_xor(float4 a, int o) {
    a.x = __shfl_xor_sync(0xffffffffu, a.x, o);
    a.y = __shfl_xor_sync(0xffffffffu, a.y, o);
    a.z = __shfl_xor_sync(0xffffffffu, a.z, o);
    a.w = __shfl_xor_sync(0xffffffffu, a.w, o);
    return a;
}

// bf16 <-> fp32 by bit manipulation (bf16 is the upper half of an fp32 word).
EIF_DEV float bf16lo_to_f32(uint32_t packed) { return __uint_as_float(packed << 16); }
EIF_DEV float bf16hi_to_f32(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }

// Load n consecutive KV elements as fp32 (n = 2, 4 or 8; the address is aligned to n elements).
template <typename T, int N>
struct KvLoad;

template <int N>
struct KvLoad<float, N> {
    static EIF_DEV void load(const float *p, float *out) {
        if constexpr (N == 2) {
            float2 a = *reinterpret_cast<const float2 *>(p);
            out[0] = a.x; out[1] = a.y;
        } else if constexpr (N == 4) {
            float4 a = *reinterpret_cast<const float4 *>(p);
            out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        } else {
            float4 a = reinterpret_cast<const float4 *>(p)[0];
            float4 b = reinterpret_cast<const float4 *>(p)[1];
            out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
            out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
        }
    }
};

template <int N>
struct KvLoad<__nv_bfloat16, N> {
    static EIF_DEV void load(const __nv_bfloat16 *p, float *out) {
        if constexpr (N == 2) {
            uint32_t a = *reinterpret_cast<const uint32_t *>(p);
            out[0] = bf16lo_to_f32(a); out[1] = bf16hi_to_f32(a);
        } else if constexpr (N == 4) {
            uint2 a = *reinterpret_cast<const uint2 *>(p);
            out[0] = bf16lo_to_f32(a.x); out[1] = bf16hi_to_f32(a.x);
            out[2] = bf16lo_to_f32(a.y); out[3] = bf16hi_to_f32(a.y);
        } else {
            uint4 a = *reinterpret_cast<const uint4 *>(p);
            out[0] = bf16lo_to_f32(a.x); out[1] = bf16hi_to_f32(a.x);
            out[2] = bf16lo_to_f32(a.y); out[3] = bf16hi_to_f32(a.y);
            out[4] = bf16lo_to_f32(a.z); out[5] = bf16hi_to_f32(a.z);
            out[6] = bf16lo_to_f32(a.w); out[7] = bf16hi_to_f32(a.w);
        }
    }
};
