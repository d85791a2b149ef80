// common.cuh -- small device helpers shared by the kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define EIF_DEV __device__ __forceinline__

// Programmatic dependent launch (sm_90+): let the next kernel on the stream begin launching its CTAs, and wait
// until the previous kernel has completed with its memory visible (no-ops for a kernel launched without the
// programmatic-serialization attribute, or with no kernel before it).
EIF_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
EIF_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// ---- INT8 KV cache (tinyllm kv_type 1) ----

// Four packed int8 values -> fp32, exactly: the byte x + 128 is placed in the low mantissa bits of 2^23
// (0x4B0000uu == 2^23 + uu), and 2^23 + 128 is subtracted.  One byte permute and one add per value.
EIF_DEV void i8x4_to_f32(uint32_t w, float *o) {
    const uint32_t u = w ^ 0x80808080u;
    o[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
    o[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
    o[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
    o[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}

template <int N>
struct KvLoad<int8_t, N> {
    static EIF_DEV void load(const int8_t *p, float *out) {
        if constexpr (N == 2) {
            const uint32_t a = *reinterpret_cast<const uint16_t *>(p);
            float t[4];
            i8x4_to_f32(a, t);
            out[0] = t[0]; out[1] = t[1];
        } else if constexpr (N == 4) {
            i8x4_to_f32(*reinterpret_cast<const uint32_t *>(p), out);
        } else if constexpr (N == 8) {
            const uint2 a = *reinterpret_cast<const uint2 *>(p);
            i8x4_to_f32(a.x, out);
            i8x4_to_f32(a.y, out + 4);
        } else {
            static_assert(N == 16, "2, 4, 8 or 16 int8 values");
            const uint4 a = *reinterpret_cast<const uint4 *>(p);
            i8x4_to_f32(a.x, out);
            i8x4_to_f32(a.y, out + 4);
            i8x4_to_f32(a.z, out + 8);
            i8x4_to_f32(a.w, out + 12);
        }
    }
};

// Quantise one head of `hd` = 32 * VPL values held by a warp (lane l owns x[l*VPL .. l*VPL+VPL)) the way
// tinyllm's cache write does (src/eif_tinyllm.c:509-553): amax over the head; scale = amax / 127 and
// inv = 127 / amax (1 / 127 both when amax < 1e-12); code = trunc(x * inv +- 0.5) clamped to [-128, 127].
// The reference is built with -ffast-math (CMakeLists.txt:19), under which its compiler turns amax / 127.0f
// into amax * (1 / 127.0f) and fuses x * inv + 0.5 into one fma; both forms are reproduced here, so codes
// and scales are bit-identical to the compiled reference.  Writes the lane's VPL codes to dst + l*VPL and,
// from lane 0, the scale.
template <int VPL>
EIF_DEV void quantize_head_warp(const float (&x)[VPL], int8_t *dst, float *scale_out, int lane) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = warp_max(amax);
    const bool tiny = amax < 1e-12f;
    const float scale = tiny ? 1.0f : amax * (1.0f / 127.0f);
    const float inv = __fdiv_rn(127.0f, tiny ? 1.0f : amax);
    uint32_t packed[(VPL + 3) / 4] = {};
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        int c = __float2int_rz(__fmaf_rn(x[i], inv, x[i] >= 0.f ? 0.5f : -0.5f));
        c = max(-128, min(127, c));
        packed[i / 4] |= (uint32_t)(c & 0xff) << (8 * (i % 4));
    }
    int8_t *d = dst + lane * VPL;
    if constexpr (VPL == 2) {
        *reinterpret_cast<uint16_t *>(d) = (uint16_t)packed[0];
    } else if constexpr (VPL == 4) {
        *reinterpret_cast<uint32_t *>(d) = packed[0];
    } else {
        static_assert(VPL == 8, "head_dim 64, 128 or 256");
        *reinterpret_cast<uint2 *>(d) = make_uint2(packed[0], packed[1]);
    }
    if (lane == 0) *scale_out = scale;
}
