// rope.cu -- tinyllm's rotary position embedding and cache write on the device.
//
// Reference: tinyllm_forward_embedding_ex rotates q and k of the new token with per-position tables
// (src/eif_tinyllm.c:395-405: freq_j = 1 / theta^(2j/head_dim), cos / sin of pos * freq_j) -- NeoX
// half-split pairs (j, j + head_dim/2) for Qwen2, adjacent pairs (2j, 2j+1) when rope_interleaved
// (:481-507) -- and the rotated k and v land in cache row pos (:415-418); the batched prefill does the same
// per token of the chunk (:994-1006).  The tables are computed on the host by the same float formula
// (eif_cuda_kv_set_rope) and read here by position, so the device rotation multiplies the same numbers.
//
// rope_append_kernel: one CTA per token row r = (sequence b, token i): position pos[b] (one token per
// sequence) or start_pos + i (a chunk); every thread takes (head, pair) items of q and k, then the v row.
// An INT8 cache stages the rotated k row in shared memory and quantises k and v per head, one warp each.
#include "internal.h"
#include "common.cuh"

namespace {

// INT8 cache: one warp quantises one head of hd = 32 * VPL values read from src (shared or global memory).
template <int VPL>
__device__ void quantize_from(const float *src, int8_t *dst, float *scale_out, int lane) {
    float x[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) x[i] = src[lane * VPL + i];
    quantize_head_warp<VPL>(x, dst, scale_out, lane);
}

__global__ void __launch_bounds__(256) rope_append_kernel(const RopeArgs a) {
    extern __shared__ float krot[];  // INT8 caches: the rotated k row [nkv][hd], quantised once complete
    const int r = blockIdx.x, b = r / a.n_tok;
    const int hd = a.hd, half = hd / 2, nh = a.nh, nkv = a.nkv;
    const int p = a.pos ? a.pos[b] : a.start_pos + r % a.n_tok;
    const bool pos_ok = p >= 0 && p < a.max_seq;
    if (!pos_ok && threadIdx.x == 0) atomicOr(a.dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
    const float *cs = a.cos_t + (size_t)(pos_ok ? p : 0) * half;
    const float *sn = a.sin_t + (size_t)(pos_ok ? p : 0) * half;
    const size_t crow = ((size_t)b * a.max_seq + p) * nkv * hd;  // cache row of (b, p)
    for (int it = threadIdx.x; it < (nh + nkv) * half; it += blockDim.x) {
        const int hh = it / half, j = it - hh * half;
        const bool isq = hh < nh;
        const int hi = isq ? hh : hh - nh;
        const float *src = isq ? a.q + ((size_t)r * nh + hi) * hd : a.k + ((size_t)r * nkv + hi) * hd;
        const int ia = a.interleaved ? 2 * j : j, ib = a.interleaved ? 2 * j + 1 : j + half;
        const float x0 = src[ia], x1 = src[ib], c = cs[j], s = sn[j];
        // x0 c - x1 s and x1 c + x0 s with the first product fused, as the reference's -mfma build contracts
        // them: bit-identical rotated rows (and so INT8 scales, which inherit amax's last bit)
        const float y0 = __fmaf_rn(x0, c, -__fmul_rn(x1, s)), y1 = __fmaf_rn(x1, c, __fmul_rn(x0, s));
        if (isq) {
            const size_t o = ((size_t)r * nh + hi) * hd;
            if (a.q_out_bf16) {
                a.q_out_bf16[o + ia] = __float2bfloat16_rn(y0);
                a.q_out_bf16[o + ib] = __float2bfloat16_rn(y1);
            } else {
                a.q_out[o + ia] = y0;
                a.q_out[o + ib] = y1;
            }
        } else if (pos_ok) {
            const size_t o = crow + (size_t)hi * hd;
            if (a.dtype == EIF_CUDA_INT8) {
                krot[hi * hd + ia] = y0;
                krot[hi * hd + ib] = y1;
            } else if (a.dtype == EIF_CUDA_F32) {
                static_cast<float *>(a.Kc)[o + ia] = y0;
                static_cast<float *>(a.Kc)[o + ib] = y1;
            } else {
                static_cast<__nv_bfloat16 *>(a.Kc)[o + ia] = __float2bfloat16_rn(y0);
                static_cast<__nv_bfloat16 *>(a.Kc)[o + ib] = __float2bfloat16_rn(y1);
            }
        }
    }
    if (a.dtype == EIF_CUDA_INT8) {
        // the quantised write of the rotated k and of v (src/eif_tinyllm.c:509-553): one warp per head
        __syncthreads();
        if (!pos_ok) return;
        const int lane = threadIdx.x & 31;
        for (int it = threadIdx.x >> 5; it < 2 * nkv; it += blockDim.x >> 5) {
            const bool is_v = it >= nkv;
            const int h = is_v ? it - nkv : it;
            const float *src = is_v ? a.v + ((size_t)r * nkv + h) * hd : krot + h * hd;
            int8_t *dst = static_cast<int8_t *>(is_v ? a.Vc : a.Kc) + crow + (size_t)h * hd;
            float *sc = (is_v ? a.v_scale : a.k_scale) + ((size_t)b * nkv + h) * a.scale_stride + p;
            if (hd == 64)
                quantize_from<2>(src, dst, sc, lane);
            else if (hd == 128)
                quantize_from<4>(src, dst, sc, lane);
            else
                quantize_from<8>(src, dst, sc, lane);
        }
        return;
    }
    if (pos_ok)
        for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
            const float v = a.v[(size_t)r * nkv * hd + i];
            if (a.dtype == EIF_CUDA_F32)
                static_cast<float *>(a.Vc)[crow + i] = v;
            else
                static_cast<__nv_bfloat16 *>(a.Vc)[crow + i] = __float2bfloat16_rn(v);
        }
}

}  // namespace

cudaError_t launch_rope_append(cudaStream_t st, const RopeArgs &a) {
    const size_t smem = a.dtype == EIF_CUDA_INT8 ? (size_t)a.nkv * a.hd * sizeof(float) : 0;
    rope_append_kernel<<<a.B * a.n_tok, 256, smem, st>>>(a);
    return cudaGetLastError();
}
