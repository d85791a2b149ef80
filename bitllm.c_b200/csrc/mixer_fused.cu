// mixer_fused.cu -- the whole per-token Qwen3.5 token-mixer bodies as single kernels.
//
// deltanet_core_kernel: deltanet_core (src/eif_qwen35.c:546-656) for one token of every sequence:
//   causal conv1d over the sliding window + SiLU (:560-572), per-head L2 norm of q and k, q scaled by
//   1/sqrt(d_k) (:579-585), beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias) (:587-592), the
//   delta rule (:594-639) and the gated RMSNorm o * rsqrt(mean(o^2) + 1e-6) * norm_w * silu(z)
//   (:642-653).  One CTA per (sequence, head): it owns that head's q, k and v conv channels (so every
//   conv-window row is updated by exactly one CTA) and all d_v columns of S (so the RMSNorm of the
//   head's output row closes inside the CTA).  S crosses HBM once each way.
//   The S reads are all issued when the CTA starts, before the conv: the first half of the head's rows
//   by bulk copies into shared memory, the second half by each thread into registers (eight float4
//   rows), so one memory round trip overlaps the conv and the norms, and both passes over S (retrieve,
//   then update + output) read on-chip copies.  32 KB of shared memory and 64 registers per CTA: four CTAs
//   fit per SM, so up to 4 x SMs heads run in one wave (a whole head in shared memory allows three, and at
//   small batches its second wave of a few CTAs set the time).
//
// fullatt_prep_kernel: fullatt_prep (src/eif_qwen35.c:699-737) for one token of every sequence:
//   split the interleaved [q | gate] heads, RMSNorm q and k per head with q_norm / k_norm (eps 1e-6),
//   rotate the first head_dim/4 dims of q and k (half-split pairs, theta 1e7: rope_partial,
//   :502-535) with a cos / sin table computed on the host by the reference's formula, and write k, v
//   into cache row pos[b].  fullatt_prep_warp_kernel does the same with one warp per (row, head) and
//   vector loads (head_dim 64 / 128 / 256, aligned rows); fullatt_prep_kernel, one CTA per row with
//   scalar accesses, takes every other shape.
#include <math.h>

#include "internal.h"
#include "common.cuh"
#include "ptx.cuh"

namespace {

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <int DK, int DV, int THREADS>
__global__ void __launch_bounds__(THREADS, 4) deltanet_core_kernel(const DeltaCoreArgs a) {
    constexpr int LPR = DV / 4;        // threads per S row (float4 each)
    constexpr int RP = THREADS / LPR;  // rows per pass
    constexpr int NP = DK / RP;        // passes
    constexpr int NW = THREADS / 32;
    static_assert(LPR <= 32 && 32 % LPR == 0 && DK % RP == 0, "tile shape");
    // launched as a programmatic dependent.  prefetch (set by the host when the kernel launched just before this one
    // on the stream does not write this layer's state): the state (S, conv windows) and the layer's weights are
    // read before griddepcontrol.wait -- every grid before that kernel has completed, since each of the library's
    // grids triggers its dependents only after its own wait -- and only the inputs after it
    const bool pre = a.prefetch != 0;
    if (!pre) {
        griddep_wait();
        griddep_launch_dependents();  // after the wait: a dependent that starts early finds every earlier grid complete
    }
    const int h = blockIdx.x, b = blockIdx.y;
    const int H = a.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int lc = tid % LPR, rg = tid / LPR;
    const size_t bh = (size_t)b * H + h;
    const int key_dim = H * DK, conv_dim = 2 * key_dim + H * DV;

    constexpr int NH = NP / 2;  // passes over the rows staged in shared memory; the other NH in registers
    constexpr int NC = 2 * DK + DV;  // the head's conv channels: q, k, v
    __shared__ float sq[DK], sk[DK], sv[DV];
    __shared__ float2 red[NW];
    __shared__ float gates[2];
    __shared__ __align__(8) uint64_t s_bar;
    // dynamic: S rows [0, DK/2) | z, norm_w [2][DV] | staging: conv windows [NC][ck], conv weights [NC][ck],
    // inputs [NC] (stage_inputs), dead after the conv and then reused for the two column-sum buffers
    extern __shared__ __align__(128) float Ssm[];
    float *zn = Ssm + DK / 2 * DV;
    float *stg = zn + 2 * DV;
    float4(*cred)[NW][LPR] = reinterpret_cast<float4(*)[NW][LPR]>(stg);  // [2][NW][LPR]: no barrier between uses
    const bool staged = a.stage_inputs != 0;

    float *Sh = a.S + bh * DK * DV;
    const int col0 = lc * 4;
    const float4 *Srow = reinterpret_cast<const float4 *>(Sh) + col0 / 4;
    const float4 *Smem = reinterpret_cast<const float4 *>(Ssm) + col0 / 4;
    // S rows [0, DK/2) into shared memory (bulk copies completing on s_bar), rows [DK/2, DK) into registers
    const uint32_t sbar = smem_u32(&s_bar);
    const int ck = a.conv_k;
    if (tid == 0) {
        constexpr uint32_t bytes = DK / 2 * DV * 4, piece = bytes < 16384 ? bytes : 16384;
        mbar_init(sbar, 1);
        fence_barrier_init();
        // staged: everything else the CTA reads rides on the same barrier, so its inputs cost one round trip
        // (the conv windows of the q, k and v channel blocks, their weights, the raw inputs, z and norm_w)
        const uint32_t wbytes = (uint32_t)(NC * ck * 4);
        mbar_arrive_expect_tx(sbar, bytes + (staged ? 2 * DV * 4 + 2 * wbytes + NC * 4 : 0));
        for (uint32_t off = 0; off < bytes; off += piece)
            bulk_load(smem_u32(Ssm) + off, reinterpret_cast<const char *>(Sh) + off, piece, sbar);
        if (staged) {
            bulk_load(smem_u32(zn + DV), a.norm_w, DV * 4, sbar);
#pragma unroll
            for (int blk = 0; blk < 3; ++blk) {  // local channels [i0, i0 + n) = global channels [c0, c0 + n)
                const int i0 = blk * DK, n = blk < 2 ? DK : DV;
                const int c0 = blk == 0 ? h * DK : (blk == 1 ? key_dim + h * DK : 2 * key_dim + h * DV);
                bulk_load(smem_u32(stg + i0 * ck), a.conv + ((size_t)b * conv_dim + c0) * ck, n * ck * 4, sbar);
                bulk_load(smem_u32(stg + (NC + i0) * ck), a.conv_w + (size_t)c0 * ck, n * ck * 4, sbar);
            }
        }
    }
    float4 sreg[NH];
#pragma unroll
    for (int u = 0; u < NH; ++u) sreg[u] = Srow[(rg + (NH + u) * RP) * (DV / 4)];
    if (pre) {
        griddep_wait();  // the inputs (qkv, z, the gates' inputs) may be the previous kernel's output
        griddep_launch_dependents();
    }
    if (tid == 0 && staged) {  // the inputs, on the same barrier
        bulk_load(smem_u32(zn), a.z + bh * DV, DV * 4, sbar);
#pragma unroll
        for (int blk = 0; blk < 3; ++blk) {
            const int i0 = blk * DK, n = blk < 2 ? DK : DV;
            const int c0 = blk == 0 ? h * DK : (blk == 1 ? key_dim + h * DK : 2 * key_dim + h * DV);
            bulk_load(smem_u32(stg + 2 * NC * ck + i0), a.qkv + (size_t)b * conv_dim + c0, n * 4, sbar);
        }
    }
    // the gates' inputs, loaded now so that their latency overlaps the conv
    float braw = 0.f, araw = 0.f, dtb = 0.f, aex = 0.f;
    if (tid == 0) {
        braw = a.b_raw[bh];
        araw = a.a_raw[bh];
        dtb = a.dt_bias[h];
        aex = a.a_exp[h];
    }

    // causal conv1d + SiLU on this head's channels: q [h*DK, +DK), k [key_dim + h*DK, +DK), v [2*key_dim + h*DV, +DV)
    __syncthreads();  // the barrier's initialisation is visible to every thread
    // a wait that gives up leaves S and the conv windows untouched (the error word tells the host)
    const bool s_ok0 = staged ? mbar_wait(sbar, 0, a.dev_err) : true;
    if (staged) {
        const float *cwin = stg, *cwt = stg + NC * ck, *cx = stg + 2 * NC * ck;
        for (int i = tid; i < NC; i += THREADS) {
            const int c = i < DK ? h * DK + i : (i < 2 * DK ? key_dim + h * DK + (i - DK) : 2 * key_dim + h * DV + (i - 2 * DK));
            const float *wr = cwin + i * ck, *w = cwt + i * ck;
            const float xin = cx[i];
            float acc = 0.f;
            for (int j = 0; j < ck - 1; ++j) acc += wr[j + 1] * w[j];
            acc += xin * w[ck - 1];
            if (s_ok0) {
                float *row = a.conv + ((size_t)b * conv_dim + c) * ck;
                for (int j = 0; j < ck - 1; ++j) row[j] = wr[j + 1];
                row[ck - 1] = xin;
            }
            const float y = silu_f(acc);
            if (i < DK) sq[i] = y;
            else if (i < 2 * DK) sk[i - DK] = y;
            else sv[i - 2 * DK] = y;
        }
    } else {  // conv state arrays not staged: read in place
        for (int i = tid; i < 2 * DK + DV; i += THREADS) {
            const int c = i < DK ? h * DK + i : (i < 2 * DK ? key_dim + h * DK + (i - DK) : 2 * key_dim + h * DV + (i - 2 * DK));
            float *row = a.conv + ((size_t)b * conv_dim + c) * ck;
            const float *w = a.conv_w + (size_t)c * ck;
            const float xin = a.qkv[(size_t)b * conv_dim + c];
            float acc = 0.f;
            for (int j = 0; j < ck - 1; ++j) {
                const float v = row[j + 1];
                row[j] = v;
                acc += v * w[j];
            }
            row[ck - 1] = xin;
            acc += xin * w[ck - 1];
            const float y = silu_f(acc);
            if (i < DK) sq[i] = y;
            else if (i < 2 * DK) sk[i - DK] = y;
            else sv[i - 2 * DK] = y;
        }
    }
    if (tid == 0) {
        gates[0] = 1.0f / (1.0f + expf(-braw));
        gates[1] = -aex * logf(1.0f + expf(araw + dtb));
    }
    __syncthreads();

    // L2 norms (eps 1e-12 inside the root), q also scaled by 1/sqrt(d_k): both sums in one block reduction
    float pq = 0.f, pk = 0.f;
    for (int i = tid; i < DK; i += THREADS) {
        pq += sq[i] * sq[i];
        pk += sk[i] * sk[i];
    }
    pq = warp_sum(pq);
    pk = warp_sum(pk);
    if (lane == 0) red[warp] = make_float2(pq, pk);
    __syncthreads();
    float ssq = 0.f, ssk = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        ssq += red[w].x;
        ssk += red[w].y;
    }
    const float iq = 1.0f / sqrtf(ssq + 1e-12f), ik = 1.0f / sqrtf(ssk + 1e-12f);
    const float q_scale = 1.0f / sqrtf((float)DK);
    for (int i = tid; i < DK; i += THREADS) {
        sq[i] = sq[i] * iq * q_scale;
        sk[i] = sk[i] * ik;
    }
    __syncthreads();

    // column sums over the row groups; every thread gets its columns' totals (buffer `cb`, used once)
    auto colsum = [&](float4 x, int cb) -> float4 {
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) x = f4_add(x, f4_shfl_xor(x, off));
        if (lane < LPR) cred[cb][warp][lc] = x;
        __syncthreads();
        float4 t = cred[cb][0][lc];
#pragma unroll
        for (int w = 1; w < NW; ++w) t = f4_add(t, cred[cb][w][lc]);
        return t;
    };

    const float decay = expf(gates[1]), bet = gates[0];
    const bool s_ok = staged ? s_ok0 : mbar_wait(sbar, 0, a.dev_err);
    // pass p reads row rg + p * RP: from shared memory for p < NH, from registers after
    auto row = [&](int p) -> float4 { return p < NH ? Smem[(rg + p * RP) * (DV / 4)] : sreg[p - NH]; };
    float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const float ki = sk[rg + p * RP];
        float4 s = row(p);
        s.x *= decay; s.y *= decay; s.z *= decay; s.w *= decay;
        e.x += s.x * ki; e.y += s.y * ki; e.z += s.z * ki; e.w += s.w * ki;
    }
    e = colsum(e, 0);
    const float4 vv = make_float4(sv[col0], sv[col0 + 1], sv[col0 + 2], sv[col0 + 3]);
    const float4 dlt = make_float4(vv.x - e.x, vv.y - e.y, vv.z - e.z, vv.w - e.w);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int i = rg + p * RP;
        const float ki = bet * sk[i];
        float4 s = row(p);
        s.x *= decay; s.y *= decay; s.z *= decay; s.w *= decay;  // as in the first pass
        s.x += ki * dlt.x; s.y += ki * dlt.y; s.z += ki * dlt.z; s.w += ki * dlt.w;
        if (s_ok) __stcs(reinterpret_cast<float4 *>(Sh + (size_t)i * DV + col0), s);
        const float qi = sq[i];
        o.x += s.x * qi; o.y += s.y * qi; o.z += s.z * qi; o.w += s.w * qi;
    }
    o = colsum(o, 1);
    // gated RMSNorm over the head's d_v outputs: the LPR lanes of a row group hold the whole row, so the sum
    // of squares is a shuffle reduction (no block barrier); row group 0 writes
    float ss = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
#pragma unroll
    for (int off = 1; off < LPR; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (rg == 0) {
        const float rms = 1.0f / sqrtf(ss / DV + 1e-6f);
        const float *z = (staged ? zn : a.z + bh * DV) + col0;
        const float *nw = (staged ? zn + DV : a.norm_w) + col0;
        float4 y;
        y.x = o.x * rms * nw[0] * silu_f(z[0]);
        y.y = o.y * rms * nw[1] * silu_f(z[1]);
        y.z = o.z * rms * nw[2] * silu_f(z[2]);
        y.w = o.w * rms * nw[3] * silu_f(z[3]);
        *reinterpret_cast<float4 *>(a.out + bh * DV + col0) = y;
    }
}

// One CTA per sequence.
// One CTA per token row r = (sequence b, token i of n_tok): at position pos[b] (decode, n_tok = 1) or
// start_pos + i (a prefill chunk, pos null).  Input and output rows are indexed by r, cache rows by (b, p).
__global__ void __launch_bounds__(256) fullatt_prep_kernel(const AttnPrepArgs a) {
    const int r = blockIdx.x, b = r / a.n_tok;
    const int hd = a.hd, nh = a.nh, nkv = a.nkv, n_rot = a.n_rot, half = n_rot / 2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int p = a.pos ? a.pos[b] : a.start_pos + r % a.n_tok;
    const bool pos_ok = p >= 0 && p < a.max_seq;
    if (!pos_ok && tid == 0) atomicOr(a.dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
    const float *cs = a.rope_cos + (size_t)(pos_ok ? p : 0) * half;
    const float *sn = a.rope_sin + (size_t)(pos_ok ? p : 0) * half;
    // one warp per head: q heads then k heads
    for (int hh = warp; hh < nh + nkv; hh += nw) {
        const bool isq = hh < nh;
        const int hi = isq ? hh : hh - nh;
        const float *src = isq ? a.qg + ((size_t)r * nh + hi) * 2 * hd : a.k + ((size_t)r * nkv + hi) * hd;
        const float *wn = isq ? a.q_norm : a.k_norm;
        float ss = 0.f;
        for (int i = lane; i < hd; i += 32) ss += src[i] * src[i];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / hd + 1e-6f);
        const size_t qrow = ((size_t)r * nh + hi) * hd;
        for (int i = lane; i < hd; i += 32) {
            float y = src[i] * inv * wn[i];
            if (i < n_rot) {
                // rotated pair (i, i + half) within the first n_rot dims
                const int j = i < half ? i : i - half;
                const float x0 = src[j] * inv * wn[j], x1 = src[j + half] * inv * wn[j + half];
                y = i < half ? x0 * cs[j] - x1 * sn[j] : x0 * sn[j] + x1 * cs[j];
            }
            if (isq) {
                if (a.q_out_bf16)
                    a.q_out_bf16[qrow + i] = __float2bfloat16_rn(y);
                else
                    a.q_out[qrow + i] = y;
            } else if (pos_ok) {
                const size_t row = (((size_t)b * a.max_seq + p) * nkv + hi) * hd + i;
                if (a.dtype == EIF_CUDA_F32)
                    static_cast<float *>(a.Kc)[row] = y;
                else
                    static_cast<__nv_bfloat16 *>(a.Kc)[row] = __float2bfloat16_rn(y);
            }
        }
        if (isq)
            for (int i = lane; i < hd; i += 32) a.gate_out[qrow + i] = src[hd + i];
    }
    if (pos_ok)
        for (int i = tid; i < nkv * hd; i += blockDim.x) {
            const size_t row = ((size_t)b * a.max_seq + p) * nkv * hd + i;
            const float v = a.v[(size_t)r * nkv * hd + i];
            if (a.dtype == EIF_CUDA_F32)
                static_cast<float *>(a.Vc)[row] = v;
            else
                static_cast<__nv_bfloat16 *>(a.Vc)[row] = __float2bfloat16_rn(v);
        }
}

// The same prep with one warp per (token row, head) -- q heads, k heads, then one warp for the row's v --
// and every lane holding VPL = hd / 32 consecutive elements: each row of q, gate, k, v and the norm
// weights is read with one vector load per lane, all before any store, and the rotation partner
// (element i +- n_rot / 2) comes from lane +- n_rot / (2 VPL) by a shuffle.  Same arithmetic per element
// as fullatt_prep_kernel; the sum of squares is taken in another order (within float rounding).
template <int VPL>
__device__ __forceinline__ void load_vec(float (&x)[VPL], const float *src) {
    if constexpr (VPL == 2) {
        const float2 t = *reinterpret_cast<const float2 *>(src);
        x[0] = t.x; x[1] = t.y;
    } else {
#pragma unroll
        for (int k = 0; k < VPL; k += 4) {
            const float4 t = *reinterpret_cast<const float4 *>(src + k);
            x[k] = t.x; x[k + 1] = t.y; x[k + 2] = t.z; x[k + 3] = t.w;
        }
    }
}
template <int VPL>
__device__ __forceinline__ void store_vec(float *dst, const float (&x)[VPL]) {
    if constexpr (VPL == 2) {
        *reinterpret_cast<float2 *>(dst) = make_float2(x[0], x[1]);
    } else {
#pragma unroll
        for (int k = 0; k < VPL; k += 4)
            *reinterpret_cast<float4 *>(dst + k) = make_float4(x[k], x[k + 1], x[k + 2], x[k + 3]);
    }
}
template <int VPL>
__device__ __forceinline__ void store_vec_bf16(__nv_bfloat16 *dst, const float (&x)[VPL]) {
    uint32_t w[VPL / 2];
#pragma unroll
    for (int k = 0; k < VPL / 2; ++k) w[k] = pack_bf16x2(x[2 * k], x[2 * k + 1]);
    if constexpr (VPL == 2) *reinterpret_cast<uint32_t *>(dst) = w[0];
    else if constexpr (VPL == 4) *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
    else
#pragma unroll
        for (int k = 0; k < VPL / 2; k += 4) *reinterpret_cast<uint4 *>(dst + 2 * k) = make_uint4(w[k], w[k + 1], w[k + 2], w[k + 3]);
}

template <int VPL>
__global__ void __launch_bounds__(256) fullatt_prep_warp_kernel(const AttnPrepArgs a) {
    const int hd = a.hd, nh = a.nh, nkv = a.nkv, half = a.n_rot / 2;
    const int per_row = nh + nkv + 1;
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    griddep_wait();  // launched as a programmatic dependent: wait for the previous kernels' writes
    griddep_launch_dependents();  // after the wait: a dependent that starts early finds every earlier grid complete
    if (gw >= a.B * a.n_tok * per_row) return;  // warp-uniform; the kernel has no block barrier
    const int r = gw / per_row, hh = gw % per_row, b = r / a.n_tok;
    const int p = a.pos ? a.pos[b] : a.start_pos + r % a.n_tok;
    const bool pos_ok = p >= 0 && p < a.max_seq;
    if (hh == nh + nkv) {  // v row -> cache
        if (!pos_ok) return;
        const float *src = a.v + (size_t)r * nkv * hd;
        const size_t row = ((size_t)b * a.max_seq + p) * nkv * hd;
        for (int i = lane * VPL; i < nkv * hd; i += 32 * VPL) {
            float x[VPL];
            load_vec<VPL>(x, src + i);
            if (a.dtype == EIF_CUDA_F32)
                store_vec<VPL>(static_cast<float *>(a.Vc) + row + i, x);
            else
                store_vec_bf16<VPL>(static_cast<__nv_bfloat16 *>(a.Vc) + row + i, x);
        }
        return;
    }
    if (!pos_ok && hh == 0 && lane == 0) atomicOr(a.dev_err, (unsigned)EIF_DEVERR_POS_RANGE);
    const bool isq = hh < nh;
    const int hi = isq ? hh : hh - nh, i0 = lane * VPL;
    const float *src = isq ? a.qg + ((size_t)r * nh + hi) * 2 * hd : a.k + ((size_t)r * nkv + hi) * hd;
    float x[VPL], w[VPL], g[VPL];
    load_vec<VPL>(x, src + i0);
    load_vec<VPL>(w, (isq ? a.q_norm : a.k_norm) + i0);
    if (isq) load_vec<VPL>(g, src + hd + i0);
    const bool rot = i0 < 2 * half;  // whole lanes: half is a multiple of VPL
    float cs[VPL], sn[VPL];
    if (rot) {
        const int j0 = i0 < half ? i0 : i0 - half;
        const float *c = a.rope_cos + (size_t)(pos_ok ? p : 0) * half + j0;
        const float *t = a.rope_sin + (size_t)(pos_ok ? p : 0) * half + j0;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            cs[k] = c[k];
            sn[k] = t[k];
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) ss += x[k] * x[k];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / hd + 1e-6f);
    float y[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) y[k] = x[k] * inv * w[k];
    const int dl = half / VPL;
    const int partner = !rot ? lane : (i0 < half ? lane + dl : lane - dl);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
        const float o = __shfl_sync(0xffffffffu, y[k], partner);
        if (rot) {
            const float x0 = i0 < half ? y[k] : o, x1 = i0 < half ? o : y[k];
            y[k] = i0 < half ? x0 * cs[k] - x1 * sn[k] : x0 * sn[k] + x1 * cs[k];
        }
    }
    if (isq) {
        const size_t qrow = ((size_t)r * nh + hi) * hd + i0;
        if (a.q_out_bf16)
            store_vec_bf16<VPL>(a.q_out_bf16 + qrow, y);
        else
            store_vec<VPL>(a.q_out + qrow, y);
        store_vec<VPL>(a.gate_out + qrow, g);
    } else if (pos_ok) {
        const size_t row = (((size_t)b * a.max_seq + p) * nkv + hi) * hd + i0;
        if (a.dtype == EIF_CUDA_F32)
            store_vec<VPL>(static_cast<float *>(a.Kc) + row, y);
        else
            store_vec_bf16<VPL>(static_cast<__nv_bfloat16 *>(a.Kc) + row, y);
    }
}

}  // namespace

cudaError_t launch_deltanet_core(cudaStream_t st, const DeltaCoreArgs &a0, bool *supported) {
    *supported = true;
    const dim3 grid(a0.H, a0.B);
    // the inputs ride on the S barrier as bulk copies when every array is 16-byte aligned (the channel blocks'
    // offsets then are too: d_k and d_v are multiples of 4) and the windows are short enough to stage
    DeltaCoreArgs a = a0;
    auto al = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    a.stage_inputs = a.conv_k >= 1 && a.conv_k <= 4 && al(a.conv) && al(a.conv_w) && al(a.qkv) && al(a.z) &&
                     al(a.norm_w);
    auto run = [&](auto kernel, int threads) {
        // dynamic shared memory: S rows [0, dk/2) | z, norm_w | the larger of the staged inputs and the two
        // column-sum buffers (one float4 per thread each)
        const size_t nc = 2 * (size_t)a.dk + a.dv;
        const size_t csum = 2 * (size_t)threads * 16, staging = a.stage_inputs ? nc * (2 * a.conv_k + 1) * 4 : 0;
        const size_t smem = (size_t)a.dk / 2 * a.dv * 4 + 2 * (size_t)a.dv * 4 + (staging > csum ? staging : csum);
        // static + dynamic shared memory above 48 KB needs the opt-in (the static part is under 8 KB)
        if (smem > 40 * 1024) {
            const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        launch_pdl(kernel, grid, dim3(threads), smem, st, a);
        return cudaGetLastError();
    };
    if (a.dk == 128 && a.dv == 128) return run(deltanet_core_kernel<128, 128, 256>, 256);
    if (a.dk == 128 && a.dv == 64) return run(deltanet_core_kernel<128, 64, 256>, 256);
    if (a.dk == 64 && a.dv == 64) return run(deltanet_core_kernel<64, 64, 128>, 128);
    *supported = false;
    return cudaSuccess;
}

cudaError_t launch_fullatt_prep(cudaStream_t st, const AttnPrepArgs &a) {
    // the warp-per-head form needs hd in {64, 128, 256}, whole lanes of rotated pairs and vector-aligned rows
    const int vpl = a.hd / 32, half = a.n_rot / 2;
    auto al = [&](const void *q) { return ((uintptr_t)q % (vpl == 2 ? 8 : 16)) == 0; };
    const bool warp_form = (a.hd == 64 || a.hd == 128 || a.hd == 256) && half % vpl == 0 && a.n_rot <= a.hd &&
                           al(a.qg) && al(a.k) && al(a.v) && al(a.q_norm) && al(a.k_norm) && al(a.Kc) && al(a.Vc) &&
                           al(a.gate_out) && (a.q_out_bf16 ? al(a.q_out_bf16) : al(a.q_out));
    if (!warp_form) {
        fullatt_prep_kernel<<<a.B * a.n_tok, 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    const long warps = (long)a.B * a.n_tok * (a.nh + a.nkv + 1);
    const unsigned blocks = (unsigned)((warps + 7) / 8);
    if (vpl == 2) launch_pdl(fullatt_prep_warp_kernel<2>, dim3(blocks), dim3(256), 0, st, a);
    else if (vpl == 4) launch_pdl(fullatt_prep_warp_kernel<4>, dim3(blocks), dim3(256), 0, st, a);
    else launch_pdl(fullatt_prep_warp_kernel<8>, dim3(blocks), dim3(256), 0, st, a);
    return cudaGetLastError();
}
