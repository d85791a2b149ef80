// internal.h -- shared between the .cu files of libeif_cuda.so (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/eif_cuda.h"

// Device-side error word bits (set by kernels, read back by eif_cuda_synchronize / host entry points).
enum : unsigned {
    EIF_DEVERR_POS_RANGE = 1u,   // a pos[] value outside [0, max_seq_len)
    EIF_DEVERR_WAIT_LIMIT = 2u,  // a bounded pipeline wait ran out of iterations
};

struct eif_cuda_ctx {
    int device = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    int timeout_ms = 120000;
    uint64_t launches = 0;
    char err[512] = {0};
    // device scratch (split-K partials etc.), grown on demand
    void *ws = nullptr;
    size_t ws_bytes = 0;
    // device staging for the host-pointer entry points, grown on demand
    void *stage = nullptr;
    size_t stage_bytes = 0;
    // device q / gate between the two halves of eif_cuda_fullatt_decode_dev, grown on demand
    void *mix = nullptr;
    size_t mix_bytes = 0;
    // device (cache sequence, pos) of every query row of a prefill over an fp32 / INT8 cache, grown on demand
    void *rowbuf = nullptr;
    size_t rowbuf_bytes = 0;
    // device error word: the first 16 bytes of io, whose remaining kSmallIo bytes take the outputs of
    // small host-pointer calls, so that the word and the output come back in one copy
    void *io = nullptr;
    unsigned *dev_err = nullptr;
    // pinned host copy of the error word
    unsigned *host_err = nullptr;
    // pinned host staging of small host-pointer calls: [inputs, packed | error word + output]
    void *pin = nullptr;
    // the DeltaNet state written by the most recent deltanet_core launch, and `launches` right after it: the next
    // deltanet_core may read its own state before its grid-dependency wait unless it is that state and no other
    // launch came in between
    const void *last_state = nullptr;
    uint64_t last_state_launches = 0;
};

// Host-pointer calls whose inputs (together) and output are at most this many bytes go through the pinned
// staging block: one host-to-device copy of the packed inputs, one copy back of the error word + output.
constexpr size_t kSmallIo = 256 << 10;

struct eif_cuda_kv {
    eif_cuda_ctx_t *ctx = nullptr;
    int n_layers = 0, batch = 0, max_seq = 0, n_kv = 0, hd = 0;
    eif_cuda_dtype_t dtype = EIF_CUDA_F32;
    size_t layer_elems = 0;  // batch * max_seq * n_kv * hd
    void **k = nullptr;      // [n_layers] device pointers
    void **v = nullptr;
    // INT8 caches: per-layer scales of K and V, head-major [batch][n_kv][scale_stride] with scale_stride =
    // max_seq rounded up to 64, so the 64 scales of a key tile are one aligned 256-byte run (nullptr otherwise)
    float **ks = nullptr, **vs = nullptr;
    int scale_stride = 0;
    // TMA descriptors of the layers (the decode kernels' boxes for the cache dtype), made on first use
    CUtensorMap *tmk = nullptr;
    CUtensorMap *tmv = nullptr;
    bool *tm_ready = nullptr;
    // Qwen3.5 attention prep: per-layer q_norm / k_norm [hd] and the partial-RoPE cos / sin table
    float **q_norm = nullptr, **k_norm = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;  // [max_seq][hd/8], theta 1e7 (made on first use)
    // tinyllm RoPE: full-width tables [max_seq][hd/2] for the model's theta (eif_cuda_kv_set_rope)
    float *tl_cos = nullptr, *tl_sin = nullptr;
    int tl_interleaved = 0;
};

struct eif_cuda_delta {
    eif_cuda_ctx_t *ctx = nullptr;
    int n_layers = 0, batch = 0, H = 0, dk = 0, dv = 0, conv_k = 0, conv_dim = 0;
    float **S = nullptr;     // [n_layers] -> [batch][H][dk][dv]
    float **conv = nullptr;  // [n_layers] -> [batch][conv_dim][conv_k] (nullptr when conv_k == 0)
    // per-layer weights of deltanet_core, uploaded by eif_cuda_delta_set_weights: one device block
    // [conv_dim*conv_k | H dt_bias | H exp(A_log) | dv norm_w]
    float **weights = nullptr;
};

// ---- launchers (return cudaError_t of the launch) ----
cudaError_t launch_delta_rule(cudaStream_t st, float *S, const float *q, const float *k, const float *v,
                              const float *beta, const float *g, float q_scale, float *o, int B, int H, int dk,
                              int dv, int sm_count, bool *supported);

struct DecodeArgs {
    const void *K;
    const void *V;
    eif_cuda_dtype_t dtype;
    const float *q;
    const int *pos;
    int B, Hq, Hkv, D, max_seq;
    int max_len;  // upper bound of pos[b] + 1
    float scale;
    const float *gate;
    int subln;
    const float *sub_norm;
    float *out;
    unsigned *dev_err;
    const CUtensorMap *tmk = nullptr;  // TMA descriptors of K / V (nullptr -> SIMT kernel)
    const CUtensorMap *tmv = nullptr;
    bool force_simt = false;
    size_t max_ws_bytes = 0;  // 0: the split may use any amount of scratch; else it must fit in this many bytes
    const float *k_scale = nullptr;  // INT8 caches: [B][Hkv][scale_stride] scales of K and V
    const float *v_scale = nullptr;
    int scale_stride = 0;
    // nullptr: query row b reads cache sequence b.  Else [B] cache sequence of each query row (prefill over
    // fp32 / INT8 caches runs every token of a chunk as one decode row at its own pos)
    const int *row_seq = nullptr;
};

// Fused per-token mixer bodies (mixer_fused.cu).
struct DeltaCoreArgs {
    float *S, *conv;  // layer state [B][H][dk][dv], conv windows [B][conv_dim][conv_k]
    const float *qkv, *z, *b_raw, *a_raw;  // [B][conv_dim], [B][H*dv], [B][H], [B][H]
    const float *conv_w, *dt_bias, *a_exp, *norm_w;  // layer weights: [conv_dim][conv_k], [H], [H], [dv]
    float *out;  // [B][H*dv]
    int B, H, dk, dv, conv_k;
    unsigned *dev_err;
    int stage_inputs;  // set by launch_deltanet_core: the conv windows, weights, inputs, z and norm_w come by bulk copies
    int prefetch;      // the kernel launched just before this one on the stream does not write this layer's state
};
cudaError_t launch_deltanet_core(cudaStream_t st, const DeltaCoreArgs &a, bool *supported);

struct AttnPrepArgs {
    const float *qg, *k, *v;  // rows r = (b, token): [B*n_tok][nh][2*hd], [B*n_tok][nkv*hd], [B*n_tok][nkv*hd]
    const float *q_norm, *k_norm;  // [hd]
    const float *rope_cos, *rope_sin;  // [max_seq][n_rot/2]
    const int *pos;  // [B] (one token per sequence), or null: row (b, i) sits at start_pos + i
    void *Kc, *Vc;   // layer cache
    eif_cuda_dtype_t dtype;
    float *q_out, *gate_out;  // [B*n_tok][nh*hd] (q_out unused when q_out_bf16 is set)
    int B, nh, nkv, hd, n_rot, max_seq;
    unsigned *dev_err;
    __nv_bfloat16 *q_out_bf16;  // q as bf16 (the prefill attention's input), or null
    int n_tok, start_pos;
};
cudaError_t launch_fullatt_prep(cudaStream_t st, const AttnPrepArgs &a);

// tinyllm RoPE + cache write (rope.cu): rows r = (b, token) as in AttnPrepArgs.
struct RopeArgs {
    const float *q, *k, *v;            // [B*n_tok][nh*hd], [B*n_tok][nkv*hd], [B*n_tok][nkv*hd]
    const float *cos_t, *sin_t;        // [max_seq][hd/2]
    const int *pos;                    // [B] or null (row (b, i) at start_pos + i)
    void *Kc, *Vc;
    eif_cuda_dtype_t dtype;
    float *q_out;                      // [B*n_tok][nh*hd] fp32, unless q_out_bf16 is set
    __nv_bfloat16 *q_out_bf16;
    int B, n_tok, start_pos, nh, nkv, hd, max_seq, interleaved;
    unsigned *dev_err;
    float *k_scale = nullptr, *v_scale = nullptr;  // INT8 caches: [B][nkv][scale_stride]
    int scale_stride = 0;
};
cudaError_t launch_rope_append(cudaStream_t st, const RopeArgs &a);

// Chunked (WY / UT) DeltaNet prefill (deltanet_chunked.cu).
bool deltanet_chunked_supported(int dk, int dv);
// Scratch of the chunked prefill: per (sequence, head, chunk) the bf16 [128][64] pair T diag(-b e^G) ; T diag(b)
// (deltanet_chunked_tmat_bytes, at the start), then the fp32 [64] cumulative log decays G.
size_t deltanet_chunked_tmat_bytes(int B, int T, int H);
size_t deltanet_chunked_workspace(int B, int T, int H);
cudaError_t launch_deltanet_chunked(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                    const CUtensorMap &tv, const CUtensorMap &tt, void *t_ws, const float *beta,
                                    const float *g, __nv_bfloat16 *o, float *o_f32, float *S, int B, int T, int H,
                                    int dv, float q_scale, unsigned *dev_err, int *n_launches);  // o_f32: fp32 out

// Chunk-level DeltaNet pre / post ops of the prefill core (deltanet_prefill_ops.cu).
struct DeltaPrefillArgs {
    const float *qkv, *z, *b_raw, *a_raw;  // [B][n_tok][conv_dim], [B][n_tok][H*dv], [B][n_tok][H] x 2
    float *conv;                           // [B][conv_dim][conv_k] window, updated to the chunk's last inputs
    const float *conv_w, *dt_bias, *a_exp, *norm_w;
    __nv_bfloat16 *q, *k, *v;              // [B][n_tok][H][dk | dk | dv] (q L2-normalised and scaled)
    float *beta, *g;                       // [B][n_tok][H]
    const float *o;                        // [B][n_tok][H][dv] fp32, the rule's output
    float *out;                            // [B][n_tok][H*dv]
    int B, n_tok, H, dk, dv, conv_k;
};
cudaError_t launch_deltanet_prefill_pre(cudaStream_t st, const DeltaPrefillArgs &a);
cudaError_t launch_deltanet_prefill_post(cudaStream_t st, const DeltaPrefillArgs &a);

// Causal prefill attention on tcgen05 (attn_prefill_tc.cu), head_dim D.
bool prefill_tc_supported(int D);
cudaError_t launch_attend_prefill_tc(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                     const CUtensorMap &tv, int B, int n_tok, int start_pos, int Hq, int Hkv,
                                     int max_seq, int D, float scale, __nv_bfloat16 *out, float *out_f32,
                                     unsigned *dev_err);  // out_f32 set: fp32 output there instead of bf16
// Row epilogue after prefill (gate_subln.cu): out = SubLN(o * sigmoid(gate)) per row of `dim` values.
cudaError_t launch_gate_subln(cudaStream_t st, const float *o, const float *gate, int rows, int dim, int subln,
                              const float *sub_norm, float *out);
// head_dim 256 (attn_prefill_hd256.cu): one query tile per CTA, double-buffered S.
cudaError_t launch_attend_prefill_hd256(cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk,
                                        const CUtensorMap &tv, int B, int n_tok, int start_pos, int Hq, int Hkv,
                                        int max_seq, float scale, __nv_bfloat16 *out, float *out_f32,
                                        unsigned *dev_err);

// Fills the TMA descriptors (made on first use per layer) and the kernel choice of `a` (eif_cuda.cu).
void decode_prepare(eif_cuda_kv_t *kv, int layer, DecodeArgs &a);

// Tensor-core decode path (attn_decode_tc.cu).
bool decode_tc_supported(int D, int G);
int decode_tc_partials(int D);  // partials per item of the bf16 kernel (one per consumer warp)
cudaError_t launch_attend_decode_tc(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                    const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                    float2 *part_ml, int sm_count);
// TMA-fed decode over an fp32 cache (attn_decode_f32.cu); tk / tv: 32-key x 32-float boxes, 128-byte swizzle.
// One tinyllm decode step in one launch for small batches (attn_decode_step.cu): RoPE of q and k, the new
// K / V row, GQA attention over [0, pos] split over a cluster of nc CTAs per (sequence, kv head).
struct DecodeStepArgs {
    const float *q, *k, *v;       // [B][Hq*D], [B][Hkv*D], [B][Hkv*D] fp32, un-rotated
    const int *pos;               // [B]
    const float *cos_t, *sin_t;   // [max_seq][D/2]
    void *Kc, *Vc;                // the layer's cache
    eif_cuda_dtype_t dtype;
    float *out;                   // [B][Hq*D]
    int B, Hq, Hkv, D, max_seq, interleaved, nc;
    float scale;
    unsigned *dev_err;
    int chunk_cap;                // keys of the largest chunk (sizes the staged rows)
};
// Chunks per (sequence, kv head) of the one-launch step for this shape (and the largest chunk in
// *chunk_cap), or 0 when it does not take it.
int decode_step_chunks(eif_cuda_dtype_t dtype, int D, int G, int B, int Hkv, int max_len, int sm_count,
                       int *chunk_cap);
cudaError_t launch_attend_decode_step(cudaStream_t st, const DecodeStepArgs &a);

bool decode_f32_supported(int D, int G);
cudaError_t launch_attend_decode_f32(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                     const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                     float2 *part_ml, int sm_count);
// Tensor-core decode over an INT8 cache (attn_decode_i8.cu); tk / tv: 64-byte-swizzled int8 tensor maps.
cudaError_t launch_attend_decode_i8(cudaStream_t st, const CUtensorMap &tk, const CUtensorMap &tv,
                                    const DecodeArgs &a, int nchunk, int chunk_keys, float *part_o,
                                    float2 *part_ml, int sm_count);
// Launch `kernel` as a programmatic dependent of the previous kernel on `st`: its CTAs may start while that kernel
// drains, so the kernel must call griddepcontrol.wait (griddep_wait) before it reads anything the previous kernels
// wrote, and may call griddepcontrol.launch_dependents to let the next one do the same.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// KV heads a work item of the INT8 tensor-core decode covers: both heads of a 128-byte cache row at head_dim 64
// with an even kv-head count (attn_decode_i8.cu), else one.
inline int decode_i8_heads_per_item(int D, int Hkv) { return D == 64 && Hkv % 2 == 0 ? 2 : 1; }
// Workspace bytes needed by launch_attend_decode for these args and the chosen split.
size_t decode_workspace_bytes(const DecodeArgs &a, int sm_count);
// The split launch_attend_decode would use: key chunks per (sequence, kv head), keys per chunk, scratch bytes.
void decode_plan(const DecodeArgs &a, int sm_count, int *nchunk, int *chunk_keys, size_t *ws_bytes);
// Query rows of a prefill chunk as decode rows: row i = token i % n_tok of sequence i / n_tok at start_pos + i % n_tok.
cudaError_t launch_prefill_rows(cudaStream_t st, int *row_seq, int *pos, int batch, int n_tok, int start_pos);
// A projection's weights on the device (linear.cu): the engine's packed rows, each padded with zeros to `stride`
// bytes (a multiple of 64), and the scales (rows x n_scales_row floats; none for fp32).
struct eif_cuda_linear {
    eif_cuda_ctx_t *ctx = nullptr;
    int wtype = 0, group = 0, rows = 0, cols = 0;
    size_t row_bytes = 0, stride = 0;
    int n_scales_row = 0;
    uint8_t *W = nullptr;
    float *scales = nullptr;
};
// The engine's bytes a row of the format (row_bytes, src/eif_qwen35.c:110-116; INT8: a byte a weight).
size_t linear_row_bytes(int wtype, int cols);
// Whether a row of `stride` bytes fits the kernel's shared-memory token tile.
bool linear_fits(int wtype, size_t stride);
// out[t][rows] = W x[t] for n tokens (fp32 device arrays): the tensor-core kernel where it supports the format and
// n >= 4 (linear_mma.cu), else the CUDA-core kernel (linear.cu).
cudaError_t launch_linear(cudaStream_t st, const eif_cuda_linear &lin, const float *x, int n, float *out,
                          int sm_count);
bool linear_mma_supported(const eif_cuda_linear &lin);
cudaError_t launch_linear_mma(cudaStream_t st, const eif_cuda_linear &lin, const float *x, int n, float *out,
                              int sm_count);
// Bytes of the fixed scratch array of eif_cuda_attend_decode_noalloc_dev (noalloc.cu).
size_t noalloc_scratch_capacity();
cudaError_t launch_attend_decode(cudaStream_t st, const DecodeArgs &a, void *ws, size_t ws_bytes, int sm_count,
                                 bool *supported, int *n_launches);

cudaError_t launch_kv_append(cudaStream_t st, void *K, void *V, eif_cuda_dtype_t dtype, const int *pos,
                             const float *k, const float *v, int B, int max_seq, int kv_dim, unsigned *dev_err);
// INT8 caches (kv.cu).  Quantise fp32 rows (k, v: [n_rows][nkv*hd]) into the cache: row r lands in
// sequence r at position pos[r] when pos is set (one new token per sequence), else in sequence `seq` at
// position t0 + r.  Scales are [B][nkv][scale_stride].
cudaError_t launch_kv_quantize(cudaStream_t st, int8_t *K, int8_t *V, float *ks, float *vs, const int *pos,
                               int seq, int t0, const float *k, const float *v, int n_rows, int max_seq, int nkv,
                               int hd, int scale_stride, unsigned *dev_err);
// code * scale of rows [t0, t0 + n_rows) of sequence `seq`, into fp32 [n_rows][nkv*hd].
cudaError_t launch_kv_dequantize(cudaStream_t st, const int8_t *K, const float *ks, int seq, int t0, float *out,
                                 int n_rows, int max_seq, int nkv, int hd, int scale_stride);
cudaError_t launch_f32_to_bf16(cudaStream_t st, const float *src, __nv_bfloat16 *dst, size_t n);
cudaError_t launch_bf16_to_f32(cudaStream_t st, const __nv_bfloat16 *src, float *dst, size_t n);
