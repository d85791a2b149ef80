// eif_cuda.cu -- the C ABI of include/eif_cuda.h: contexts, device mirrors of the engine's KV cache
// and DeltaNet state, argument checking, host<->device staging and kernel dispatch.
//
// Every entry point validates its arguments on the host before anything is launched and returns an
// eif_status_t (include/eif_status.h:8-19 in bitllm.c); there is no CPU fallback.  Host-pointer
// entry points wait with a deadline (EIF_STATUS_TIMEOUT) instead of blocking forever.
#include <errno.h>
#include <math.h>
#include <sched.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <new>

#include "internal.h"

#define EIF_API extern "C" __attribute__((visibility("default")))

namespace {

eif_status_t fail(eif_cuda_ctx_t *ctx, eif_status_t st, const char *fmt, ...) {
    if (ctx) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(ctx->err, sizeof ctx->err, fmt, ap);
        va_end(ap);
    }
    return st;
}

eif_status_t cuda_fail(eif_cuda_ctx_t *ctx, cudaError_t e, const char *what) {
    const eif_status_t st = (e == cudaErrorMemoryAllocation) ? EIF_STATUS_OUT_OF_MEMORY : EIF_STATUS_ERROR;
    return fail(ctx, st, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call)                                                      \
    do {                                                              \
        cudaError_t _e = (call);                                      \
        if (_e != cudaSuccess) return cuda_fail(ctx, _e, #call);      \
    } while (0)

bool no_cuda_env() {
    const char *e = getenv("BITLLM_NO_CUDA");
    return e && *e && strcmp(e, "0") != 0;
}

// Makes ctx->device current for the scope and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(const eif_cuda_ctx_t *ctx) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != ctx->device) ok = cudaSetDevice(ctx->device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

// Grow a device buffer; waits for the stream first because queued work may still use the old one.
eif_status_t ensure_buffer(eif_cuda_ctx_t *ctx, void **buf, size_t *cap, size_t bytes) {
    if (bytes <= *cap) return EIF_STATUS_OK;
    CK(cudaStreamSynchronize(ctx->stream));
    if (*buf) CK(cudaFree(*buf));
    *buf = nullptr;
    *cap = 0;
    const size_t want = std::max(bytes, (size_t)1 << 20);
    CK(cudaMalloc(buf, want));
    *cap = want;
    return EIF_STATUS_OK;
}

// Wait for the context's stream with the deadline (the work queued so far, copies included).
static eif_status_t wait_done(eif_cuda_ctx_t *ctx) {
    cudaError_t e = cudaEventRecord(ctx->done, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "queue completion event");
    const double t0 = now_ms();
    int spins = 0;
    for (;;) {
        e = cudaEventQuery(ctx->done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_fail(ctx, e, "device work failed");
        if (ctx->timeout_ms > 0 && now_ms() - t0 > ctx->timeout_ms)
            return fail(ctx, EIF_STATUS_TIMEOUT, "device work did not finish within %d ms", ctx->timeout_ms);
        if (++spins < 2000)
            sched_yield();
        else
            usleep(50);
    }
    return EIF_STATUS_OK;
}

// The device error word read back after the work: clears it and reports what it says.
static eif_status_t check_err_word(eif_cuda_ctx_t *ctx, unsigned derr) {
    if (derr) {
        CK(cudaMemsetAsync(ctx->dev_err, 0, sizeof(unsigned), ctx->stream));
        if (derr & EIF_DEVERR_POS_RANGE)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "a kernel saw pos outside [0, max_seq_len) or above the call's max_pos");
        if (derr & EIF_DEVERR_WAIT_LIMIT)
            return fail(ctx, EIF_STATUS_TIMEOUT, "a kernel pipeline wait ran out of iterations");
        return fail(ctx, EIF_STATUS_INTERNAL_ERROR, "device error word 0x%x", derr);
    }
    return EIF_STATUS_OK;
}

// Wait for the context's stream with the deadline, then report any device-side error word.
eif_status_t wait_stream(eif_cuda_ctx_t *ctx) {
    *ctx->host_err = 0;
    CK(cudaMemcpyAsync(ctx->host_err, ctx->dev_err, sizeof(unsigned), cudaMemcpyDeviceToHost, ctx->stream));
    const eif_status_t st = wait_done(ctx);
    if (st != EIF_STATUS_OK) return st;
    return check_err_word(ctx, *ctx->host_err);
}

// Small host-pointer calls.  send_packed copies n host arrays (total at most kSmallIo, each at a 16-byte
// aligned offset off[i]) into the pinned block and sends them to dst in one copy; the call's kernels write
// an output of at most kSmallIo bytes to small_out(ctx); finish_small brings back the error word and that
// output in one copy, waits, and hands the output to the caller.  The pinned block is reused only after
// the wait, so no copy still reads it.
static size_t a16(size_t x) { return (x + 15) & ~(size_t)15; }

static float *small_out(eif_cuda_ctx_t *ctx) { return reinterpret_cast<float *>(static_cast<char *>(ctx->io) + 16); }

static eif_status_t send_packed(eif_cuda_ctx_t *ctx, char *dst, int n, const void *const *src, const size_t *bytes,
                                size_t *off) {
    char *h = static_cast<char *>(ctx->pin);
    size_t o = 0;
    for (int i = 0; i < n; ++i) {
        off[i] = o;
        if (bytes[i]) memcpy(h + o, src[i], bytes[i]);
        o += a16(bytes[i]);
    }
    CK(cudaMemcpyAsync(dst, h, o, cudaMemcpyHostToDevice, ctx->stream));
    return EIF_STATUS_OK;
}

static eif_status_t finish_small(eif_cuda_ctx_t *ctx, void *out, size_t bytes) {
    char *h = static_cast<char *>(ctx->pin) + kSmallIo;
    CK(cudaMemcpyAsync(h, ctx->io, 16 + bytes, cudaMemcpyDeviceToHost, ctx->stream));
    eif_status_t st = wait_done(ctx);
    if (st != EIF_STATUS_OK) return st;
    st = check_err_word(ctx, *reinterpret_cast<const unsigned *>(h));
    if (st != EIF_STATUS_OK) return st;
    memcpy(out, h + 16, bytes);
    return EIF_STATUS_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link dependency on libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// TMA descriptor of one cache array [batch*max_seq][n_kv][hd] as a 3-D tensor (hd, n_kv, rows) with the boxes
// and swizzle each decode kernel's shared-memory addressing expects: bf16 64 dims x 64 keys (128-byte rows,
// 128-byte swizzle), INT8 128 dims x 64 keys (128-byte rows, 128-byte swizzle; 64 dims and the 64-byte
// swizzle at head_dim 64), fp32 32 dims x 32 keys (128-byte rows, 128-byte swizzle).
bool make_kv_tensor_map(CUtensorMap *map, void *base, const eif_cuda_kv_t *kv) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc || kv->hd % 64) return false;
    const bool i8 = kv->dtype == EIF_CUDA_INT8, f32 = kv->dtype == EIF_CUDA_F32;
    const cuuint64_t elt = i8 ? 1 : f32 ? 4 : 2;
    const cuuint64_t dims[3] = {(cuuint64_t)kv->hd, (cuuint64_t)kv->n_kv, (cuuint64_t)kv->batch * kv->max_seq};
    const cuuint64_t strides[2] = {(cuuint64_t)kv->hd * elt, (cuuint64_t)kv->n_kv * kv->hd * elt};
    // INT8: 128-byte rows (128 dims) from head_dim 128 up; 64-byte rows at head_dim 64
    const cuuint32_t box0 = f32 ? 32u : (i8 && kv->hd >= 128) ? 128u : 64u;
    // fp32: 32-key boxes, 16 at head_dim 256 (the fp32 decode kernel's tile there)
    const cuuint32_t box[3] = {box0, 1, f32 ? (kv->hd == 256 ? 16u : 32u) : 64u};
    const cuuint32_t es[3] = {1, 1, 1};
    // L2 promotion no wider than what a tile reads of a cache row: one kv head's row, or two heads' at INT8 head_dim
    // 64 with an even kv-head count (the INT8 decode kernel's stages then hold both halves of each 128-byte row);
    // a wider promotion would fetch rows of other work items from HBM with every tile
    const size_t head_row = (size_t)kv->hd * elt * ((i8 && kv->hd == 64 && kv->n_kv % 2 == 0) ? 2 : 1);
    const CUtensorMapL2promotion promo = head_row >= 256   ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                         : head_row >= 128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                                           : CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
    return enc(map, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides,
               box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               (i8 && kv->hd < 128) ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
               promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool env_flag(const char *name) {
    const char *e = getenv(name);
    return e && *e && strcmp(e, "0") != 0;
}

// Carve consecutive 256-byte aligned slices out of the staging buffer.
struct Carver {
    size_t off = 0;
    size_t take(size_t bytes) {
        const size_t o = off;
        off += a256(bytes);
        return o;
    }
};

}  // namespace

// =================================================================================================
// Context
// =================================================================================================

EIF_API int eif_cuda_device_count(void) {
    if (no_cuda_env()) return 0;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

EIF_API eif_status_t eif_cuda_init(eif_cuda_ctx_t **out, int device) {
    if (!out) return EIF_STATUS_INVALID_ARGUMENT;
    *out = nullptr;
    if (no_cuda_env()) return EIF_STATUS_NOT_SUPPORTED;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return EIF_STATUS_NOT_SUPPORTED;
    }
    if (device < 0 || device >= n) return EIF_STATUS_NOT_SUPPORTED;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return EIF_STATUS_NOT_SUPPORTED;
    if (prop.major != 10 || prop.minor != 0) return EIF_STATUS_NOT_SUPPORTED;  // built for sm_100a only

    eif_cuda_ctx_t *ctx = new eif_cuda_ctx_t();
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    ctx->cc_major = prop.major;
    ctx->cc_minor = prop.minor;
    DeviceGuard g(ctx);
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->io, 16 + kSmallIo);
    if (e == cudaSuccess) e = cudaMemset(ctx->io, 0, 16);
    if (e == cudaSuccess) e = cudaMallocHost(&ctx->host_err, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMallocHost(&ctx->pin, 2 * kSmallIo + 16);
    ctx->dev_err = static_cast<unsigned *>(ctx->io);
    if (e != cudaSuccess) {
        eif_cuda_free(ctx);
        return e == cudaErrorMemoryAllocation ? EIF_STATUS_OUT_OF_MEMORY : EIF_STATUS_ERROR;
    }
    ctx->stream = ctx->own_stream;
    *out = ctx;
    return EIF_STATUS_OK;
}

EIF_API void eif_cuda_free(eif_cuda_ctx_t *ctx) {
    if (!ctx) return;
    {
        DeviceGuard g(ctx);
        if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
        if (ctx->stream && ctx->stream != ctx->own_stream) cudaStreamSynchronize(ctx->stream);
        if (ctx->ws) cudaFree(ctx->ws);
        if (ctx->stage) cudaFree(ctx->stage);
        if (ctx->mix) cudaFree(ctx->mix);
        if (ctx->rowbuf) cudaFree(ctx->rowbuf);
        if (ctx->io) cudaFree(ctx->io);
        if (ctx->host_err) cudaFreeHost(ctx->host_err);
        if (ctx->pin) cudaFreeHost(ctx->pin);
        if (ctx->done) cudaEventDestroy(ctx->done);
        if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    }
    delete ctx;
}

EIF_API const char *eif_cuda_last_error(const eif_cuda_ctx_t *ctx) { return ctx ? ctx->err : "no context"; }

EIF_API eif_status_t eif_cuda_set_stream(eif_cuda_ctx_t *ctx, void *stream) {
    if (!ctx) return EIF_STATUS_INVALID_ARGUMENT;
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    return EIF_STATUS_OK;
}

EIF_API void *eif_cuda_get_stream(const eif_cuda_ctx_t *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

EIF_API eif_status_t eif_cuda_set_timeout(eif_cuda_ctx_t *ctx, int timeout_ms) {
    if (!ctx || timeout_ms < 0) return EIF_STATUS_INVALID_ARGUMENT;
    ctx->timeout_ms = timeout_ms;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_synchronize(eif_cuda_ctx_t *ctx) {
    if (!ctx) return EIF_STATUS_INVALID_ARGUMENT;
    DeviceGuard g(ctx);
    return wait_stream(ctx);
}

EIF_API uint64_t eif_cuda_launch_count(const eif_cuda_ctx_t *ctx) { return ctx ? ctx->launches : 0; }

// =================================================================================================
// KV cache
// =================================================================================================

static size_t dtype_size(eif_cuda_dtype_t t) { return t == EIF_CUDA_INT8 ? 1 : t == EIF_CUDA_BF16 ? 2 : 4; }

// Bytes of one layer's K (or V) scale array of an INT8 cache: [batch][n_kv][scale_stride] fp32.
static size_t scale_bytes(const eif_cuda_kv_t *kv) { return (size_t)kv->batch * kv->n_kv * kv->scale_stride * 4; }

EIF_API eif_status_t eif_cuda_kv_alloc(eif_cuda_ctx_t *ctx, int n_layers, int batch, int max_seq_len,
                                       int n_kv_heads, int head_dim, eif_cuda_dtype_t dtype, eif_cuda_kv_t **out) {
    if (!ctx || !out) return EIF_STATUS_INVALID_ARGUMENT;
    *out = nullptr;
    if (n_layers <= 0 || batch <= 0 || max_seq_len <= 0 || n_kv_heads <= 0 || head_dim <= 0 || head_dim % 8)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_alloc: bad shape");
    if (dtype != EIF_CUDA_F32 && dtype != EIF_CUDA_BF16 && dtype != EIF_CUDA_INT8)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_alloc: dtype must be F32, BF16 or INT8");
    if (dtype == EIF_CUDA_INT8 && head_dim != 64 && head_dim != 128 && head_dim != 256)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "kv_alloc: an INT8 cache needs head_dim 64, 128 or 256");
    DeviceGuard g(ctx);
    eif_cuda_kv_t *kv = new eif_cuda_kv_t();
    kv->ctx = ctx;
    kv->n_layers = n_layers;
    kv->batch = batch;
    kv->max_seq = max_seq_len;
    kv->n_kv = n_kv_heads;
    kv->hd = head_dim;
    kv->dtype = dtype;
    kv->layer_elems = (size_t)batch * max_seq_len * n_kv_heads * head_dim;
    kv->k = (void **)calloc(n_layers, sizeof(void *));
    kv->v = (void **)calloc(n_layers, sizeof(void *));
    kv->tmk = static_cast<CUtensorMap *>(aligned_alloc(64, sizeof(CUtensorMap) * n_layers));
    kv->tmv = static_cast<CUtensorMap *>(aligned_alloc(64, sizeof(CUtensorMap) * n_layers));
    kv->tm_ready = (bool *)calloc(n_layers, sizeof(bool));
    kv->q_norm = (float **)calloc(n_layers, sizeof(float *));
    kv->k_norm = (float **)calloc(n_layers, sizeof(float *));
    if (dtype == EIF_CUDA_INT8) {
        kv->ks = (float **)calloc(n_layers, sizeof(float *));
        kv->vs = (float **)calloc(n_layers, sizeof(float *));
        kv->scale_stride = (max_seq_len + 63) / 64 * 64;
    }
    const size_t bytes = kv->layer_elems * dtype_size(dtype);
    for (int l = 0; l < n_layers; ++l) {
        cudaError_t e = cudaMalloc(&kv->k[l], bytes);
        if (e == cudaSuccess) e = cudaMalloc(&kv->v[l], bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(kv->k[l], 0, bytes, ctx->stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(kv->v[l], 0, bytes, ctx->stream);
        if (e == cudaSuccess && kv->ks) {
            e = cudaMalloc(&kv->ks[l], scale_bytes(kv));
            if (e == cudaSuccess) e = cudaMalloc(&kv->vs[l], scale_bytes(kv));
            if (e == cudaSuccess) e = cudaMemsetAsync(kv->ks[l], 0, scale_bytes(kv), ctx->stream);
            if (e == cudaSuccess) e = cudaMemsetAsync(kv->vs[l], 0, scale_bytes(kv), ctx->stream);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            eif_cuda_kv_free(kv);
            return fail(ctx, EIF_STATUS_OUT_OF_MEMORY, "kv_alloc: %s (layer %d, %zu bytes each)",
                        cudaGetErrorString(e), l, bytes);
        }
    }
    eif_status_t st = wait_stream(ctx);
    if (st != EIF_STATUS_OK) {
        eif_cuda_kv_free(kv);
        return st;
    }
    *out = kv;
    return EIF_STATUS_OK;
}

EIF_API void eif_cuda_kv_free(eif_cuda_kv_t *kv) {
    if (!kv) return;
    {
        DeviceGuard g(kv->ctx);
        cudaStreamSynchronize(kv->ctx->stream);
        for (int l = 0; l < kv->n_layers; ++l) {
            if (kv->k && kv->k[l]) cudaFree(kv->k[l]);
            if (kv->v && kv->v[l]) cudaFree(kv->v[l]);
            if (kv->q_norm && kv->q_norm[l]) cudaFree(kv->q_norm[l]);
            if (kv->ks && kv->ks[l]) cudaFree(kv->ks[l]);
            if (kv->vs && kv->vs[l]) cudaFree(kv->vs[l]);
        }
    }
    free(kv->k);
    free(kv->v);
    free(kv->ks);
    free(kv->vs);
    free(kv->tmk);
    free(kv->tmv);
    free(kv->tm_ready);
    if (kv->rope_cos) {
        DeviceGuard g(kv->ctx);
        cudaFree(kv->rope_cos);
    }
    if (kv->tl_cos) {
        DeviceGuard g(kv->ctx);
        cudaFree(kv->tl_cos);
    }
    free(kv->q_norm);
    free(kv->k_norm);
    delete kv;
}

EIF_API eif_status_t eif_cuda_kv_reset(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    DeviceGuard g(ctx);
    const size_t bytes = kv->layer_elems * dtype_size(kv->dtype);
    for (int l = 0; l < kv->n_layers; ++l) {
        CK(cudaMemsetAsync(kv->k[l], 0, bytes, ctx->stream));
        CK(cudaMemsetAsync(kv->v[l], 0, bytes, ctx->stream));
        if (kv->ks) {  // tinyllm_reset zeroes the scales too (src/eif_tinyllm.c:180-187)
            CK(cudaMemsetAsync(kv->ks[l], 0, scale_bytes(kv), ctx->stream));
            CK(cudaMemsetAsync(kv->vs[l], 0, scale_bytes(kv), ctx->stream));
        }
    }
    return wait_stream(ctx);
}

static eif_status_t kv_rows_check(eif_cuda_ctx_t *ctx, const eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                  int n_rows) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (seq < 0 || seq >= kv->batch) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "seq %d out of range", seq);
    if (row0 < 0 || n_rows < 0 || row0 + n_rows > kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rows [%d, %d) outside [0, %d)", row0, row0 + n_rows,
                    kv->max_seq);
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_kv_upload(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                        int n_rows, const float *k_rows, const float *v_rows) {
    eif_status_t st = kv_rows_check(ctx, kv, layer, seq, row0, n_rows);
    if (st != EIF_STATUS_OK) return st;
    if (!k_rows || !v_rows) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_upload: NULL rows");
    if (n_rows == 0) return EIF_STATUS_OK;
    DeviceGuard g(ctx);
    const size_t kv_dim = (size_t)kv->n_kv * kv->hd;
    const size_t n = (size_t)n_rows * kv_dim;
    const size_t off = ((size_t)seq * kv->max_seq + row0) * kv_dim;
    if (kv->dtype == EIF_CUDA_F32) {
        CK(cudaMemcpyAsync(static_cast<float *>(kv->k[layer]) + off, k_rows, n * 4, cudaMemcpyHostToDevice,
                           ctx->stream));
        CK(cudaMemcpyAsync(static_cast<float *>(kv->v[layer]) + off, v_rows, n * 4, cudaMemcpyHostToDevice,
                           ctx->stream));
    } else {
        st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, 2 * a256(n * 4));
        if (st != EIF_STATUS_OK) return st;
        float *sk = static_cast<float *>(ctx->stage);
        float *sv = reinterpret_cast<float *>(static_cast<char *>(ctx->stage) + a256(n * 4));
        CK(cudaMemcpyAsync(sk, k_rows, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(cudaMemcpyAsync(sv, v_rows, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        if (kv->dtype == EIF_CUDA_INT8) {
            CK(launch_kv_quantize(ctx->stream, static_cast<int8_t *>(kv->k[layer]), static_cast<int8_t *>(kv->v[layer]),
                                  kv->ks[layer], kv->vs[layer], nullptr, seq, row0, sk, sv, n_rows, kv->max_seq,
                                  kv->n_kv, kv->hd, kv->scale_stride, ctx->dev_err));
            ctx->launches += 1;
        } else {
            CK(launch_f32_to_bf16(ctx->stream, sk, static_cast<__nv_bfloat16 *>(kv->k[layer]) + off, n));
            CK(launch_f32_to_bf16(ctx->stream, sv, static_cast<__nv_bfloat16 *>(kv->v[layer]) + off, n));
            ctx->launches += 2;
        }
    }
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_kv_download(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                          int n_rows, float *k_rows, float *v_rows) {
    eif_status_t st = kv_rows_check(ctx, kv, layer, seq, row0, n_rows);
    if (st != EIF_STATUS_OK) return st;
    if (!k_rows || !v_rows) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_download: NULL rows");
    if (n_rows == 0) return EIF_STATUS_OK;
    DeviceGuard g(ctx);
    const size_t kv_dim = (size_t)kv->n_kv * kv->hd;
    const size_t n = (size_t)n_rows * kv_dim;
    const size_t off = ((size_t)seq * kv->max_seq + row0) * kv_dim;
    if (kv->dtype == EIF_CUDA_F32) {
        CK(cudaMemcpyAsync(k_rows, static_cast<float *>(kv->k[layer]) + off, n * 4, cudaMemcpyDeviceToHost,
                           ctx->stream));
        CK(cudaMemcpyAsync(v_rows, static_cast<float *>(kv->v[layer]) + off, n * 4, cudaMemcpyDeviceToHost,
                           ctx->stream));
    } else {
        st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, 2 * a256(n * 4));
        if (st != EIF_STATUS_OK) return st;
        float *sk = static_cast<float *>(ctx->stage);
        float *sv = reinterpret_cast<float *>(static_cast<char *>(ctx->stage) + a256(n * 4));
        if (kv->dtype == EIF_CUDA_INT8) {
            CK(launch_kv_dequantize(ctx->stream, static_cast<int8_t *>(kv->k[layer]), kv->ks[layer], seq, row0, sk,
                                    n_rows, kv->max_seq, kv->n_kv, kv->hd, kv->scale_stride));
            CK(launch_kv_dequantize(ctx->stream, static_cast<int8_t *>(kv->v[layer]), kv->vs[layer], seq, row0, sv,
                                    n_rows, kv->max_seq, kv->n_kv, kv->hd, kv->scale_stride));
        } else {
            CK(launch_bf16_to_f32(ctx->stream, static_cast<__nv_bfloat16 *>(kv->k[layer]) + off, sk, n));
            CK(launch_bf16_to_f32(ctx->stream, static_cast<__nv_bfloat16 *>(kv->v[layer]) + off, sv, n));
        }
        ctx->launches += 2;
        CK(cudaMemcpyAsync(k_rows, sk, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaMemcpyAsync(v_rows, sv, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    }
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_kv_layer_ptrs(const eif_cuda_kv_t *kv, int layer, void **k_dev, void **v_dev) {
    if (!kv || layer < 0 || layer >= kv->n_layers) return EIF_STATUS_INVALID_ARGUMENT;
    if (k_dev) *k_dev = kv->k[layer];
    if (v_dev) *v_dev = kv->v[layer];
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_kv_download_int8(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int seq, int row0,
                                               int n_rows, int8_t *k_codes, int8_t *v_codes, float *k_scale,
                                               float *v_scale) {
    eif_status_t st = kv_rows_check(ctx, kv, layer, seq, row0, n_rows);
    if (st != EIF_STATUS_OK) return st;
    if (kv->dtype != EIF_CUDA_INT8) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_download_int8: not an INT8 cache");
    if (!k_codes || !v_codes || !k_scale || !v_scale)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "kv_download_int8: NULL output");
    if (n_rows == 0) return EIF_STATUS_OK;
    DeviceGuard g(ctx);
    const size_t r0 = (size_t)seq * kv->max_seq + row0;
    const size_t n = (size_t)n_rows * kv->n_kv * kv->hd;
    const size_t off = r0 * kv->n_kv * kv->hd;
    CK(cudaMemcpyAsync(k_codes, static_cast<int8_t *>(kv->k[layer]) + off, n, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaMemcpyAsync(v_codes, static_cast<int8_t *>(kv->v[layer]) + off, n, cudaMemcpyDeviceToHost, ctx->stream));
    // the device keeps scales head-major; the engine's order is [row][kv head]: one strided copy per head
    for (int h = 0; h < kv->n_kv; ++h) {
        const size_t soff = ((size_t)seq * kv->n_kv + h) * kv->scale_stride + row0;
        CK(cudaMemcpy2DAsync(k_scale + h, (size_t)kv->n_kv * 4, kv->ks[layer] + soff, 4, 4, n_rows,
                             cudaMemcpyDeviceToHost, ctx->stream));
        CK(cudaMemcpy2DAsync(v_scale + h, (size_t)kv->n_kv * 4, kv->vs[layer] + soff, 4, 4, n_rows,
                             cudaMemcpyDeviceToHost, ctx->stream));
    }
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_kv_layer_scales(const eif_cuda_kv_t *kv, int layer, float **k_scale_dev,
                                              float **v_scale_dev) {
    if (!kv || layer < 0 || layer >= kv->n_layers || kv->dtype != EIF_CUDA_INT8) return EIF_STATUS_INVALID_ARGUMENT;
    if (k_scale_dev) *k_scale_dev = kv->ks[layer];
    if (v_scale_dev) *v_scale_dev = kv->vs[layer];
    return EIF_STATUS_OK;
}

static eif_status_t kv_append_impl(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const int *pos_dev,
                                   const float *k_dev, const float *v_dev) {
    if (kv->dtype == EIF_CUDA_INT8)
        CK(launch_kv_quantize(ctx->stream, static_cast<int8_t *>(kv->k[layer]), static_cast<int8_t *>(kv->v[layer]),
                              kv->ks[layer], kv->vs[layer], pos_dev, 0, 0, k_dev, v_dev, kv->batch, kv->max_seq,
                              kv->n_kv, kv->hd, kv->scale_stride, ctx->dev_err));
    else
        CK(launch_kv_append(ctx->stream, kv->k[layer], kv->v[layer], kv->dtype, pos_dev, k_dev, v_dev, kv->batch,
                            kv->max_seq, kv->n_kv * kv->hd, ctx->dev_err));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_kv_append_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const int *pos_dev,
                                            const float *k_dev, const float *v_dev) {
    if (!ctx || !kv || kv->ctx != ctx || !pos_dev || !k_dev || !v_dev) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    DeviceGuard g(ctx);
    return kv_append_impl(ctx, kv, layer, pos_dev, k_dev, v_dev);
}

EIF_API eif_status_t eif_cuda_kv_append(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const int *pos,
                                        const float *k, const float *v) {
    if (!ctx || !kv || kv->ctx != ctx || !pos || !k || !v) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    for (int b = 0; b < kv->batch; ++b)
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
    DeviceGuard g(ctx);
    const size_t n = (size_t)kv->batch * kv->n_kv * kv->hd;
    Carver cv;
    const size_t o_k = cv.take(n * 4), o_v = cv.take(n * 4), o_p = cv.take((size_t)kv->batch * 4);
    eif_status_t st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_k, k, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_p, pos, (size_t)kv->batch * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = kv_append_impl(ctx, kv, layer, reinterpret_cast<int *>(s + o_p), reinterpret_cast<float *>(s + o_k),
                        reinterpret_cast<float *>(s + o_v));
    if (st != EIF_STATUS_OK) return st;
    return wait_stream(ctx);
}

// =================================================================================================
// Decode attention
// =================================================================================================

static eif_status_t decode_check(eif_cuda_ctx_t *ctx, const eif_cuda_kv_t *kv, int layer, int n_heads,
                                 eif_cuda_subln_t subln) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_heads <= 0 || n_heads % kv->n_kv)
        return fail(ctx, EIF_STATUS_SHAPE_MISMATCH, "n_heads %d is not a multiple of n_kv_heads %d", n_heads, kv->n_kv);
    if (subln != EIF_CUDA_SUBLN_NONE && subln != EIF_CUDA_SUBLN_RMS && subln != EIF_CUDA_SUBLN_WEIGHT)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "bad subln mode %d", (int)subln);
    return EIF_STATUS_OK;
}

void decode_prepare(eif_cuda_kv_t *kv, int layer, DecodeArgs &a) {
    if (!kv->tm_ready[layer]) {
        kv->tm_ready[layer] = make_kv_tensor_map(&kv->tmk[layer], kv->k[layer], kv) &&
                              make_kv_tensor_map(&kv->tmv[layer], kv->v[layer], kv);
    }
    if (kv->tm_ready[layer]) {
        a.tmk = &kv->tmk[layer];
        a.tmv = &kv->tmv[layer];
    }
    if (kv->dtype == EIF_CUDA_INT8) {
        a.k_scale = kv->ks[layer];
        a.v_scale = kv->vs[layer];
        a.scale_stride = kv->scale_stride;
    }
    a.force_simt = env_flag("BITLLM_DECODE_SIMT");
}

static eif_status_t decode_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, DecodeArgs &a) {
    decode_prepare(kv, layer, a);
    const size_t ws = decode_workspace_bytes(a, ctx->sm_count);
    eif_status_t st = ensure_buffer(ctx, &ctx->ws, &ctx->ws_bytes, ws);
    if (st != EIF_STATUS_OK) return st;
    bool ok = true;
    int nl = 0;
    cudaError_t e = launch_attend_decode(ctx->stream, a, ctx->ws, ctx->ws_bytes, ctx->sm_count, &ok, &nl);
    ctx->launches += nl;
    if (!ok)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "decode attention: head_dim %d / group %d not supported", a.D,
                    a.Hq / a.Hkv);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attend_decode launch");
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_attend_decode_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                const float *q_dev, const int *pos_dev, int max_pos, int n_heads,
                                                float scale, const float *gate_dev, eif_cuda_subln_t subln,
                                                const float *sub_norm_dev, float *out_dev) {
    eif_status_t st = decode_check(ctx, kv, layer, n_heads, subln);
    if (st != EIF_STATUS_OK) return st;
    if (!q_dev || !pos_dev || !out_dev || (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm_dev))
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_decode_dev: NULL pointer");
    if (max_pos < 0 || max_pos >= kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "max_pos %d outside [0, %d)", max_pos, kv->max_seq);
    DeviceGuard g(ctx);
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, q_dev, pos_dev, kv->batch, n_heads, kv->n_kv, kv->hd,
                 kv->max_seq, max_pos + 1, scale, gate_dev, (int)subln, sub_norm_dev, out_dev, ctx->dev_err};
    return decode_run(ctx, kv, layer, a);
}

EIF_API eif_status_t eif_cuda_attend_decode(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                            const int *pos, int n_heads, float scale, const float *gate,
                                            eif_cuda_subln_t subln, const float *sub_norm, float *out) {
    eif_status_t st = decode_check(ctx, kv, layer, n_heads, subln);
    if (st != EIF_STATUS_OK) return st;
    if (!q || !pos || !out || (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm))
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_decode: NULL pointer");
    int max_pos = 0;
    for (int b = 0; b < kv->batch; ++b) {
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
        max_pos = std::max(max_pos, pos[b]);
    }
    DeviceGuard g(ctx);
    const size_t row = (size_t)n_heads * kv->hd;
    const size_t nq = (size_t)kv->batch * row;
    // inputs q, pos, gate, sub_norm (absent ones are empty), packed in one copy when small
    const bool wn = subln == EIF_CUDA_SUBLN_WEIGHT;
    const void *src[4] = {q, pos, gate, sub_norm};
    const size_t bytes[4] = {nq * 4, (size_t)kv->batch * 4, gate ? nq * 4 : 0, wn ? row * 4 : 0};
    size_t off[4], in_total = 0;
    for (int i = 0; i < 4; ++i) {
        off[i] = in_total;
        in_total += a16(bytes[i]);
    }
    const bool small = in_total <= kSmallIo && nq * 4 <= kSmallIo;
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, a256(in_total) + (small ? 0 : nq * 4));
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    if (small) {
        st = send_packed(ctx, s, 4, src, bytes, off);
        if (st != EIF_STATUS_OK) return st;
    } else {
        for (int i = 0; i < 4; ++i)
            if (bytes[i]) CK(cudaMemcpyAsync(s + off[i], src[i], bytes[i], cudaMemcpyHostToDevice, ctx->stream));
    }
    float *dout = small ? small_out(ctx) : reinterpret_cast<float *>(s + a256(in_total));
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, reinterpret_cast<float *>(s + off[0]),
                 reinterpret_cast<int *>(s + off[1]), kv->batch, n_heads, kv->n_kv, kv->hd, kv->max_seq, max_pos + 1,
                 scale, gate ? reinterpret_cast<float *>(s + off[2]) : nullptr, (int)subln,
                 wn ? reinterpret_cast<float *>(s + off[3]) : nullptr, dout, ctx->dev_err};
    st = decode_run(ctx, kv, layer, a);
    if (st != EIF_STATUS_OK) return st;
    if (small) return finish_small(ctx, out, nq * 4);
    CK(cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_attend_decode_plan(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_heads,
                                                 int max_pos, int noalloc, int *n_chunks, int *chunk_keys,
                                                 size_t *scratch_bytes) {
    eif_status_t st = decode_check(ctx, kv, layer, n_heads, EIF_CUDA_SUBLN_NONE);
    if (st != EIF_STATUS_OK) return st;
    if (!n_chunks || !chunk_keys || !scratch_bytes)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_decode_plan: NULL pointer");
    if (max_pos < 0 || max_pos >= kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "max_pos %d outside [0, %d)", max_pos, kv->max_seq);
    DeviceGuard g(ctx);
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, nullptr, nullptr, kv->batch, n_heads, kv->n_kv, kv->hd,
                 kv->max_seq, max_pos + 1, 1.0f, nullptr, 0, nullptr, nullptr, ctx->dev_err};
    if (noalloc) a.max_ws_bytes = noalloc_scratch_capacity();
    decode_prepare(kv, layer, a);
    decode_plan(a, ctx->sm_count, n_chunks, chunk_keys, scratch_bytes);
    return EIF_STATUS_OK;
}

// =================================================================================================
// Causal prefill attention
// =================================================================================================

static eif_status_t prefill_check(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_tok, int start_pos,
                                  int n_heads) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_heads <= 0 || n_heads % kv->n_kv)
        return fail(ctx, EIF_STATUS_SHAPE_MISMATCH, "n_heads %d is not a multiple of n_kv_heads %d", n_heads, kv->n_kv);
    if (n_tok < 1 || start_pos < 0 || start_pos + n_tok > kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rows [%d, %d) outside the cache [0, %d)", start_pos,
                    start_pos + n_tok, kv->max_seq);
    if (kv->hd != 64 && kv->hd != 128 && kv->hd != 256)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "prefill attention: head_dim %d (64, 128 or 256)", kv->hd);
    if ((size_t)kv->batch * n_tok * kv->n_kv > 0x3fffffffull)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "too many rows");
    return EIF_STATUS_OK;
}

// bf16 caches run the causal prefill on the tensor-core kernels (bf16 q / out); fp32 and INT8 caches run every
// token of the chunk as one decode row at its own position on the decode kernels, in fp32 arithmetic over the
// cache's own values (fp32 q / out) -- the reference's per-token loop (src/eif_tinyllm.c:1158-1268,
// src/eif_qwen35.c:1122-1133), with the split-K work spread over (token, kv head, key chunk) items.
static bool prefill_by_rows(const eif_cuda_kv_t *kv) { return kv->dtype != EIF_CUDA_BF16; }

static eif_status_t prefill_rows_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                     int n_tok, int start_pos, int n_heads, float scale, const float *gate_dev,
                                     eif_cuda_subln_t subln, const float *sub_norm_dev, float *out_dev) {
    const int rows = kv->batch * n_tok;
    eif_status_t st = ensure_buffer(ctx, &ctx->rowbuf, &ctx->rowbuf_bytes, 2 * a256((size_t)rows * 4));
    if (st != EIF_STATUS_OK) return st;
    int *row_seq = static_cast<int *>(ctx->rowbuf);
    int *pos = reinterpret_cast<int *>(static_cast<char *>(ctx->rowbuf) + a256((size_t)rows * 4));
    CK(launch_prefill_rows(ctx->stream, row_seq, pos, kv->batch, n_tok, start_pos));
    ctx->launches += 1;
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, q_dev, pos, rows, n_heads, kv->n_kv, kv->hd, kv->max_seq,
                 start_pos + n_tok, scale, gate_dev, (int)subln, sub_norm_dev, out_dev, ctx->dev_err};
    a.row_seq = row_seq;
    return decode_run(ctx, kv, layer, a);
}

// TMA descriptor of the queries [B*n_tok][Hq][hd] bf16: boxes of 64 dims x 1 head x 128 tokens.
static bool make_q_tensor_map(CUtensorMap *map, const void *q, int rows, int Hq, int hd) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)Hq, (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)Hq * hd * 2};
    const cuuint32_t box[3] = {64, 1, 128};
    const cuuint32_t es[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(q), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// out_f32 set: the attention goes there as fp32 (out_dev unused), else as bf16 to out_dev.
static eif_status_t prefill_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const void *q_dev, int n_tok,
                                int start_pos, int n_heads, float scale, void *out_dev, float *out_f32 = nullptr) {
    if ((reinterpret_cast<uintptr_t>(q_dev) | reinterpret_cast<uintptr_t>(out_dev) |
         reinterpret_cast<uintptr_t>(out_f32)) & 15)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "prefill: q and out must be 16-byte aligned");
    DecodeArgs probe{};
    decode_prepare(kv, layer, probe);  // makes the layer's K / V tensor maps
    if (!probe.tmk || !probe.tmv) return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "prefill: no TMA descriptors");
    alignas(64) CUtensorMap tq;
    if (!make_q_tensor_map(&tq, q_dev, kv->batch * n_tok, n_heads, kv->hd))
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "prefill: cannot describe q for TMA");
    CK(launch_attend_prefill_tc(ctx->stream, tq, *probe.tmk, *probe.tmv, kv->batch, n_tok, start_pos, n_heads,
                                kv->n_kv, kv->max_seq, kv->hd, scale, static_cast<__nv_bfloat16 *>(out_dev), out_f32,
                                ctx->dev_err));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_attend_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                 const void *q_dev, int n_tok, int start_pos, int n_heads,
                                                 float scale, void *out_dev) {
    eif_status_t st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    if (!q_dev || !out_dev) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_prefill_dev: NULL pointer");
    DeviceGuard g(ctx);
    if (prefill_by_rows(kv))
        return prefill_rows_run(ctx, kv, layer, static_cast<const float *>(q_dev), n_tok, start_pos, n_heads, scale,
                                nullptr, EIF_CUDA_SUBLN_NONE, nullptr, static_cast<float *>(out_dev));
    return prefill_run(ctx, kv, layer, q_dev, n_tok, start_pos, n_heads, scale, out_dev);
}

EIF_API eif_status_t eif_cuda_attend_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                             int n_tok, int start_pos, int n_heads, float scale, float *out) {
    eif_status_t st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    if (!q || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_prefill: NULL pointer");
    DeviceGuard g(ctx);
    const size_t n = (size_t)kv->batch * n_tok * n_heads * kv->hd;
    if (prefill_by_rows(kv)) {
        Carver cr;
        const size_t o_q = cr.take(n * 4), o_o = cr.take(n * 4);
        st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cr.off);
        if (st != EIF_STATUS_OK) return st;
        char *s = static_cast<char *>(ctx->stage);
        CK(cudaMemcpyAsync(s + o_q, q, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        st = prefill_rows_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_q), n_tok, start_pos, n_heads, scale,
                              nullptr, EIF_CUDA_SUBLN_NONE, nullptr, reinterpret_cast<float *>(s + o_o));
        if (st != EIF_STATUS_OK) return st;
        CK(cudaMemcpyAsync(out, s + o_o, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
        return wait_stream(ctx);
    }
    Carver cv;
    const size_t o_f = cv.take(n * 4), o_q = cv.take(n * 2), o_o = cv.take(n * 2);
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_f, q, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(launch_f32_to_bf16(ctx->stream, reinterpret_cast<float *>(s + o_f), reinterpret_cast<__nv_bfloat16 *>(s + o_q), n));
    ctx->launches += 1;
    st = prefill_run(ctx, kv, layer, s + o_q, n_tok, start_pos, n_heads, scale, s + o_o);
    if (st != EIF_STATUS_OK) return st;
    CK(launch_bf16_to_f32(ctx->stream, reinterpret_cast<__nv_bfloat16 *>(s + o_o), reinterpret_cast<float *>(s + o_f), n));
    ctx->launches += 1;
    CK(cudaMemcpyAsync(out, s + o_f, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// Gated prefill: the raw attention goes to the context scratch in fp32, then the row epilogue writes
// SubLN(o * sigmoid(gate)) as fp32.
static eif_status_t prefill_gated_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const void *q_dev, int n_tok,
                                      int start_pos, int n_heads, float scale, const float *gate_dev,
                                      eif_cuda_subln_t subln, const float *sub_norm_dev, float *out_dev) {
    const int dim = n_heads * kv->hd;
    const size_t n = (size_t)kv->batch * n_tok * dim;
    eif_status_t st = ensure_buffer(ctx, &ctx->ws, &ctx->ws_bytes, n * 4);
    if (st != EIF_STATUS_OK) return st;
    float *raw = static_cast<float *>(ctx->ws);
    st = prefill_run(ctx, kv, layer, q_dev, n_tok, start_pos, n_heads, scale, nullptr, raw);
    if (st != EIF_STATUS_OK) return st;
    CK(launch_gate_subln(ctx->stream, raw, gate_dev, kv->batch * n_tok, dim, (int)subln, sub_norm_dev, out_dev));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

static eif_status_t subln_check(eif_cuda_ctx_t *ctx, eif_cuda_subln_t subln, const void *sub_norm) {
    if (subln != EIF_CUDA_SUBLN_NONE && subln != EIF_CUDA_SUBLN_RMS && subln != EIF_CUDA_SUBLN_WEIGHT)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "unknown SubLN mode %d", (int)subln);
    if (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "SubLN with weights needs sub_norm");
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_attend_prefill_gated_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                       const void *q_dev, int n_tok, int start_pos, int n_heads,
                                                       float scale, const float *gate_dev, eif_cuda_subln_t subln,
                                                       const float *sub_norm_dev, float *out_dev) {
    eif_status_t st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    st = subln_check(ctx, subln, sub_norm_dev);
    if (st != EIF_STATUS_OK) return st;
    if (!q_dev || !out_dev) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_prefill_gated_dev: NULL pointer");
    DeviceGuard g(ctx);
    if (prefill_by_rows(kv))
        return prefill_rows_run(ctx, kv, layer, static_cast<const float *>(q_dev), n_tok, start_pos, n_heads, scale,
                                gate_dev, subln, sub_norm_dev, out_dev);
    return prefill_gated_run(ctx, kv, layer, q_dev, n_tok, start_pos, n_heads, scale, gate_dev, subln, sub_norm_dev,
                             out_dev);
}

EIF_API eif_status_t eif_cuda_attend_prefill_gated(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                                   int n_tok, int start_pos, int n_heads, float scale,
                                                   const float *gate, eif_cuda_subln_t subln, const float *sub_norm,
                                                   float *out) {
    eif_status_t st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    st = subln_check(ctx, subln, sub_norm);
    if (st != EIF_STATUS_OK) return st;
    if (!q || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_prefill_gated: NULL pointer");
    DeviceGuard g(ctx);
    const size_t row = (size_t)n_heads * kv->hd, n = (size_t)kv->batch * n_tok * row;
    const bool rows = prefill_by_rows(kv);  // fp32 q on the decode kernels, else bf16 q on the prefill kernels
    Carver cv;
    const size_t o_f = cv.take(n * 4), o_q = cv.take(rows ? n * 4 : n * 2), o_g = gate ? cv.take(n * 4) : 0,
                 o_n = subln == EIF_CUDA_SUBLN_WEIGHT ? cv.take(row * 4) : 0;
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    float *f = reinterpret_cast<float *>(s + o_f);
    if (rows) {
        CK(cudaMemcpyAsync(s + o_q, q, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    } else {
        CK(cudaMemcpyAsync(f, q, n * 4, cudaMemcpyHostToDevice, ctx->stream));
        CK(launch_f32_to_bf16(ctx->stream, f, reinterpret_cast<__nv_bfloat16 *>(s + o_q), n));
        ctx->launches += 1;
    }
    if (gate) CK(cudaMemcpyAsync(s + o_g, gate, n * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (subln == EIF_CUDA_SUBLN_WEIGHT) CK(cudaMemcpyAsync(s + o_n, sub_norm, row * 4, cudaMemcpyHostToDevice, ctx->stream));
    const float *gd = gate ? reinterpret_cast<float *>(s + o_g) : nullptr;
    const float *nd = subln == EIF_CUDA_SUBLN_WEIGHT ? reinterpret_cast<float *>(s + o_n) : nullptr;
    if (rows)
        st = prefill_rows_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_q), n_tok, start_pos, n_heads, scale, gd,
                              subln, nd, f);
    else
        st = prefill_gated_run(ctx, kv, layer, s + o_q, n_tok, start_pos, n_heads, scale, gd, subln, nd, f);
    if (st != EIF_STATUS_OK) return st;
    CK(cudaMemcpyAsync(out, f, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// DeltaNet state
// =================================================================================================

EIF_API eif_status_t eif_cuda_delta_alloc(eif_cuda_ctx_t *ctx, int n_layers, int batch, int n_heads, int d_k,
                                          int d_v, int conv_k, eif_cuda_delta_t **out) {
    if (!ctx || !out) return EIF_STATUS_INVALID_ARGUMENT;
    *out = nullptr;
    if (n_layers <= 0 || batch <= 0 || n_heads <= 0 || d_k <= 0 || d_v <= 0 || conv_k < 0 || d_k % 4 || d_v % 4)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "delta_alloc: bad shape");
    DeviceGuard g(ctx);
    eif_cuda_delta_t *st = new eif_cuda_delta_t();
    st->ctx = ctx;
    st->n_layers = n_layers;
    st->batch = batch;
    st->H = n_heads;
    st->dk = d_k;
    st->dv = d_v;
    st->conv_k = conv_k;
    st->conv_dim = 2 * n_heads * d_k + n_heads * d_v;
    st->S = (float **)calloc(n_layers, sizeof(float *));
    st->conv = (float **)calloc(n_layers, sizeof(float *));
    st->weights = (float **)calloc(n_layers, sizeof(float *));
    const size_t s_bytes = (size_t)batch * n_heads * d_k * d_v * 4;
    const size_t c_bytes = (size_t)batch * st->conv_dim * conv_k * 4;
    for (int l = 0; l < n_layers; ++l) {
        cudaError_t e = cudaMalloc(&st->S[l], s_bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(st->S[l], 0, s_bytes, ctx->stream);
        if (e == cudaSuccess && c_bytes) e = cudaMalloc(&st->conv[l], c_bytes);
        if (e == cudaSuccess && c_bytes) e = cudaMemsetAsync(st->conv[l], 0, c_bytes, ctx->stream);
        if (e != cudaSuccess) {
            cudaGetLastError();
            eif_cuda_delta_free(st);
            return fail(ctx, EIF_STATUS_OUT_OF_MEMORY, "delta_alloc: %s (layer %d)", cudaGetErrorString(e), l);
        }
    }
    eif_status_t rs = wait_stream(ctx);
    if (rs != EIF_STATUS_OK) {
        eif_cuda_delta_free(st);
        return rs;
    }
    *out = st;
    return EIF_STATUS_OK;
}

EIF_API void eif_cuda_delta_free(eif_cuda_delta_t *st) {
    if (!st) return;
    {
        DeviceGuard g(st->ctx);
        cudaStreamSynchronize(st->ctx->stream);
        for (int l = 0; l < st->n_layers; ++l) {
            if (st->S && st->S[l]) cudaFree(st->S[l]);
            if (st->conv && st->conv[l]) cudaFree(st->conv[l]);
            if (st->weights && st->weights[l]) cudaFree(st->weights[l]);
        }
    }
    free(st->S);
    free(st->conv);
    free(st->weights);
    delete st;
}

EIF_API eif_status_t eif_cuda_delta_reset(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st) {
    if (!ctx || !st || st->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    DeviceGuard g(ctx);
    const size_t s_bytes = (size_t)st->batch * st->H * st->dk * st->dv * 4;
    const size_t c_bytes = (size_t)st->batch * st->conv_dim * st->conv_k * 4;
    for (int l = 0; l < st->n_layers; ++l) {
        CK(cudaMemsetAsync(st->S[l], 0, s_bytes, ctx->stream));
        if (c_bytes) CK(cudaMemsetAsync(st->conv[l], 0, c_bytes, ctx->stream));
    }
    return wait_stream(ctx);
}

static eif_status_t delta_seq_check(eif_cuda_ctx_t *ctx, const eif_cuda_delta_t *st, int layer, int seq) {
    if (!ctx || !st || st->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (seq < 0 || seq >= st->batch) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "seq %d out of range", seq);
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_delta_upload(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int seq,
                                           const float *S, const float *conv_state) {
    eif_status_t rs = delta_seq_check(ctx, st, layer, seq);
    if (rs != EIF_STATUS_OK) return rs;
    if (conv_state && !st->conv_k) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "state has no conv window");
    DeviceGuard g(ctx);
    const size_t s_n = (size_t)st->H * st->dk * st->dv, c_n = (size_t)st->conv_dim * st->conv_k;
    if (S) CK(cudaMemcpyAsync(st->S[layer] + seq * s_n, S, s_n * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (conv_state)
        CK(cudaMemcpyAsync(st->conv[layer] + seq * c_n, conv_state, c_n * 4, cudaMemcpyHostToDevice, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_delta_download(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int seq,
                                             float *S, float *conv_state) {
    eif_status_t rs = delta_seq_check(ctx, st, layer, seq);
    if (rs != EIF_STATUS_OK) return rs;
    if (conv_state && !st->conv_k) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "state has no conv window");
    DeviceGuard g(ctx);
    const size_t s_n = (size_t)st->H * st->dk * st->dv, c_n = (size_t)st->conv_dim * st->conv_k;
    if (S) CK(cudaMemcpyAsync(S, st->S[layer] + seq * s_n, s_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    if (conv_state)
        CK(cudaMemcpyAsync(conv_state, st->conv[layer] + seq * c_n, c_n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_delta_layer_ptrs(const eif_cuda_delta_t *st, int layer, float **S_dev,
                                               float **conv_dev) {
    if (!st || layer < 0 || layer >= st->n_layers) return EIF_STATUS_INVALID_ARGUMENT;
    if (S_dev) *S_dev = st->S[layer];
    if (conv_dev) *conv_dev = st->conv[layer];
    return EIF_STATUS_OK;
}

static eif_status_t rule_run(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q, const float *k,
                             const float *v, const float *beta, const float *g, float q_scale, float *o) {
    bool ok = true;
    cudaError_t e = launch_delta_rule(ctx->stream, st->S[layer], q, k, v, beta, g, q_scale, o, st->batch, st->H,
                                      st->dk, st->dv, ctx->sm_count, &ok);
    if (!ok)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "deltanet_step: d_k %d / d_v %d not supported", st->dk, st->dv);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "deltanet_step launch");
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_deltanet_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                const float *q_dev, const float *k_dev, const float *v_dev,
                                                const float *beta_dev, const float *g_dev, float q_scale,
                                                float *o_dev) {
    if (!ctx || !st || st->ctx != ctx || !q_dev || !k_dev || !v_dev || !beta_dev || !g_dev || !o_dev)
        return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    DeviceGuard gd(ctx);
    return rule_run(ctx, st, layer, q_dev, k_dev, v_dev, beta_dev, g_dev, q_scale, o_dev);
}

EIF_API eif_status_t eif_cuda_deltanet_step(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q,
                                            const float *k, const float *v, const float *beta, const float *g,
                                            float q_scale, float *o) {
    if (!ctx || !st || st->ctx != ctx || !q || !k || !v || !beta || !g || !o) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    DeviceGuard gd(ctx);
    const size_t nqk = (size_t)st->batch * st->H * st->dk, nv = (size_t)st->batch * st->H * st->dv;
    const size_t nh = (size_t)st->batch * st->H;
    Carver cv;
    const size_t o_q = cv.take(nqk * 4), o_k = cv.take(nqk * 4), o_v = cv.take(nv * 4), o_o = cv.take(nv * 4);
    const size_t o_b = cv.take(nh * 4), o_g = cv.take(nh * 4);
    eif_status_t rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_q, q, nqk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nqk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nv * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_b, beta, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_g, g, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = rule_run(ctx, st, layer, reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_k),
                  reinterpret_cast<float *>(s + o_v), reinterpret_cast<float *>(s + o_b),
                  reinterpret_cast<float *>(s + o_g), q_scale, reinterpret_cast<float *>(s + o_o));
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(o, s + o_o, nv * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// Whole DeltaNet mixer (deltanet_core)
// =================================================================================================

EIF_API eif_status_t eif_cuda_delta_set_weights(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                const float *conv_w, const float *dt_bias, const float *A_log,
                                                const float *norm_w) {
    if (!ctx || !st || st->ctx != ctx || !conv_w || !dt_bias || !A_log || !norm_w) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (st->conv_k < 1) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "state was allocated without a conv window");
    DeviceGuard g(ctx);
    const size_t ncw = (size_t)st->conv_dim * st->conv_k, n = ncw + 2 * st->H + st->dv;
    if (!st->weights[layer]) CK(cudaMalloc(&st->weights[layer], n * 4));
    // a_exp = expf(A_log) on the host, exactly as the engine's loader does (src/eif_qwen35.c:1362)
    float *a_exp = (float *)malloc(sizeof(float) * st->H);
    for (int h = 0; h < st->H; ++h) a_exp[h] = expf(A_log[h]);
    float *w = st->weights[layer];
    cudaError_t e = cudaMemcpyAsync(w, conv_w, ncw * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w + ncw, dt_bias, st->H * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w + ncw + st->H, a_exp, st->H * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w + ncw + 2 * st->H, norm_w, st->dv * 4, cudaMemcpyHostToDevice, ctx->stream);
    eif_status_t rs = e == cudaSuccess ? wait_stream(ctx) : cuda_fail(ctx, e, "delta_set_weights");
    free(a_exp);
    return rs;
}

static eif_status_t core_check(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer) {
    if (!ctx || !st || st->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (!st->weights[layer]) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "layer %d has no weights (delta_set_weights)", layer);
    return EIF_STATUS_OK;
}

static eif_status_t core_run(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv, const float *z,
                             const float *b_raw, const float *a_raw, float *out) {
    const size_t ncw = (size_t)st->conv_dim * st->conv_k;
    const float *w = st->weights[layer];
    DeltaCoreArgs a{st->S[layer], st->conv[layer], qkv, z, b_raw, a_raw, w, w + ncw, w + ncw + st->H,
                    w + ncw + 2 * st->H, out, st->batch, st->H, st->dk, st->dv, st->conv_k, ctx->dev_err};
    // every library kernel launched as a programmatic dependent triggers its own dependents only after its
    // grid-dependency wait, so when this kernel starts early only the launch just before it can still be running:
    // the state may be read ahead of the wait unless that launch wrote it
    a.prefetch = !(ctx->last_state == st->S[layer] && ctx->last_state_launches == ctx->launches);
    bool ok = true;
    cudaError_t e = launch_deltanet_core(ctx->stream, a, &ok);
    if (!ok) return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "deltanet_core: d_k %d / d_v %d not supported", st->dk, st->dv);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "deltanet_core launch");
    ctx->launches += 1;
    ctx->last_state = st->S[layer];
    ctx->last_state_launches = ctx->launches;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_deltanet_core_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                const float *qkv_dev, const float *z_dev, const float *b_dev,
                                                const float *a_dev, float *out_dev) {
    eif_status_t rs = core_check(ctx, st, layer);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qkv_dev || !z_dev || !b_dev || !a_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_core_dev: NULL pointer");
    DeviceGuard g(ctx);
    return core_run(ctx, st, layer, qkv_dev, z_dev, b_dev, a_dev, out_dev);
}

EIF_API eif_status_t eif_cuda_deltanet_core(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv,
                                            const float *z, const float *b_raw, const float *a_raw, float *out) {
    eif_status_t rs = core_check(ctx, st, layer);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qkv || !z || !b_raw || !a_raw || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_core: NULL pointer");
    DeviceGuard g(ctx);
    const size_t B = st->batch, nq = B * st->conv_dim, nz = B * st->H * st->dv, nh = B * st->H;
    Carver cv;
    const size_t o_q = cv.take(nq * 4), o_z = cv.take(nz * 4), o_b = cv.take(nh * 4), o_a = cv.take(nh * 4),
                 o_o = cv.take(nz * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_q, qkv, nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_z, z, nz * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_b, b_raw, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_a, a_raw, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = core_run(ctx, st, layer, reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_z),
                  reinterpret_cast<float *>(s + o_b), reinterpret_cast<float *>(s + o_a),
                  reinterpret_cast<float *>(s + o_o));
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(out, s + o_o, nz * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// Chunked DeltaNet prefill
// =================================================================================================

// TMA descriptor of a token-major bf16 array [rows][H][d] as (d, H, rows), boxes of 64 x 1 x 64.
static bool make_tok_tensor_map(CUtensorMap *map, const void *base, int rows, int H, int d) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)H, (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)H * d * 2};
    const cuuint32_t box[3] = {64, 1, 64};
    const cuuint32_t es[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static eif_status_t chunked_check(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int n_tok) {
    if (!ctx || !st || st->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= st->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_tok < 1) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "n_tok %d", n_tok);
    if (!deltanet_chunked_supported(st->dk, st->dv))
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "chunked prefill: d_k %d / d_v %d not supported", st->dk, st->dv);
    if ((size_t)st->batch * n_tok > 0x7fffffffull) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "too many rows");
    return EIF_STATUS_OK;
}

// The chunked rule with its per-chunk scratch at t_ws (deltanet_chunked_workspace bytes): o as bf16, or as
// fp32 to o_f32 when that is set.
static eif_status_t chunked_launch(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const void *q, const void *k,
                                   const void *v, const float *beta, const float *g, int n_tok, float q_scale, void *o,
                                   float *o_f32, void *t_ws) {
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(o_f32)) & 15)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "chunked prefill: q, k, v, o must be 16-byte aligned");
    alignas(64) CUtensorMap tq, tk, tv, tt;
    const int rows = st->batch * n_tok;
    const int t_rows = (int)(deltanet_chunked_tmat_bytes(st->batch, n_tok, st->H) / 128);  // 64 bf16 per row
    if (!make_tok_tensor_map(&tq, q, rows, st->H, st->dk) || !make_tok_tensor_map(&tk, k, rows, st->H, st->dk) ||
        !make_tok_tensor_map(&tv, v, rows, st->H, st->dv) || !make_tok_tensor_map(&tt, t_ws, t_rows, 1, 64))
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "chunked prefill: cannot describe q / k / v for TMA");
    int nl = 0;
    const cudaError_t e = launch_deltanet_chunked(ctx->stream, tq, tk, tv, tt, t_ws, beta, g,
                                                  static_cast<__nv_bfloat16 *>(o), o_f32, st->S[layer], st->batch,
                                                  n_tok, st->H, st->dv, q_scale, ctx->dev_err, &nl);
    ctx->launches += nl;
    if (e != cudaSuccess) return cuda_fail(ctx, e, "deltanet_chunked launch");
    return EIF_STATUS_OK;
}

static eif_status_t chunked_run(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const void *q, const void *k,
                                const void *v, const float *beta, const float *g, int n_tok, float q_scale, void *o) {
    // scratch: per chunk T diag(-b e^G) and T diag(b) with T = (I + A)^-1 (bf16 [batch][H][chunk][128][64]),
    // then the cumulative log decays (fp32 [batch][H][chunk][64])
    eif_status_t rs = ensure_buffer(ctx, &ctx->ws, &ctx->ws_bytes, deltanet_chunked_workspace(st->batch, n_tok, st->H));
    if (rs != EIF_STATUS_OK) return rs;
    return chunked_launch(ctx, st, layer, q, k, v, beta, g, n_tok, q_scale, o, nullptr, ctx->ws);
}

// The whole deltanet_core over a prefill chunk: pre ops -> chunked rule (fp32 output) -> gated RMSNorm.
static eif_status_t prefill_core_run(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *qkv,
                                     const float *z, const float *b_raw, const float *a_raw, int n_tok, float *out) {
    const size_t tok = (size_t)st->batch * n_tok * st->H;
    Carver cv;
    const size_t o_q = cv.take(tok * st->dk * 2), o_k = cv.take(tok * st->dk * 2), o_v = cv.take(tok * st->dv * 2),
                 o_b = cv.take(tok * 4), o_g = cv.take(tok * 4), o_o = cv.take(tok * st->dv * 4),
                 o_t = cv.take(deltanet_chunked_workspace(st->batch, n_tok, st->H));
    eif_status_t rs = ensure_buffer(ctx, &ctx->ws, &ctx->ws_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->ws);
    const size_t ncw = (size_t)st->conv_dim * st->conv_k;
    const float *w = st->weights[layer];
    DeltaPrefillArgs a{qkv, z, b_raw, a_raw, st->conv[layer], w, w + ncw, w + ncw + st->H, w + ncw + 2 * st->H,
                       reinterpret_cast<__nv_bfloat16 *>(s + o_q), reinterpret_cast<__nv_bfloat16 *>(s + o_k),
                       reinterpret_cast<__nv_bfloat16 *>(s + o_v), reinterpret_cast<float *>(s + o_b),
                       reinterpret_cast<float *>(s + o_g), reinterpret_cast<float *>(s + o_o), out, st->batch, n_tok,
                       st->H, st->dk, st->dv, st->conv_k};
    CK(launch_deltanet_prefill_pre(ctx->stream, a));
    ctx->launches += 2;
    rs = chunked_launch(ctx, st, layer, a.q, a.k, a.v, a.beta, a.g, n_tok, 1.0f, nullptr,
                        reinterpret_cast<float *>(s + o_o), s + o_t);
    if (rs != EIF_STATUS_OK) return rs;
    CK(launch_deltanet_prefill_post(ctx->stream, a));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

static eif_status_t prefill_core_check(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, int n_tok) {
    eif_status_t rs = core_check(ctx, st, layer);
    if (rs != EIF_STATUS_OK) return rs;
    rs = chunked_check(ctx, st, layer, n_tok);
    if (rs != EIF_STATUS_OK) return rs;
    if (st->conv_k < 1) return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "deltanet prefill core: the state has no conv window");
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_deltanet_prefill_core_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                        const float *qkv_dev, const float *z_dev, const float *b_dev,
                                                        const float *a_dev, int n_tok, float *out_dev) {
    eif_status_t rs = prefill_core_check(ctx, st, layer, n_tok);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qkv_dev || !z_dev || !b_dev || !a_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_prefill_core_dev: NULL pointer");
    DeviceGuard gd(ctx);
    return prefill_core_run(ctx, st, layer, qkv_dev, z_dev, b_dev, a_dev, n_tok, out_dev);
}

EIF_API eif_status_t eif_cuda_deltanet_prefill_core(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                    const float *qkv, const float *z, const float *b_raw,
                                                    const float *a_raw, int n_tok, float *out) {
    eif_status_t rs = prefill_core_check(ctx, st, layer, n_tok);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qkv || !z || !b_raw || !a_raw || !out)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_prefill_core: NULL pointer");
    DeviceGuard gd(ctx);
    const size_t tok = (size_t)st->batch * n_tok, nq = tok * st->conv_dim, nz = tok * st->H * st->dv,
                 nh = tok * st->H;
    Carver cv;
    const size_t o_q = cv.take(nq * 4), o_z = cv.take(nz * 4), o_b = cv.take(nh * 4), o_a = cv.take(nh * 4),
                 o_o = cv.take(nz * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_q, qkv, nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_z, z, nz * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_b, b_raw, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_a, a_raw, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = prefill_core_run(ctx, st, layer, reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_z),
                          reinterpret_cast<float *>(s + o_b), reinterpret_cast<float *>(s + o_a), n_tok,
                          reinterpret_cast<float *>(s + o_o));
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(out, s + o_o, nz * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_deltanet_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer,
                                                   const void *q_dev, const void *k_dev, const void *v_dev,
                                                   const float *beta_dev, const float *g_dev, int n_tok, float q_scale,
                                                   void *o_dev) {
    eif_status_t rs = chunked_check(ctx, st, layer, n_tok);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q_dev || !k_dev || !v_dev || !beta_dev || !g_dev || !o_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_prefill_dev: NULL pointer");
    DeviceGuard gd(ctx);
    return chunked_run(ctx, st, layer, q_dev, k_dev, v_dev, beta_dev, g_dev, n_tok, q_scale, o_dev);
}

EIF_API eif_status_t eif_cuda_deltanet_prefill(eif_cuda_ctx_t *ctx, eif_cuda_delta_t *st, int layer, const float *q,
                                               const float *k, const float *v, const float *beta, const float *g,
                                               int n_tok, float q_scale, float *o) {
    eif_status_t rs = chunked_check(ctx, st, layer, n_tok);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q || !k || !v || !beta || !g || !o) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "deltanet_prefill: NULL pointer");
    DeviceGuard gd(ctx);
    const size_t rows = (size_t)st->batch * n_tok, nqk = rows * st->H * st->dk, nv = rows * st->H * st->dv,
                 nh = rows * st->H;
    Carver cv;
    const size_t o_f = cv.take(std::max(nqk, nv) * 4), o_q = cv.take(nqk * 2), o_k = cv.take(nqk * 2),
                 o_v = cv.take(nv * 2), o_o = cv.take(nv * 2), o_b = cv.take(nh * 4), o_g = cv.take(nh * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    float *f = reinterpret_cast<float *>(s + o_f);
    CK(cudaMemcpyAsync(f, q, nqk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(launch_f32_to_bf16(ctx->stream, f, reinterpret_cast<__nv_bfloat16 *>(s + o_q), nqk));
    CK(cudaMemcpyAsync(f, k, nqk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(launch_f32_to_bf16(ctx->stream, f, reinterpret_cast<__nv_bfloat16 *>(s + o_k), nqk));
    CK(cudaMemcpyAsync(f, v, nv * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(launch_f32_to_bf16(ctx->stream, f, reinterpret_cast<__nv_bfloat16 *>(s + o_v), nv));
    CK(cudaMemcpyAsync(s + o_b, beta, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_g, g, nh * 4, cudaMemcpyHostToDevice, ctx->stream));
    ctx->launches += 3;
    rs = chunked_run(ctx, st, layer, s + o_q, s + o_k, s + o_v, reinterpret_cast<float *>(s + o_b),
                     reinterpret_cast<float *>(s + o_g), n_tok, q_scale, s + o_o);
    if (rs != EIF_STATUS_OK) return rs;
    CK(launch_bf16_to_f32(ctx->stream, reinterpret_cast<__nv_bfloat16 *>(s + o_o), f, nv));
    ctx->launches += 1;
    CK(cudaMemcpyAsync(o, f, nv * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// tinyllm RoPE + cache write
// =================================================================================================

EIF_API eif_status_t eif_cuda_kv_set_rope(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, float theta, int interleaved) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (!(theta > 0.f)) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rope theta %g", (double)theta);
    if (kv->hd % 2 || kv->hd > 256)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "rope: head_dim %d (even, <= 256)", kv->hd);
    DeviceGuard g(ctx);
    const int half = kv->hd / 2;
    const size_t n = (size_t)kv->max_seq * half;
    float *hc = (float *)malloc(2 * n * sizeof(float));
    if (!hc) return fail(ctx, EIF_STATUS_OUT_OF_MEMORY, "rope table");
    // the reference's per-position table (src/eif_tinyllm.c:399-404), for every position of the cache.  Its
    // source reads freq = 1.0f / powf(theta, e); its build (-ffast-math, CMakeLists.txt:19) folds that into
    // powf(theta, -e), which rounds differently in the last bit for some j, so the folded form is computed
    // here and the tables equal the compiled reference's bit for bit.
    for (int j = 0; j < half; ++j) {
        const float freq = powf(theta, -((float)(2 * j) / (float)kv->hd));
        for (int pos = 0; pos < kv->max_seq; ++pos) {
            const float val = (float)pos * freq;
            hc[(size_t)pos * half + j] = cosf(val);
            hc[n + (size_t)pos * half + j] = sinf(val);
        }
    }
    cudaError_t e = cudaSuccess;
    if (!kv->tl_cos) {
        float *d = nullptr;
        e = cudaMalloc(&d, 2 * n * sizeof(float));
        if (e == cudaSuccess) {
            kv->tl_cos = d;
            kv->tl_sin = d + n;
        }
    }
    if (e == cudaSuccess) e = cudaMemcpy(kv->tl_cos, hc, 2 * n * sizeof(float), cudaMemcpyHostToDevice);
    free(hc);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "rope table");
    kv->tl_interleaved = interleaved != 0;
    return EIF_STATUS_OK;
}

static eif_status_t rope_check(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_heads) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_heads <= 0 || n_heads % kv->n_kv)
        return fail(ctx, EIF_STATUS_SHAPE_MISMATCH, "n_heads %d is not a multiple of n_kv_heads %d", n_heads, kv->n_kv);
    if (!kv->tl_cos) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "no RoPE table (eif_cuda_kv_set_rope)");
    if (kv->dtype == EIF_CUDA_INT8 && (size_t)kv->n_kv * kv->hd * 4 > 48 * 1024)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "INT8 rope_append: n_kv_heads * head_dim %d above 12288",
                    kv->n_kv * kv->hd);
    return EIF_STATUS_OK;
}

static eif_status_t rope_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, const float *k,
                             const float *v, const int *pos, int n_tok, int start_pos, int n_heads, float *q_out,
                             __nv_bfloat16 *q_out_bf16) {
    RopeArgs a{q, k, v, kv->tl_cos, kv->tl_sin, pos, kv->k[layer], kv->v[layer], kv->dtype, q_out, q_out_bf16,
               kv->batch, n_tok, start_pos, n_heads, kv->n_kv, kv->hd, kv->max_seq, kv->tl_interleaved, ctx->dev_err};
    if (kv->dtype == EIF_CUDA_INT8) {
        a.k_scale = kv->ks[layer];
        a.v_scale = kv->vs[layer];
        a.scale_stride = kv->scale_stride;
    }
    CK(launch_rope_append(ctx->stream, a));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_rope_append_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                              const float *k_dev, const float *v_dev, const int *pos_dev, int n_heads,
                                              float *q_out_dev) {
    eif_status_t rs = rope_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q_dev || !k_dev || !v_dev || !pos_dev || !q_out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rope_append_dev: NULL pointer");
    DeviceGuard g(ctx);
    return rope_run(ctx, kv, layer, q_dev, k_dev, v_dev, pos_dev, 1, 0, n_heads, q_out_dev, nullptr);
}

static eif_status_t stage_step_inputs(eif_cuda_ctx_t *ctx, const float *q, const float *k, const float *v,
                                      const int *pos, size_t nq, size_t nk, size_t B, char **s_out, size_t *off,
                                      float **dout);

EIF_API eif_status_t eif_cuda_rope_append(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                          const float *k, const float *v, const int *pos, int n_heads, float *q_out) {
    eif_status_t rs = rope_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q || !k || !v || !pos || !q_out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rope_append: NULL pointer");
    for (int b = 0; b < kv->batch; ++b)
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
    DeviceGuard g(ctx);
    const size_t B = kv->batch, nq = B * n_heads * kv->hd, nk = B * kv->n_kv * kv->hd;
    char *s = nullptr;
    size_t off[4];
    float *dout = nullptr;
    rs = stage_step_inputs(ctx, q, k, v, pos, nq, nk, B, &s, off, &dout);
    if (rs != EIF_STATUS_OK) return rs;
    rs = rope_run(ctx, kv, layer, reinterpret_cast<float *>(s + off[0]), reinterpret_cast<float *>(s + off[1]),
                  reinterpret_cast<float *>(s + off[2]), reinterpret_cast<int *>(s + off[3]), 1, 0, n_heads, dout,
                  nullptr);
    if (rs != EIF_STATUS_OK) return rs;
    if (dout == small_out(ctx)) return finish_small(ctx, q_out, nq * 4);
    CK(cudaMemcpyAsync(q_out, dout, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// ---- the whole decode step of a layer: RoPE, the new row, attention -------------------------------------

// Host inputs q, k, v, pos of a decode step into the stage buffer (packed in one copy when small); *dout is
// where the step's output [B][nq / B] goes: small_out(ctx) when it fits, else the stage after the inputs,
// followed by nq floats of scratch.
static eif_status_t stage_step_inputs(eif_cuda_ctx_t *ctx, const float *q, const float *k, const float *v,
                                      const int *pos, size_t nq, size_t nk, size_t B, char **s_out, size_t *off,
                                      float **dout) {
    const void *src[4] = {q, k, v, pos};
    const size_t bytes[4] = {nq * 4, nk * 4, nk * 4, B * 4};
    size_t in_total = 0;
    for (int i = 0; i < 4; ++i) {
        off[i] = in_total;
        in_total += a16(bytes[i]);
    }
    const bool small = in_total <= kSmallIo && nq * 4 <= kSmallIo;
    eif_status_t st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, a256(in_total) + 2 * a256(nq * 4));
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    if (small) {
        st = send_packed(ctx, s, 4, src, bytes, off);
        if (st != EIF_STATUS_OK) return st;
    } else {
        for (int i = 0; i < 4; ++i) CK(cudaMemcpyAsync(s + off[i], src[i], bytes[i], cudaMemcpyHostToDevice, ctx->stream));
    }
    *s_out = s;
    *dout = small ? small_out(ctx) : reinterpret_cast<float *>(s + a256(in_total));
    return EIF_STATUS_OK;
}

// The step on device arrays: one launch (attn_decode_step.cu) when the shape is small enough, else
// rope_append's kernel (the rotated q into q_rot) and the split-K decode.
static eif_status_t step_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q, const float *k,
                             const float *v, const int *pos, int max_len, int n_heads, float scale, float *out,
                             float *q_rot) {
    int cap = 0;
    const int nc = decode_step_chunks(kv->dtype, kv->hd, n_heads / kv->n_kv, kv->batch, kv->n_kv, max_len,
                                      ctx->sm_count, &cap);
    if (nc > 0) {
        DecodeStepArgs a{q, k, v, pos, kv->tl_cos, kv->tl_sin, kv->k[layer], kv->v[layer], kv->dtype, out,
                         kv->batch, n_heads, kv->n_kv, kv->hd, kv->max_seq, kv->tl_interleaved, nc, scale,
                         ctx->dev_err, cap};
        CK(launch_attend_decode_step(ctx->stream, a));
        ctx->launches += 1;
        return EIF_STATUS_OK;
    }
    eif_status_t st = rope_run(ctx, kv, layer, q, k, v, pos, 1, 0, n_heads, q_rot, nullptr);
    if (st != EIF_STATUS_OK) return st;
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, q_rot, pos, kv->batch, n_heads, kv->n_kv, kv->hd,
                 kv->max_seq, max_len, scale, nullptr, (int)EIF_CUDA_SUBLN_NONE, nullptr, out, ctx->dev_err};
    return decode_run(ctx, kv, layer, a);
}

EIF_API eif_status_t eif_cuda_decode_step(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                          const float *k, const float *v, const int *pos, int n_heads, float scale,
                                          float *out) {
    eif_status_t rs = rope_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q || !k || !v || !pos || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "decode_step: NULL pointer");
    int max_pos = 0;
    for (int b = 0; b < kv->batch; ++b) {
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
        max_pos = std::max(max_pos, pos[b]);
    }
    DeviceGuard g(ctx);
    const size_t B = kv->batch, nq = B * n_heads * kv->hd, nk = B * kv->n_kv * kv->hd;
    char *s = nullptr;
    size_t off[4];
    float *dout = nullptr;
    rs = stage_step_inputs(ctx, q, k, v, pos, nq, nk, B, &s, off, &dout);
    if (rs != EIF_STATUS_OK) return rs;
    const bool small = dout == small_out(ctx);
    float *q_rot = small ? reinterpret_cast<float *>(s + a256(off[3] + B * 4))
                         : reinterpret_cast<float *>(reinterpret_cast<char *>(dout) + a256(nq * 4));
    rs = step_run(ctx, kv, layer, reinterpret_cast<float *>(s + off[0]), reinterpret_cast<float *>(s + off[1]),
                  reinterpret_cast<float *>(s + off[2]), reinterpret_cast<int *>(s + off[3]), max_pos + 1, n_heads,
                  scale, dout, q_rot);
    if (rs != EIF_STATUS_OK) return rs;
    if (small) return finish_small(ctx, out, nq * 4);
    CK(cudaMemcpyAsync(out, dout, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_decode_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                              const float *k_dev, const float *v_dev, const int *pos_dev, int max_pos,
                                              int n_heads, float scale, float *out_dev) {
    eif_status_t rs = rope_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q_dev || !k_dev || !v_dev || !pos_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "decode_step_dev: NULL pointer");
    if (max_pos < 0 || max_pos >= kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "max_pos %d outside [0, %d)", max_pos, kv->max_seq);
    DeviceGuard g(ctx);
    // scratch for the rotated q of the two-launch form
    const size_t nq = (size_t)kv->batch * n_heads * kv->hd;
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, a256(nq * 4));
    if (rs != EIF_STATUS_OK) return rs;
    return step_run(ctx, kv, layer, q_dev, k_dev, v_dev, pos_dev, max_pos + 1, n_heads, scale, out_dev,
                    static_cast<float *>(ctx->stage));
}

static eif_status_t rope_prefill_check(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_tok, int start_pos,
                                       int n_heads) {
    eif_status_t rs = rope_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (n_tok < 1 || start_pos < 0 || start_pos + n_tok > kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rows [%d, %d) outside the cache [0, %d)", start_pos,
                    start_pos + n_tok, kv->max_seq);
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_rope_append_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                      const float *q_dev, const float *k_dev, const float *v_dev,
                                                      int n_tok, int start_pos, int n_heads, void *q_out_dev) {
    eif_status_t rs = rope_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q_dev || !k_dev || !v_dev || !q_out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rope_append_prefill_dev: NULL pointer");
    DeviceGuard g(ctx);
    if (prefill_by_rows(kv))  // fp32 / INT8 caches: the prefill attention reads fp32 queries
        return rope_run(ctx, kv, layer, q_dev, k_dev, v_dev, nullptr, n_tok, start_pos, n_heads,
                        static_cast<float *>(q_out_dev), nullptr);
    return rope_run(ctx, kv, layer, q_dev, k_dev, v_dev, nullptr, n_tok, start_pos, n_heads, nullptr,
                    static_cast<__nv_bfloat16 *>(q_out_dev));
}

EIF_API eif_status_t eif_cuda_rope_append_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                                  const float *k, const float *v, int n_tok, int start_pos,
                                                  int n_heads, float *q_out) {
    eif_status_t rs = rope_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!q || !k || !v || !q_out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rope_append_prefill: NULL pointer");
    DeviceGuard g(ctx);
    const size_t rows = (size_t)kv->batch * n_tok, nq = rows * n_heads * kv->hd, nk = rows * kv->n_kv * kv->hd;
    Carver cv;
    const size_t o_q = cv.take(nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4), o_o = cv.take(nq * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_q, q, nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = rope_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_k),
                  reinterpret_cast<float *>(s + o_v), nullptr, n_tok, start_pos, n_heads,
                  reinterpret_cast<float *>(s + o_o), nullptr);
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(q_out, s + o_o, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// Qwen3.5 attention prep (fullatt_prep)
// =================================================================================================

EIF_API eif_status_t eif_cuda_kv_set_norms(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_norm,
                                           const float *k_norm) {
    if (!ctx || !kv || kv->ctx != ctx || !q_norm || !k_norm) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    DeviceGuard g(ctx);
    if (!kv->q_norm[layer]) {
        CK(cudaMalloc(&kv->q_norm[layer], 2 * (size_t)kv->hd * 4));
        kv->k_norm[layer] = kv->q_norm[layer] + kv->hd;
    }
    CK(cudaMemcpyAsync(kv->q_norm[layer], q_norm, kv->hd * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(kv->k_norm[layer], k_norm, kv->hd * 4, cudaMemcpyHostToDevice, ctx->stream));
    return wait_stream(ctx);
}

// cos / sin of rope_partial (src/eif_qwen35.c:502-535) for every cache row: n_rot = head_dim * 0.25,
// angle = pos * inv_freq_i.  The source reads inv_freq_i = 1.0f / powf(1e7f, 2i / n_rot); the reference's
// build (-O3 -ffast-math, CMakeLists.txt:19) turns a power of the constant 1e7 into an exponential,
// inv_freq_i = expf(-(2i / n_rot) * logf(1e7)), which differs from 1 / powf in the last bit for most i.
// At positions in the tens of thousands one ulp of inv_freq moves the angle by ~1e-3 rad, so the table
// takes the compiled form: the float product, then its exponential rounded to nearest from double.
static eif_status_t ensure_rope_table(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv) {
    if (kv->rope_cos) return EIF_STATUS_OK;
    const int n_rot = (int)(kv->hd * 0.25f), half = n_rot / 2;
    if (half < 1) return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "head_dim %d too small for partial RoPE", kv->hd);
    const size_t n = (size_t)kv->max_seq * half;
    float *hc = (float *)malloc(2 * n * sizeof(float));
    if (!hc) return fail(ctx, EIF_STATUS_OUT_OF_MEMORY, "rope table");
    float inv[128];
    const float ln_theta = (float)log(10000000.0);
    for (int i = 0; i < half && i < 128; ++i) {
        const float y = -(2.0f * i / (float)n_rot) * ln_theta;
        inv[i] = (float)exp((double)y);
    }
    for (int pos = 0; pos < kv->max_seq; ++pos)
        for (int i = 0; i < half; ++i) {
            const float theta = pos * inv[i];
            hc[(size_t)pos * half + i] = cosf(theta);
            hc[n + (size_t)pos * half + i] = sinf(theta);
        }
    float *d = nullptr;
    cudaError_t e = cudaMalloc(&d, 2 * n * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(d, hc, 2 * n * sizeof(float), cudaMemcpyHostToDevice);
    free(hc);
    if (e != cudaSuccess) {
        if (d) cudaFree(d);
        return cuda_fail(ctx, e, "rope table");
    }
    kv->rope_cos = d;
    kv->rope_sin = d + n;
    return EIF_STATUS_OK;
}

static eif_status_t prep_check(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_heads) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return fail(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_heads <= 0 || n_heads % kv->n_kv)
        return fail(ctx, EIF_STATUS_SHAPE_MISMATCH, "n_heads %d is not a multiple of n_kv_heads %d", n_heads, kv->n_kv);
    if (!kv->q_norm[layer]) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "layer %d has no q/k norms (kv_set_norms)", layer);
    if (kv->hd > 1024) return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "head_dim %d", kv->hd);
    if (kv->dtype == EIF_CUDA_INT8)  // Qwen3.5 keeps an fp32 cache (include/eif_qwen35.h:204-208)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "Qwen3.5 attention prep writes fp32 or bf16 caches, not INT8");
    return EIF_STATUS_OK;
}

// pos set: one token per sequence at pos[b]; else n_tok tokens per sequence at start_pos + i.
static eif_status_t prep_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg, const float *k,
                             const float *v, const int *pos, int n_heads, float *q_out, float *gate_out,
                             int n_tok = 1, int start_pos = 0, __nv_bfloat16 *q_out_bf16 = nullptr) {
    eif_status_t rs = ensure_rope_table(ctx, kv);
    if (rs != EIF_STATUS_OK) return rs;
    AttnPrepArgs a{qg, k, v, kv->q_norm[layer], kv->k_norm[layer], kv->rope_cos, kv->rope_sin, pos, kv->k[layer],
                   kv->v[layer], kv->dtype, q_out, gate_out, kv->batch, n_heads, kv->n_kv, kv->hd,
                   (int)(kv->hd * 0.25f), kv->max_seq, ctx->dev_err, q_out_bf16, n_tok, start_pos};
    CK(launch_fullatt_prep(ctx->stream, a));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

static eif_status_t prep_prefill_check(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, int n_tok, int start_pos,
                                       int n_heads) {
    eif_status_t rs = prep_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (n_tok < 1 || start_pos < 0 || start_pos + n_tok > kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "rows [%d, %d) outside the cache [0, %d)", start_pos,
                    start_pos + n_tok, kv->max_seq);
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_fullatt_prep_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                       const float *qg_dev, const float *k_dev, const float *v_dev,
                                                       int n_tok, int start_pos, int n_heads, void *q_out_dev,
                                                       float *gate_out_dev) {
    eif_status_t rs = prep_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qg_dev || !k_dev || !v_dev || !q_out_dev || !gate_out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prep_prefill_dev: NULL pointer");
    DeviceGuard g(ctx);
    if (prefill_by_rows(kv))  // an fp32 cache: the prefill attention reads fp32 queries
        return prep_run(ctx, kv, layer, qg_dev, k_dev, v_dev, nullptr, n_heads, static_cast<float *>(q_out_dev),
                        gate_out_dev, n_tok, start_pos);
    return prep_run(ctx, kv, layer, qg_dev, k_dev, v_dev, nullptr, n_heads, nullptr, gate_out_dev, n_tok, start_pos,
                    static_cast<__nv_bfloat16 *>(q_out_dev));
}

EIF_API eif_status_t eif_cuda_fullatt_prep_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                                   const float *k, const float *v, int n_tok, int start_pos,
                                                   int n_heads, float *q_out, float *gate_out) {
    eif_status_t rs = prep_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qg || !k || !v || !q_out || !gate_out)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prep_prefill: NULL pointer");
    DeviceGuard g(ctx);
    const size_t rows = (size_t)kv->batch * n_tok, nq = rows * n_heads * kv->hd, nk = rows * kv->n_kv * kv->hd;
    Carver cv;
    const size_t o_qg = cv.take(2 * nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4), o_q = cv.take(nq * 4),
                 o_g = cv.take(nq * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_qg, qg, 2 * nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = prep_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_qg), reinterpret_cast<float *>(s + o_k),
                  reinterpret_cast<float *>(s + o_v), nullptr, n_heads, reinterpret_cast<float *>(s + o_q),
                  reinterpret_cast<float *>(s + o_g), n_tok, start_pos);
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(q_out, s + o_q, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaMemcpyAsync(gate_out, s + o_g, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

EIF_API eif_status_t eif_cuda_fullatt_prep_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg_dev,
                                               const float *k_dev, const float *v_dev, const int *pos_dev,
                                               int n_heads, float *q_out_dev, float *gate_out_dev) {
    eif_status_t rs = prep_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qg_dev || !k_dev || !v_dev || !pos_dev || !q_out_dev || !gate_out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prep_dev: NULL pointer");
    DeviceGuard g(ctx);
    return prep_run(ctx, kv, layer, qg_dev, k_dev, v_dev, pos_dev, n_heads, q_out_dev, gate_out_dev);
}

EIF_API eif_status_t eif_cuda_fullatt_prep(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                           const float *k, const float *v, const int *pos, int n_heads,
                                           float *q_out, float *gate_out) {
    eif_status_t rs = prep_check(ctx, kv, layer, n_heads);
    if (rs != EIF_STATUS_OK) return rs;
    if (!qg || !k || !v || !pos || !q_out || !gate_out)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prep: NULL pointer");
    for (int b = 0; b < kv->batch; ++b)
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
    DeviceGuard g(ctx);
    const size_t B = kv->batch, nq = B * n_heads * kv->hd, nk = B * kv->n_kv * kv->hd;
    Carver cv;
    const size_t o_qg = cv.take(2 * nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4), o_p = cv.take(B * 4),
                 o_q = cv.take(nq * 4), o_g = cv.take(nq * 4);
    rs = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (rs != EIF_STATUS_OK) return rs;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_qg, qg, 2 * nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_p, pos, B * 4, cudaMemcpyHostToDevice, ctx->stream));
    rs = prep_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_qg), reinterpret_cast<float *>(s + o_k),
                  reinterpret_cast<float *>(s + o_v), reinterpret_cast<int *>(s + o_p), n_heads,
                  reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_g));
    if (rs != EIF_STATUS_OK) return rs;
    CK(cudaMemcpyAsync(q_out, s + o_q, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaMemcpyAsync(gate_out, s + o_g, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// The Qwen3.5 attention mixer of one token: fullatt_prep + fullatt_attend in one call
// =================================================================================================

static eif_status_t fullatt_decode_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                       const float *k, const float *v, const int *pos, int max_pos, int n_heads,
                                       float scale, eif_cuda_subln_t subln, const float *sub_norm, float *out,
                                       float *q_buf, float *gate_buf) {
    eif_status_t st = prep_run(ctx, kv, layer, qg, k, v, pos, n_heads, q_buf, gate_buf);
    if (st != EIF_STATUS_OK) return st;
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, q_buf, pos, kv->batch, n_heads, kv->n_kv, kv->hd,
                 kv->max_seq, max_pos + 1, scale, gate_buf, (int)subln, sub_norm, out, ctx->dev_err};
    return decode_run(ctx, kv, layer, a);
}

EIF_API eif_status_t eif_cuda_fullatt_decode_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                 const float *qg_dev, const float *k_dev, const float *v_dev,
                                                 const int *pos_dev, int max_pos, int n_heads, float scale,
                                                 eif_cuda_subln_t subln, const float *sub_norm_dev, float *out_dev) {
    eif_status_t st = prep_check(ctx, kv, layer, n_heads);
    if (st == EIF_STATUS_OK) st = decode_check(ctx, kv, layer, n_heads, subln);
    if (st != EIF_STATUS_OK) return st;
    if (!qg_dev || !k_dev || !v_dev || !pos_dev || !out_dev || (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm_dev))
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_decode_dev: NULL pointer");
    if (max_pos < 0 || max_pos >= kv->max_seq)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "max_pos %d outside [0, %d)", max_pos, kv->max_seq);
    DeviceGuard g(ctx);
    const size_t nq = (size_t)kv->batch * n_heads * kv->hd;
    st = ensure_buffer(ctx, &ctx->mix, &ctx->mix_bytes, 2 * a256(nq * 4));
    if (st != EIF_STATUS_OK) return st;
    float *qb = static_cast<float *>(ctx->mix);
    float *gb = reinterpret_cast<float *>(static_cast<char *>(ctx->mix) + a256(nq * 4));
    return fullatt_decode_run(ctx, kv, layer, qg_dev, k_dev, v_dev, pos_dev, max_pos, n_heads, scale, subln,
                              sub_norm_dev, out_dev, qb, gb);
}

EIF_API eif_status_t eif_cuda_fullatt_decode(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                             const float *k, const float *v, const int *pos, int n_heads, float scale,
                                             eif_cuda_subln_t subln, const float *sub_norm, float *out) {
    eif_status_t st = prep_check(ctx, kv, layer, n_heads);
    if (st == EIF_STATUS_OK) st = decode_check(ctx, kv, layer, n_heads, subln);
    if (st != EIF_STATUS_OK) return st;
    if (!qg || !k || !v || !pos || !out || (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm))
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_decode: NULL pointer");
    int max_pos = 0;
    for (int b = 0; b < kv->batch; ++b) {
        if (pos[b] < 0 || pos[b] >= kv->max_seq)
            return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "pos[%d] = %d outside [0, %d)", b, pos[b], kv->max_seq);
        max_pos = std::max(max_pos, pos[b]);
    }
    DeviceGuard g(ctx);
    const size_t B = kv->batch, row = (size_t)n_heads * kv->hd, nq = B * row, nk = B * kv->n_kv * kv->hd;
    const bool wn = subln == EIF_CUDA_SUBLN_WEIGHT;
    Carver cv;
    const size_t o_qg = cv.take(2 * nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4), o_p = cv.take(B * 4),
                 o_n = cv.take(wn ? row * 4 : 0), o_q = cv.take(nq * 4), o_g = cv.take(nq * 4), o_o = cv.take(nq * 4);
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_qg, qg, 2 * nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_p, pos, B * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (wn) CK(cudaMemcpyAsync(s + o_n, sub_norm, row * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = fullatt_decode_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_qg), reinterpret_cast<float *>(s + o_k),
                            reinterpret_cast<float *>(s + o_v), reinterpret_cast<int *>(s + o_p), max_pos, n_heads,
                            scale, subln, wn ? reinterpret_cast<float *>(s + o_n) : nullptr,
                            reinterpret_cast<float *>(s + o_o), reinterpret_cast<float *>(s + o_q),
                            reinterpret_cast<float *>(s + o_g));
    if (st != EIF_STATUS_OK) return st;
    CK(cudaMemcpyAsync(out, s + o_o, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// =================================================================================================
// Whole attention blocks of a prefill chunk in one call (queries stay on the device between the halves)
// =================================================================================================

// tinyllm: RoPE + cache write of the chunk, then causal attention; q_buf holds the rotated queries (bf16 for a
// bf16 cache, fp32 otherwise), out is fp32.
static eif_status_t prefill_step_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                     const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                     float scale, float *out, void *q_buf) {
    const bool rows = prefill_by_rows(kv);
    eif_status_t st = rope_run(ctx, kv, layer, q, k, v, nullptr, n_tok, start_pos, n_heads,
                               rows ? static_cast<float *>(q_buf) : nullptr,
                               rows ? nullptr : static_cast<__nv_bfloat16 *>(q_buf));
    if (st != EIF_STATUS_OK) return st;
    if (rows)
        return prefill_rows_run(ctx, kv, layer, static_cast<float *>(q_buf), n_tok, start_pos, n_heads, scale, nullptr,
                                EIF_CUDA_SUBLN_NONE, nullptr, out);
    return prefill_run(ctx, kv, layer, q_buf, n_tok, start_pos, n_heads, scale, nullptr, out);
}

EIF_API eif_status_t eif_cuda_prefill_step_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q_dev,
                                               const float *k_dev, const float *v_dev, int n_tok, int start_pos,
                                               int n_heads, float scale, float *out_dev) {
    eif_status_t st = rope_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    if (!q_dev || !k_dev || !v_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "prefill_step_dev: NULL pointer");
    DeviceGuard g(ctx);
    const size_t nq = (size_t)kv->batch * n_tok * n_heads * kv->hd;
    st = ensure_buffer(ctx, &ctx->mix, &ctx->mix_bytes, a256(nq * 4));
    if (st != EIF_STATUS_OK) return st;
    return prefill_step_run(ctx, kv, layer, q_dev, k_dev, v_dev, n_tok, start_pos, n_heads, scale, out_dev, ctx->mix);
}

EIF_API eif_status_t eif_cuda_prefill_step(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *q,
                                           const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                           float scale, float *out) {
    eif_status_t st = rope_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st != EIF_STATUS_OK) return st;
    if (!q || !k || !v || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "prefill_step: NULL pointer");
    DeviceGuard g(ctx);
    const size_t rows = (size_t)kv->batch * n_tok, nq = rows * n_heads * kv->hd, nk = rows * kv->n_kv * kv->hd;
    Carver cv;
    const size_t o_q = cv.take(nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4), o_r = cv.take(nq * 4),
                 o_o = cv.take(nq * 4);
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_q, q, nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = prefill_step_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_q), reinterpret_cast<float *>(s + o_k),
                          reinterpret_cast<float *>(s + o_v), n_tok, start_pos, n_heads, scale,
                          reinterpret_cast<float *>(s + o_o), s + o_r);
    if (st != EIF_STATUS_OK) return st;
    CK(cudaMemcpyAsync(out, s + o_o, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// Qwen3.5: fullatt_prep of the chunk, then the gated causal attention; q_buf as above, gate_buf fp32.
static eif_status_t fullatt_prefill_run(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                        const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                        float scale, eif_cuda_subln_t subln, const float *sub_norm, float *out,
                                        void *q_buf, float *gate_buf) {
    const bool rows = prefill_by_rows(kv);
    eif_status_t st = prep_run(ctx, kv, layer, qg, k, v, nullptr, n_heads, rows ? static_cast<float *>(q_buf) : nullptr,
                               gate_buf, n_tok, start_pos, rows ? nullptr : static_cast<__nv_bfloat16 *>(q_buf));
    if (st != EIF_STATUS_OK) return st;
    if (rows)
        return prefill_rows_run(ctx, kv, layer, static_cast<float *>(q_buf), n_tok, start_pos, n_heads, scale, gate_buf,
                                subln, sub_norm, out);
    return prefill_gated_run(ctx, kv, layer, q_buf, n_tok, start_pos, n_heads, scale, gate_buf, subln, sub_norm, out);
}

EIF_API eif_status_t eif_cuda_fullatt_prefill_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                  const float *qg_dev, const float *k_dev, const float *v_dev,
                                                  int n_tok, int start_pos, int n_heads, float scale,
                                                  eif_cuda_subln_t subln, const float *sub_norm_dev, float *out_dev) {
    eif_status_t st = prep_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = subln_check(ctx, subln, sub_norm_dev);
    if (st != EIF_STATUS_OK) return st;
    if (!qg_dev || !k_dev || !v_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prefill_dev: NULL pointer");
    DeviceGuard g(ctx);
    const size_t nq = (size_t)kv->batch * n_tok * n_heads * kv->hd;
    st = ensure_buffer(ctx, &ctx->mix, &ctx->mix_bytes, 2 * a256(nq * 4));
    if (st != EIF_STATUS_OK) return st;
    float *gb = reinterpret_cast<float *>(static_cast<char *>(ctx->mix) + a256(nq * 4));
    return fullatt_prefill_run(ctx, kv, layer, qg_dev, k_dev, v_dev, n_tok, start_pos, n_heads, scale, subln,
                               sub_norm_dev, out_dev, ctx->mix, gb);
}

EIF_API eif_status_t eif_cuda_fullatt_prefill(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer, const float *qg,
                                              const float *k, const float *v, int n_tok, int start_pos, int n_heads,
                                              float scale, eif_cuda_subln_t subln, const float *sub_norm,
                                              float *out) {
    eif_status_t st = prep_prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = prefill_check(ctx, kv, layer, n_tok, start_pos, n_heads);
    if (st == EIF_STATUS_OK) st = subln_check(ctx, subln, sub_norm);
    if (st != EIF_STATUS_OK) return st;
    if (!qg || !k || !v || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "fullatt_prefill: NULL pointer");
    DeviceGuard g(ctx);
    const size_t rows = (size_t)kv->batch * n_tok, row = (size_t)n_heads * kv->hd, nq = rows * row,
                 nk = rows * kv->n_kv * kv->hd;
    const bool wn = subln == EIF_CUDA_SUBLN_WEIGHT;
    Carver cv;
    const size_t o_qg = cv.take(2 * nq * 4), o_k = cv.take(nk * 4), o_v = cv.take(nk * 4),
                 o_n = cv.take(wn ? row * 4 : 0), o_q = cv.take(nq * 4), o_g = cv.take(nq * 4), o_o = cv.take(nq * 4);
    st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, cv.off);
    if (st != EIF_STATUS_OK) return st;
    char *s = static_cast<char *>(ctx->stage);
    CK(cudaMemcpyAsync(s + o_qg, qg, 2 * nq * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_k, k, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    CK(cudaMemcpyAsync(s + o_v, v, nk * 4, cudaMemcpyHostToDevice, ctx->stream));
    if (wn) CK(cudaMemcpyAsync(s + o_n, sub_norm, row * 4, cudaMemcpyHostToDevice, ctx->stream));
    st = fullatt_prefill_run(ctx, kv, layer, reinterpret_cast<float *>(s + o_qg), reinterpret_cast<float *>(s + o_k),
                             reinterpret_cast<float *>(s + o_v), n_tok, start_pos, n_heads, scale, subln,
                             wn ? reinterpret_cast<float *>(s + o_n) : nullptr, reinterpret_cast<float *>(s + o_o),
                             s + o_q, reinterpret_cast<float *>(s + o_g));
    if (st != EIF_STATUS_OK) return st;
    CK(cudaMemcpyAsync(out, s + o_o, nq * 4, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}

// ---------------------------------------------------------------------------------------------------------------
// Projections: linear_gemv / linear_gemm / int8_gemv (src/eif_qwen35.c:384-443, 1033-1063) on resident weights.

EIF_API eif_status_t eif_cuda_linear_upload(eif_cuda_ctx_t *ctx, int quant_type, int rows, int cols, const void *W,
                                            const float *scales, eif_cuda_linear_t **out) {
    if (!ctx || !out) return EIF_STATUS_INVALID_ARGUMENT;
    *out = nullptr;
    const int wt = quant_type & 0xff, group = quant_type >> 8;
    if (wt < EIF_CUDA_W_F32 || wt > EIF_CUDA_W_INT8 || group < 0)
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "linear: unknown quant type %d", quant_type);
    if (rows <= 0 || cols <= 0 || !W || (wt != EIF_CUDA_W_F32 && !scales))
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "linear_upload: rows %d cols %d or a NULL pointer", rows, cols);
    if (group > 0 && (wt != EIF_CUDA_W_TERNARY2 || group % 16 || cols % group))
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED,
                    "linear: scale group %d (2-bit ternary only, a multiple of 16 dividing cols %d)", group, cols);
    const size_t row_bytes = linear_row_bytes(wt, cols), stride = (row_bytes + 63) & ~(size_t)63;
    if (!linear_fits(wt, stride))
        return fail(ctx, EIF_STATUS_NOT_SUPPORTED, "linear: %d columns exceed the shared-memory token tile", cols);
    DeviceGuard g(ctx);
    if (!g.ok) return fail(ctx, EIF_STATUS_ERROR, "cannot select device %d", ctx->device);
    eif_cuda_linear_t *lin = new (std::nothrow) eif_cuda_linear_t();
    if (!lin) return fail(ctx, EIF_STATUS_OUT_OF_MEMORY, "linear_upload: host allocation");
    lin->ctx = ctx;
    lin->wtype = wt;
    lin->group = group;
    lin->rows = rows;
    lin->cols = cols;
    lin->row_bytes = row_bytes;
    lin->stride = stride;
    lin->n_scales_row = wt == EIF_CUDA_W_F32 ? 0 : (group ? cols / group : 1);
    cudaError_t e = cudaMalloc(&lin->W, stride * (size_t)rows);
    if (e == cudaSuccess && stride != row_bytes) e = cudaMemset(lin->W, 0, stride * (size_t)rows);
    if (e == cudaSuccess) e = cudaMemcpy2D(lin->W, stride, W, row_bytes, row_bytes, rows, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && lin->n_scales_row) {
        const size_t ns = (size_t)rows * lin->n_scales_row * sizeof(float);
        e = cudaMalloc(&lin->scales, ns);
        if (e == cudaSuccess) e = cudaMemcpy(lin->scales, scales, ns, cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        if (lin->W) cudaFree(lin->W);
        if (lin->scales) cudaFree(lin->scales);
        delete lin;
        return cuda_fail(ctx, e, "linear_upload");
    }
    *out = lin;
    return EIF_STATUS_OK;
}

EIF_API void eif_cuda_linear_free(eif_cuda_linear_t *lin) {
    if (!lin) return;
    DeviceGuard g(lin->ctx);
    cudaStreamSynchronize(lin->ctx->stream);  // queued projections may still read the weights
    if (lin->W) cudaFree(lin->W);
    if (lin->scales) cudaFree(lin->scales);
    delete lin;
}

EIF_API eif_status_t eif_cuda_linear_forward_dev(eif_cuda_ctx_t *ctx, const eif_cuda_linear_t *lin,
                                                 const float *x_dev, int n, float *out_dev) {
    if (!ctx || !lin) return EIF_STATUS_INVALID_ARGUMENT;
    if (lin->ctx != ctx) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "linear: weights of another context");
    if (n < 1 || !x_dev || !out_dev)
        return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "linear_forward_dev: n %d or a NULL pointer", n);
    DeviceGuard g(ctx);
    CK(launch_linear(ctx->stream, *lin, x_dev, n, out_dev, ctx->sm_count));
    ctx->launches += 1;
    return EIF_STATUS_OK;
}

EIF_API eif_status_t eif_cuda_linear_forward(eif_cuda_ctx_t *ctx, const eif_cuda_linear_t *lin, const float *x,
                                             int n, float *out) {
    if (!ctx || !lin) return EIF_STATUS_INVALID_ARGUMENT;
    if (lin->ctx != ctx) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "linear: weights of another context");
    if (n < 1 || !x || !out) return fail(ctx, EIF_STATUS_INVALID_ARGUMENT, "linear_forward: n %d or a NULL pointer", n);
    DeviceGuard g(ctx);
    const size_t xb = (size_t)n * lin->cols * 4, ob = (size_t)n * lin->rows * 4;
    eif_status_t st = ensure_buffer(ctx, &ctx->stage, &ctx->stage_bytes, a256(xb) + ob);
    if (st != EIF_STATUS_OK) return st;
    float *xd = static_cast<float *>(ctx->stage);
    float *od = reinterpret_cast<float *>(static_cast<char *>(ctx->stage) + a256(xb));
    CK(cudaMemcpyAsync(xd, x, xb, cudaMemcpyHostToDevice, ctx->stream));
    CK(launch_linear(ctx->stream, *lin, xd, n, od, ctx->sm_count));
    ctx->launches += 1;
    CK(cudaMemcpyAsync(out, od, ob, cudaMemcpyDeviceToHost, ctx->stream));
    return wait_stream(ctx);
}
