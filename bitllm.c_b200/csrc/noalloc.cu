// noalloc.cu -- decode attention for callers that must not allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc once they are running: an inference engine that
// sizes all device memory at start-up and forbids allocation on its decode path (so a long-running
// server never fragments or runs out mid-request), or a caller that holds the GPU under an external
// memory budget where any allocation can fail or stall.  eif_cuda_attend_decode_dev grows a per-context
// scratch buffer with cudaMalloc the first time a split needs more room, which such callers cannot
// accept.  eif_cuda_attend_decode_noalloc_dev runs the same kernels with their split-K partials placed
// in one fixed array that lives in the library's own device image instead.
//
// The array: kNoallocScratchBytes (16 MiB) of device memory, reserved on every GPU that loads this
// library and held until the process exits.  Host code never dereferences its name (on the host the
// symbol is only a stand-in, not a device address); the device address is fetched once per device
// with cudaGetSymbolAddress, with that device current, and handed to the kernels.  The first call on a
// device does that set-up, so make the first call on each device before any stream capture begins.  The
// address is kept per device ordinal and belongs to the device's primary context, the one the CUDA
// runtime (and this library's contexts) use: a host that drives the library from another driver context,
// or that reset the device (cudaDeviceReset) after the first call, must not use this entry point.
//
// All calls in the process share the array and find the previous call's contents in it.  The decode
// kernels overwrite every partial they later read, so nothing has to be cleared between calls; calls
// that overlap on the GPU (different streams or contexts of one device running at the same time)
// race on the array and must be ordered by the caller.
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>

#include "internal.h"

#define EIF_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr size_t kNoallocScratchBytes = (size_t)16 << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

void *g_scratch_addr[kMaxDevices];
pthread_mutex_t g_scratch_lock = PTHREAD_MUTEX_INITIALIZER;

eif_status_t set_err(eif_cuda_ctx_t *ctx, eif_status_t st, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(ctx->err, sizeof ctx->err, fmt, ap);
    va_end(ap);
    return st;
}

// Device address of g_noalloc_scratch on ctx's device, looked up once per device with it current.
eif_status_t scratch_address(eif_cuda_ctx_t *ctx, void **addr) {
    if (ctx->device < 0 || ctx->device >= kMaxDevices)
        return set_err(ctx, EIF_STATUS_NOT_SUPPORTED, "noalloc: device %d beyond the table", ctx->device);
    pthread_mutex_lock(&g_scratch_lock);
    void *p = g_scratch_addr[ctx->device];
    cudaError_t e = cudaSuccess;
    if (!p) {
        int prev = -1;
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        e = cudaSetDevice(ctx->device);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (prev >= 0) cudaSetDevice(prev);
        if (e == cudaSuccess && p) g_scratch_addr[ctx->device] = p;
    }
    pthread_mutex_unlock(&g_scratch_lock);
    if (e != cudaSuccess || !p)
        return set_err(ctx, EIF_STATUS_ERROR, "noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    *addr = p;
    return EIF_STATUS_OK;
}

}  // namespace

size_t noalloc_scratch_capacity() { return kNoallocScratchBytes; }

EIF_API eif_status_t eif_cuda_attend_decode_noalloc_dev(eif_cuda_ctx_t *ctx, eif_cuda_kv_t *kv, int layer,
                                                        const float *q_dev, const int *pos_dev, int max_pos,
                                                        int n_heads, float scale, const float *gate_dev,
                                                        eif_cuda_subln_t subln, const float *sub_norm_dev,
                                                        float *out_dev) {
    if (!ctx || !kv || kv->ctx != ctx) return EIF_STATUS_INVALID_ARGUMENT;
    if (layer < 0 || layer >= kv->n_layers) return set_err(ctx, EIF_STATUS_INVALID_LAYER, "layer %d out of range", layer);
    if (n_heads <= 0 || n_heads % kv->n_kv)
        return set_err(ctx, EIF_STATUS_SHAPE_MISMATCH, "n_heads %d is not a multiple of n_kv_heads %d", n_heads,
                       kv->n_kv);
    if (subln != EIF_CUDA_SUBLN_NONE && subln != EIF_CUDA_SUBLN_RMS && subln != EIF_CUDA_SUBLN_WEIGHT)
        return set_err(ctx, EIF_STATUS_INVALID_ARGUMENT, "bad subln mode %d", (int)subln);
    if (!q_dev || !pos_dev || !out_dev || (subln == EIF_CUDA_SUBLN_WEIGHT && !sub_norm_dev))
        return set_err(ctx, EIF_STATUS_INVALID_ARGUMENT, "attend_decode_noalloc_dev: NULL pointer");
    if (max_pos < 0 || max_pos >= kv->max_seq)
        return set_err(ctx, EIF_STATUS_INVALID_ARGUMENT, "max_pos %d outside [0, %d)", max_pos, kv->max_seq);

    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != ctx->device && cudaSetDevice(ctx->device) != cudaSuccess)
        return set_err(ctx, EIF_STATUS_ERROR, "cannot select device %d", ctx->device);

    eif_status_t st = EIF_STATUS_OK;
    void *scratch = nullptr;
    DecodeArgs a{kv->k[layer], kv->v[layer], kv->dtype, q_dev, pos_dev, kv->batch, n_heads, kv->n_kv, kv->hd,
                 kv->max_seq, max_pos + 1, scale, gate_dev, (int)subln, sub_norm_dev, out_dev, ctx->dev_err};
    a.max_ws_bytes = kNoallocScratchBytes;
    decode_prepare(kv, layer, a);
    const size_t need = decode_workspace_bytes(a, ctx->sm_count);
    if (need > kNoallocScratchBytes) {
        st = set_err(ctx, EIF_STATUS_INVALID_ARGUMENT,
                     "attend_decode_noalloc_dev: batch %d x %d kv heads x %d q heads/group x head_dim %d needs %zu "
                     "bytes of scratch; the fixed array holds %zu",
                     kv->batch, kv->n_kv, n_heads / kv->n_kv, kv->hd, need, kNoallocScratchBytes);
    } else {
        st = scratch_address(ctx, &scratch);
    }
    if (st == EIF_STATUS_OK) {
        bool ok = true;
        int nl = 0;
        const cudaError_t e =
            launch_attend_decode(ctx->stream, a, scratch, kNoallocScratchBytes, ctx->sm_count, &ok, &nl);
        ctx->launches += nl;
        if (!ok)
            st = set_err(ctx, EIF_STATUS_NOT_SUPPORTED, "decode attention: head_dim %d / group %d not supported",
                         kv->hd, n_heads / kv->n_kv);
        else if (e != cudaSuccess)
            st = set_err(ctx, EIF_STATUS_ERROR, "attend_decode_noalloc_dev launch: %s", cudaGetErrorString(e));
    }
    if (prev >= 0 && prev != ctx->device) cudaSetDevice(prev);
    return st;
}
