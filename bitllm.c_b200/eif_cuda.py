"""ctypes binding of include/eif_cuda.h (the C ABI of libeif_cuda.so).

This is the host-side mirror a Python caller uses; a C99 engine calls the same entry points
directly.  Host arrays are numpy float32/int32; `_dev` methods take raw device
addresses (ints), e.g. torch's tensor.data_ptr(), and run asynchronously on the context's stream.

Errors come back as EifCudaError carrying the eif_status_t code and the library's message; there is
no CPU fallback, and a missing library raises at import time of lib().
"""
from __future__ import annotations

import ctypes
import os
import re
import weakref

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeif_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "eif_cuda.h")

# eif_status_t (include/eif_status.h:8-19 of bitllm.c)
STATUS = {0: "OK", -1: "ERROR", -2: "INVALID_ARGUMENT", -3: "OUT_OF_MEMORY", -4: "NOT_IMPLEMENTED",
          -5: "NOT_SUPPORTED", -6: "TIMEOUT", -7: "INTERNAL_ERROR", -8: "INVALID_LAYER", -9: "SHAPE_MISMATCH"}
F32, BF16, INT8 = 0, 1, 2
# projection weight formats (eif_cuda_wtype_t): the engine's quant types (include/eif_qwen35.h:83-86) + INT8 head
W_F32, W_INT4, W_TERNARY2, W_TERNARY_DENSE, W_INT8 = 0, 1, 2, 3, 4
SUBLN_NONE, SUBLN_RMS, SUBLN_WEIGHT = 0, 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_lib = None


class EifCudaError(RuntimeError):
    def __init__(self, status: int, where: str, message: str = ""):
        self.status = status
        self.name = STATUS.get(status, str(status))
        super().__init__(f"{where}: EIF_STATUS_{self.name}" + (f" ({message})" if message else ""))


def header_functions() -> list[str]:
    """Names of every function the C header declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(eif_cuda_\w+)\s*\(", src)))


def lib() -> ctypes.CDLL:
    """Load libeif_cuda.so (built by bitllm.c_b200/build.py); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} not built: run python bitllm.c_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    sig = {
        "eif_cuda_device_count": (_I, []),
        "eif_cuda_init": (_I, [ctypes.POINTER(_P), _I]),
        "eif_cuda_free": (None, [_P]),
        "eif_cuda_last_error": (ctypes.c_char_p, [_P]),
        "eif_cuda_set_stream": (_I, [_P, _P]),
        "eif_cuda_get_stream": (_P, [_P]),
        "eif_cuda_set_timeout": (_I, [_P, _I]),
        "eif_cuda_synchronize": (_I, [_P]),
        "eif_cuda_launch_count": (ctypes.c_uint64, [_P]),
        "eif_cuda_kv_alloc": (_I, [_P, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
        "eif_cuda_kv_free": (None, [_P]),
        "eif_cuda_kv_reset": (_I, [_P, _P]),
        "eif_cuda_kv_upload": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
        "eif_cuda_kv_download": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
        "eif_cuda_kv_layer_ptrs": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
        "eif_cuda_kv_download_int8": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
        "eif_cuda_kv_layer_scales": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
        "eif_cuda_kv_append": (_I, [_P, _P, _I, _P, _P, _P]),
        "eif_cuda_kv_append_dev": (_I, [_P, _P, _I, _P, _P, _P]),
        "eif_cuda_kv_set_rope": (_I, [_P, _P, _F, _I]),
        "eif_cuda_rope_append": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P]),
        "eif_cuda_rope_append_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P]),
        "eif_cuda_decode_step": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, ctypes.c_float, _P]),
        "eif_cuda_decode_step_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _I, ctypes.c_float, _P]),
        "eif_cuda_rope_append_prefill": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _P]),
        "eif_cuda_rope_append_prefill_dev": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _P]),
        "eif_cuda_attend_decode": (_I, [_P, _P, _I, _P, _P, _I, _F, _P, _I, _P, _P]),
        "eif_cuda_attend_decode_dev": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _P, _I, _P, _P]),
        "eif_cuda_attend_decode_noalloc_dev": (_I, [_P, _P, _I, _P, _P, _I, _I, _F, _P, _I, _P, _P]),
        "eif_cuda_attend_decode_plan": (_I, [_P, _P, _I, _I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I),
                                             ctypes.POINTER(ctypes.c_size_t)]),
        "eif_cuda_fullatt_decode": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _F, _I, _P, _P]),
        "eif_cuda_fullatt_decode_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _I, _F, _I, _P, _P]),
        "eif_cuda_fullatt_prefill": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _F, _I, _P, _P]),
        "eif_cuda_fullatt_prefill_dev": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _F, _I, _P, _P]),
        "eif_cuda_prefill_step": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _F, _P]),
        "eif_cuda_prefill_step_dev": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _F, _P]),
        "eif_cuda_attend_prefill": (_I, [_P, _P, _I, _P, _I, _I, _I, _F, _P]),
        "eif_cuda_attend_prefill_dev": (_I, [_P, _P, _I, _P, _I, _I, _I, _F, _P]),
        "eif_cuda_attend_prefill_gated": (_I, [_P, _P, _I, _P, _I, _I, _I, _F, _P, _I, _P, _P]),
        "eif_cuda_attend_prefill_gated_dev": (_I, [_P, _P, _I, _P, _I, _I, _I, _F, _P, _I, _P, _P]),
        "eif_cuda_delta_alloc": (_I, [_P, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_P)]),
        "eif_cuda_delta_free": (None, [_P]),
        "eif_cuda_delta_reset": (_I, [_P, _P]),
        "eif_cuda_delta_upload": (_I, [_P, _P, _I, _I, _P, _P]),
        "eif_cuda_delta_download": (_I, [_P, _P, _I, _I, _P, _P]),
        "eif_cuda_delta_layer_ptrs": (_I, [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
        "eif_cuda_deltanet_step": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _F, _P]),
        "eif_cuda_deltanet_step_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _F, _P]),
        "eif_cuda_delta_set_weights": (_I, [_P, _P, _I, _P, _P, _P, _P]),
        "eif_cuda_deltanet_core": (_I, [_P, _P, _I, _P, _P, _P, _P, _P]),
        "eif_cuda_deltanet_core_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _P]),
        "eif_cuda_deltanet_prefill_core": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P]),
        "eif_cuda_deltanet_prefill_core_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P]),
        "eif_cuda_deltanet_prefill": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _I, _F, _P]),
        "eif_cuda_deltanet_prefill_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _P, _I, _F, _P]),
        "eif_cuda_kv_set_norms": (_I, [_P, _P, _I, _P, _P]),
        "eif_cuda_fullatt_prep": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P, _P]),
        "eif_cuda_fullatt_prep_dev": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _P, _P]),
        "eif_cuda_fullatt_prep_prefill": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P]),
        "eif_cuda_fullatt_prep_prefill_dev": (_I, [_P, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P]),
        "eif_cuda_linear_upload": (_I, [_P, _I, _I, _I, _P, _P, ctypes.POINTER(_P)]),
        "eif_cuda_linear_free": (None, [_P]),
        "eif_cuda_linear_forward": (_I, [_P, _P, _P, _I, _P]),
        "eif_cuda_linear_forward_dev": (_I, [_P, _P, _P, _I, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ptr(a):
    """Host numpy array -> its data address for a void* argument (None passes NULL).  The address comes from
    the array interface rather than a.ctypes, whose per-call object costs microseconds on short calls; the
    caller keeps the array alive across the call."""
    if a is None:
        return None
    return a.__array_interface__["data"][0]


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _out(a, shape):
    """A caller-provided fp32 output array of exactly `shape` (C-contiguous), or a fresh zeroed one."""
    if a is None:
        return np.zeros(shape, np.float32)
    if a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"] or a.shape != tuple(shape):
        raise ValueError(f"output array must be C-contiguous float32 of shape {tuple(shape)}")
    return a


def device_count() -> int:
    return lib().eif_cuda_device_count()


class Context:
    """One device, one stream (eif_cuda_ctx_t).  Not thread-safe, like the engine's eif_gpu context."""

    def __init__(self, device: int = 0):
        self._h = _P()
        st = lib().eif_cuda_init(ctypes.byref(self._h), int(device))
        if st != 0:
            raise EifCudaError(st, f"eif_cuda_init(device={device})")
        self.device = device
        # device objects made on this context; they must be freed before the context itself
        self._children = weakref.WeakSet()

    @property
    def handle(self):
        return self._h

    def check(self, st: int, where: str):
        if st != 0:
            msg = lib().eif_cuda_last_error(self._h)
            raise EifCudaError(st, where, msg.decode() if msg else "")

    def close(self):
        if self._h:
            for c in list(self._children):
                c.free()
            lib().eif_cuda_free(self._h)
            self._h = _P()

    @property
    def alive(self) -> bool:
        return bool(self._h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_handle: int | None):
        self.check(lib().eif_cuda_set_stream(self._h, stream_handle), "set_stream")

    @property
    def stream(self) -> int:
        return lib().eif_cuda_get_stream(self._h) or 0

    def set_timeout(self, ms: int):
        self.check(lib().eif_cuda_set_timeout(self._h, int(ms)), "set_timeout")

    def synchronize(self):
        self.check(lib().eif_cuda_synchronize(self._h), "synchronize")

    @property
    def launch_count(self) -> int:
        return int(lib().eif_cuda_launch_count(self._h))

    @property
    def last_error(self) -> str:
        m = lib().eif_cuda_last_error(self._h)
        return m.decode() if m else ""


class KVCache:
    """Device KV cache (eif_cuda_kv_t): per layer [batch][max_seq_len][n_kv_heads][head_dim]."""

    def __init__(self, ctx: Context, n_layers: int, batch: int, max_seq_len: int, n_kv_heads: int, head_dim: int,
                 dtype: int = F32):
        self.ctx = ctx
        self.n_layers, self.batch, self.max_seq_len = n_layers, batch, max_seq_len
        self.n_kv_heads, self.head_dim, self.dtype = n_kv_heads, head_dim, dtype
        self._h = _P()
        ctx.check(lib().eif_cuda_kv_alloc(ctx.handle, n_layers, batch, max_seq_len, n_kv_heads, head_dim, dtype,
                                          ctypes.byref(self._h)), "kv_alloc")
        ctx._children.add(self)

    @property
    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    def free(self):
        if self._h and self.ctx.alive:
            lib().eif_cuda_kv_free(self._h)
        self._h = _P()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def reset(self):
        self.ctx.check(lib().eif_cuda_kv_reset(self.ctx.handle, self._h), "kv_reset")

    def upload(self, layer: int, seq: int, row0: int, k_rows, v_rows):
        k, v = _f32(k_rows), _f32(v_rows)
        n = k.size // self.kv_dim
        self.ctx.check(lib().eif_cuda_kv_upload(self.ctx.handle, self._h, layer, seq, row0, n, _ptr(k), _ptr(v)),
                       "kv_upload")

    def download(self, layer: int, seq: int, row0: int, n_rows: int):
        k = np.zeros((n_rows, self.kv_dim), np.float32)
        v = np.zeros((n_rows, self.kv_dim), np.float32)
        self.ctx.check(lib().eif_cuda_kv_download(self.ctx.handle, self._h, layer, seq, row0, n_rows, _ptr(k),
                                                  _ptr(v)), "kv_download")
        return k, v

    def layer_ptrs(self, layer: int):
        k, v = _P(), _P()
        self.ctx.check(lib().eif_cuda_kv_layer_ptrs(self._h, layer, ctypes.byref(k), ctypes.byref(v)),
                       "kv_layer_ptrs")
        return k.value, v.value

    def download_int8(self, layer: int, seq: int, row0: int, n_rows: int):
        """INT8 caches: (k_codes, v_codes) int8 [n_rows][kv_dim] and (k_scale, v_scale) fp32 [n_rows][n_kv]."""
        kc = np.zeros((n_rows, self.kv_dim), np.int8)
        vc = np.zeros((n_rows, self.kv_dim), np.int8)
        ks = np.zeros((n_rows, self.n_kv_heads), np.float32)
        vs = np.zeros((n_rows, self.n_kv_heads), np.float32)
        self.ctx.check(lib().eif_cuda_kv_download_int8(self.ctx.handle, self._h, layer, seq, row0, n_rows, _ptr(kc),
                                                       _ptr(vc), _ptr(ks), _ptr(vs)), "kv_download_int8")
        return kc, vc, ks, vs

    def layer_scales(self, layer: int):
        """INT8 caches: device pointers of the layer's K / V scales, head-major [batch][n_kv_heads][stride] fp32,
        stride = max_seq_len rounded up to 64."""
        k, v = _P(), _P()
        self.ctx.check(lib().eif_cuda_kv_layer_scales(self._h, layer, ctypes.byref(k), ctypes.byref(v)),
                       "kv_layer_scales")
        return k.value, v.value

    def append(self, layer: int, pos, k, v):
        p, kk, vv = _i32(pos), _f32(k), _f32(v)
        self.ctx.check(lib().eif_cuda_kv_append(self.ctx.handle, self._h, layer, _ptr(p), _ptr(kk), _ptr(vv)),
                       "kv_append")

    def append_dev(self, layer: int, pos_dev: int, k_dev: int, v_dev: int):
        self.ctx.check(lib().eif_cuda_kv_append_dev(self.ctx.handle, self._h, layer, pos_dev, k_dev, v_dev),
                       "kv_append_dev")

    def set_rope(self, theta: float, interleaved: bool = False):
        """tinyllm RoPE tables of the model's theta; interleaved = adjacent pairs (llama-style)."""
        self.ctx.check(lib().eif_cuda_kv_set_rope(self.ctx.handle, self._h, float(theta), int(bool(interleaved))),
                       "kv_set_rope")

    def rope_append(self, layer: int, q, k, v, pos, n_heads: int, q_out=None):
        """RoPE of q and k at pos[b] and the cache write of k, v: returns the rotated q [batch][n_heads*hd]."""
        qq, kk, vv, pp = _f32(q), _f32(k), _f32(v), _i32(pos)
        out = _out(q_out, (self.batch, n_heads * self.head_dim))
        self.ctx.check(lib().eif_cuda_rope_append(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                  _ptr(pp), n_heads, _ptr(out)), "rope_append")
        return out

    def rope_append_dev(self, layer: int, q_dev, k_dev, v_dev, pos_dev, n_heads: int, q_out_dev):
        self.ctx.check(lib().eif_cuda_rope_append_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev, pos_dev,
                                                      n_heads, q_out_dev), "rope_append_dev")

    def decode_step(self, layer: int, q, k, v, pos, n_heads: int, scale: float, out=None):
        """The whole decode step of the layer (RoPE, the new K / V row at pos[b], attention over [0, pos[b]]):
        returns out [batch][n_heads*hd] (written into `out` when given)."""
        qq, kk, vv, pp = _f32(q), _f32(k), _f32(v), _i32(pos)
        o = _out(out, (self.batch, n_heads * self.head_dim))
        self.ctx.check(lib().eif_cuda_decode_step(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                  _ptr(pp), n_heads, float(scale), _ptr(o)), "decode_step")
        return o

    def decode_step_dev(self, layer: int, q_dev, k_dev, v_dev, pos_dev, max_pos: int, n_heads: int, scale: float,
                        out_dev):
        self.ctx.check(lib().eif_cuda_decode_step_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev, pos_dev,
                                                      int(max_pos), n_heads, float(scale), out_dev), "decode_step_dev")

    def rope_append_prefill(self, layer: int, q, k, v, n_tok: int, start_pos: int, n_heads: int):
        """RoPE + cache write for n_tok tokens per sequence at start_pos + i: returns the rotated q."""
        qq, kk, vv = _f32(q), _f32(k), _f32(v)
        out = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        self.ctx.check(lib().eif_cuda_rope_append_prefill(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk),
                                                          _ptr(vv), n_tok, start_pos, n_heads, _ptr(out)),
                       "rope_append_prefill")
        return out

    def rope_append_prefill_dev(self, layer: int, q_dev, k_dev, v_dev, n_tok: int, start_pos: int, n_heads: int,
                                q_out_dev):
        """q_out as bf16 device array (the prefill attention's input); q / k / v fp32 device arrays."""
        self.ctx.check(lib().eif_cuda_rope_append_prefill_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev,
                                                              n_tok, start_pos, n_heads, q_out_dev),
                       "rope_append_prefill_dev")

    def attend_decode(self, layer: int, q, pos, n_heads: int, scale: float, gate=None, subln: int = SUBLN_NONE,
                      sub_norm=None, out=None):
        """q [batch][n_heads*head_dim] fp32 -> out [batch][n_heads*head_dim] fp32 (written into `out` when
        given, e.g. a pinned host array)."""
        qq, pp = _f32(q), _i32(pos)
        gg = _f32(gate) if gate is not None else None
        nn = _f32(sub_norm) if sub_norm is not None else None
        out = _out(out, (self.batch, n_heads * self.head_dim))
        self.ctx.check(lib().eif_cuda_attend_decode(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(pp), n_heads,
                                                    float(scale), _ptr(gg), int(subln), _ptr(nn), _ptr(out)),
                       "attend_decode")
        return out

    def set_norms(self, layer: int, q_norm, k_norm):
        """Per-layer q_norm / k_norm [head_dim] of the Qwen3.5 attention prep."""
        qn, kn = _f32(q_norm), _f32(k_norm)
        self.ctx.check(lib().eif_cuda_kv_set_norms(self.ctx.handle, self._h, layer, _ptr(qn), _ptr(kn)), "kv_set_norms")

    def fullatt_prep(self, layer: int, qg, k, v, pos, n_heads: int, q_out=None, gate_out=None):
        """fullatt_prep for one token per sequence: returns (q, gate) [batch][n_heads*head_dim] (in q_out /
        gate_out when given); writes k, v (normed and rotated k) into cache row pos[b]."""
        qq, kk, vv, pp = _f32(qg), _f32(k), _f32(v), _i32(pos)
        q = _out(q_out, (self.batch, n_heads * self.head_dim))
        g = _out(gate_out, (self.batch, n_heads * self.head_dim))
        self.ctx.check(lib().eif_cuda_fullatt_prep(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                   _ptr(pp), n_heads, _ptr(q), _ptr(g)), "fullatt_prep")
        return q, g

    def fullatt_prep_dev(self, layer: int, qg_dev, k_dev, v_dev, pos_dev, n_heads: int, q_out_dev, gate_out_dev):
        self.ctx.check(lib().eif_cuda_fullatt_prep_dev(self.ctx.handle, self._h, layer, qg_dev, k_dev, v_dev, pos_dev,
                                                       n_heads, q_out_dev, gate_out_dev), "fullatt_prep_dev")

    def fullatt_prep_prefill(self, layer: int, qg, k, v, n_tok: int, start_pos: int, n_heads: int):
        """fullatt_prep for n_tok tokens per sequence at start_pos + i: returns (q, gate)
        [batch][n_tok][n_heads*head_dim] and writes the chunk's cache rows."""
        qq, kk, vv = _f32(qg), _f32(k), _f32(v)
        q = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        g = np.zeros_like(q)
        self.ctx.check(lib().eif_cuda_fullatt_prep_prefill(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk),
                                                           _ptr(vv), n_tok, start_pos, n_heads, _ptr(q), _ptr(g)),
                       "fullatt_prep_prefill")
        return q, g

    def fullatt_prep_prefill_dev(self, layer: int, qg_dev, k_dev, v_dev, n_tok: int, start_pos: int, n_heads: int,
                                 q_out_dev, gate_out_dev):
        """q_out as bf16 device array; the rest fp32 device arrays; asynchronous."""
        self.ctx.check(lib().eif_cuda_fullatt_prep_prefill_dev(self.ctx.handle, self._h, layer, qg_dev, k_dev, v_dev,
                                                               n_tok, start_pos, n_heads, q_out_dev, gate_out_dev),
                       "fullatt_prep_prefill_dev")

    def attend_prefill(self, layer: int, q, n_tok: int, start_pos: int, n_heads: int, scale: float):
        """Causal prefill: q [batch][n_tok][n_heads*head_dim] fp32 -> out of the same shape (fp32)."""
        qq = _f32(q)
        out = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        self.ctx.check(lib().eif_cuda_attend_prefill(self.ctx.handle, self._h, layer, _ptr(qq), n_tok, start_pos,
                                                     n_heads, float(scale), _ptr(out)), "attend_prefill")
        return out

    def attend_prefill_dev(self, layer: int, q_dev: int, n_tok: int, start_pos: int, n_heads: int, scale: float,
                           out_dev: int):
        """bf16 device arrays [batch][n_tok][n_heads*head_dim]; asynchronous on the context's stream."""
        self.ctx.check(lib().eif_cuda_attend_prefill_dev(self.ctx.handle, self._h, layer, q_dev, n_tok, start_pos,
                                                         n_heads, float(scale), out_dev), "attend_prefill_dev")

    def attend_prefill_gated(self, layer: int, q, n_tok: int, start_pos: int, n_heads: int, scale: float,
                             gate=None, subln: int = SUBLN_NONE, sub_norm=None):
        """Qwen3.5 prefill attention with the output gate and SubLN: fp32 host arrays in and out."""
        qq = _f32(q)
        gg = _f32(gate) if gate is not None else None
        nn = _f32(sub_norm) if sub_norm is not None else None
        out = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        self.ctx.check(lib().eif_cuda_attend_prefill_gated(self.ctx.handle, self._h, layer, _ptr(qq), n_tok, start_pos,
                                                           n_heads, float(scale), _ptr(gg), int(subln), _ptr(nn),
                                                           _ptr(out)), "attend_prefill_gated")
        return out

    def attend_prefill_gated_dev(self, layer: int, q_dev: int, n_tok: int, start_pos: int, n_heads: int,
                                 scale: float, out_dev: int, gate_dev: int | None = None, subln: int = SUBLN_NONE,
                                 sub_norm_dev: int | None = None):
        """q bf16, gate / sub_norm / out fp32 device arrays; asynchronous on the context's stream."""
        self.ctx.check(lib().eif_cuda_attend_prefill_gated_dev(self.ctx.handle, self._h, layer, q_dev, n_tok, start_pos,
                                                               n_heads, float(scale), gate_dev, int(subln),
                                                               sub_norm_dev, out_dev), "attend_prefill_gated_dev")

    def decode_plan(self, layer: int, n_heads: int, max_pos: int, noalloc: bool = False):
        """(key chunks per (sequence, kv head), keys per chunk, scratch bytes) of decode attention's split."""
        nc, ck, wb = _I(), _I(), ctypes.c_size_t()
        self.ctx.check(lib().eif_cuda_attend_decode_plan(self.ctx.handle, self._h, layer, n_heads, int(max_pos),
                                                         int(bool(noalloc)), ctypes.byref(nc), ctypes.byref(ck),
                                                         ctypes.byref(wb)), "attend_decode_plan")
        return nc.value, ck.value, wb.value

    def fullatt_decode(self, layer: int, qg, k, v, pos, n_heads: int, scale: float, subln: int = SUBLN_NONE,
                       sub_norm=None, out=None):
        """The Qwen3.5 attention mixer of one token (fullatt_prep + fullatt_attend) from host arrays."""
        qq, kk, vv, pp = _f32(qg), _f32(k), _f32(v), _i32(pos)
        nn = _f32(sub_norm) if sub_norm is not None else None
        o = _out(out, (self.batch, n_heads * self.head_dim))
        self.ctx.check(lib().eif_cuda_fullatt_decode(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                     _ptr(pp), n_heads, float(scale), int(subln), _ptr(nn), _ptr(o)),
                       "fullatt_decode")
        return o

    def fullatt_prefill(self, layer: int, qg, k, v, n_tok: int, start_pos: int, n_heads: int, scale: float,
                        subln: int = SUBLN_NONE, sub_norm=None):
        """The Qwen3.5 attention block of a prefill chunk (fullatt_prep + gated causal attention), host arrays."""
        qq, kk, vv = _f32(qg), _f32(k), _f32(v)
        nn = _f32(sub_norm) if sub_norm is not None else None
        o = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        self.ctx.check(lib().eif_cuda_fullatt_prefill(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                      n_tok, start_pos, n_heads, float(scale), int(subln), _ptr(nn),
                                                      _ptr(o)), "fullatt_prefill")
        return o

    def fullatt_prefill_dev(self, layer: int, qg_dev, k_dev, v_dev, n_tok: int, start_pos: int, n_heads: int,
                            scale: float, out_dev, subln: int = SUBLN_NONE, sub_norm_dev=None):
        self.ctx.check(lib().eif_cuda_fullatt_prefill_dev(self.ctx.handle, self._h, layer, qg_dev, k_dev, v_dev, n_tok,
                                                          start_pos, n_heads, float(scale), int(subln), sub_norm_dev,
                                                          out_dev), "fullatt_prefill_dev")

    def prefill_step(self, layer: int, q, k, v, n_tok: int, start_pos: int, n_heads: int, scale: float):
        """The tinyllm attention block of a prefill chunk (RoPE, cache writes, causal attention), host arrays."""
        qq, kk, vv = _f32(q), _f32(k), _f32(v)
        o = np.zeros((self.batch, n_tok, n_heads * self.head_dim), np.float32)
        self.ctx.check(lib().eif_cuda_prefill_step(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv), n_tok,
                                                   start_pos, n_heads, float(scale), _ptr(o)), "prefill_step")
        return o

    def prefill_step_dev(self, layer: int, q_dev, k_dev, v_dev, n_tok: int, start_pos: int, n_heads: int,
                         scale: float, out_dev):
        self.ctx.check(lib().eif_cuda_prefill_step_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev, n_tok,
                                                       start_pos, n_heads, float(scale), out_dev), "prefill_step_dev")

    def fullatt_decode_dev(self, layer: int, qg_dev, k_dev, v_dev, pos_dev, max_pos: int, n_heads: int,
                           scale: float, out_dev, subln: int = SUBLN_NONE, sub_norm_dev=None):
        self.ctx.check(lib().eif_cuda_fullatt_decode_dev(self.ctx.handle, self._h, layer, qg_dev, k_dev, v_dev,
                                                         pos_dev, int(max_pos), n_heads, float(scale), int(subln),
                                                         sub_norm_dev, out_dev), "fullatt_decode_dev")

    def attend_decode_dev(self, layer: int, q_dev: int, pos_dev: int, max_pos: int, n_heads: int, scale: float,
                          out_dev: int, gate_dev: int | None = None, subln: int = SUBLN_NONE,
                          sub_norm_dev: int | None = None):
        self.ctx.check(lib().eif_cuda_attend_decode_dev(self.ctx.handle, self._h, layer, q_dev, pos_dev, int(max_pos),
                                                        n_heads, float(scale), gate_dev, int(subln), sub_norm_dev,
                                                        out_dev), "attend_decode_dev")


class DeltaState:
    """Device DeltaNet states (eif_cuda_delta_t): per layer S [batch][H][d_k][d_v] and conv windows."""

    def __init__(self, ctx: Context, n_layers: int, batch: int, n_heads: int, d_k: int, d_v: int, conv_k: int = 0):
        self.ctx = ctx
        self.n_layers, self.batch, self.H, self.dk, self.dv, self.conv_k = n_layers, batch, n_heads, d_k, d_v, conv_k
        self.conv_dim = 2 * n_heads * d_k + n_heads * d_v
        self._h = _P()
        ctx.check(lib().eif_cuda_delta_alloc(ctx.handle, n_layers, batch, n_heads, d_k, d_v, conv_k,
                                             ctypes.byref(self._h)), "delta_alloc")
        ctx._children.add(self)

    def free(self):
        if self._h and self.ctx.alive:
            lib().eif_cuda_delta_free(self._h)
        self._h = _P()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def reset(self):
        self.ctx.check(lib().eif_cuda_delta_reset(self.ctx.handle, self._h), "delta_reset")

    def upload(self, layer: int, seq: int, S=None, conv_state=None):
        s = _f32(S) if S is not None else None
        c = _f32(conv_state) if conv_state is not None else None
        self.ctx.check(lib().eif_cuda_delta_upload(self.ctx.handle, self._h, layer, seq, _ptr(s), _ptr(c)),
                       "delta_upload")

    def download(self, layer: int, seq: int):
        S = np.zeros((self.H, self.dk, self.dv), np.float32)
        c = np.zeros((self.conv_dim, self.conv_k), np.float32) if self.conv_k else None
        self.ctx.check(lib().eif_cuda_delta_download(self.ctx.handle, self._h, layer, seq, _ptr(S), _ptr(c)),
                       "delta_download")
        return S, c

    def layer_ptrs(self, layer: int):
        s, c = _P(), _P()
        self.ctx.check(lib().eif_cuda_delta_layer_ptrs(self._h, layer, ctypes.byref(s), ctypes.byref(c)),
                       "delta_layer_ptrs")
        return s.value, c.value

    def step(self, layer: int, q, k, v, beta, g, q_scale: float, out=None):
        """One token of the delta rule for every sequence: returns o [batch][H*d_v] (written into `out` when
        given, e.g. a pinned host array)."""
        qq, kk, vv, bb, gg = _f32(q), _f32(k), _f32(v), _f32(beta), _f32(g)
        o = _out(out, (self.batch, self.H * self.dv))
        self.ctx.check(lib().eif_cuda_deltanet_step(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                    _ptr(bb), _ptr(gg), float(q_scale), _ptr(o)), "deltanet_step")
        return o

    def set_weights(self, layer: int, conv_w, dt_bias, A_log, norm_w):
        """Per-layer weights of deltanet_core: conv_w [conv_dim][conv_k], dt_bias [H], A_log [H], norm_w [d_v]."""
        a = [_f32(x) for x in (conv_w, dt_bias, A_log, norm_w)]
        self.ctx.check(lib().eif_cuda_delta_set_weights(self.ctx.handle, self._h, layer, *[_ptr(x) for x in a]),
                       "delta_set_weights")

    def core(self, layer: int, qkv, z, b_raw, a_raw, out=None):
        """deltanet_core for one token of every sequence: returns out [batch][H*d_v] (written into `out`
        when given, e.g. a pinned host array)."""
        a = [_f32(x) for x in (qkv, z, b_raw, a_raw)]
        out = _out(out, (self.batch, self.H * self.dv))
        self.ctx.check(lib().eif_cuda_deltanet_core(self.ctx.handle, self._h, layer, *[_ptr(x) for x in a], _ptr(out)),
                       "deltanet_core")
        return out

    def core_dev(self, layer: int, qkv_dev, z_dev, b_dev, a_dev, out_dev):
        self.ctx.check(lib().eif_cuda_deltanet_core_dev(self.ctx.handle, self._h, layer, qkv_dev, z_dev, b_dev, a_dev,
                                                        out_dev), "deltanet_core_dev")

    def prefill_core(self, layer: int, qkv, z, b_raw, a_raw):
        """deltanet_core over a chunk of n_tok tokens per sequence (qkv [batch][n_tok][conv_dim], z
        [batch][n_tok][H*d_v], b, a [batch][n_tok][H]); returns out [batch][n_tok][H*d_v]."""
        a = [_f32(x) for x in (qkv, z, b_raw, a_raw)]
        n_tok = a[0].shape[1]
        out = np.zeros((self.batch, n_tok, self.H * self.dv), np.float32)
        self.ctx.check(lib().eif_cuda_deltanet_prefill_core(self.ctx.handle, self._h, layer, *[_ptr(x) for x in a],
                                                            n_tok, _ptr(out)), "deltanet_prefill_core")
        return out

    def prefill_core_dev(self, layer: int, qkv_dev, z_dev, b_dev, a_dev, n_tok: int, out_dev):
        self.ctx.check(lib().eif_cuda_deltanet_prefill_core_dev(self.ctx.handle, self._h, layer, qkv_dev, z_dev, b_dev,
                                                                a_dev, n_tok, out_dev), "deltanet_prefill_core_dev")

    def prefill(self, layer: int, q, k, v, beta, g, q_scale: float, out=None):
        """Chunked prefill of n_tok tokens per sequence (fp32 host arrays; q, k [batch][n_tok][H][d_k],
        v [batch][n_tok][H][d_v], beta, g [batch][n_tok][H]); returns o [batch][n_tok][H][d_v] (in `out`
        when given)."""
        qq, kk, vv, bb, gg = (_f32(x) for x in (q, k, v, beta, g))
        n_tok = qq.shape[1]
        o = _out(out, (self.batch, n_tok, self.H, self.dv))
        self.ctx.check(lib().eif_cuda_deltanet_prefill(self.ctx.handle, self._h, layer, _ptr(qq), _ptr(kk), _ptr(vv),
                                                       _ptr(bb), _ptr(gg), n_tok, float(q_scale), _ptr(o)),
                       "deltanet_prefill")
        return o

    def prefill_dev(self, layer: int, q_dev, k_dev, v_dev, beta_dev, g_dev, n_tok: int, q_scale: float, o_dev):
        self.ctx.check(lib().eif_cuda_deltanet_prefill_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev,
                                                           beta_dev, g_dev, n_tok, float(q_scale), o_dev),
                       "deltanet_prefill_dev")

    def step_dev(self, layer: int, q_dev, k_dev, v_dev, beta_dev, g_dev, q_scale: float, o_dev):
        self.ctx.check(lib().eif_cuda_deltanet_step_dev(self.ctx.handle, self._h, layer, q_dev, k_dev, v_dev,
                                                        beta_dev, g_dev, float(q_scale), o_dev), "deltanet_step_dev")


def packed_row_bytes(cols: int, wtype: int) -> int:
    """Bytes of one packed weight row of the format (row_bytes, src/eif_qwen35.c:110-116; INT8 a byte a weight)."""
    return {W_F32: 4 * cols, W_INT4: (cols + 1) // 2, W_TERNARY2: (cols + 3) // 4,
            W_TERNARY_DENSE: (cols + 4) // 5}.get(wtype, cols)


class Linear:
    """A projection's weights resident on the device (eif_cuda_linear_t): linear_gemv / linear_gemm / int8_gemv
    (src/eif_qwen35.c:384-443, 1033-1063) on the GPU.  `quant_type` is the engine's packed quant type (base in the
    low byte, the 2-bit ternary scale group in the bits above); W is the engine's packed rows (uint8, rows x
    row_bytes) and scales its fp32 scales (None for fp32 weights)."""

    def __init__(self, ctx: Context, quant_type: int, rows: int, cols: int, W, scales=None):
        self.ctx, self.quant_type, self.rows, self.cols = ctx, int(quant_type), int(rows), int(cols)
        w = np.ascontiguousarray(W).view(np.uint8)
        need = rows * packed_row_bytes(cols, quant_type & 0xFF)
        if (quant_type & 0xFF) <= W_INT8 and w.size != need:  # an unknown format is the library's to reject
            raise ValueError(f"W holds {w.size} bytes, the format needs {need}")
        sc = _f32(scales) if scales is not None else None
        self._h = _P()
        ctx.check(lib().eif_cuda_linear_upload(ctx.handle, self.quant_type, self.rows, self.cols, _ptr(w), _ptr(sc),
                                               ctypes.byref(self._h)), "linear_upload")
        ctx._children.add(self)

    def free(self):
        if self._h and self.ctx.alive:
            lib().eif_cuda_linear_free(self._h)
        self._h = _P()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def forward(self, x, out=None):
        """out [n][rows] = W x[t] for x [n][cols] (fp32 host arrays; a 1-D x is one token)."""
        xx = _f32(x).reshape(-1, self.cols)
        o = _out(out, (xx.shape[0], self.rows))
        self.ctx.check(lib().eif_cuda_linear_forward(self.ctx.handle, self._h, _ptr(xx), xx.shape[0], _ptr(o)),
                       "linear_forward")
        return o

    def forward_dev(self, x_dev, n: int, out_dev):
        self.ctx.check(lib().eif_cuda_linear_forward_dev(self.ctx.handle, self._h, x_dev, int(n), out_dev),
                       "linear_forward_dev")
