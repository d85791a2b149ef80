"""ctypes front-end to the CPU checker (TEST INFRASTRUCTURE ONLY).

Two libraries live under oracle/:
  * liboracle.so           -- oracle.c, the C restatement ("port") of the reference hot path;
  * _ref/libbitllm_ref.so  -- the reference's own src/eif_qwen35.c compiled from its sources
                              (built only where the reference tree is present).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import this module; the
product (libeif_cuda.so and its Python host mirror) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libbitllm_ref.so")

_F = ctypes.POINTER(ctypes.c_float)
_I8 = ctypes.POINTER(ctypes.c_int8)
_port = None
_ref = None


def build(ref: bool = False) -> None:
    """Compile the port (and, when asked and the reference tree exists, the reference shim)."""
    targets = ["all"]
    if ref:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "oracle buffers are contiguous float32"
    return a.ctypes.data_as(_F)


def port():
    """The C restatement (liboracle.so), built on first use if missing."""
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(ref=False)
        _port = ctypes.CDLL(PORT_SO)
        i, f = ctypes.c_int, ctypes.c_float
        _port.orc_deltanet_rule.argtypes = [_F, _F, _F, _F, _F, _F, f, _F, i, i, i]
        _port.orc_deltanet_core.argtypes = [_F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _F, i, i, i, i]
        _port.orc_attend_decode.argtypes = [_F, _F, _F, i, i, i, i, f, _F, _F]
        _port.orc_subln.argtypes = [_F, _F, i, i]
        _port.orc_attend_prefill.argtypes = [_F, _F, _F, i, i, i, i, i, f, _F]
        _port.orc_rope_table.argtypes = [i, i, f, _F, _F]
        _port.orc_rope_apply.argtypes = [_F, i, i, _F, _F, i]
        _port.orc_rope_partial.argtypes = [_F, i, i, i]
        _port.orc_fullatt_prep.argtypes = [_F, _F, _F, _F, _F, _F, _F, _F, _F, i, i, i, i]
        _port.orc_round_bf16.argtypes = [_F, ctypes.c_size_t]
        _port.orc_kv_quantize.argtypes = [_F, i, i, _I8, _F]
        _port.orc_attend_decode_i8.argtypes = [_F, _I8, _F, _I8, _F, i, i, i, i, f, _F]
        _port.orc_linear.argtypes = [_F, ctypes.c_void_p, _F, _F, i, i, i, i]
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own code (oracle/_ref/libbitllm_ref.so); raises if it was not built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError("oracle/_ref/libbitllm_ref.so not built (needs the reference tree)")
        _ref = ctypes.CDLL(REF_SO)
        i = ctypes.c_int
        _ref.ref_deltanet_core.argtypes = [_F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _F, i, i, i, i]
        _ref.ref_fullatt_prep.argtypes = [_F, _F, _F, _F, _F, _F, _F, _F, _F, i, i, i, i]
        _ref.ref_fullatt_attend.argtypes = [_F, _F, _F, _F, _F, _F, i, i, i, i, i]
        _ref.ref_omp_threads.restype = i
        _ref.ref_tinyllm_decode_steps.argtypes = [i, i, i, i, ctypes.c_float, i, i, i, _F, _F, _F, _F, _F, _F,
                                                  _I8, _I8, _F, _F, _F]
        _ref.ref_tinyllm_decode_steps.restype = i
        _ref.ref_tinyllm_decode_time.argtypes = [i, i, i, i, ctypes.c_float, i, i, i]
        _ref.ref_tinyllm_decode_time.restype = ctypes.c_double
        _ref.ref_set_threads.argtypes = [i]
        _ref.ref_linear.argtypes = [_F, ctypes.c_void_p, _F, _F, i, i, i, i]
        _ref.ref_linear_time.argtypes = [_F, ctypes.c_void_p, _F, _F, i, i, i, i, i]
        _ref.ref_linear_time.restype = ctypes.c_double
    return _ref


def c32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------------------------------------
# Port wrappers (numpy in, numpy out; inputs are not modified unless stated)
# ------------------------------------------------------------------------------------------------

def deltanet_rule(S, q, k, v, beta, g, q_scale):
    """One token, one sequence: S [H,dk,dv] is updated IN PLACE; returns o [H*dv]."""
    H, dk, dv = S.shape
    o = np.zeros(H * dv, np.float32)
    port().orc_deltanet_rule(_fp(S), _fp(c32(q)), _fp(c32(k)), _fp(c32(v)), _fp(c32(beta)), _fp(c32(g)),
                             float(q_scale), _fp(o), H, dk, dv)
    return o


def deltanet_core(qkv_raw, z, b_raw, a_raw, conv_state, S, conv_w, dt_bias, A_log, norm_w, lib=None):
    """deltanet_core on one token; conv_state and S are updated IN PLACE; returns out [H*dv].

    lib=None uses the port; lib=ref() runs the reference's own function."""
    H, dk, dv = S.shape
    conv_k = conv_state.shape[-1]
    qkv = c32(qkv_raw).copy()
    out = np.zeros(H * dv, np.float32)
    args = (_fp(qkv), _fp(c32(z).copy()), _fp(c32(b_raw).copy()), _fp(c32(a_raw).copy()), _fp(conv_state), _fp(S),
            _fp(c32(conv_w)), _fp(c32(dt_bias)), _fp(c32(A_log)), _fp(c32(norm_w)), _fp(out), H, dk, dv, conv_k)
    if lib is None:
        port().orc_deltanet_core(*args)
    else:
        lib.ref_deltanet_core(*args)
    return out


def attend_decode(q, k_cache, v_cache, pos, nh, nkv, hd, scale, gate=None):
    out = np.zeros(nh * hd, np.float32)
    port().orc_attend_decode(_fp(c32(q)), _fp(c32(k_cache)), _fp(c32(v_cache)), int(pos), nh, nkv, hd, float(scale),
                             _fp(c32(gate)) if gate is not None else None, _fp(out))
    return out


def subln(x, sub_norm, mode):
    y = c32(x).copy()
    port().orc_subln(_fp(y), _fp(c32(sub_norm)) if sub_norm is not None else None, int(mode), y.size)
    return y


def attend_prefill(q, k_cache, v_cache, n_tok, start_pos, nh, nkv, hd, scale):
    out = np.zeros((n_tok, nh * hd), np.float32)
    port().orc_attend_prefill(_fp(c32(q)), _fp(c32(k_cache)), _fp(c32(v_cache)), n_tok, start_pos, nh, nkv, hd,
                              float(scale), _fp(out))
    return out


def rope_table(pos, hd, theta):
    c = np.zeros(hd // 2, np.float32)
    s = np.zeros(hd // 2, np.float32)
    port().orc_rope_table(int(pos), hd, float(theta), _fp(c), _fp(s))
    return c, s


def rope_apply(x, n_heads, hd, pos, theta, interleaved=False):
    """tinyllm RoPE of x [n_heads*hd] at pos (returns a rotated copy)."""
    c, s = rope_table(pos, hd, theta)
    y = c32(x).copy()
    port().orc_rope_apply(_fp(y), n_heads, hd, _fp(c), _fp(s), int(bool(interleaved)))
    return y


def rope_partial(x, pos, n_heads, hd):
    y = c32(x).copy()
    port().orc_rope_partial(_fp(y), int(pos), n_heads, hd)
    return y


def fullatt_prep(qg, k, v, q_norm, k_norm, k_cache, v_cache, pos, nh, nkv, hd, lib=None):
    """Returns (q, gate, k_rotated); writes cache row pos IN PLACE."""
    q = np.zeros(nh * hd, np.float32)
    gate = np.zeros(nh * hd, np.float32)
    kk = c32(k).copy()
    args = (_fp(c32(qg)), _fp(kk), _fp(c32(v)), _fp(q), _fp(gate), _fp(c32(q_norm)), _fp(c32(k_norm)),
            _fp(k_cache), _fp(v_cache), int(pos), nh, nkv, hd)
    if lib is None:
        port().orc_fullatt_prep(*args)
    else:
        lib.ref_fullatt_prep(*args)
    return q, gate, kk


def ref_fullatt_attend(q, gate, k_cache, v_cache, sub_norm, plain_linear, pos, nh, nkv, hd):
    """The reference's fullatt_attend (needs oracle/_ref)."""
    o = np.zeros(nh * hd, np.float32)
    ref().ref_fullatt_attend(_fp(c32(q)), _fp(c32(gate)), _fp(o), _fp(k_cache), _fp(v_cache),
                             _fp(c32(sub_norm)) if sub_norm is not None else None, int(plain_linear), int(pos),
                             nh, nkv, hd)
    return o


def _i8p(a):
    assert a.dtype == np.int8 and a.flags["C_CONTIGUOUS"], "oracle code buffers are contiguous int8"
    return a.ctypes.data_as(_I8)


def kv_quantize(x, nkv, hd):
    """tinyllm INT8 cache write of rows x [..., nkv*hd]: returns (codes int8 [..., nkv*hd], scales [..., nkv])."""
    x = c32(x)
    rows = x.reshape(-1, nkv * hd)
    codes = np.zeros(rows.shape, np.int8)
    scales = np.zeros((rows.shape[0], nkv), np.float32)
    for r in range(rows.shape[0]):
        port().orc_kv_quantize(_fp(c32(rows[r])), nkv, hd, _i8p(codes[r]), _fp(scales[r]))
    return codes.reshape(x.shape), scales.reshape(x.shape[:-1] + (nkv,))


def attend_decode_i8(q, k_codes, k_scale, v_codes, v_scale, pos, nh, nkv, hd, scale):
    """tinyllm decode attention of one token over INT8 cache rows [0, pos]."""
    out = np.zeros(nh * hd, np.float32)
    port().orc_attend_decode_i8(_fp(c32(q)), _i8p(np.ascontiguousarray(k_codes, np.int8)), _fp(c32(k_scale)),
                                _i8p(np.ascontiguousarray(v_codes, np.int8)), _fp(c32(v_scale)), int(pos), nh, nkv,
                                hd, float(scale), _fp(out))
    return out


def ref_tinyllm_decode_steps(q, k, v, nh, nkv, hd, seq_len, theta, interleaved, kv_type):
    """The reference's own tinyllm forward over len(q) decode steps (oracle/ref_shim.c); needs oracle/_ref.

    Returns a dict of per-step arrays: q_rot, k_row, v_row, (INT8) k_codes, v_codes, k_scale, v_scale, attn."""
    n = q.shape[0]
    o = dict(q_rot=np.zeros((n, nh * hd), np.float32), k_row=np.zeros((n, nkv * hd), np.float32),
             v_row=np.zeros((n, nkv * hd), np.float32), k_codes=np.zeros((n, nkv * hd), np.int8),
             v_codes=np.zeros((n, nkv * hd), np.int8), k_scale=np.zeros((n, nkv), np.float32),
             v_scale=np.zeros((n, nkv), np.float32), attn=np.zeros((n, nh * hd), np.float32))
    rc = ref().ref_tinyllm_decode_steps(nh, nkv, hd, seq_len, float(theta), int(interleaved), int(kv_type), n,
                                        _fp(c32(q)), _fp(c32(k)), _fp(c32(v)), _fp(o["q_rot"]), _fp(o["k_row"]),
                                        _fp(o["v_row"]), _i8p(o["k_codes"]), _i8p(o["v_codes"]), _fp(o["k_scale"]),
                                        _fp(o["v_scale"]), _fp(o["attn"]))
    if rc != 0:
        raise RuntimeError("the reference rejected the tinyllm configuration")
    return o


def ref_tinyllm_decode_time(nh, nkv, hd, seq_len, theta, kv_type, pos, n_steps):
    """Seconds the reference's own tinyllm forward takes for n_steps decode steps at position pos over a
    pre-filled fp32 (kv_type 0) or INT8 (kv_type 1) cache (oracle/ref_shim.c); needs oracle/_ref."""
    t = ref().ref_tinyllm_decode_time(nh, nkv, hd, seq_len, float(theta), int(kv_type), int(pos), int(n_steps))
    if t < 0:
        raise RuntimeError("the reference rejected the tinyllm configuration")
    return t


def round_bf16(x):
    y = c32(x).copy()
    port().orc_round_bf16(_fp(y), y.size)
    return y


def deltanet_core_bf16_rule(qkv_raw, z, b_raw, a_raw, conv_state, S, conv_w, dt_bias, A_log, norm_w):
    """deltanet_core over consecutive tokens with the rule's q / k / v rounded to bf16: the recurrent
    reference "on the same bf16-rounded inputs" for a path whose rule runs on bf16 operands.

    The steps around the rule follow src/eif_qwen35.c in float64: causal conv1d over the conv_k window +
    SiLU (:560-572), L2 norms with eps 1e-12 and q scaled by 1/sqrt(d_k) (:579-585), beta = sigmoid(b),
    g = -exp(A_log) softplus(a + dt_bias) (:587-592); q / k / v are then rounded to bf16 and the port's rule
    (:594-639) runs token by token in fp32; the gated RMSNorm (:642-653) closes in float64.
    qkv_raw [T][conv_dim], z [T][H*dv], b_raw / a_raw [T][H]; conv_state [conv_dim][conv_k] and S [H][dk][dv]
    are updated IN PLACE; returns out [T][H*dv]."""
    H, dk, dv = S.shape
    T, conv_dim = qkv_raw.shape
    ck = conv_state.shape[-1]
    silu = lambda x: x / (1.0 + np.exp(-x))  # noqa: E731
    win = np.concatenate([conv_state.T.astype(np.float64), np.asarray(qkv_raw, np.float64)], 0)
    y = np.stack([silu((win[t + 1:t + 1 + ck] * np.asarray(conv_w, np.float64).T).sum(0)) for t in range(T)])
    conv_state[:] = win[T:T + ck].T if T >= ck else win[T:].T
    q = y[:, :H * dk].reshape(T, H, dk)
    k = y[:, H * dk:2 * H * dk].reshape(T, H, dk)
    v = y[:, 2 * H * dk:].reshape(T, H, dv)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-12) / np.sqrt(dk)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-12)
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b_raw, np.float64)))
    g = -np.exp(np.asarray(A_log, np.float64)) * np.log1p(np.exp(np.asarray(a_raw, np.float64) + dt_bias))
    out = np.zeros((T, H * dv), np.float32)
    zz = np.asarray(z, np.float64).reshape(T, H, dv)
    for t in range(T):
        o = deltanet_rule(S, round_bf16(q[t]).ravel(), round_bf16(k[t]).ravel(), round_bf16(v[t]).ravel(),
                          beta[t].astype(np.float32), g[t].astype(np.float32), 1.0).reshape(H, dv).astype(np.float64)
        o = o / np.sqrt((o * o).mean(-1, keepdims=True) + 1e-6) * np.asarray(norm_w, np.float64) * silu(zz[t])
        out[t] = o.ravel()
    return out


# ------------------------------------------------------------------------------------------------
# Projections: the engine's packed weight rows (src/eif_qwen35.c:110-116) and linear_gemv / linear_gemm /
# int8_gemv (src/eif_qwen35.c:384-443, 1033-1063)
# ------------------------------------------------------------------------------------------------

W_F32, W_INT4, W_TERNARY2, W_TERNARY_DENSE, W_INT8 = 0, 1, 2, 3, 4


def row_bytes(cols, base):
    return {0: 4 * cols, 1: (cols + 1) // 2, 2: (cols + 3) // 4, 3: (cols + 4) // 5}.get(base, cols)


def pack_weights(values, base, rng=None):
    """Pack a [rows][cols] array of weight values into the engine's row layout of quant type `base`:
    fp32 values as they are; INT4 values in [-8, 7] (even column in the high nibble, value + 8); 2-bit ternary
    values in {-1, 0, 1} (column c at bits 2(c mod 4), +1 -> code 1, -1 -> code 2, 0 -> code 0, or code 3 at
    random when `rng` is given: the reference reads code 3 as 0); dense ternary in {-1, 0, 1} (five base-3 digits
    a byte, least significant first, +1 -> 1, -1 -> 2); INT8 values in [-128, 127]."""
    v = np.asarray(values)
    rows, cols = v.shape
    if base == 0:
        return np.ascontiguousarray(v, dtype=np.float32).view(np.uint8).reshape(rows, 4 * cols)
    if base == 4:
        return np.ascontiguousarray(v.astype(np.int8)).view(np.uint8)
    out = np.zeros((rows, row_bytes(cols, base)), dtype=np.uint8)
    vi = v.astype(np.int64)
    if base == 1:
        nib = (vi + 8).astype(np.uint8)
        out[:, :] = 0
        out[:, : (cols + 1) // 2] |= (nib[:, 0::2] << 4).astype(np.uint8)
        out[:, : cols // 2] |= nib[:, 1::2]
        return out
    if base == 2:
        code = np.where(vi == 1, 1, np.where(vi == -1, 2, 0)).astype(np.uint8)
        if rng is not None:
            code = np.where((vi == 0) & (rng.random(vi.shape) < 0.5), 3, code).astype(np.uint8)
        for q in range(4):
            part = code[:, q::4]
            out[:, : part.shape[1]] |= (part << (2 * q)).astype(np.uint8)
        return out
    digit = np.where(vi == 1, 1, np.where(vi == -1, 2, 0)).astype(np.int64)
    acc = np.zeros((rows, out.shape[1]), dtype=np.int64)
    for p in range(5):
        part = digit[:, p::5]
        acc[:, : part.shape[1]] += part * 3 ** p
    return acc.astype(np.uint8)


def _linear_call(fn, W, scales, x, rows, cols, quant_type):
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = c32(x).reshape(-1, cols)
    sc = None if scales is None else c32(scales)
    out = np.zeros((x.shape[0], rows), dtype=np.float32)
    fn(_fp(out), W.ctypes.data_as(ctypes.c_void_p), _fp(sc), _fp(x), x.shape[0], rows, cols, quant_type)
    return out


def linear(W, scales, x, rows, cols, quant_type):
    """out[n][rows] = W x[t] (the port of linear_gemv / int8_gemv in each kernel's scalar order)."""
    return _linear_call(port().orc_linear, W, scales, x, rows, cols, quant_type)


def ref_linear(W, scales, x, rows, cols, quant_type):
    """The reference's own linear_gemv (one token), linear_gemm (several) or int8_gemv (quant type 4)."""
    return _linear_call(ref().ref_linear, W, scales, x, rows, cols, quant_type)


def ref_linear_time(W, scales, x, rows, cols, quant_type, reps):
    """Seconds the reference's projection takes for `reps` calls on these inputs."""
    W = np.ascontiguousarray(W, dtype=np.uint8)
    x = c32(x).reshape(-1, cols)
    sc = None if scales is None else c32(scales)
    out = np.zeros((x.shape[0], rows), dtype=np.float32)
    return ref().ref_linear_time(_fp(out), W.ctypes.data_as(ctypes.c_void_p), _fp(sc), _fp(x), x.shape[0], rows,
                                 cols, quant_type, reps)
