"""Generate the golden fixtures of the hot path from the REFERENCE's own code.

Run in a container that holds the reference tree (the fixtures are committed; the GPU box never
runs this script):

    make -C oracle all ref            # builds oracle/_ref/libbitllm_ref.so from the reference sources
    python tests/golden/gen_golden.py

Every fixture stores its seeded inputs and the outputs of the reference function named in it, so
the tests can check both the C restatement (oracle/oracle.c) and the CUDA kernels against the
reference without the reference being present.

  deltanet_core_*.npz   deltanet_core          src/eif_qwen35.c:546-656  (several tokens in a row)
  fullatt_prep.npz      fullatt_prep           src/eif_qwen35.c:699-737
  fullatt_attend.npz    fullatt_attend         src/eif_qwen35.c:741-790  (gate + SubLN, and plain)
  decode_cfg1.npz       fullatt_attend, gate=+100 (sigmoid == 1.0f), plain: the ungated GQA core at
                        the Qwen2.5-0.5B decode shape of BASELINE config 1, RoPE (NeoX, theta 1e6)
                        applied by the tinyllm restatement before the cache is filled
  prefill_small.npz     fullatt_attend per token with the causal bound pos = start_pos + i, which is
                        what tinyllm_forward_batch_embeddings (src/eif_tinyllm.c:1158-1268) computes
  tinyllm_*.npz         tinyllm_forward_embedding_ex (src/eif_tinyllm.c:371-857) over consecutive decode
                        steps of a one-layer model whose attention is observable (oracle/ref_shim.c,
                        ref_tinyllm_decode_steps): RoPE (:481-507), the cache write -- fp32, or INT8 codes
                        and scales (:509-553) -- and the attention output (:555-656)
  linear_formats.npz    linear_gemv (one token) and linear_gemm (several) of src/eif_qwen35.c:422-443, 1033-1063
                        for every weight format -- fp32, INT4, 2-bit ternary (a scale a row, and grouped
                        scales; code-3 bytes included), dense base-3 ternary -- and int8_gemv (:384-420),
                        at ragged widths (cols not a multiple of the weights a byte)

    python tests/golden/gen_golden.py [fixture-name ...]   # default: every fixture
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))
from oracle import oracle as orc  # noqa: E402

GATE_ONE = 100.0  # 1/(1+expf(-100)) rounds to exactly 1.0f


def gen_deltanet_core(name, seed, H, dk, dv, conv_k, n_steps):
    rng = np.random.default_rng(seed)
    conv_dim = 2 * H * dk + H * dv
    S0 = (rng.standard_normal((H, dk, dv)) * 0.02).astype(np.float32)
    conv0 = rng.standard_normal((conv_dim, conv_k)).astype(np.float32)
    conv_w = (rng.standard_normal((conv_dim, conv_k)) * 0.5).astype(np.float32)
    dt_bias = rng.standard_normal(H).astype(np.float32)
    A_log = (rng.standard_normal(H) * 0.5).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(dv)).astype(np.float32)
    qkv = rng.standard_normal((n_steps, conv_dim)).astype(np.float32)
    z = rng.standard_normal((n_steps, H * dv)).astype(np.float32)
    b = rng.standard_normal((n_steps, H)).astype(np.float32)
    a = rng.standard_normal((n_steps, H)).astype(np.float32)
    S = S0.copy()
    conv = conv0.copy()
    outs = []
    lib = orc.ref()
    for t in range(n_steps):
        outs.append(orc.deltanet_core(qkv[t], z[t], b[t], a[t], conv, S, conv_w, dt_bias, A_log, norm_w, lib=lib))
    np.savez(os.path.join(HERE, name), S0=S0, conv0=conv0, conv_w=conv_w, dt_bias=dt_bias, A_log=A_log,
             norm_w=norm_w, qkv=qkv, z=z, b=b, a=a, out=np.stack(outs), S_final=S, conv_final=conv,
             meta=np.array([H, dk, dv, conv_k, n_steps], np.int32))


def gen_fullatt_prep(seed, nh, nkv, hd, max_seq, pos):
    rng = np.random.default_rng(seed)
    kv_dim = nkv * hd
    qg = rng.standard_normal(nh * 2 * hd).astype(np.float32)
    k = rng.standard_normal(kv_dim).astype(np.float32)
    v = rng.standard_normal(kv_dim).astype(np.float32)
    q_norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    k_norm = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kc = np.zeros((max_seq, kv_dim), np.float32)
    vc = np.zeros((max_seq, kv_dim), np.float32)
    q, gate, k_rot = orc.fullatt_prep(qg, k, v, q_norm, k_norm, kc, vc, pos, nh, nkv, hd, lib=orc.ref())
    np.savez(os.path.join(HERE, "fullatt_prep.npz"), qg=qg, k=k, v=v, q_norm=q_norm, k_norm=k_norm, q=q,
             gate=gate, k_rot=k_rot, k_row=kc[pos], v_row=vc[pos], meta=np.array([nh, nkv, hd, pos], np.int32))


def gen_fullatt_attend(seed, nh, nkv, hd, n_rows, pos):
    rng = np.random.default_rng(seed)
    kv_dim = nkv * hd
    kc = rng.standard_normal((n_rows, kv_dim)).astype(np.float32)
    vc = rng.standard_normal((n_rows, kv_dim)).astype(np.float32)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    gate = rng.standard_normal(nh * hd).astype(np.float32)
    sub_norm = (1.0 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    out_subln = orc.ref_fullatt_attend(q, gate, kc, vc, sub_norm, 0, pos, nh, nkv, hd)
    out_rms = orc.ref_fullatt_attend(q, gate, kc, vc, None, 0, pos, nh, nkv, hd)
    out_plain = orc.ref_fullatt_attend(q, gate, kc, vc, None, 1, pos, nh, nkv, hd)
    np.savez(os.path.join(HERE, "fullatt_attend.npz"), k_cache=kc, v_cache=vc, q=q, gate=gate, sub_norm=sub_norm,
             out_subln=out_subln, out_rms=out_rms, out_plain=out_plain, meta=np.array([nh, nkv, hd, pos], np.int32))


def gen_decode_cfg1(seed):
    """B1, 14 Q / 2 KV heads, hd 64, KV length 512, fp32, NeoX RoPE theta 1e6."""
    nh, nkv, hd, T, theta = 14, 2, 64, 512, 1e6
    rng = np.random.default_rng(seed)
    kv_dim = nkv * hd
    k_raw = rng.standard_normal((T, kv_dim)).astype(np.float32)
    vc = rng.standard_normal((T, kv_dim)).astype(np.float32)
    q_raw = rng.standard_normal(nh * hd).astype(np.float32)
    kc = np.stack([orc.rope_apply(k_raw[t], nkv, hd, t, theta) for t in range(T)])
    q = orc.rope_apply(q_raw, nh, hd, T - 1, theta)
    gate = np.full(nh * hd, GATE_ONE, np.float32)
    out = orc.ref_fullatt_attend(q, gate, kc, vc, None, 1, T - 1, nh, nkv, hd)
    np.savez(os.path.join(HERE, "decode_cfg1.npz"), q=q, k_cache=kc, v_cache=vc, out=out,
             meta=np.array([nh, nkv, hd, T - 1], np.int32))


def gen_prefill_small(seed, nh, nkv, hd, n_tok, start_pos):
    rng = np.random.default_rng(seed)
    kv_dim = nkv * hd
    rows = start_pos + n_tok
    kc = rng.standard_normal((rows, kv_dim)).astype(np.float32)
    vc = rng.standard_normal((rows, kv_dim)).astype(np.float32)
    q = rng.standard_normal((n_tok, nh * hd)).astype(np.float32)
    gate = np.full(nh * hd, GATE_ONE, np.float32)
    out = np.stack([orc.ref_fullatt_attend(q[i], gate, kc, vc, None, 1, start_pos + i, nh, nkv, hd)
                    for i in range(n_tok)])
    np.savez(os.path.join(HERE, "prefill_small.npz"), q=q, k_cache=kc, v_cache=vc, out=out,
             meta=np.array([nh, nkv, hd, n_tok, start_pos], np.int32))


def gen_tinyllm(name, seed, nh, nkv, hd, n_steps, theta, interleaved, kv_type, check_steps):
    """Decode steps 0..n_steps-1 through the reference's tinyllm forward.  k rows span two decades of
    scale; for the INT8 cache, k row 5 is zero (amax 0 -> scale 1), v row 9's first head is below the
    1e-12 floor, and v rows 20-23 sit next to rounding boundaries of code = trunc(x * inv +- 0.5)."""
    rng = np.random.default_rng(seed)
    kv_dim = nkv * hd
    q = rng.standard_normal((n_steps, nh * hd)).astype(np.float32)
    k = (rng.standard_normal((n_steps, kv_dim)) * rng.uniform(0.1, 10.0, (n_steps, 1))).astype(np.float32)
    v = (rng.standard_normal((n_steps, kv_dim)) * rng.uniform(0.3, 3.0, (n_steps, 1))).astype(np.float32)
    if kv_type == 1:
        k[5] = 0.0
        v[9, :hd] = 1e-13
        inv = np.float32(127) / np.float32(100)
        for t in range(20, 24):
            m = rng.integers(-127, 127, kv_dim)
            base = ((m + 0.5) / np.float64(inv)).astype(np.float32)
            step = rng.integers(-1, 2, kv_dim)
            row = np.where(step == 0, base, np.nextafter(base, np.where(step > 0, np.inf, -np.inf).astype(np.float32)))
            row = np.clip(row, -100.0, 100.0).astype(np.float32)
            row[::hd] = 100.0  # amax of every head: inv = 127 / 100, inexact
            v[t] = row
    o = orc.ref_tinyllm_decode_steps(q, k, v, nh, nkv, hd, n_steps, theta, interleaved, kv_type)
    steps = np.array(check_steps, np.int32)
    extra = dict(k_codes=o["k_codes"], v_codes=o["v_codes"], k_scale=o["k_scale"], v_scale=o["v_scale"]) \
        if kv_type == 1 else {}
    np.savez(os.path.join(HERE, name), q=q, k=k, v=v, steps=steps, q_rot=o["q_rot"][steps], attn=o["attn"][steps],
             k_row=o["k_row"], v_row=o["v_row"], theta=np.float32(theta),
             meta=np.array([nh, nkv, hd, n_steps, interleaved, kv_type], np.int32), **extra)


FIXTURES = {
    "deltanet_core_h2d128.npz": lambda: gen_deltanet_core("deltanet_core_h2d128.npz", 1001, H=2, dk=128, dv=128,
                                                          conv_k=4, n_steps=6),
    "deltanet_core_h3d64.npz": lambda: gen_deltanet_core("deltanet_core_h3d64.npz", 1002, H=3, dk=64, dv=64,
                                                         conv_k=4, n_steps=5),
    "fullatt_prep.npz": lambda: gen_fullatt_prep(1003, nh=8, nkv=2, hd=256, max_seq=16, pos=11),
    "fullatt_attend.npz": lambda: gen_fullatt_attend(1004, nh=8, nkv=2, hd=256, n_rows=40, pos=37),
    "decode_cfg1.npz": lambda: gen_decode_cfg1(1005),
    "prefill_small.npz": lambda: gen_prefill_small(1006, nh=6, nkv=2, hd=64, n_tok=24, start_pos=8),
    # BASELINE config 1's heads (14 / 2, hd 64, NeoX theta 1e6), fp32 cache, past the reference's
    # OpenMP threshold pos >= 64 (src/eif_tinyllm.c:557)
    "tinyllm_f32_cfg1.npz": lambda: gen_tinyllm("tinyllm_f32_cfg1.npz", 1007, 14, 2, 64, 72, 1e6, 0, 0,
                                                [0, 1, 2, 31, 63, 64, 65, 71]),
    "tinyllm_int8_hd64.npz": lambda: gen_tinyllm("tinyllm_int8_hd64.npz", 1008, 4, 2, 64, 72, 1e6, 0, 1,
                                                 [0, 1, 5, 9, 23, 63, 64, 71]),
    "tinyllm_int8_hd128.npz": lambda: gen_tinyllm("tinyllm_int8_hd128.npz", 1009, 4, 1, 128, 40, 1e4, 1, 1,
                                                  [0, 1, 5, 9, 22, 39]),
    "tinyllm_int8_hd256.npz": lambda: gen_tinyllm("tinyllm_int8_hd256.npz", 1010, 2, 1, 256, 24, 5e5, 0, 1,
                                                  [0, 3, 9, 21, 23]),
}


LINEAR_CASES = [  # name, quant_type, rows, cols, n
    ("f32", 0, 24, 96, 1), ("f32_n3", 0, 24, 96, 3),
    ("int4", 1, 24, 97, 1), ("int4_n5", 1, 24, 97, 5),
    ("tern2", 2, 24, 130, 1), ("tern2_n5", 2, 24, 130, 5),
    ("tern2_g32", 2 | (32 << 8), 24, 128, 1), ("tern2_g32_n5", 2 | (32 << 8), 24, 128, 5),
    ("dense", 3, 24, 101, 1), ("dense_n5", 3, 24, 101, 5),
    ("int8", 4, 24, 96, 1), ("int8_n3", 4, 24, 96, 3),
]


def linear_case(rng, quant_type, rows, cols, n):
    """Seeded weights of the format (values, packed rows, scales) and n input tokens."""
    base, group = quant_type & 0xFF, quant_type >> 8
    if base == 0:
        v = (0.05 * rng.standard_normal((rows, cols))).astype(np.float32)
    elif base == 1:
        v = rng.integers(-8, 8, (rows, cols))
    elif base == 4:
        v = rng.integers(-128, 128, (rows, cols))
    else:
        v = rng.integers(-1, 2, (rows, cols))
    W = orc.pack_weights(v, base, rng if base == 2 else None)
    sc = None if base == 0 else (0.01 + 0.1 * rng.random((rows, cols // group) if group else rows)).astype(np.float32)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    return v, W, sc, x


def gen_linear(seed):
    rng = np.random.default_rng(seed)
    arrays = {}
    for name, qt, rows, cols, n in LINEAR_CASES:
        _, W, sc, x = linear_case(rng, qt, rows, cols, n)
        arrays[f"{name}_W"] = W
        arrays[f"{name}_sc"] = sc if sc is not None else np.zeros(0, np.float32)
        arrays[f"{name}_x"] = x
        arrays[f"{name}_out"] = orc.ref_linear(W, sc, x, rows, cols, qt)
        arrays[f"{name}_shape"] = np.array([qt, rows, cols, n], np.int64)
    np.savez(os.path.join(HERE, "linear_formats.npz"), **arrays)


FIXTURES["linear_formats.npz"] = lambda: gen_linear(1100)


def main():
    orc.build(ref=True)
    names = sys.argv[1:] or list(FIXTURES)
    for n in names:
        FIXTURES[n]()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"{f:32s} {os.path.getsize(os.path.join(HERE, f)):>9d} B")


if __name__ == "__main__":
    main()
