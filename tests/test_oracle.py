"""The CPU checker (oracle/oracle.c) against the reference's own outputs.

The fixtures under tests/golden/ were produced by the reference's src/eif_qwen35.c compiled from its
sources (tests/golden/gen_golden.py); where that build is present (oracle/_ref/) the restatement is
also compared with it on fresh seeded inputs.  No GPU needed."""
import numpy as np
import pytest

from conftest import golden, rel_l2


@pytest.mark.parametrize("name", ["deltanet_core_h2d128.npz", "deltanet_core_h3d64.npz"])
def test_deltanet_core_golden(orc, name):
    d = golden(name)
    H, dk, dv, ck, n = (int(x) for x in d["meta"])
    S, conv = d["S0"].copy(), d["conv0"].copy()
    outs = [orc.deltanet_core(d["qkv"][t], d["z"][t], d["b"][t], d["a"][t], conv, S, d["conv_w"], d["dt_bias"],
                              d["A_log"], d["norm_w"]) for t in range(n)]
    assert rel_l2(np.stack(outs), d["out"]) < 1e-6
    assert rel_l2(S, d["S_final"]) < 1e-6
    assert rel_l2(conv, d["conv_final"]) < 1e-6


def test_decode_cfg1_golden(orc):
    d = golden("decode_cfg1.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    o = orc.attend_decode(d["q"], d["k_cache"], d["v_cache"], pos, nh, nkv, hd, 1.0 / np.sqrt(hd))
    assert rel_l2(o, d["out"]) < 1e-6


def test_fullatt_attend_golden(orc):
    d = golden("fullatt_attend.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    o = orc.attend_decode(d["q"], d["k_cache"], d["v_cache"], pos, nh, nkv, hd, scale, gate=d["gate"])
    assert rel_l2(o, d["out_plain"]) < 1e-6
    assert rel_l2(orc.subln(o, None, 1), d["out_rms"]) < 1e-6
    assert rel_l2(orc.subln(o, d["sub_norm"], 2), d["out_subln"]) < 1e-6


def test_prefill_golden(orc):
    d = golden("prefill_small.npz")
    nh, nkv, hd, n, sp = (int(x) for x in d["meta"])
    o = orc.attend_prefill(d["q"], d["k_cache"], d["v_cache"], n, sp, nh, nkv, hd, 1.0 / np.sqrt(hd))
    assert rel_l2(o, d["out"]) < 1e-6


def test_fullatt_prep_golden(orc):
    d = golden("fullatt_prep.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    kc = np.zeros((16, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    q, g, kr = orc.fullatt_prep(d["qg"], d["k"], d["v"], d["q_norm"], d["k_norm"], kc, vc, pos, nh, nkv, hd)
    assert rel_l2(q, d["q"]) < 1e-6 and rel_l2(g, d["gate"]) == 0.0
    assert rel_l2(kr, d["k_rot"]) < 1e-6 and rel_l2(kc[pos], d["k_row"]) < 1e-6
    assert np.array_equal(vc[pos], d["v_row"])


def test_pos0_attention_copies_v(orc):
    """Known answer of the reference's tests/test_gguf_gqa_layout.c:105: at pos 0 attention returns v_0
    of each query head's kv group (GQA mapping h -> h / (nh/nkv))."""
    rng = np.random.default_rng(3)
    nh, nkv, hd = 4, 2, 16
    kc = rng.standard_normal((1, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((1, nkv * hd)).astype(np.float32)
    o = orc.attend_decode(rng.standard_normal(nh * hd), kc, vc, 0, nh, nkv, hd, 0.25)
    for h in range(nh):
        kvh = h // (nh // nkv)
        assert np.allclose(o[h * hd:(h + 1) * hd], vc[0, kvh * hd:(kvh + 1) * hd], rtol=0, atol=1e-6)


ref_only = pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).ref_available()",
                              reason="reference build (oracle/_ref) absent")


@ref_only
def test_port_vs_reference_deltanet_random(orc):
    rng = np.random.default_rng(11)
    for H, dk, ck in [(16, 128, 4), (1, 32, 3)]:
        conv_dim = 3 * H * dk
        args = dict(conv_w=(rng.standard_normal((conv_dim, ck)) * 0.5).astype(np.float32),
                    dt_bias=rng.standard_normal(H).astype(np.float32),
                    A_log=rng.standard_normal(H).astype(np.float32) * 0.5,
                    norm_w=(1 + 0.1 * rng.standard_normal(dk)).astype(np.float32))
        S1 = (rng.standard_normal((H, dk, dk)) * 0.02).astype(np.float32)
        c1 = rng.standard_normal((conv_dim, ck)).astype(np.float32)
        S2, c2 = S1.copy(), c1.copy()
        for _ in range(3):
            x = [rng.standard_normal(n).astype(np.float32) for n in (conv_dim, H * dk, H, H)]
            o1 = orc.deltanet_core(*x, c1, S1, **args)
            o2 = orc.deltanet_core(*x, c2, S2, **args, lib=orc.ref())
            assert rel_l2(o1, o2) < 1e-6
        assert rel_l2(S1, S2) < 1e-6


@ref_only
def test_port_vs_reference_attend_random(orc):
    rng = np.random.default_rng(12)
    for nh, nkv, hd, T in [(14, 2, 64, 300), (8, 2, 256, 64), (9, 3, 128, 17), (4, 4, 64, 1)]:
        kc = rng.standard_normal((T, nkv * hd)).astype(np.float32)
        vc = rng.standard_normal((T, nkv * hd)).astype(np.float32)
        q = rng.standard_normal(nh * hd).astype(np.float32)
        gate = rng.standard_normal(nh * hd).astype(np.float32)
        scale = np.float32(1.0) / np.sqrt(np.float32(hd))
        o = orc.attend_decode(q, kc, vc, T - 1, nh, nkv, hd, scale, gate=gate)
        r = orc.ref_fullatt_attend(q, gate, kc, vc, None, 1, T - 1, nh, nkv, hd)
        assert rel_l2(o, r) < 1e-6


TINYLLM = ["tinyllm_f32_cfg1.npz", "tinyllm_int8_hd64.npz", "tinyllm_int8_hd128.npz", "tinyllm_int8_hd256.npz"]


@pytest.mark.parametrize("name", TINYLLM)
def test_tinyllm_golden(orc, name):
    """tinyllm's own forward (src/eif_tinyllm.c:371-857) over decode steps: RoPE, the fp32 or INT8 cache write
    and the attention output, against the restatement.  INT8 codes and scales are bit-exact."""
    d = golden(name)
    nh, nkv, hd, n, inter, kv_type = (int(x) for x in d["meta"])
    theta = float(d["theta"])
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    k_rot = np.stack([orc.rope_apply(d["k"][t], nkv, hd, t, theta, inter) for t in range(n)])
    for i, t in enumerate(d["steps"]):  # RoPE tables and rotation bit-identical to the compiled reference
        assert np.array_equal(orc.rope_apply(d["q"][t], nh, hd, t, theta, inter), d["q_rot"][i]), t
    if kv_type == 0:
        assert np.array_equal(k_rot, d["k_row"]) and np.array_equal(d["v_row"], d["v"])
        for i, t in enumerate(d["steps"]):
            o = orc.attend_decode(d["q_rot"][i], d["k_row"][:t + 1], d["v_row"][:t + 1], t, nh, nkv, hd, scale)
            assert rel_l2(o, d["attn"][i]) <= 1e-6, t
        return
    # the fp32 row of step 0 is overwritten by the reference's INT8 rows (they alias one buffer,
    # src/eif_tinyllm.c:136-138); rows >= 1 are intact when read right after their step
    assert np.array_equal(k_rot[1:], d["k_row"][1:]) and np.array_equal(d["v_row"][1:], d["v"][1:])
    kc, ks = orc.kv_quantize(np.concatenate([k_rot[:1], d["k_row"][1:]]), nkv, hd)
    vc, vs = orc.kv_quantize(d["v"], nkv, hd)
    assert np.array_equal(kc, d["k_codes"]) and np.array_equal(vc, d["v_codes"])
    assert np.array_equal(ks.view(np.uint32), d["k_scale"].view(np.uint32))
    assert np.array_equal(vs.view(np.uint32), d["v_scale"].view(np.uint32))
    for i, t in enumerate(d["steps"]):
        o = orc.attend_decode_i8(d["q_rot"][i], d["k_codes"][:t + 1], d["k_scale"][:t + 1], d["v_codes"][:t + 1],
                                 d["v_scale"][:t + 1], t, nh, nkv, hd, scale)
        assert rel_l2(o, d["attn"][i]) <= 1e-6, t


def test_int8_quantize_edges(orc):
    """The quantiser's edge rows: all zero (amax 0 -> scale 1, codes 0), below the 1e-12 floor, a head whose
    amax sits at the clamp (+-127 reached, -128 never produced by the symmetric scale), and sign handling."""
    hd = 64
    x = np.zeros((4, 2 * hd), np.float32)
    x[1, :hd] = 5e-13
    x[1, hd:] = -5e-13
    x[2, :hd] = np.linspace(-3.0, 3.0, hd, dtype=np.float32)
    x[3, :hd] = -1.0
    x[3, hd:] = 0.25
    c, s = orc.kv_quantize(x, 2, hd)
    assert np.all(c[0] == 0) and np.all(s[0] == 1.0)
    assert np.all(c[1] == 0) and np.all(s[1] == 1.0)
    assert c[2, 0] == -127 and c[2, hd - 1] == 127 and np.isclose(s[2, 0], 3.0 / 127)
    assert np.all(c[3, :hd] == -127) and np.all(c[3, hd:] == 127)
    assert s[2, 1] == 1.0 and np.all(c[2, hd:] == 0)


def test_rope_table_folded_form(orc):
    """The device tables (eif_cuda_kv_set_rope) compute freq = powf(theta, -2j/hd) with libm, the form the
    reference's -ffast-math build gives its 1.0f / powf(theta, 2j/hd); check that form against the
    restatement compiled with the reference's flags, over the thetas and head sizes of the tinyllm models."""
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("powf", "cosf", "sinf"):
        getattr(libm, fn).restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    libm.cosf.argtypes = [ctypes.c_float]
    libm.sinf.argtypes = [ctypes.c_float]
    f32 = np.float32
    for theta in (1e4, 1e5, 5e5, 1e6, 5e6):
        for hd in (64, 128, 256):
            freq = [f32(libm.powf(f32(theta), -(f32(2 * j) / f32(hd)))) for j in range(hd // 2)]
            for pos in range(0, 4096, 251):
                c, s = orc.rope_table(pos, hd, theta)
                vals = [f32(pos) * f for f in freq]
                assert np.array_equal(c, np.array([libm.cosf(v) for v in vals], f32)), (theta, hd, pos)
                assert np.array_equal(s, np.array([libm.sinf(v) for v in vals], f32)), (theta, hd, pos)


# ------------------------------------------------------------------------------------------------
# Projections (linear_gemv / linear_gemm / int8_gemv, src/eif_qwen35.c:384-443, 1033-1063)
# ------------------------------------------------------------------------------------------------

LINEAR_NAMES = ["f32", "f32_n3", "int4", "int4_n5", "tern2", "tern2_n5", "tern2_g32", "tern2_g32_n5", "dense",
                "dense_n5", "int8", "int8_n3"]


def linear_golden(name):
    d = golden("linear_formats.npz")
    qt, rows, cols, n = (int(v) for v in d[f"{name}_shape"])
    sc = d[f"{name}_sc"]
    return qt, rows, cols, n, d[f"{name}_W"], (sc if sc.size else None), d[f"{name}_x"], d[f"{name}_out"]


@pytest.mark.parametrize("name", LINEAR_NAMES)
def test_linear_golden(orc, name):
    """The restatement against the reference's own projections on every weight format (rel-L2 <= 1e-5: both
    sum in fp32, in different orders; a decoding mistake is O(1))."""
    qt, rows, cols, n, W, sc, x, out = linear_golden(name)
    assert rel_l2(orc.linear(W, sc, x, rows, cols, qt), out) <= 1e-5


@pytest.mark.parametrize("base", [0, 1, 2, 3, 4])
def test_linear_pack_decode_exact(orc, base):
    """Packing and the restatement's decoding are inverse: integer weights and inputs with a power-of-two scale
    give the exact integer product (every partial sum is an integer below 2^24)."""
    rng = np.random.default_rng(70 + base)
    rows, cols = 19, 203
    lo, hi = {0: (-8, 8), 1: (-8, 8), 4: (-128, 128)}.get(base, (-1, 2))
    v = rng.integers(lo, hi, (rows, cols))
    W = orc.pack_weights(v.astype(np.float32) if base == 0 else v, base, rng if base == 2 else None)
    sc = None if base == 0 else np.full(rows, 0.5, np.float32)
    x = rng.integers(-4, 5, (3, cols)).astype(np.float32)
    want = (x.astype(np.int64) @ v.T.astype(np.int64)).astype(np.float64) * (1.0 if base == 0 else 0.5)
    assert np.array_equal(orc.linear(W, sc, x, rows, cols, base).astype(np.float64), want)


def test_port_vs_reference_linear_random(orc):
    """Where the reference build is present: the restatement against it at a Qwen3.5 projection width."""
    if not orc.ref_available():
        pytest.skip("reference build absent")
    rng = np.random.default_rng(71)
    for qt, rows, cols in [(2, 96, 1024), (2 | (64 << 8), 96, 1024), (1, 64, 2048), (3, 64, 1024), (4, 128, 1024),
                           (0, 64, 1024)]:
        base, group = qt & 0xFF, qt >> 8
        v = (rng.integers(-1, 2, (rows, cols)) if base in (2, 3) else rng.integers(-8, 8, (rows, cols)) if base == 1
             else rng.integers(-128, 128, (rows, cols)) if base == 4 else rng.standard_normal((rows, cols)) * 0.05)
        W = orc.pack_weights(v, base, rng if base == 2 else None)
        sc = None if base == 0 else (0.01 + rng.random((rows, cols // group) if group else rows)).astype(np.float32)
        for n in (1, 6):
            x = rng.standard_normal((n, cols)).astype(np.float32)
            assert rel_l2(orc.linear(W, sc, x, rows, cols, qt), orc.ref_linear(W, sc, x, rows, cols, qt)) <= 1e-5, qt
