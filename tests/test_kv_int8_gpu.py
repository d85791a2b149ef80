"""tinyllm's INT8 KV cache on the device (EIF_CUDA_INT8): the quantised cache write (src/eif_tinyllm.c:509-553)
through kv_upload / kv_append / rope_append, and the decode attention over codes and scales (:555-571, 615-625),
through the C ABI.  Codes and scales: bit-exact against the reference's own forward (tests/golden/tinyllm_int8_*)
and the C restatement; attention: rel-L2 <= 1e-5 (the fp32 decode tolerance)."""
import numpy as np
import pytest

from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("name", ["tinyllm_int8_hd64.npz", "tinyllm_int8_hd128.npz", "tinyllm_int8_hd256.npz"])
def test_decode_chain_vs_reference(pkg, ctx, name):
    """Every decode step of the reference's tinyllm forward: rope_append into the INT8 cache, attend_decode;
    codes and scales of every row bit-exact, the attention of the recorded steps within 1e-5."""
    d = golden(name)
    nh, nkv, hd, n, inter, _ = (int(x) for x in d["meta"])
    kv = pkg.KVCache(ctx, 1, 1, n, nkv, hd, pkg.INT8)
    kv.set_rope(float(d["theta"]), bool(inter))
    steps = list(d["steps"])
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    for t in range(n):
        pos = np.array([t], np.int32)
        qr = kv.rope_append(0, d["q"][t][None], d["k"][t][None], d["v"][t][None], pos, nh)
        if t in steps:
            i = steps.index(t)
            assert np.array_equal(qr[0], d["q_rot"][i]), t  # the reference's tables and rounding
            out = kv.attend_decode(0, qr, pos, nh, scale)
            assert rel_l2(out[0], d["attn"][i]) <= TOL, t
    kc, vc, ks, vs = kv.download_int8(0, 0, 0, n)
    assert np.array_equal(kc, d["k_codes"]) and np.array_equal(vc, d["v_codes"])
    assert bits_equal(ks, d["k_scale"]) and bits_equal(vs, d["v_scale"])


def test_upload_and_download(pkg, ctx, orc):
    """kv_upload quantises each (row, kv head); kv_download returns code * scale; reset zeroes codes and scales."""
    rng = np.random.default_rng(3)
    nkv, hd, T = 3, 128, 40
    kv = pkg.KVCache(ctx, 2, 2, T, nkv, hd, pkg.INT8)
    k = (rng.standard_normal((T, nkv * hd)) * rng.uniform(0.01, 50, (T, 1))).astype(np.float32)
    v = rng.standard_normal((T, nkv * hd)).astype(np.float32)
    k[3] = 0.0
    v[4, hd:2 * hd] = 1e-13
    kv.upload(1, 1, 0, k, v)
    kc, vc, ks, vs = kv.download_int8(1, 1, 0, T)
    rk, rks = orc.kv_quantize(k, nkv, hd)
    rv, rvs = orc.kv_quantize(v, nkv, hd)
    assert np.array_equal(kc, rk) and np.array_equal(vc, rv) and bits_equal(ks, rks) and bits_equal(vs, rvs)
    kd, vd = kv.download(1, 1, 0, T)
    want = (rk.reshape(T, nkv, hd).astype(np.float32) * rks[:, :, None]).reshape(T, -1)
    assert np.array_equal(kd, want)
    # other (layer, sequence) slots untouched
    kc0, _, ks0, _ = kv.download_int8(0, 1, 0, T)
    assert not kc0.any() and not ks0.any()
    kv.reset()
    kc, vc, ks, vs = kv.download_int8(1, 1, 0, T)
    assert not kc.any() and not vc.any() and not ks.any() and not vs.any()


def test_append_batch(pkg, ctx, orc):
    """kv_append of one token per sequence at different positions."""
    rng = np.random.default_rng(4)
    B, nkv, hd, T = 5, 2, 256, 33
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.INT8)
    pos = np.array([0, 7, 32, 1, 16], np.int32)
    k = rng.standard_normal((B, nkv * hd)).astype(np.float32) * 3
    v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    kv.append(0, pos, k, v)
    rk, rks = orc.kv_quantize(k, nkv, hd)
    rv, rvs = orc.kv_quantize(v, nkv, hd)
    for b in range(B):
        kc, vc, ks, vs = kv.download_int8(0, b, int(pos[b]), 1)
        assert np.array_equal(kc[0], rk[b]) and np.array_equal(vc[0], rv[b])
        assert bits_equal(ks[0], rks[b]) and bits_equal(vs[0], rvs[b])


@pytest.mark.parametrize("simt", [False, True], ids=["tensor-core", "simt"])
@pytest.mark.parametrize("nh,nkv,hd,T", [(14, 2, 64, 700), (8, 2, 128, 1500), (8, 1, 256, 300), (6, 6, 64, 129),
                                         (16, 2, 128, 64), (3, 1, 64, 4000)])
def test_decode_vs_oracle(pkg, ctx, orc, monkeypatch, simt, nh, nkv, hd, T):
    """attend_decode over an uploaded INT8 cache, a batch of sequences at different positions (split-K chunks,
    groups 1..8, ragged last tiles), against the restatement's INT8 attention on the same codes; both the
    tensor-core kernel and the SIMT kernel (BITLLM_DECODE_SIMT=1)."""
    if simt:
        monkeypatch.setenv("BITLLM_DECODE_SIMT", "1")
    rng = np.random.default_rng(nh * 1000 + hd + T)
    B = 3
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.INT8)
    pos = np.array([T - 1, T // 2, 0], np.int32)
    codes = []
    for b in range(B):
        k = (rng.standard_normal((T, nkv * hd)) * rng.uniform(0.2, 4, (T, 1))).astype(np.float32)
        v = rng.standard_normal((T, nkv * hd)).astype(np.float32)
        kv.upload(0, b, 0, k, v)
        codes.append(kv.download_int8(0, b, 0, T))
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_decode(0, q, pos, nh, scale)
    for b in range(B):
        kc, vc, ks, vs = codes[b]
        ref = orc.attend_decode_i8(q[b], kc, ks, vc, vs, int(pos[b]), nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= TOL, b


@pytest.mark.parametrize("vmag", [1e-7, 1.0, 3e3, 1e6], ids=["v1e-7", "v1", "v3e3", "v1e6"])
@pytest.mark.parametrize("nh,nkv,hd", [(14, 2, 64), (8, 2, 128)])
def test_decode_value_range(pkg, ctx, orc, nh, nkv, hd, vmag):
    """V rows whose INT8 scales are tiny or far above 16 (p * v_scale then leaves f16's range unless the kernel
    rescales its P operand), and rows of one sequence spanning four orders of magnitude, through the tensor-core
    kernel against the restatement's INT8 attention on the same codes."""
    rng = np.random.default_rng(int(hd + nh + np.log10(vmag) * 7 + 100))
    B, T = 2, 900
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.INT8)
    pos = np.array([T - 1, T // 3], np.int32)
    codes = []
    for b in range(B):
        k = (rng.standard_normal((T, nkv * hd)) * rng.uniform(0.2, 4, (T, 1))).astype(np.float32)
        v = (rng.standard_normal((T, nkv * hd)) * vmag * 10.0 ** rng.uniform(-2, 2, (T, 1))).astype(np.float32)
        kv.upload(0, b, 0, k, v)
        codes.append(kv.download_int8(0, b, 0, T))
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_decode(0, q, pos, nh, scale)
    assert np.isfinite(out).all()
    for b in range(B):
        kc, vc, ks, vs = codes[b]
        ref = orc.attend_decode_i8(q[b], kc, ks, vc, vs, int(pos[b]), nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= TOL, b


def test_int8_rejections(pkg, ctx):
    """INT8 caches: head_dim 64/128/256 only; no Qwen3.5 prep over them (its cache is fp32); the raw download
    needs an INT8 cache."""
    with pytest.raises(pkg.EifCudaError) as e:
        pkg.KVCache(ctx, 1, 1, 8, 2, 96, pkg.INT8)
    assert e.value.name == "NOT_SUPPORTED"
    kv = pkg.KVCache(ctx, 1, 1, 64, 2, 64, pkg.INT8)
    kv.set_norms(0, np.ones(64, np.float32), np.ones(64, np.float32))
    with pytest.raises(pkg.EifCudaError) as e:
        kv.fullatt_prep(0, np.zeros((1, 4 * 128), np.float32), np.zeros((1, 128), np.float32),
                        np.zeros((1, 128), np.float32), np.array([0]), 4)
    assert e.value.name == "NOT_SUPPORTED"
    f32 = pkg.KVCache(ctx, 1, 1, 8, 2, 64, pkg.F32)
    with pytest.raises(pkg.EifCudaError) as e:
        f32.download_int8(0, 0, 0, 1)
    assert e.value.name == "INVALID_ARGUMENT"


@pytest.mark.parametrize("hd,nh,nkv", [(64, 14, 2), (128, 8, 2), (256, 8, 2)])
def test_int8_prefill_chain(pkg, ctx, orc, hd, nh, nkv):
    """The batched prefill over an INT8 cache (src/eif_tinyllm.c:1158-1268 with kv_type 1, :1172-1235): a chunk's
    RoPE and quantised cache writes (rope_append_prefill: codes and scales bit-identical to per-token
    rope_append), then causal attention of every chunk token over the codes and scales, against the
    restatement of the INT8 loop token by token (rel-L2 <= 1e-5); a second chunk continues at start_pos > 0."""
    rng = np.random.default_rng(hd + nh)
    B, T = 2, 300
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.INT8)
    kv.set_rope(1e6)
    one = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.INT8)  # the same rows written one token at a time
    one.set_rope(1e6)
    scale = 1.0 / np.sqrt(hd)
    start = 0
    for n_tok in (130, 67):
        q = rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32)
        k = rng.standard_normal((B, n_tok, nkv * hd)).astype(np.float32)
        v = rng.standard_normal((B, n_tok, nkv * hd)).astype(np.float32)
        qr = kv.rope_append_prefill(0, q, k, v, n_tok, start, nh)
        for t in range(n_tok):
            pos = np.full(B, start + t, np.int32)
            qt = one.rope_append(0, q[:, t], k[:, t], v[:, t], pos, nh)
            assert np.array_equal(qt, qr[:, t]), t
        out = kv.attend_prefill(0, qr, n_tok, start, nh, scale)
        for b in range(B):
            got = kv.download_int8(0, b, 0, start + n_tok)
            want = one.download_int8(0, b, 0, start + n_tok)
            for g_, w_ in zip(got, want):
                assert np.array_equal(g_, w_)
            kc, vc, ks, vs = got
            for t in range(n_tok):
                ref = orc.attend_decode_i8(qr[b, t], kc, ks, vc, vs, start + t, nh, nkv, hd, scale)
                assert rel_l2(out[b, t], ref) <= TOL, (b, t)
        start += n_tok
