"""tinyllm RoPE + cache write on the device (eif_cuda_kv_set_rope, eif_cuda_rope_append[_prefill]) against
the C restatement of src/eif_tinyllm.c:395-405 (tables) and :481-507 (rotation, NeoX or adjacent pairs),
through the C ABI.  fp32 paths: rel-L2 <= 1e-5; bf16 cache rows: within one bf16 ulp of the rotated fp32
row; the prefill attention after it: rel-L2 <= 1e-2, max-abs <= 2e-2."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def one_ulp(got, want):
    return np.all(np.abs(got - want) <= 2.0 ** -7 * np.abs(want) + 1e-30)


@pytest.mark.parametrize("hd,nh,nkv,theta,inter,dtype", [(64, 14, 2, 1e6, False, "f32"), (128, 8, 2, 1e4, True, "f32"),
                                                        (64, 14, 2, 1e6, False, "bf16"), (128, 12, 4, 5e5, True, "bf16")])
def test_rope_append_vs_oracle(pkg, ctx, orc, hd, nh, nkv, theta, inter, dtype):
    rng = np.random.default_rng(hd + nh)
    B, T = 3, 520
    dt = pkg.F32 if dtype == "f32" else pkg.BF16
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    kv.set_rope(theta, inter)
    pos = np.array([0, 5, 511], np.int32)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    qr = kv.rope_append(0, q, k, v, pos, nh)
    for b in range(B):
        assert rel_l2(qr[b], orc.rope_apply(q[b], nh, hd, pos[b], theta, inter)) <= TOL, b
        kd, vd = kv.download(0, b, pos[b], 1)
        kref = orc.rope_apply(k[b], nkv, hd, pos[b], theta, inter)
        if dt == pkg.F32:
            assert rel_l2(kd[0], kref) <= TOL and np.array_equal(vd[0], v[b])
        else:
            assert one_ulp(kd[0], kref) and np.array_equal(vd[0], orc.round_bf16(v[b]))


def test_tinyllm_decode_chain(pkg, ctx, orc):
    """BASELINE config 1's head shape (14 q / 2 kv heads, hd 64, NeoX RoPE theta 1e6, fp32 cache): 40 decode
    steps of rope_append + attend_decode against the restatement's rotation + attention."""
    rng = np.random.default_rng(1)
    nh, nkv, hd, theta, T = 14, 2, 64, 1e6, 48
    kv = pkg.KVCache(ctx, 1, 1, T, nkv, hd, pkg.F32)
    kv.set_rope(theta, False)
    kc = np.zeros((T, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    for t in range(40):
        q = rng.standard_normal(nh * hd).astype(np.float32)
        k = rng.standard_normal(nkv * hd).astype(np.float32)
        v = rng.standard_normal(nkv * hd).astype(np.float32)
        pos = np.array([t], np.int32)
        qr = kv.rope_append(0, q[None], k[None], v[None], pos, nh)
        out = kv.attend_decode(0, qr, pos, nh, 1.0 / 8)
        kc[t] = orc.rope_apply(k, nkv, hd, t, theta)
        vc[t] = v
        ref = orc.attend_decode(orc.rope_apply(q, nh, hd, t, theta), kc, vc, t, nh, nkv, hd, 1.0 / 8)
        assert rel_l2(out[0], ref) <= TOL, t


def test_rope_append_prefill_then_attention(pkg, ctx, orc):
    """A tinyllm prefill chunk: RoPE of all its tokens + cache rows in one launch, then the causal prefill
    attention over the cache, on a bf16 cache that already holds earlier rows."""
    rng = np.random.default_rng(2)
    B, nh, nkv, hd, theta, start, n = 2, 14, 2, 64, 1e6, 30, 100
    T = start + n + 2
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.BF16)
    kv.set_rope(theta, False)
    kc = np.zeros((B, T, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:, :start] = orc.round_bf16(rng.standard_normal((B, start, nkv * hd))).reshape(B, start, -1)
    vc[:, :start] = orc.round_bf16(rng.standard_normal((B, start, nkv * hd))).reshape(B, start, -1)
    for b in range(B):
        kv.upload(0, b, 0, kc[b, :start], vc[b, :start])
    q = rng.standard_normal((B, n, nh * hd)).astype(np.float32)
    k = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    qr = kv.rope_append_prefill(0, q, k, v, n, start, nh)
    out = kv.attend_prefill(0, qr, n, start, nh, 1.0 / 8)
    for b in range(B):
        qref = np.stack([orc.rope_apply(q[b, i], nh, hd, start + i, theta) for i in range(n)])
        assert rel_l2(qr[b], qref) <= TOL
        for i in range(n):
            kc[b, start + i] = orc.round_bf16(orc.rope_apply(k[b, i], nkv, hd, start + i, theta))
            vc[b, start + i] = orc.round_bf16(v[b, i])
        kd, vd = kv.download(0, b, 0, start + n)
        assert one_ulp(kd, kc[b, :start + n]) and np.array_equal(vd, vc[b, :start + n])
        ref = orc.attend_prefill(orc.round_bf16(qref).reshape(n, -1), kd, vd, n, start, nh, nkv, hd, 1.0 / 8)
        assert rel_l2(out[b], ref) <= 1e-2 and np.max(np.abs(out[b] - ref)) <= 2e-2


@pytest.mark.parametrize("dtype", ["f32", "bf16", "int8"])
def test_prefill_step_one_call(pkg, ctx, orc, dtype):
    """eif_cuda_prefill_step (RoPE, cache writes and causal attention of a chunk in one call) against the two
    calls rope_append_prefill + attend_prefill on a second cache: the same cache rows, and the same attention
    (fp32 / INT8 caches: rel-L2 <= 1e-5 and the fp32 cache also against the restatement; bf16: the prefill
    tolerance, the two-call host path rounds its output to bf16)."""
    rng = np.random.default_rng(17)
    dt = {"f32": pkg.F32, "bf16": pkg.BF16, "int8": pkg.INT8}[dtype]
    B, nh, nkv, hd, theta, start, n = 2, 14, 2, 64, 1e6, 40, 90
    T = start + n + 2
    kvs = []
    for _ in range(2):
        kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
        kv.set_rope(theta, False)
        kvs.append(kv)
    k0 = rng.standard_normal((B, start, nkv * hd)).astype(np.float32)
    v0 = rng.standard_normal((B, start, nkv * hd)).astype(np.float32)
    for kv in kvs:
        for b in range(B):
            kv.upload(0, b, 0, k0[b], v0[b])
    q = rng.standard_normal((B, n, nh * hd)).astype(np.float32)
    k = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    qr = kvs[0].rope_append_prefill(0, q, k, v, n, start, nh)
    two = kvs[0].attend_prefill(0, qr, n, start, nh, 1.0 / 8)
    one = kvs[1].prefill_step(0, q, k, v, n, start, nh, 1.0 / 8)
    for b in range(B):
        if dt == pkg.INT8:
            for a_, b_ in zip(kvs[0].download_int8(0, b, 0, T), kvs[1].download_int8(0, b, 0, T)):
                assert np.array_equal(a_, b_)
        else:
            for a_, b_ in zip(kvs[0].download(0, b, 0, T), kvs[1].download(0, b, 0, T)):
                assert np.array_equal(a_, b_)
        if dt == pkg.BF16:
            assert rel_l2(one[b], two[b]) <= 1e-2
        else:
            assert rel_l2(one[b], two[b]) <= 1e-5
        if dt == pkg.F32:
            kd, vd = kvs[1].download(0, b, 0, start + n)
            assert rel_l2(one[b], orc.attend_prefill(qr[b], kd, vd, n, start, nh, nkv, hd, 1.0 / 8)) <= 1e-5
    for kv in kvs:
        kv.free()


def test_rope_needs_table(pkg, ctx):
    kv = pkg.KVCache(ctx, 1, 1, 8, 2, 64, pkg.F32)
    with pytest.raises(pkg.EifCudaError) as e:
        kv.rope_append(0, np.zeros((1, 128), np.float32), np.zeros((1, 128), np.float32),
                       np.zeros((1, 128), np.float32), np.array([0]), 2)
    assert e.value.name == "INVALID_ARGUMENT"


def test_tinyllm_decode_vs_reference(pkg, ctx):
    """The reference's own tinyllm forward (tests/golden/tinyllm_f32_cfg1.npz: BASELINE config 1's heads, fp32
    cache, 72 steps past its OpenMP threshold): rope_append + attend_decode per step, rel-L2 <= 1e-5."""
    from conftest import golden
    d = golden("tinyllm_f32_cfg1.npz")
    nh, nkv, hd, n, inter, _ = (int(x) for x in d["meta"])
    kv = pkg.KVCache(ctx, 1, 1, n, nkv, hd, pkg.F32)
    kv.set_rope(float(d["theta"]), bool(inter))
    steps = list(d["steps"])
    for t in range(n):
        pos = np.array([t], np.int32)
        qr = kv.rope_append(0, d["q"][t][None], d["k"][t][None], d["v"][t][None], pos, nh)
        if t in steps:
            i = steps.index(t)
            assert np.array_equal(qr[0], d["q_rot"][i])  # the reference's tables and rounding, bit for bit
            assert rel_l2(kv.attend_decode(0, qr, pos, nh, 0.125)[0], d["attn"][i]) <= TOL, t
    kd, vd = kv.download(0, 0, 0, n)
    assert np.array_equal(kd, d["k_row"]) and np.array_equal(vd, d["v_row"])
