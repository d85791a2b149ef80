"""The whole Qwen3.5 mixer bodies through the C ABI: deltanet_core (src/eif_qwen35.c:546-656) and
fullatt_prep (src/eif_qwen35.c:699-737) -> attend (gate + SubLN), against the reference's own outputs
(tests/golden/*.npz, recorded from the compiled reference) and the C restatement.  fp32 paths:
rel-L2 <= 1e-5."""
import numpy as np
import pytest

from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.mark.parametrize("name", ["deltanet_core_h2d128.npz", "deltanet_core_h3d64.npz"])
def test_deltanet_core_golden(pkg, ctx, name):
    """Consecutive tokens through the reference's deltanet_core (conv window, norms, gates, rule, gated
    RMSNorm); the same tokens through eif_cuda_deltanet_core, state carried on the device."""
    d = golden(name)
    H, dk, dv, ck, n = (int(x) for x in d["meta"])
    st = pkg.DeltaState(ctx, 1, 1, H, dk, dv, ck)
    st.set_weights(0, d["conv_w"], d["dt_bias"], d["A_log"], d["norm_w"])
    st.upload(0, 0, S=d["S0"], conv_state=d["conv0"])
    outs = [st.core(0, d["qkv"][t][None], d["z"][t][None], d["b"][t][None], d["a"][t][None])[0] for t in range(n)]
    assert rel_l2(np.stack(outs), d["out"]) <= TOL
    S, conv = st.download(0, 0)
    assert rel_l2(S, d["S_final"]) <= TOL
    assert rel_l2(conv, d["conv_final"]) <= TOL


def test_deltanet_core_batched_vs_port(pkg, ctx, orc):
    """Qwen3.5-0.8B mixer shape (16 heads, d 128, conv 4) for a batch of 5 sequences, 4 tokens."""
    rng = np.random.default_rng(77)
    B, H, d, ck = 5, 16, 128, 4
    conv_dim = 3 * H * d
    w = dict(conv_w=(rng.standard_normal((conv_dim, ck)) * 0.5).astype(np.float32),
             dt_bias=rng.standard_normal(H).astype(np.float32), A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
             norm_w=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    st = pkg.DeltaState(ctx, 2, B, H, d, d, ck)
    st.set_weights(1, **w)
    S = (0.02 * rng.standard_normal((B, H, d, d))).astype(np.float32)
    conv = rng.standard_normal((B, conv_dim, ck)).astype(np.float32)
    for b in range(B):
        st.upload(1, b, S=S[b], conv_state=conv[b])
    for t in range(4):
        qkv = rng.standard_normal((B, conv_dim)).astype(np.float32)
        z = rng.standard_normal((B, H * d)).astype(np.float32)
        bb = rng.standard_normal((B, H)).astype(np.float32)
        aa = rng.standard_normal((B, H)).astype(np.float32)
        out = st.core(1, qkv, z, bb, aa)
        for b in range(B):
            ref = orc.deltanet_core(qkv[b], z[b], bb[b], aa[b], conv[b], S[b], **w)
            assert rel_l2(out[b], ref) <= TOL, (t, b)
    for b in range(B):
        Sg, cg = st.download(1, b)
        assert rel_l2(Sg, S[b]) <= TOL and rel_l2(cg, conv[b]) <= TOL


def test_deltanet_core_needs_weights(pkg, ctx):
    st = pkg.DeltaState(ctx, 1, 1, 2, 128, 128, 4)
    z = np.zeros((1, 256), np.float32)
    with pytest.raises(pkg.EifCudaError) as e:
        st.core(0, np.zeros((1, 768), np.float32), z, np.zeros((1, 2), np.float32), np.zeros((1, 2), np.float32))
    assert e.value.name == "INVALID_ARGUMENT"


def test_fullatt_prep_golden(pkg, ctx):
    """The reference's fullatt_prep at pos 11: q, gate, and the cache rows it writes."""
    d = golden("fullatt_prep.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    kv = pkg.KVCache(ctx, 1, 1, 16, nkv, hd, pkg.F32)
    kv.set_norms(0, d["q_norm"], d["k_norm"])
    q, g = kv.fullatt_prep(0, d["qg"][None], d["k"][None], d["v"][None], np.array([pos]), nh)
    assert rel_l2(q[0], d["q"]) <= TOL
    assert np.array_equal(g[0], d["gate"])
    kd, vd = kv.download(0, 0, pos, 1)
    assert rel_l2(kd[0], d["k_row"]) <= TOL
    assert np.array_equal(vd[0], d["v_row"])


def test_fullatt_prep_large_positions(pkg, ctx, orc):
    """Partial RoPE far into a long context (rows up to 32767): at such positions one ulp of an inverse
    frequency moves the angle by ~1e-3 rad, so the device table must hold the compiled reference's own
    inverse frequencies (its -ffast-math build evaluates 1/powf(1e7, x) as expf(-x * logf(1e7))).  q and the
    written k row against the reference's fullatt_prep (the restatement, built the same way, where the
    reference build is absent)."""
    rng = np.random.default_rng(90)
    B, nh, nkv, hd, T = 4, 8, 2, 256, 32768
    lib = orc.ref() if orc.ref_available() else None
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.F32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kv.set_norms(0, qn, kn)
    pos = np.array([4095, 20001, 32766, 32767], np.int32)
    qg = rng.standard_normal((B, nh * 2 * hd)).astype(np.float32)
    k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    q, g = kv.fullatt_prep(0, qg, k, v, pos, nh)
    for b in range(B):
        kc = np.zeros((int(pos[b]) + 1, nkv * hd), np.float32)
        rq, rg, rk = orc.fullatt_prep(qg[b], k[b], v[b], qn, kn, kc, kc.copy(), int(pos[b]), nh, nkv, hd, lib=lib)
        assert rel_l2(q[b], rq) <= 1e-6, (b, rel_l2(q[b], rq))
        kd, _ = kv.download(0, b, int(pos[b]), 1)
        assert rel_l2(kd[0], rk) <= 1e-6, b
    kv.free()


def test_deltanet_core_batch_independent(pkg, ctx, orc):
    """40 sequences x 16 heads (more heads than one wave of CTAs) and the first 5 of them alone give the
    same bits (outputs and states), and the large batch matches the port."""
    rng = np.random.default_rng(79)
    H, d, ck = 16, 128, 4
    conv_dim = 3 * H * d
    w = dict(conv_w=(rng.standard_normal((conv_dim, ck)) * 0.5).astype(np.float32),
             dt_bias=rng.standard_normal(H).astype(np.float32), A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
             norm_w=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    outs, states = {}, {}
    S = (0.02 * rng.standard_normal((40, H, d, d))).astype(np.float32)
    conv = rng.standard_normal((40, conv_dim, ck)).astype(np.float32)
    xs = [(rng.standard_normal((40, conv_dim)).astype(np.float32), rng.standard_normal((40, H * d)).astype(np.float32),
           rng.standard_normal((40, H)).astype(np.float32), rng.standard_normal((40, H)).astype(np.float32))
          for _ in range(2)]
    for B in (40, 5):
        st = pkg.DeltaState(ctx, 1, B, H, d, d, ck)
        st.set_weights(0, **w)
        for b in range(B):
            st.upload(0, b, S=S[b], conv_state=conv[b])
        outs[B] = [st.core(0, *(x[:B] for x in xt)) for xt in xs]
        states[B] = [st.download(0, b)[0] for b in range(5)]
    for t in range(2):
        assert np.array_equal(outs[40][t][:5], outs[5][t])
    for b in range(5):
        assert np.array_equal(states[40][b], states[5][b])
    Sr, cr = S.copy(), conv.copy()
    for t, (qkv, z, bb, aa) in enumerate(xs):
        for b in (0, 17, 39):
            ref = orc.deltanet_core(qkv[b], z[b], bb[b], aa[b], cr[b], Sr[b], **w)
            assert rel_l2(outs[40][t][b], ref) <= TOL, (t, b)


@pytest.mark.parametrize("hd", [64, 128, 256])
def test_fullatt_prep_head_dims(pkg, ctx, orc, hd):
    """fullatt_prep for 2 sequences at head_dim 64 / 128 / 256 (2, 4, 8 elements per lane in the
    warp-per-head kernel), fp32 cache, against the restatement; then the same rows through the
    device-pointer entry with every array one float off 16-byte alignment (the per-row kernel)."""
    import torch
    rng = np.random.default_rng(92 + hd)
    B, nh, nkv, T = 2, 4, 2, 16
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.F32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kv.set_norms(0, qn, kn)
    qg = rng.standard_normal((B, nh * 2 * hd)).astype(np.float32)
    k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    pos = np.array([3, 9], np.int32)
    q, g = kv.fullatt_prep(0, qg, k, v, pos, nh)
    kc = np.zeros((T, nkv * hd), np.float32)
    for b in range(B):
        rq, rg, rk = orc.fullatt_prep(qg[b], k[b], v[b], qn, kn, kc.copy(), kc.copy(), pos[b], nh, nkv, hd)
        assert rel_l2(q[b], rq) <= TOL and np.array_equal(g[b], rg)
        kd, vd = kv.download(0, b, pos[b], 1)
        assert rel_l2(kd[0], rk) <= TOL and np.array_equal(vd[0], v[b])

    def off(a):  # a device copy starting one float past a 16-byte boundary
        t = torch.zeros(a.size + 1, dtype=torch.float32, device="cuda")
        t[1:] = torch.from_numpy(np.ascontiguousarray(a).ravel()).cuda()
        return t
    tq, tk, tv = off(qg), off(k), off(v)
    tqo, tgo = off(np.zeros_like(q)), off(np.zeros_like(g))
    tpos = torch.from_numpy(pos + 1).cuda()
    torch.cuda.synchronize()
    kv.fullatt_prep_dev(0, tq.data_ptr() + 4, tk.data_ptr() + 4, tv.data_ptr() + 4, tpos.data_ptr(), nh,
                        tqo.data_ptr() + 4, tgo.data_ptr() + 4)
    ctx.synchronize()
    q2 = tqo[1:].cpu().numpy().reshape(q.shape)
    assert np.array_equal(tgo[1:].cpu().numpy().reshape(g.shape), g)
    for b in range(B):  # rows at pos + 1
        rq, _, rk = orc.fullatt_prep(qg[b], k[b], v[b], qn, kn, kc.copy(), kc.copy(), pos[b] + 1, nh, nkv, hd)
        assert rel_l2(q2[b], rq) <= TOL
        kd, vd = kv.download(0, b, pos[b] + 1, 1)
        assert rel_l2(kd[0], rk) <= TOL and np.array_equal(vd[0], v[b])


@pytest.mark.parametrize("api", ["two_calls", "one_call"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_qwen35_attention_layer_chain(pkg, ctx, orc, dtype, api):
    """Several decode steps of a Qwen3.5 full-attention layer for a batch with ragged positions:
    fullatt_prep (norms, partial RoPE, append) then attend with the sigmoid gate and SubLN -- as two calls, or
    as the one call eif_cuda_fullatt_decode -- against the restatement of fullatt_prep + fullatt_attend."""
    rng = np.random.default_rng(88)
    B, nh, nkv, hd, T = 3, 8, 2, 256, 48
    dt = pkg.F32 if dtype == "f32" else pkg.BF16
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    sub = (1 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    kv.set_norms(0, qn, kn)
    kc = np.zeros((B, T, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    pos = np.array([0, 5, 20], np.int32)
    for step in range(6):
        qg = rng.standard_normal((B, nh * 2 * hd)).astype(np.float32)
        k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        if api == "two_calls":
            q, g = kv.fullatt_prep(0, qg, k, v, pos, nh)
            out = kv.attend_decode(0, q, pos, nh, 1.0 / 16, gate=g, subln=pkg.SUBLN_WEIGHT, sub_norm=sub)
        else:
            out = kv.fullatt_decode(0, qg, k, v, pos, nh, 1.0 / 16, subln=pkg.SUBLN_WEIGHT, sub_norm=sub)
        for b in range(B):
            rq, rg, _ = orc.fullatt_prep(qg[b], k[b], v[b], qn, kn, kc[b], vc[b], pos[b], nh, nkv, hd)
            if dt == pkg.BF16:
                kc[b, pos[b]] = orc.round_bf16(kc[b, pos[b]])
                vc[b, pos[b]] = orc.round_bf16(vc[b, pos[b]])
            if api == "two_calls":
                assert rel_l2(q[b], rq) <= TOL and np.array_equal(g[b], rg)
            ref = orc.subln(orc.attend_decode(rq, kc[b], vc[b], pos[b], nh, nkv, hd, 1.0 / 16, gate=rg), sub, 2)
            assert rel_l2(out[b], ref) <= TOL, (step, b)
        pos = pos + 1


def test_qwen35_attention_prefill_chain(pkg, ctx, orc):
    """A Qwen3.5 full-attention layer over a prefill chunk as prefill_chunk runs it (src/eif_qwen35.c:1122-1133):
    fullatt_prep for every token of the chunk (one launch), then the gated causal prefill attention, on a bf16
    cache that already holds earlier rows; against fullatt_prep + attention + gate + SubLN token by token.
    fp32 prep outputs: rel-L2 <= 1e-5; the bf16 prefill attention: rel-L2 <= 1e-2, max-abs <= 2e-2."""
    rng = np.random.default_rng(91)
    B, nh, nkv, hd, start, n = 2, 8, 2, 256, 20, 100
    T = start + n + 4
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.BF16)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    sub = (1 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    kv.set_norms(0, qn, kn)
    kc = np.zeros((B, T, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:, :start] = orc.round_bf16(rng.standard_normal((B, start, nkv * hd))).reshape(B, start, -1)
    vc[:, :start] = orc.round_bf16(rng.standard_normal((B, start, nkv * hd))).reshape(B, start, -1)
    for b in range(B):
        kv.upload(0, b, 0, kc[b, :start], vc[b, :start])
    qg = rng.standard_normal((B, n, nh * 2 * hd)).astype(np.float32)
    k = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    q, g = kv.fullatt_prep_prefill(0, qg, k, v, n, start, nh)
    out = kv.attend_prefill_gated(0, q, n, start, nh, 1.0 / 16, g, pkg.SUBLN_WEIGHT, sub)
    for b in range(B):
        rq = np.zeros((n, nh * hd), np.float32)
        for i in range(n):
            rq[i], rg, _ = orc.fullatt_prep(qg[b, i], k[b, i], v[b, i], qn, kn, kc[b], vc[b], start + i, nh, nkv, hd)
            assert np.array_equal(g[b, i], rg)
            kc[b, start + i] = orc.round_bf16(kc[b, start + i])
            vc[b, start + i] = orc.round_bf16(vc[b, start + i])
        assert rel_l2(q[b], rq) <= TOL
        kd, vd = kv.download(0, b, 0, start + n)
        assert np.array_equal(vd, vc[b, :start + n])
        # k is normed and rotated in fp32 on both sides (rel ~1e-7 apart), then rounded to bf16: one ulp at most
        assert np.all(np.abs(kd - kc[b, :start + n]) <= 2.0 ** -7 * np.abs(kc[b, :start + n]) + 1e-30)
        q16 = orc.round_bf16(rq).reshape(n, -1)
        ref = np.stack([orc.subln(orc.attend_decode(q16[i], kc[b], vc[b], start + i, nh, nkv, hd, 1.0 / 16, gate=g[b, i]),
                                  sub, 2) for i in range(n)])
        assert rel_l2(out[b], ref) <= 1e-2 and np.max(np.abs(out[b] - ref)) <= 2e-2


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_fullatt_prefill_one_call(pkg, ctx, orc, dtype):
    """eif_cuda_fullatt_prefill (the chunk's fullatt_prep and the gated causal attention in one call) against
    fullatt_prep_prefill + attend_prefill_gated on a second cache; over the reference's own fp32 cache, also
    against fullatt_prep + fullatt_attend token by token at the fp32 tolerance (rel-L2 <= 1e-5)."""
    rng = np.random.default_rng(92)
    dt = pkg.F32 if dtype == "f32" else pkg.BF16
    B, nh, nkv, hd, start, n = 2, 8, 2, 256, 20, 70
    T = start + n + 4
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    sub = (1 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    k0 = rng.standard_normal((B, start, nkv * hd)).astype(np.float32)
    v0 = rng.standard_normal((B, start, nkv * hd)).astype(np.float32)
    kvs = []
    for _ in range(2):
        kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
        kv.set_norms(0, qn, kn)
        for b in range(B):
            kv.upload(0, b, 0, k0[b], v0[b])
        kvs.append(kv)
    qg = rng.standard_normal((B, n, nh * 2 * hd)).astype(np.float32)
    k = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, n, nkv * hd)).astype(np.float32)
    q, g = kvs[0].fullatt_prep_prefill(0, qg, k, v, n, start, nh)
    two = kvs[0].attend_prefill_gated(0, q, n, start, nh, 1.0 / 16, g, pkg.SUBLN_WEIGHT, sub)
    one = kvs[1].fullatt_prefill(0, qg, k, v, n, start, nh, 1.0 / 16, subln=pkg.SUBLN_WEIGHT, sub_norm=sub)
    for b in range(B):
        for a_, b_ in zip(kvs[0].download(0, b, 0, T), kvs[1].download(0, b, 0, T)):
            assert np.array_equal(a_, b_)
        assert rel_l2(one[b], two[b]) <= (1e-5 if dt == pkg.F32 else 1e-2)
    if dt == pkg.F32:
        for b in range(B):
            kc = np.zeros((T, nkv * hd), np.float32)
            vc = np.zeros_like(kc)
            kc[:start], vc[:start] = k0[b], v0[b]
            for i in range(n):
                rq, rg, _ = orc.fullatt_prep(qg[b, i], k[b, i], v[b, i], qn, kn, kc, vc, start + i, nh, nkv, hd)
                ref = orc.subln(orc.attend_decode(rq, kc, vc, start + i, nh, nkv, hd, 1.0 / 16, gate=rg), sub, 2)
                assert rel_l2(one[b, i], ref) <= 1e-5, (b, i)
    for kv in kvs:
        kv.free()


def test_deltanet_core_host_matches_dev(pkg, ctx):
    """A host-pointer deltanet_core at a serving batch (160 sequences, 5.3 MB of inputs per call) against the
    device-pointer call on a twin state: the same bits, outputs and states."""
    import torch

    class CudaArray:  # a library allocation seen by torch without a copy
        def __init__(self, ptr, shape, typestr):
            self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr, "version": 3}
    rng = np.random.default_rng(93)
    B, H, d, ck = 160, 16, 128, 4
    conv_dim = 3 * H * d
    w = dict(conv_w=(rng.standard_normal((conv_dim, ck)) * 0.5).astype(np.float32),
             dt_bias=rng.standard_normal(H).astype(np.float32), A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
             norm_w=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32))
    sts = [pkg.DeltaState(ctx, 1, B, H, d, d, ck) for _ in range(2)]
    views = []
    for st in sts:
        st.set_weights(0, **w)
        s_ptr, c_ptr = st.layer_ptrs(0)
        views.append((torch.as_tensor(CudaArray(s_ptr, (B * H * d * d,), "<f4"), device="cuda"),
                      torch.as_tensor(CudaArray(c_ptr, (B * conv_dim * ck,), "<f4"), device="cuda")))
    gen = torch.Generator(device="cuda").manual_seed(3)
    views[0][0].normal_(0, 0.02, generator=gen)
    views[0][1].normal_(generator=gen)
    views[1][0].copy_(views[0][0])
    views[1][1].copy_(views[0][1])
    torch.cuda.synchronize()
    for t in range(2):
        qkv = rng.standard_normal((B, conv_dim)).astype(np.float32)
        z = rng.standard_normal((B, H * d)).astype(np.float32)
        bb = rng.standard_normal((B, H)).astype(np.float32)
        aa = rng.standard_normal((B, H)).astype(np.float32)
        out_host = sts[0].core(0, qkv, z, bb, aa)
        dev = [torch.from_numpy(x).cuda() for x in (qkv, z, bb, aa)]
        out_dev = torch.zeros((B, H * d), device="cuda")
        torch.cuda.synchronize()
        sts[1].core_dev(0, *(x.data_ptr() for x in dev), out_dev.data_ptr())
        ctx.synchronize()
        assert np.array_equal(out_host, out_dev.cpu().numpy()), t
    assert torch.equal(views[0][0], views[1][0]) and torch.equal(views[0][1], views[1][1])


def test_deltanet_core_back_to_back_launches(pkg, ctx):
    """deltanet_core launches as a programmatic dependent and, when the launch just before it wrote another
    layer's state, reads its own state before its grid-dependency wait.  A run of device-pointer calls with
    nothing between them (the same layer twice in a row, then alternating layers) must leave the same bits as
    the same calls with a synchronisation after each, where no launch can overlap another."""
    import torch

    class CudaArray:
        def __init__(self, ptr, shape, typestr):
            self.__cuda_array_interface__ = {"data": (ptr, False), "shape": shape, "typestr": typestr, "version": 3}
    rng = np.random.default_rng(97)
    B, H, d, ck = 24, 16, 128, 4
    conv_dim = 3 * H * d
    order = [0, 0, 1, 0, 1, 1, 0, 1]
    sts = [pkg.DeltaState(ctx, 2, B, H, d, d, ck) for _ in range(2)]
    views = []
    # the same weights for both twins
    wts = [dict(conv_w=(0.5 * rng.standard_normal((conv_dim, ck))).astype(np.float32),
                dt_bias=rng.standard_normal(H).astype(np.float32),
                A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
                norm_w=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32)) for _ in range(2)]
    for st in sts:
        for layer in range(2):
            st.set_weights(layer, **wts[layer])
            s_ptr, c_ptr = st.layer_ptrs(layer)
            views.append((torch.as_tensor(CudaArray(s_ptr, (B * H * d * d,), "<f4"), device="cuda"),
                          torch.as_tensor(CudaArray(c_ptr, (B * conv_dim * ck,), "<f4"), device="cuda")))
    gen = torch.Generator(device="cuda").manual_seed(5)
    for layer in range(2):  # views: [twin 0 layer 0, twin 0 layer 1, twin 1 layer 0, twin 1 layer 1]
        views[layer][0].normal_(0, 0.02, generator=gen)
        views[layer][1].normal_(generator=gen)
        views[2 + layer][0].copy_(views[layer][0])
        views[2 + layer][1].copy_(views[layer][1])
    ins = [[torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).cuda()
            for shape in ((B, conv_dim), (B, H * d), (B, H), (B, H))] for _ in order]
    outs = [[torch.zeros((B, H * d), device="cuda") for _ in order] for _ in range(2)]
    torch.cuda.synchronize()
    for k, layer in enumerate(order):  # twin 0: back to back
        sts[0].core_dev(layer, *(x.data_ptr() for x in ins[k]), outs[0][k].data_ptr())
    ctx.synchronize()
    for k, layer in enumerate(order):  # twin 1: one call at a time
        sts[1].core_dev(layer, *(x.data_ptr() for x in ins[k]), outs[1][k].data_ptr())
        ctx.synchronize()
    for k in range(len(order)):
        assert torch.equal(outs[0][k], outs[1][k]), k
    for layer in range(2):
        assert torch.equal(views[layer][0], views[2 + layer][0]) and torch.equal(views[layer][1], views[2 + layer][1])
