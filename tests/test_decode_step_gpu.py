"""The whole tinyllm decode step in one call (eif_cuda_decode_step[_dev]: RoPE of q and k, the new K / V row,
attention over [0, pos]) against the C restatement of src/eif_tinyllm.c:395-405 / :480-507 (RoPE), :509-549
(INT8 row) and :555-656 (the head loop), step after step on ragged positions.  Small batches of fp32 / bf16
caches take the one-launch cluster kernel; INT8 caches and large batches take rope_append's kernel and the
split-K decode.  fp32 arithmetic throughout: rel-L2 <= 1e-5."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def run_chain(pkg, ctx, orc, B, hd, nh, nkv, theta, inter, dtype, steps, pos0, T, seed):
    """Rows [0, pos0[b]) uploaded, then `steps` decode steps of every sequence from pos0[b] on; returns the
    worst rel-L2 of the outputs against the port."""
    rng = np.random.default_rng(seed)
    dt = {"f32": pkg.F32, "bf16": pkg.BF16, "int8": pkg.INT8}[dtype]
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    kv.set_rope(theta, inter)
    scale = 1.0 / np.sqrt(hd)
    kc = np.zeros((B, T, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    ks = np.zeros((B, T, nkv), np.float32)
    vs = np.zeros_like(ks)
    k8 = np.zeros((B, T, nkv * hd), np.int8)
    v8 = np.zeros_like(k8)

    def put(b, t0, kr, vr):  # the cache content the device holds for rows [t0, t0 + len)
        n = kr.shape[0]
        if dtype == "int8":
            k8[b, t0:t0 + n], ks[b, t0:t0 + n] = orc.kv_quantize(kr, nkv, hd)
            v8[b, t0:t0 + n], vs[b, t0:t0 + n] = orc.kv_quantize(vr, nkv, hd)
        elif dtype == "bf16":
            kc[b, t0:t0 + n], vc[b, t0:t0 + n] = orc.round_bf16(kr), orc.round_bf16(vr)
        else:
            kc[b, t0:t0 + n], vc[b, t0:t0 + n] = kr, vr
    for b in range(B):
        if pos0[b]:
            kr = rng.standard_normal((pos0[b], nkv * hd)).astype(np.float32)
            vr = rng.standard_normal((pos0[b], nkv * hd)).astype(np.float32)
            kv.upload(0, b, 0, kr, vr)
            put(b, 0, kr, vr)
    worst = 0.0
    for step in range(steps):
        p = (np.array(pos0) + step).astype(np.int32)
        q = rng.standard_normal((B, nh * hd)).astype(np.float32)
        k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        out = kv.decode_step(0, q, k, v, p, nh, scale)
        for b in range(B):
            t = int(p[b])
            put(b, t, orc.rope_apply(k[b], nkv, hd, t, theta, inter)[None], v[b][None])
            qr = orc.rope_apply(q[b], nh, hd, t, theta, inter)
            if dtype == "int8":
                ref = orc.attend_decode_i8(qr, k8[b], ks[b], v8[b], vs[b], t, nh, nkv, hd, scale)
            else:
                ref = orc.attend_decode(qr, kc[b], vc[b], t, nh, nkv, hd, scale)
            worst = max(worst, rel_l2(out[b], ref))
    return worst


@pytest.mark.parametrize("B,hd,nh,nkv,theta,inter,dtype", [
    (1, 64, 14, 2, 1e6, False, "f32"),    # BASELINE config 1's heads: one launch, up to 8 CTAs per kv head
    (3, 128, 8, 2, 1e4, True, "bf16"),    # adjacent pairs, bf16 rows
    (2, 64, 16, 2, 1e6, False, "f32"),    # 8 q heads per kv head
    (2, 128, 4, 4, 5e5, False, "bf16"),   # G = 1
    (2, 64, 14, 2, 1e6, False, "int8"),   # INT8 cache: rope_append's kernel + the INT8 decode
    (160, 64, 14, 2, 1e6, False, "f32"),  # 320 (sequence, kv head) units: the two-launch form
])
def test_decode_step_vs_port(pkg, ctx, orc, B, hd, nh, nkv, theta, inter, dtype):
    pos0 = [(137 * b + 511) % 590 for b in range(B)]  # 511 first: 8 CTAs of 64 keys per kv head
    worst = run_chain(pkg, ctx, orc, B, hd, nh, nkv, theta, inter, dtype, steps=3, pos0=pos0, T=600, seed=B + hd)
    assert worst <= TOL


def test_decode_step_long_context(pkg, ctx, orc):
    """One step at pos 4999 over rows uploaded before (fp32, 14 / 2 heads): more keys than the one-launch
    kernel stages, so rope_append's kernel and the split-K decode."""
    rng = np.random.default_rng(11)
    nh, nkv, hd, T, t = 14, 2, 64, 5008, 4999
    kv = pkg.KVCache(ctx, 1, 1, T, nkv, hd, pkg.F32)
    kv.set_rope(1e6, False)
    kc = rng.standard_normal((T, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((T, nkv * hd)).astype(np.float32)
    kv.upload(0, 0, 0, kc[:t], vc[:t])
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    v = rng.standard_normal(nkv * hd).astype(np.float32)
    out = kv.decode_step(0, q[None], k[None], v[None], np.array([t], np.int32), nh, 0.125)
    kc[t], vc[t] = orc.rope_apply(k, nkv, hd, t, 1e6), v
    ref = orc.attend_decode(orc.rope_apply(q, nh, hd, t, 1e6), kc, vc, t, nh, nkv, hd, 0.125)
    assert rel_l2(out[0], ref) <= TOL
    kd, vd = kv.download(0, 0, t, 1)
    assert rel_l2(kd[0], kc[t]) <= TOL and np.array_equal(vd[0], v)


def test_decode_step_matches_two_calls(pkg, ctx):
    """The one-launch step against rope_append + attend_decode on a twin cache: same rows, outputs within 1e-6."""
    import torch
    rng = np.random.default_rng(12)
    B, nh, nkv, hd, T = 2, 14, 2, 64, 300
    a = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.F32)
    c = pkg.KVCache(ctx, 1, B, T, nkv, hd, pkg.F32)
    for kv in (a, c):
        kv.set_rope(1e6, False)
    rows = rng.standard_normal((B, 200, nkv * hd)).astype(np.float32)
    for b in range(B):
        a.upload(0, b, 0, rows[b], 2 * rows[b])
        c.upload(0, b, 0, rows[b], 2 * rows[b])
    pos = np.array([200, 150], np.int32)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    k = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((B, nkv * hd)).astype(np.float32)
    tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    tp = torch.from_numpy(pos).cuda()
    to = torch.zeros((B, nh * hd), device="cuda")
    torch.cuda.synchronize()
    a.decode_step_dev(0, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tp.data_ptr(), 200, nh, 0.125, to.data_ptr())
    ctx.synchronize()
    qr = c.rope_append(0, q, k, v, pos, nh)
    ref = c.attend_decode(0, qr, pos, nh, 0.125)
    assert rel_l2(to.cpu().numpy(), ref) <= 1e-6
    for b in range(B):
        assert np.array_equal(a.download(0, b, pos[b], 1)[0], c.download(0, b, pos[b], 1)[0])


def test_decode_step_rejections(pkg, ctx):
    kv = pkg.KVCache(ctx, 1, 1, 16, 2, 64, pkg.F32)
    z = np.zeros((1, 14 * 64), np.float32)
    zk = np.zeros((1, 128), np.float32)
    with pytest.raises(pkg.EifCudaError) as e:  # no RoPE table yet
        kv.decode_step(0, z, zk, zk, np.array([0], np.int32), 14, 0.125)
    assert e.value.name == "INVALID_ARGUMENT"
    kv.set_rope(1e6, False)
    with pytest.raises(pkg.EifCudaError) as e:
        kv.decode_step(0, z, zk, zk, np.array([16], np.int32), 14, 0.125)
    assert e.value.name == "INVALID_ARGUMENT"
    with pytest.raises(pkg.EifCudaError) as e:
        kv.decode_step(0, z, zk, zk, np.array([0], np.int32), 13, 0.125)
    assert e.value.name == "SHAPE_MISMATCH"
