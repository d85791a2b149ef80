"""Decode attention through the C ABI against the reference (golden fixtures) and the C restatement.

Tolerance: rel-L2 <= 1e-5 for fp32 caches (the north-star bound for the fp32 decode path).  bf16
caches are compared with the fp32 oracle run on the same bf16-rounded rows, also at 1e-5: the
kernels accumulate in fp32, so only the storage is narrower."""
import numpy as np
import pytest

from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, dtype, max_seq=None):
    max_seq = max_seq or T
    kv = pkg.KVCache(ctx, 1, B, max_seq, nkv, hd, dtype)
    kc = rng.standard_normal((B, T, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((B, T, nkv * hd)).astype(np.float32)
    if dtype == pkg.BF16:
        kc = orc.round_bf16(kc).reshape(kc.shape)
        vc = orc.round_bf16(vc).reshape(vc.shape)
    for b in range(B):
        kv.upload(0, b, 0, kc[b], vc[b])
    return kv, kc, vc


def test_golden_cfg1(pkg, ctx):
    """BASELINE config 1 (Qwen2.5-0.5B decode shape) against the reference's fullatt_attend."""
    d = golden("decode_cfg1.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    kv = pkg.KVCache(ctx, 1, 1, pos + 1, nkv, hd, pkg.F32)
    kv.upload(0, 0, 0, d["k_cache"], d["v_cache"])
    out = kv.attend_decode(0, d["q"][None], np.array([pos]), nh, 1.0 / np.sqrt(hd))
    assert rel_l2(out[0], d["out"]) <= TOL


def test_golden_fullatt_gate_subln(pkg, ctx):
    d = golden("fullatt_attend.npz")
    nh, nkv, hd, pos = (int(x) for x in d["meta"])
    kv = pkg.KVCache(ctx, 1, 1, d["k_cache"].shape[0], nkv, hd, pkg.F32)
    kv.upload(0, 0, 0, d["k_cache"], d["v_cache"])
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    for mode, key, w in [(pkg.SUBLN_NONE, "out_plain", None), (pkg.SUBLN_RMS, "out_rms", None),
                         (pkg.SUBLN_WEIGHT, "out_subln", d["sub_norm"])]:
        out = kv.attend_decode(0, d["q"][None], np.array([pos]), nh, scale, gate=d["gate"][None], subln=mode,
                               sub_norm=w)
        assert rel_l2(out[0], d[key]) <= TOL, key


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("hd,nh,nkv", [(64, 14, 2), (64, 9, 3), (128, 12, 2), (128, 16, 2), (256, 8, 2),
                                       (64, 32, 32), (128, 40, 8), (256, 10, 2)])
def test_random_ragged(pkg, ctx, orc, dtype, hd, nh, nkv):
    """Ragged pos across the batch (including 0 and max_seq-1); all group sizes 1..8."""
    rng = np.random.default_rng(hd * 1000 + nh * 10 + nkv)
    dt = pkg.F32 if dtype == "f32" else pkg.BF16
    B, T = 4, 333
    kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, dt)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([T - 1, 0, 64, 129], np.int32)
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_decode(0, q, pos, nh, scale)
    for b in range(B):
        ref = orc.attend_decode(q[b], kc[b], vc[b], pos[b], nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= TOL, (b, pos[b])


@pytest.mark.parametrize("hd,nh,nkv", [(256, 8, 2), (128, 14, 2), (64, 16, 2)])
def test_bf16_tensor_core_and_simt_paths_agree(pkg, ctx, orc, monkeypatch, hd, nh, nkv):
    """The bf16 cache runs on the TMA + tensor-core kernel; BITLLM_DECODE_SIMT=1 selects the SIMT kernel.
    Both must match the oracle on the same bf16 rows (many items per persistent CTA, ragged tails)."""
    rng = np.random.default_rng(hd + nh)
    B, T = 5, 1500
    kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, pkg.BF16)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    gate = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([T - 1, 1, 63, 64, 1000], np.int32)
    scale = 1.0 / np.sqrt(hd)
    out_tc = kv.attend_decode(0, q, pos, nh, scale, gate=gate, subln=pkg.SUBLN_RMS)
    monkeypatch.setenv("BITLLM_DECODE_SIMT", "1")
    out_simt = kv.attend_decode(0, q, pos, nh, scale, gate=gate, subln=pkg.SUBLN_RMS)
    for b in range(B):
        ref = orc.subln(orc.attend_decode(q[b], kc[b], vc[b], pos[b], nh, nkv, hd, scale, gate=gate[b]), None, 1)
        assert rel_l2(out_tc[b], ref) <= TOL, ("tc", b)
        assert rel_l2(out_simt[b], ref) <= TOL, ("simt", b)


def test_rows_past_pos_are_never_used(pkg, ctx, orc):
    """Rows after pos[b] hold non-finite garbage: the output must not depend on them (the reference reads
    only rows 0..pos, src/eif_qwen35.c:757-770)."""
    rng = np.random.default_rng(21)
    nh, nkv, hd, T, B = 8, 2, 256, 300, 2
    for dt in (pkg.BF16, pkg.F32):
        kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, dt)
        pos = np.array([100, 37], np.int32)
        for b in range(B):
            junk = np.full((T - pos[b] - 1, nkv * hd), np.nan, np.float32)
            junk[::2] = np.inf
            kv.upload(0, b, int(pos[b]) + 1, junk, -junk)
        q = rng.standard_normal((B, nh * hd)).astype(np.float32)
        out = kv.attend_decode(0, q, pos, nh, 0.0625)
        assert np.all(np.isfinite(out))
        for b in range(B):
            assert rel_l2(out[b], orc.attend_decode(q[b], kc[b], vc[b], pos[b], nh, nkv, hd, 0.0625)) <= TOL


def test_pos0_copies_v(pkg, ctx, orc):
    """Known answer (reference tests/test_gguf_gqa_layout.c:105): at pos 0 the output is v_0 of the group."""
    rng = np.random.default_rng(5)
    nh, nkv, hd = 4, 2, 64
    kv, kc, vc = make_cache(pkg, ctx, orc, rng, 2, 8, nkv, hd, pkg.F32)
    out = kv.attend_decode(0, rng.standard_normal((2, nh * hd)), np.array([0, 0]), nh, 0.125)
    for b in range(2):
        for h in range(nh):
            kvh = h // (nh // nkv)
            np.testing.assert_allclose(out[b, h * hd:(h + 1) * hd], vc[b, 0, kvh * hd:(kvh + 1) * hd], rtol=0,
                                       atol=1e-6)


def test_long_context_bf16_gate(pkg, ctx, orc):
    """Qwen3.5 attention shape at a long context with the sigmoid gate (sampled sequences of a batch)."""
    rng = np.random.default_rng(9)
    nh, nkv, hd, T, B = 8, 2, 256, 8192, 3
    kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, pkg.BF16)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    gate = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([T - 1, T - 1000, 4097], np.int32)
    out = kv.attend_decode(0, q, pos, nh, 1 / 16.0, gate=gate)
    for b in range(B):
        ref = orc.attend_decode(q[b], kc[b], vc[b], pos[b], nh, nkv, hd, 1 / 16.0, gate=gate[b])
        assert rel_l2(out[b], ref) <= TOL


def test_append_then_attend(pkg, ctx, orc):
    """kv_append writes row pos[b]; attention then sees it (the engine's prep -> attend order)."""
    rng = np.random.default_rng(10)
    nh, nkv, hd, T, B = 8, 2, 128, 40, 3
    for dt in (pkg.F32, pkg.BF16):
        kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, dt)
        pos = np.array([5, 39, 17], np.int32)
        knew = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        vnew = rng.standard_normal((B, nkv * hd)).astype(np.float32)
        kv.append(0, pos, knew, vnew)
        if dt == pkg.BF16:
            knew = orc.round_bf16(knew).reshape(knew.shape)
            vnew = orc.round_bf16(vnew).reshape(vnew.shape)
        for b in range(B):
            kc[b, pos[b]] = knew[b]
            vc[b, pos[b]] = vnew[b]
            kd, vd = kv.download(0, b, 0, T)
            assert np.array_equal(kd, kc[b]) and np.array_equal(vd, vc[b])
        q = rng.standard_normal((B, nh * hd)).astype(np.float32)
        out = kv.attend_decode(0, q, pos, nh, 0.1)
        for b in range(B):
            assert rel_l2(out[b], orc.attend_decode(q[b], kc[b], vc[b], pos[b], nh, nkv, hd, 0.1)) <= TOL


def test_bad_arguments(pkg, ctx):
    kv = pkg.KVCache(ctx, 2, 2, 16, 2, 64, pkg.F32)
    q = np.zeros((2, 4 * 64), np.float32)
    with pytest.raises(pkg.EifCudaError) as e:
        kv.attend_decode(0, q, np.array([3, 16]), 4, 0.1)  # pos == max_seq_len
    assert e.value.name == "INVALID_ARGUMENT"
    with pytest.raises(pkg.EifCudaError) as e:
        kv.attend_decode(0, np.zeros((2, 3 * 64), np.float32), np.array([1, 1]), 3, 0.1)
    assert e.value.name == "SHAPE_MISMATCH"
    with pytest.raises(pkg.EifCudaError) as e:
        kv.attend_decode(2, q, np.array([1, 1]), 4, 0.1)
    assert e.value.name == "INVALID_LAYER"
    with pytest.raises(pkg.EifCudaError) as e:
        kv.append(0, np.array([0, -1]), np.zeros((2, 128), np.float32), np.zeros((2, 128), np.float32))
    assert e.value.name == "INVALID_ARGUMENT"
    # the context stays usable after refusals
    out = kv.attend_decode(0, q, np.array([0, 15]), 4, 0.1)
    assert np.all(np.isfinite(out))


def test_device_pos_out_of_range_reported(pkg, ctx):
    """A device-side pos outside the cache is caught by the kernels' bounds check, skipped, and reported
    as INVALID_ARGUMENT at the next synchronize (nothing out of bounds is read or written)."""
    import torch
    kv = pkg.KVCache(ctx, 1, 2, 16, 2, 64, pkg.F32)
    q = torch.zeros((2, 4 * 64), device="cuda")
    out = torch.zeros_like(q)
    pos = torch.tensor([3, 99], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    kv.attend_decode_dev(0, q.data_ptr(), pos.data_ptr(), 15, 4, 0.1, out.data_ptr())
    with pytest.raises(pkg.EifCudaError) as e:
        ctx.synchronize()
    assert e.value.name == "INVALID_ARGUMENT"
    ctx.synchronize()  # error word cleared
    assert torch.all(out[1] == 0)


@pytest.mark.parametrize("dtype", ["f32", "bf16", "int8", "simt"])
def test_device_pos_above_max_pos_reported(pkg, ctx, orc, monkeypatch, dtype):
    """A device-side pos inside the cache but above the call's max_pos (the bound the split was sized for)
    is skipped and reported like one outside the cache, never answered from a truncated key range; the
    other sequences of the batch are still computed."""
    import torch
    if dtype == "simt":
        monkeypatch.setenv("BITLLM_DECODE_SIMT", "1")
    dt = {"f32": pkg.F32, "bf16": pkg.BF16, "int8": pkg.INT8, "simt": pkg.BF16}[dtype]
    rng = np.random.default_rng(31)
    B, T, nh, nkv, hd = 3, 600, 8, 2, 128
    kv, kc, vc = make_cache(pkg, ctx, orc, rng, B, T, nkv, hd, dt)  # an INT8 cache quantises on upload
    qn = rng.standard_normal((B, nh * hd)).astype(np.float32)
    q = torch.from_numpy(qn).cuda()
    out = torch.full((B, nh * hd), 7.0, device="cuda")
    pos_np = np.array([100, 599, 64], np.int32)
    pos = torch.from_numpy(pos_np).cuda()
    torch.cuda.synchronize()
    kv.attend_decode_dev(0, q.data_ptr(), pos.data_ptr(), 128, nh, 0.1, out.data_ptr())  # bound 128 < 599
    with pytest.raises(pkg.EifCudaError) as e:
        ctx.synchronize()
    assert e.value.name == "INVALID_ARGUMENT"
    ctx.synchronize()
    o = out.cpu().numpy()
    assert np.all(o[1] == 0)
    for b in (0, 2):
        if dt == pkg.INT8:
            kq, vq, ks, vs = kv.download_int8(0, b, 0, T)
            ref = orc.attend_decode_i8(qn[b], kq, ks, vq, vs, int(pos_np[b]), nh, nkv, hd, 0.1)
        else:
            ref = orc.attend_decode(qn[b], kc[b], vc[b], int(pos_np[b]), nh, nkv, hd, 0.1)
        assert rel_l2(o[b], ref) <= TOL, b
    kv.free()


@pytest.mark.parametrize("dtype", ["f32", "bf16", "int8"])
@pytest.mark.parametrize("hd,nh,nkv", [(64, 14, 2), (128, 8, 2), (64, 2, 2), (256, 8, 2)])
def test_many_items_per_cta(pkg, ctx, orc, dtype, hd, nh, nkv):
    """Batches whose (sequence, kv head, chunk) items outnumber the SMs, so every persistent CTA runs several
    items and its TMA ring is reused across them and across consumer warps (the regime of the benchmarks).
    Sampled sequences against the restatement; INT8 through the codes it stored."""
    rng = np.random.default_rng(hd + nh + 7)
    B, T = 200, 700
    dt = {"f32": pkg.F32, "bf16": pkg.BF16, "int8": pkg.INT8}[dtype]
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    pos = rng.integers(T // 2, T, B).astype(np.int32)
    pos[:3] = [T - 1, 0, 63]
    sample = [0, 1, 2, 77, 150, B - 1]
    rows = {}
    for b in range(B):
        k = rng.standard_normal((T, nkv * hd)).astype(np.float32)
        v = rng.standard_normal((T, nkv * hd)).astype(np.float32)
        kv.upload(0, b, 0, k, v)
        if b in sample:
            rows[b] = (k, v)
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    for _ in range(2):  # a second call reuses the context's scratch and the layer's tensor maps
        out = kv.attend_decode(0, q, pos, nh, scale)
    for b in sample:
        if dtype == "int8":
            kc, vc, ks, vs = kv.download_int8(0, b, 0, T)
            ref = orc.attend_decode_i8(q[b], kc, ks, vc, vs, int(pos[b]), nh, nkv, hd, scale)
        else:
            k, v = rows[b]
            if dtype == "bf16":
                k, v = orc.round_bf16(k).reshape(k.shape), orc.round_bf16(v).reshape(v.shape)
            ref = orc.attend_decode(q[b], k, v, int(pos[b]), nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= TOL, (b, int(pos[b]))


@pytest.mark.parametrize("dtype", ["F32", "BF16", "INT8"])
def test_device_q_unaligned(pkg, ctx, dtype):
    """A q_dev that is 4- but not 16-byte aligned (a view one float into a buffer): the TMA-fed kernels bulk-copy
    each item's query rows and need 16-byte alignment, so such a call runs the SIMT kernel, with the results of
    the aligned (host-pointer) call."""
    import torch
    B, nh, nkv, hd, T = 3, 8, 2, 128, 300
    rng = np.random.default_rng(91)
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, getattr(pkg, dtype))
    for b in range(B):
        kv.upload(0, b, 0, rng.standard_normal((T, nkv * hd)).astype(np.float32),
                  rng.standard_normal((T, nkv * hd)).astype(np.float32))
    q = rng.standard_normal((B, nh * hd)).astype(np.float32)
    pos = np.array([T - 1, T // 2, 7], np.int32)
    scale = 1.0 / np.sqrt(hd)
    ref = kv.attend_decode(0, q, pos, nh, scale)
    buf = torch.zeros(B * nh * hd + 1, device="cuda")
    qd = buf[1:].view(B, nh * hd)
    qd.copy_(torch.from_numpy(q))
    assert qd.data_ptr() % 16 == 4
    posd = torch.from_numpy(pos).cuda()
    out = torch.zeros((B, nh * hd), device="cuda")
    torch.cuda.synchronize()
    kv.attend_decode_dev(0, qd.data_ptr(), posd.data_ptr(), T - 1, nh, scale, out.data_ptr())
    ctx.synchronize()
    assert rel_l2(out.cpu().numpy(), ref) <= TOL
