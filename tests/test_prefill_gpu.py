"""Causal prefill attention (tcgen05 + TMEM + TMA) through the C ABI against the C restatement of the
reference's batched prefill loop (src/eif_tinyllm.c:1158-1268), pinned to the reference's
fullatt_attend by tests/golden/prefill_small.npz.

Inputs are drawn in fp32 and rounded to bf16 (the kernel's input type); the oracle runs in fp32 on the
same rounded values.  Tolerance for the bf16-in / fp32-accumulate prefill path: rel-L2 <= 1e-2 and
max-abs <= 2e-2."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
REL, ABS = 1e-2, 2e-2


def bf16(orc, a):
    return orc.round_bf16(a).reshape(a.shape)


def setup(pkg, ctx, orc, rng, B, rows, max_seq, nkv, hd=128):
    kv = pkg.KVCache(ctx, 1, B, max_seq, nkv, hd, pkg.BF16)
    kc = bf16(orc, rng.standard_normal((B, rows, nkv * hd)).astype(np.float32))
    vc = bf16(orc, rng.standard_normal((B, rows, nkv * hd)).astype(np.float32))
    for b in range(B):
        kv.upload(0, b, 0, kc[b], vc[b])
    return kv, kc, vc


@pytest.mark.parametrize("B,n_tok,start_pos,nh,nkv,hd", [
    (2, 300, 0, 12, 2, 128), (1, 128, 0, 4, 4, 128), (3, 130, 200, 8, 2, 128), (2, 1, 77, 12, 2, 128),
    (1, 257, 3, 6, 1, 128),
    # head_dim 64: the Qwen2.5-0.5B attention shape (14 q / 2 kv heads) and a ragged continuation
    (2, 300, 0, 14, 2, 64), (1, 200, 130, 7, 1, 64), (2, 1, 511, 14, 2, 64),
    # head_dim 256: the Qwen3.5 full-attention shape (8 q / 2 kv heads), its own kernel
    (1, 300, 0, 8, 2, 256), (2, 130, 70, 8, 2, 256), (1, 1, 40, 8, 2, 256), (1, 64, 0, 4, 1, 256)])
def test_prefill_vs_oracle(pkg, ctx, orc, B, n_tok, start_pos, nh, nkv, hd):
    rng = np.random.default_rng(n_tok * 7 + start_pos + hd)
    rows = start_pos + n_tok
    kv, kc, vc = setup(pkg, ctx, orc, rng, B, rows, rows + 5, nkv, hd)
    q = bf16(orc, rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32))
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_prefill(0, q, n_tok, start_pos, nh, scale)
    for b in range(B):
        ref = orc.attend_prefill(q[b], kc[b], vc[b], n_tok, start_pos, nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= REL
        assert np.max(np.abs(out[b] - ref)) <= ABS


def test_config2_full_size_sampled(pkg, ctx, orc):
    """BASELINE config 2 at full size (8 x 4096 tokens, 12 q / 2 kv heads, head_dim 128, causal) on the GPU;
    64 sampled tokens across sequences and the causal range are recomputed by the oracle."""
    rng = np.random.default_rng(2)
    B, S, nh, nkv, hd = 8, 4096, 12, 2, 128
    kv, kc, vc = setup(pkg, ctx, orc, rng, B, S, S, nkv)
    q = bf16(orc, rng.standard_normal((B, S, nh * hd)).astype(np.float32))
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_prefill(0, q, S, 0, nh, scale)
    assert np.all(np.isfinite(out))
    picks = [(b, t) for b in range(B) for t in (0, 1, 127, 128, 129, 2047, 4094, 4095)]
    got, want = [], []
    for b, t in picks:
        want.append(orc.attend_prefill(q[b, t:t + 1], kc[b], vc[b], 1, t, nh, nkv, hd, scale)[0])
        got.append(out[b, t])
    got, want = np.array(got), np.array(want)
    assert rel_l2(got, want) <= REL
    assert np.max(np.abs(got - want)) <= ABS


def test_prefill_is_causal(pkg, ctx, orc):
    """Rows after a token never influence it: rewriting cache rows >= 300 (with non-finite values past
    start_pos + n_tok) leaves tokens < 300 bit-identical."""
    rng = np.random.default_rng(4)
    B, n_tok, nh, nkv, hd = 1, 600, 8, 2, 128
    kv, kc, vc = setup(pkg, ctx, orc, rng, B, n_tok, n_tok + 64, nkv)
    q = bf16(orc, rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32))
    a = kv.attend_prefill(0, q, n_tok, 0, nh, 0.0884)
    junk = rng.standard_normal((n_tok - 300, nkv * hd)).astype(np.float32) * 50
    kv.upload(0, 0, 300, junk, -junk)
    tail = np.full((64, nkv * hd), np.nan, np.float32)
    kv.upload(0, 0, n_tok, tail, tail)
    b2 = kv.attend_prefill(0, q, n_tok, 0, nh, 0.0884)
    assert np.array_equal(a[0, :300], b2[0, :300])
    assert np.all(np.isfinite(b2))


@pytest.mark.parametrize("subln,hd,nh,nkv", [(2, 256, 8, 2), (1, 256, 8, 2), (0, 256, 8, 2), (2, 128, 12, 2)])
def test_prefill_gated_vs_oracle(pkg, ctx, orc, subln, hd, nh, nkv):
    """Qwen3.5 prefill attention as prefill_chunk gets it (fullatt_attend per token with the output gate and
    SubLN, src/eif_qwen35.c:1122-1133, :773-789), against the oracle's gated attention + SubLN per token."""
    rng = np.random.default_rng(100 + subln + hd)
    B, n_tok, start_pos = 2, 150, 40
    rows = start_pos + n_tok
    kv, kc, vc = setup(pkg, ctx, orc, rng, B, rows, rows + 3, nkv, hd)
    q = bf16(orc, rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32))
    gate = rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32)
    sub_norm = (1.0 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_prefill_gated(0, q, n_tok, start_pos, nh, scale, gate, subln, sub_norm if subln == 2 else None)
    for b in range(B):
        ref = np.stack([orc.subln(orc.attend_decode(q[b, i], kc[b], vc[b], start_pos + i, nh, nkv, hd, scale, gate[b, i]),
                                  sub_norm if subln == 2 else None, subln) for i in range(n_tok)])
        assert rel_l2(out[b], ref) <= REL
        assert np.max(np.abs(out[b] - ref)) <= ABS


def test_prefill_bad_arguments(pkg, ctx):
    kv96 = pkg.KVCache(ctx, 1, 1, 64, 2, 96, pkg.F32)  # head_dim outside 64 / 128 / 256
    with pytest.raises(pkg.EifCudaError) as e:
        kv96.attend_prefill(0, np.zeros((1, 4, 192), np.float32), 4, 0, 2, 0.1)
    assert e.value.name == "NOT_SUPPORTED"
    kv = pkg.KVCache(ctx, 1, 1, 64, 2, 128, pkg.BF16)
    with pytest.raises(pkg.EifCudaError) as e:
        kv.attend_prefill(0, np.zeros((1, 8, 256), np.float32), 8, 60, 2, 0.1)
    assert e.value.name == "INVALID_ARGUMENT"
    with pytest.raises(pkg.EifCudaError) as e:
        kv.attend_prefill(0, np.zeros((1, 8, 384), np.float32), 8, 0, 3, 0.1)
    assert e.value.name == "SHAPE_MISMATCH"


@pytest.mark.parametrize("hd,nh,nkv", [(64, 14, 2), (128, 12, 2), (256, 8, 2)])
def test_prefill_fp32_cache(pkg, ctx, orc, hd, nh, nkv):
    """The reference's own cache type (fp32): every chunk token is one decode row at its own position, in fp32
    arithmetic -- the fp32 tolerance (rel-L2 <= 1e-5) against the restatement of the prefill loop; host and
    device-pointer entries, plain and gated (Qwen3.5's prefill_chunk path, src/eif_qwen35.c:1122-1133)."""
    import torch
    rng = np.random.default_rng(hd + 3 * nh)
    B, start, n_tok = 2, 77, 150
    rows = start + n_tok
    kv = pkg.KVCache(ctx, 1, B, rows + 3, nkv, hd, pkg.F32)
    kc = rng.standard_normal((B, rows, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((B, rows, nkv * hd)).astype(np.float32)
    for b in range(B):
        kv.upload(0, b, 0, kc[b], vc[b])
    q = rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32)
    gate = rng.standard_normal((B, n_tok, nh * hd)).astype(np.float32)
    sub = (1 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = kv.attend_prefill(0, q, n_tok, start, nh, scale)
    outg = kv.attend_prefill_gated(0, q, n_tok, start, nh, scale, gate=gate, subln=pkg.SUBLN_WEIGHT, sub_norm=sub)
    qd, od = torch.from_numpy(q).cuda(), torch.zeros((B, n_tok, nh * hd), device="cuda")
    torch.cuda.synchronize()
    kv.attend_prefill_dev(0, qd.data_ptr(), n_tok, start, nh, scale, od.data_ptr())
    ctx.synchronize()
    outd = od.cpu().numpy()
    for b in range(B):
        ref = orc.attend_prefill(q[b], kc[b], vc[b], n_tok, start, nh, nkv, hd, scale)
        assert rel_l2(out[b], ref) <= 1e-5 and rel_l2(outd[b], ref) <= 1e-5, b
        for t in (0, 1, n_tok // 2, n_tok - 1):
            rg = orc.subln(orc.attend_decode(q[b, t], kc[b], vc[b], start + t, nh, nkv, hd, scale, gate=gate[b, t]),
                           sub, 2)
            assert rel_l2(outg[b, t], rg) <= 1e-5, (b, t)
    kv.free()
