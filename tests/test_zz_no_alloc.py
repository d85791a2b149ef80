"""eif_cuda_attend_decode_noalloc_dev, the decode-attention entry point for callers that cannot allocate
device memory once they run (an engine that reserves all of its device memory at start-up, or one held to
a fixed memory budget).  It keeps its split-K partials in a fixed array inside the library instead of a
cudaMalloc'd buffer.

Through the C ABI: two calls in a row, each checked against eif_cuda_attend_decode_dev on the same inputs
(rel-L2 <= 1e-5, the decode tolerance of the other tests); the second call must leave the device's free
memory unchanged; a shape whose partials cannot fit the array is refused with INVALID_ARGUMENT; shapes
whose preferred split would overflow the array run a shorter split that fits (bf16, INT8 and fp32 caches),
checked against the restatement and the allocating entry point.
This file is named to be collected last."""
import ctypes

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _call(L, name, ctx, kv, q, pos, max_pos, nh, scale, gate, subln, sub_norm, out):
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    return getattr(L, name)(ctx.handle, kv._h, 0, ptr(q), ptr(pos), max_pos, nh, ctypes.c_float(scale), ptr(gate),
                            subln, ptr(sub_norm), ptr(out))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_noalloc_matches_allocating_entry_point(pkg, dtype):
    import torch
    L = pkg.lib()
    ctx = pkg.Context(0)
    rng = np.random.default_rng(2024)
    B, nh, nkv, hd, T = 6, 8, 2, 256, 700
    dt = pkg.BF16 if dtype == "bf16" else pkg.F32
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    for b in range(B):
        kv.upload(0, b, 0, rng.standard_normal((T, nkv * hd)), rng.standard_normal((T, nkv * hd)))
    scale = 1.0 / np.sqrt(hd)
    sub_norm = torch.from_numpy((1 + 0.1 * rng.standard_normal(nh * hd)).astype(np.float32)).cuda()
    free_before = None
    for call, pos_np in enumerate([np.array([699, 0, 64, 65, 300, 511]), np.array([12, 699, 698, 1, 130, 257])]):
        q = torch.from_numpy(rng.standard_normal((B, nh * hd)).astype(np.float32)).cuda()
        gate = torch.from_numpy(rng.standard_normal((B, nh * hd)).astype(np.float32)).cuda()
        pos = torch.from_numpy(pos_np.astype(np.int32)).cuda()
        out_ref = torch.zeros((B, nh * hd), device="cuda")
        out_na = torch.full((B, nh * hd), float("nan"), device="cuda")
        torch.cuda.synchronize()
        assert _call(L, "eif_cuda_attend_decode_dev", ctx, kv, q, pos, int(pos_np.max()), nh, scale, gate,
                     pkg.SUBLN_WEIGHT, sub_norm, out_ref) == 0, ctx.last_error
        assert L.eif_cuda_synchronize(ctx.handle) == 0, ctx.last_error
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
        assert _call(L, "eif_cuda_attend_decode_noalloc_dev", ctx, kv, q, pos, int(pos_np.max()), nh, scale, gate,
                     pkg.SUBLN_WEIGHT, sub_norm, out_na) == 0, ctx.last_error
        assert L.eif_cuda_synchronize(ctx.handle) == 0, ctx.last_error
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before
        a, r = out_na.cpu().numpy(), out_ref.cpu().numpy()
        assert np.all(np.isfinite(a))
        for b in range(B):
            assert rel_l2(a[b], r[b]) <= TOL, (call, b)
    kv.free()
    ctx.close()


def test_noalloc_refuses_shapes_beyond_the_array(pkg):
    import torch
    L = pkg.lib()
    ctx = pkg.Context(0)
    # 2048 sequences x 8 kv heads x head_dim 256: the unsplit partials alone exceed the 16 MiB array
    B, nkv, hd = 2048, 8, 256
    kv = pkg.KVCache(ctx, 1, B, 2, nkv, hd, pkg.BF16)
    q = torch.zeros((B, nkv * hd), device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    torch.cuda.synchronize()
    st = _call(L, "eif_cuda_attend_decode_noalloc_dev", ctx, kv, q, pos, 0, nkv, 0.0625, None, pkg.SUBLN_NONE, None,
               out)
    assert pkg.STATUS[st] == "INVALID_ARGUMENT"
    assert "fixed array" in ctx.last_error
    kv.free()
    ctx.close()


def _fill_cache(pkg, kv, seed):
    """Random cache contents written on the device: N(0, 1) rows for fp32 / bf16 caches; for INT8 caches
    codes in [-127, 127] and positive scales (any such pair is a valid quantised cache state)."""
    import torch
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    n = kv.batch * kv.max_seq_len * kv.kv_dim
    for p in kv.layer_ptrs(0):
        if kv.dtype == pkg.F32:
            torch.as_tensor(_DevArray(p, n, "<f4"), device="cuda").normal_(generator=gen)
        elif kv.dtype == pkg.BF16:
            torch.as_tensor(_DevArray(p, n, "<i2"), device="cuda").view(torch.bfloat16).normal_(generator=gen)
        else:
            torch.as_tensor(_DevArray(p, n, "|i1"), device="cuda").random_(-127, 128, generator=gen)
    if kv.dtype == pkg.INT8:
        stride = (kv.max_seq_len + 63) // 64 * 64
        for p in kv.layer_scales(0):
            torch.as_tensor(_DevArray(p, kv.batch * kv.n_kv_heads * stride, "<f4"), device="cuda").uniform_(
                0.002, 0.03, generator=gen)
    torch.cuda.synchronize()


class _DevArray:
    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (n,), "typestr": typestr, "version": 3,
                                         "strides": None}


@pytest.mark.parametrize("dtype,hd,nh,nkv,B,T", [("bf16", 128, 12, 2, 16, 4096), ("int8", 128, 14, 2, 300, 4096),
                                                 ("f32", 128, 14, 2, 300, 1024)])
def test_noalloc_caps_the_split_to_the_array(pkg, orc, dtype, hd, nh, nkv, B, T):
    """Shapes whose preferred split would leave more partials than the fixed array holds, while a shorter
    split fits: the no-allocation entry point runs the shorter split (the one path where it differs from
    eif_cuda_attend_decode_dev).  Two calls in a row, checked against the restatement on sampled sequences
    and against the allocating entry point (rel-L2 <= 1e-5)."""
    import torch
    L = pkg.lib()
    ctx = pkg.Context(0)
    dt = {"bf16": pkg.BF16, "int8": pkg.INT8, "f32": pkg.F32}[dtype]
    kv = pkg.KVCache(ctx, 1, B, T, nkv, hd, dt)
    _fill_cache(pkg, kv, 77)
    cap = 16 << 20
    nc_pref, _, ws_pref = kv.decode_plan(0, nh, T - 1)
    nc_cap, _, ws_cap = kv.decode_plan(0, nh, T - 1, noalloc=True)
    assert ws_pref > cap and ws_cap <= cap and 1 <= nc_cap < nc_pref, (nc_pref, ws_pref, nc_cap, ws_cap)
    rng = np.random.default_rng(5)
    scale = 1.0 / np.sqrt(hd)
    sample = [0, 1, B // 2, B - 1]
    rows = {}
    for b in sample:
        rows[b] = kv.download_int8(0, b, 0, T) if dt == pkg.INT8 else kv.download(0, b, 0, T)
    for call in range(2):
        pos_np = rng.integers(T // 2, T, B).astype(np.int32)
        pos_np[0], pos_np[1] = T - 1, 0
        qn = rng.standard_normal((B, nh * hd)).astype(np.float32)
        q, pos = torch.from_numpy(qn).cuda(), torch.from_numpy(pos_np).cuda()
        out_ref = torch.zeros((B, nh * hd), device="cuda")
        out_na = torch.full((B, nh * hd), float("nan"), device="cuda")
        torch.cuda.synchronize()
        assert _call(L, "eif_cuda_attend_decode_dev", ctx, kv, q, pos, T - 1, nh, scale, None, pkg.SUBLN_NONE, None,
                     out_ref) == 0, ctx.last_error
        assert _call(L, "eif_cuda_attend_decode_noalloc_dev", ctx, kv, q, pos, T - 1, nh, scale, None,
                     pkg.SUBLN_NONE, None, out_na) == 0, ctx.last_error
        assert L.eif_cuda_synchronize(ctx.handle) == 0, ctx.last_error
        a, r = out_na.cpu().numpy(), out_ref.cpu().numpy()
        assert np.all(np.isfinite(a))
        assert rel_l2(a, r) <= TOL, call
        for b in sample:
            if dt == pkg.INT8:
                kc, vc, ks, vs = rows[b]
                want = orc.attend_decode_i8(qn[b], kc, ks, vc, vs, int(pos_np[b]), nh, nkv, hd, scale)
            else:
                want = orc.attend_decode(qn[b], rows[b][0], rows[b][1], int(pos_np[b]), nh, nkv, hd, scale)
            assert rel_l2(a[b], want) <= TOL, (call, b)
    kv.free()
    ctx.close()
