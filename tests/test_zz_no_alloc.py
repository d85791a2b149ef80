"""eif_cuda_attend_decode_noalloc_dev, the decode-attention entry point for callers that cannot allocate
device memory once they run (an engine that reserves all of its device memory at start-up, or one held to
a fixed memory budget).  It keeps its split-K partials in a fixed array inside the library instead of a
cudaMalloc'd buffer.

Through the C ABI: two calls in a row, each checked against eif_cuda_attend_decode_dev on the same inputs
(rel-L2 <= 1e-5, the decode tolerance of the other tests); the second call must leave the device's free
memory unchanged; a shape whose partials cannot fit the array is refused with INVALID_ARGUMENT.
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
