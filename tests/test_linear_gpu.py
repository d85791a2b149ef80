"""The projections on the GPU (eif_cuda_linear_*): linear_gemv / linear_gemm / int8_gemv of src/eif_qwen35.c
(:384-443, 1033-1063) on weights resident in HBM, through the C ABI.

* Decoding is bit-exact: integer weights and inputs with power-of-two scales make every partial sum an exact
  integer, so the device result equals the restatement's exactly, whatever the summation order -- for every
  format, ragged widths, rows not a multiple of the warp's four, every token-tile size (1, 2, 4, 8) and partial
  tiles.
* On random fp32 inputs the device agrees with the reference's own outputs (the committed fixture, and the
  reference build where present, else the restatement) within rel-L2 1e-5: both sum in fp32, in different orders.
"""
import numpy as np
import pytest

from conftest import golden, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5
NAMES = ["f32", "f32_n3", "int4", "int4_n5", "tern2", "tern2_n5", "tern2_g32", "tern2_g32_n5", "dense", "dense_n5",
         "int8", "int8_n3"]


def _values(rng, base, rows, cols):
    if base == 0:
        return rng.standard_normal((rows, cols)).astype(np.float32) * 0.05
    if base == 1:
        return rng.integers(-8, 8, (rows, cols))
    if base == 4:
        return rng.integers(-128, 128, (rows, cols))
    return rng.integers(-1, 2, (rows, cols))


def _reference(orc, W, sc, x, rows, cols, qt):
    if orc.ref_available():
        return orc.ref_linear(W, sc, x, rows, cols, qt)
    return orc.linear(W, sc, x, rows, cols, qt)


@pytest.mark.parametrize("name", NAMES)
def test_linear_golden(pkg, ctx, name):
    d = golden("linear_formats.npz")
    qt, rows, cols, n = (int(v) for v in d[f"{name}_shape"])
    sc = d[f"{name}_sc"]
    lin = pkg.Linear(ctx, qt, rows, cols, d[f"{name}_W"], sc if sc.size else None)
    try:
        out = lin.forward(d[f"{name}_x"])
    finally:
        lin.free()
    assert out.shape == (n, rows)
    assert rel_l2(out, d[f"{name}_out"]) <= TOL


@pytest.mark.parametrize("qt", [0, 1, 2, 2 | (32 << 8), 2 | (16 << 8), 3, 4],
                         ids=["f32", "int4", "tern2", "tern2_g32", "tern2_g16", "dense", "int8"])
@pytest.mark.parametrize("rows,cols", [(1, 16), (7, 203), (66, 1024), (130, 2049)])
def test_linear_decode_bit_exact(pkg, ctx, orc, qt, rows, cols):
    base, group = qt & 0xFF, qt >> 8
    if group and cols % group:
        pytest.skip("group must divide cols")
    rng = np.random.default_rng(rows * 7 + cols + qt)
    lo, hi = {0: (-8, 8), 1: (-8, 8), 4: (-128, 128)}.get(base, (-1, 2))
    v = rng.integers(lo, hi, (rows, cols))
    W = orc.pack_weights(v.astype(np.float32) if base == 0 else v, base, rng if base == 2 else None)
    if base == 0:
        sc = None
    elif group:
        sc = np.ldexp(1.0, rng.integers(-3, 2, (rows, cols // group))).astype(np.float32)
    else:
        sc = np.ldexp(1.0, rng.integers(-3, 2, rows)).astype(np.float32)
    lin = pkg.Linear(ctx, qt, rows, cols, W, sc)
    try:
        for n in (1, 2, 3, 4, 5, 8, 9, 17):
            x = rng.integers(-4, 5, (n, cols)).astype(np.float32)
            got = lin.forward(x)
            want = orc.linear(W, sc, x, rows, cols, qt)
            assert np.array_equal(got, want), (n, np.abs(got - want).max())
    finally:
        lin.free()


@pytest.mark.parametrize("qt,rows,cols", [
    (2, 6144, 1024),             # Qwen3.5-0.8B DeltaNet in_proj_qkv, 2-bit ternary
    (2 | (64 << 8), 2048, 1024),  # the z projection with grouped scales
    (2, 1024, 3584),             # FFN down
    (1, 3584, 1024),             # INT4 FFN up
    (3, 1024, 2048),             # dense ternary out_proj
    (0, 32, 1024),               # fp32 (the small a / b projections of grouped checkpoints)
    (4, 16384, 1024),            # INT8 LM head (16384 of the vocabulary's rows)
])
def test_linear_model_shapes(pkg, ctx, orc, qt, rows, cols):
    rng = np.random.default_rng(rows + cols + qt)
    base, group = qt & 0xFF, qt >> 8
    W = orc.pack_weights(_values(rng, base, rows, cols), base, rng if base == 2 else None)
    sc = None if base == 0 else (0.01 + 0.1 * rng.random((rows, cols // group) if group else rows)).astype(np.float32)
    lin = pkg.Linear(ctx, qt, rows, cols, W, sc)
    try:
        for n in (1, 7, 64):
            x = rng.standard_normal((n, cols)).astype(np.float32)
            assert rel_l2(lin.forward(x), _reference(orc, W, sc, x, rows, cols, qt)) <= TOL, n
    finally:
        lin.free()


def test_linear_wide_rows_use_smaller_tiles(pkg, ctx, orc):
    """A 12288-column fp32 row does not fit an 8-token tile: the launch picks a smaller one, same results."""
    rng = np.random.default_rng(9)
    rows, cols = 40, 12288
    v = rng.integers(-8, 8, (rows, cols)).astype(np.float32)
    W = orc.pack_weights(v, 0)
    lin = pkg.Linear(ctx, 0, rows, cols, W)
    try:
        x = rng.integers(-4, 5, (9, cols)).astype(np.float32)
        assert np.array_equal(lin.forward(x), orc.linear(W, None, x, rows, cols, 0))
    finally:
        lin.free()


def test_linear_forward_dev(pkg, ctx, orc):
    import torch
    rng = np.random.default_rng(10)
    rows, cols, n = 300, 1024, 12
    v = rng.integers(-1, 2, (rows, cols))
    W = orc.pack_weights(v, 2, rng)
    sc = (0.01 + rng.random(rows)).astype(np.float32)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    lin = pkg.Linear(ctx, 2, rows, cols, W, sc)
    try:
        xd = torch.from_numpy(x).cuda()
        od = torch.full((n, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        lin.forward_dev(xd.data_ptr(), n, od.data_ptr())
        ctx.synchronize()
        assert rel_l2(od.cpu().numpy(), _reference(orc, W, sc, x, rows, cols, 2)) <= TOL
    finally:
        lin.free()


def test_linear_rejections(pkg, ctx):
    W = np.zeros((4, 64), np.uint8)
    sc = np.ones(4, np.float32)
    cases = [
        ((5, 4, 256, W, sc), "NOT_SUPPORTED"),               # unknown format
        ((2 | (24 << 8), 4, 256, W, np.ones((4, 10), np.float32)), "NOT_SUPPORTED"),  # group not a multiple of 16
        ((1 | (32 << 8), 4, 128, W, sc), "NOT_SUPPORTED"),   # a group on a non-ternary format
        ((2, 4, 256, W, None), "INVALID_ARGUMENT"),          # scales missing
        ((0, 0, 16, np.zeros(0, np.uint8), None), "INVALID_ARGUMENT"),
    ]
    for args, status in cases:
        with pytest.raises(pkg.EifCudaError) as e:
            pkg.Linear(ctx, *args)
        assert e.value.name == status, (args[:3], e.value)
    big = 60000  # an fp32 row of 240 kB does not fit the token tile
    with pytest.raises(pkg.EifCudaError) as e:
        pkg.Linear(ctx, 0, 1, big, np.zeros(4 * big, np.uint8))
    assert e.value.name == "NOT_SUPPORTED"
    other = pkg.Context(0)
    try:
        lin = pkg.Linear(other, 2, 4, 256, W, sc)
        x, out = np.zeros(256, np.float32), np.zeros(4, np.float32)
        with pytest.raises(pkg.EifCudaError) as e:  # weights of another context
            ctx.check(pkg.lib().eif_cuda_linear_forward(ctx.handle, lin._h, x.ctypes.data, 1, out.ctypes.data),
                      "linear_forward")
        assert e.value.name == "INVALID_ARGUMENT"
        with pytest.raises(ValueError):
            lin.forward(np.zeros((2, 256), np.float32), out=np.zeros((3, 4), np.float32))
    finally:
        other.close()


@pytest.mark.parametrize("n", [1, 6])
def test_linear_dependent_chain(pkg, ctx, orc, n):
    """Projections launched back to back as programmatic dependents, each reading the previous one's output
    (no synchronisation between them), on both kernels (one token: CUDA cores, six: tensor cores): every
    launch waits for its predecessor before it reads x, so the chain equals the reference applied in turn."""
    import torch
    rng = np.random.default_rng(20 + n)
    dims = [1024, 768, 1536, 512, 1024]
    mats = []
    for i in range(len(dims) - 1):
        rows, cols = dims[i + 1], dims[i]
        qt = 2 if i % 2 == 0 else 1
        v = _values(rng, qt, rows, cols)
        W = orc.pack_weights(v, qt, rng if qt == 2 else None)
        sc = (0.5 + rng.random(rows)).astype(np.float32) / np.sqrt(cols)
        mats.append((qt, rows, cols, W, sc, pkg.Linear(ctx, qt, rows, cols, W, sc)))
    stream = torch.cuda.Stream()
    try:
        x = rng.standard_normal((n, dims[0])).astype(np.float32)
        bufs = [torch.from_numpy(x).cuda()] + [torch.full((n, d), float("nan"), device="cuda") for d in dims[1:]]
        torch.cuda.synchronize()
        ctx.set_stream(stream.cuda_stream)
        for i, (_, _, _, _, _, lin) in enumerate(mats):
            lin.forward_dev(bufs[i].data_ptr(), n, bufs[i + 1].data_ptr())
        ctx.synchronize()
        ref = x
        for qt, rows, cols, W, sc, _ in mats:
            ref = _reference(orc, W, sc, ref, rows, cols, qt)
        assert rel_l2(bufs[-1].cpu().numpy(), ref) <= 4 * TOL
    finally:
        ctx.set_stream(None)
        for *_, lin in mats:
            lin.free()
