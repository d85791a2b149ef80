"""DeltaNet recurrent step through the C ABI against the C restatement of src/eif_qwen35.c:594-639
(itself pinned to the reference's deltanet_core by tests/test_oracle.py).  Tolerance rel-L2 <= 1e-5."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


def inputs(rng, B, H, dk, dv):
    qk = rng.standard_normal((2, B, H, dk)).astype(np.float32)
    qk /= np.sqrt((qk * qk).sum(-1, keepdims=True) + 1e-12).astype(np.float32)
    v = rng.standard_normal((B, H * dv)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((B, H))))).astype(np.float32)
    return qk[0].reshape(B, -1), qk[1].reshape(B, -1), v, beta, g


@pytest.mark.parametrize("dk,dv", [(128, 128), (64, 64), (128, 64), (64, 128), (256, 256)])
def test_rule_steps(pkg, ctx, orc, dk, dv):
    rng = np.random.default_rng(dk + dv)
    B, H, steps = 3, 5, 12
    st = pkg.DeltaState(ctx, 2, B, H, dk, dv)
    S = (rng.standard_normal((B, H, dk, dv)) * 0.02).astype(np.float32)
    for b in range(B):
        st.upload(1, b, S=S[b])
    qs = 1.0 / np.sqrt(dk)
    for t in range(steps):
        q, k, v, beta, g = inputs(rng, B, H, dk, dv)
        o = st.step(1, q, k, v, beta, g, qs)
        for b in range(B):
            ro = orc.deltanet_rule(S[b], q[b], k[b], v[b], beta[b], g[b], qs)
            assert rel_l2(o[b], ro) <= TOL, (t, b)
    for b in range(B):
        Sg, _ = st.download(1, b)
        assert rel_l2(Sg, S[b]) <= TOL
    # layer 0 untouched
    S0, _ = st.download(0, 0)
    assert not S0.any()


def test_config3_full_size(pkg, ctx, orc):
    """BASELINE config 3 at full size on the GPU (64 seqs x 16 heads x 128x128, 1024 sequential steps from
    S0 ~ N(0, 0.02)); two sampled sequences are replayed on the CPU restatement over all 1024 steps."""
    import torch
    B, H, d, steps = 64, 16, 128, 1024
    rng = np.random.default_rng(33)
    st = pkg.DeltaState(ctx, 1, B, H, d, d)
    S0 = (rng.standard_normal((B, H, d, d)) * 0.02).astype(np.float32)
    for b in range(B):
        st.upload(0, b, S=S0[b])
    gen = torch.Generator(device="cpu").manual_seed(5)
    qk = torch.randn((steps, 2, B, H, d), generator=gen)
    qk = qk / torch.sqrt((qk * qk).sum(-1, keepdim=True) + 1e-12)
    v = torch.randn((steps, B, H * d), generator=gen)
    beta = torch.sigmoid(torch.randn((steps, B, H), generator=gen))
    g = -torch.nn.functional.softplus(torch.randn((steps, B, H), generator=gen))
    dev = {n: t.contiguous().cuda() for n, t in dict(qk=qk, v=v, beta=beta, g=g).items()}
    o = torch.zeros((steps, B, H * d), device="cuda")
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    try:
        for t in range(steps):
            st.step_dev(0, dev["qk"][t, 0].data_ptr(), dev["qk"][t, 1].data_ptr(), dev["v"][t].data_ptr(),
                        dev["beta"][t].data_ptr(), dev["g"][t].data_ptr(), 1 / np.sqrt(d), o[t].data_ptr())
        ctx.synchronize()
    finally:
        ctx.set_stream(None)
    o = o.cpu().numpy()
    for b in (0, 41):
        S = S0[b].copy()
        ro = np.stack([orc.deltanet_rule(S, qk[t, 0, b].numpy().ravel(), qk[t, 1, b].numpy().ravel(),
                                         v[t, b].numpy(), beta[t, b].numpy(), g[t, b].numpy(), 1 / np.sqrt(d))
                       for t in range(steps)])
        assert rel_l2(o[:, b], ro) <= TOL
        Sg, _ = st.download(0, b)
        assert rel_l2(Sg, S) <= TOL
    assert np.all(np.isfinite(o))


def test_unsupported_dims(pkg, ctx):
    st = pkg.DeltaState(ctx, 1, 1, 2, 96, 96)
    z = np.zeros((1, 192), np.float32)
    with pytest.raises(pkg.EifCudaError) as e:
        st.step(0, z, z, z, np.zeros((1, 2), np.float32), np.zeros((1, 2), np.float32), 1.0)
    assert e.value.name == "NOT_SUPPORTED"
