"""Chunked (WY / UT) DeltaNet prefill through the C ABI against the RECURRENT restatement of the
reference's delta rule (src/eif_qwen35.c:594-639, run token by token as prefill_chunk does at
src/eif_qwen35.c:1104-1106), on the same bf16-rounded inputs.

Tolerance for this bf16-in / fp32-accumulate path: rel-L2 <= 1e-2 and max-abs <= 2e-2 on the outputs
and on the final state."""
import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
REL, ABS = 1e-2, 2e-2


def make_inputs(orc, rng, B, T, H, dk, dv):
    qk = rng.standard_normal((2, B, T, H, dk)).astype(np.float32)
    qk /= np.sqrt((qk * qk).sum(-1, keepdims=True) + 1e-12).astype(np.float32)
    q = orc.round_bf16(qk[0]).reshape(B, T, H, dk)
    k = orc.round_bf16(qk[1]).reshape(B, T, H, dk)
    v = orc.round_bf16(rng.standard_normal((B, T, H, dv)).astype(np.float32)).reshape(B, T, H, dv)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((B, T, H))))).astype(np.float32)
    return q, k, v, beta, g


def recurrent(orc, S, q, k, v, beta, g, q_scale):
    """Token by token: S [H, dk, dv] updated in place; returns o [T, H, dv]."""
    T = q.shape[0]
    return np.stack([orc.deltanet_rule(S, q[t].ravel(), k[t].ravel(), v[t].ravel(), beta[t], g[t], q_scale)
                     .reshape(S.shape[0], S.shape[2]) for t in range(T)])


@pytest.mark.parametrize("B,T,H,dv", [(2, 200, 3, 128), (1, 64, 2, 64), (1, 130, 1, 256), (3, 1, 2, 128)])
def test_chunked_vs_recurrent(pkg, ctx, orc, B, T, H, dv):
    rng = np.random.default_rng(T * 10 + H + dv)
    dk = 128
    q, k, v, beta, g = make_inputs(orc, rng, B, T, H, dk, dv)
    st = pkg.DeltaState(ctx, 1, B, H, dk, dv)
    S0 = (0.02 * rng.standard_normal((B, H, dk, dv))).astype(np.float32)
    for b in range(B):
        st.upload(0, b, S=S0[b])
    qs = 1.0 / np.sqrt(dk)
    o = st.prefill(0, q, k, v, beta, g, qs)
    for b in range(B):
        S = S0[b].copy()
        ro = recurrent(orc, S, q[b], k[b], v[b], beta[b], g[b], qs)
        assert rel_l2(o[b], ro) <= REL and np.max(np.abs(o[b] - ro)) <= ABS, b
        Sg, _ = st.download(0, b)
        assert rel_l2(Sg, S) <= REL and np.max(np.abs(Sg - S)) <= ABS, b


def test_config4_full_size(pkg, ctx, orc):
    """batch 4 x 8192 tokens, 16 heads, d 128, zero initial state; sequence 2 is
    replayed token by token on the CPU (outputs of every token and the final state)."""
    B, T, H, d = 4, 8192, 16, 128
    rng = np.random.default_rng(4)
    q, k, v, beta, g = make_inputs(orc, rng, B, T, H, d, d)
    st = pkg.DeltaState(ctx, 1, B, H, d, d)
    qs = 1.0 / np.sqrt(d)
    o = st.prefill(0, q, k, v, beta, g, qs)
    assert np.all(np.isfinite(o))
    b = 2
    S = np.zeros((H, d, d), np.float32)
    ro = recurrent(orc, S, q[b], k[b], v[b], beta[b], g[b], qs)
    assert rel_l2(o[b], ro) <= REL and np.max(np.abs(o[b] - ro)) <= ABS
    Sg, _ = st.download(0, b)
    assert rel_l2(Sg, S) <= REL and np.max(np.abs(Sg - S)) <= ABS


def test_chunked_then_recurrent_steps_continue(pkg, ctx, orc):
    """Prefill by chunks, then decode token by token with the recurrent step kernel on the same state:
    the state handed over is the recurrent one."""
    rng = np.random.default_rng(6)
    B, T, H, d = 2, 100, 4, 128
    q, k, v, beta, g = make_inputs(orc, rng, B, T + 5, H, d, d)
    st = pkg.DeltaState(ctx, 1, B, H, d, d)
    qs = 1.0 / np.sqrt(d)
    st.prefill(0, q[:, :T], k[:, :T], v[:, :T], beta[:, :T], g[:, :T], qs)
    outs = [st.step(0, q[:, t].reshape(B, -1), k[:, t].reshape(B, -1), v[:, t].reshape(B, -1), beta[:, t], g[:, t], qs)
            for t in range(T, T + 5)]
    for b in range(B):
        S = np.zeros((H, d, d), np.float32)
        ro = recurrent(orc, S, q[b], k[b], v[b], beta[b], g[b], qs)
        got = np.stack(outs)[:, b].reshape(5, H, d)
        assert rel_l2(got, ro[T:]) <= REL
