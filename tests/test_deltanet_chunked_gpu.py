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


@pytest.mark.parametrize("B,n_tok,H,dv", [(2, 150, 4, 128), (1, 3, 2, 128), (1, 70, 2, 64), (3, 64, 16, 128)])
def test_prefill_core_vs_per_token(pkg, ctx, orc, B, n_tok, H, dv):
    """eif_cuda_deltanet_prefill_core over a chunk against the C restatement of deltanet_core run token by
    token, as prefill_chunk does (src/eif_qwen35.c:1104-1106): outputs, final S, final conv window; then
    the per-token fused mixer continues on the same state.

    Tolerances: against the fp32 per-token restatement, rel-L2 <= 1e-2 on outputs and state (the conv window
    exactly); element by element, against the recurrent reference on the same bf16-rounded rule inputs
    (oracle.deltanet_core_bf16_rule), |err| <= 2e-2 + 1e-2 |ref|.  The outputs leave through the gated
    RMSNorm (unit RMS per head, times silu(z)), so they reach |out| ~ 13 here and a head whose raw output
    nearly cancels is magnified: the fp32 recurrence on bf16-rounded inputs is itself up to 0.07 away from
    the fp32 one at such elements, so the per-element bound is taken against it, with a relative term."""
    rng = np.random.default_rng(n_tok + 10 * H + dv)
    dk, ck = 128, 4
    conv_dim = 2 * H * dk + H * dv
    w = dict(conv_w=(rng.standard_normal((conv_dim, ck)) * 0.5).astype(np.float32),
             dt_bias=rng.standard_normal(H).astype(np.float32), A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
             norm_w=(1 + 0.1 * rng.standard_normal(dv)).astype(np.float32))
    st = pkg.DeltaState(ctx, 1, B, H, dk, dv, ck)
    st.set_weights(0, **w)
    S0 = (0.02 * rng.standard_normal((B, H, dk, dv))).astype(np.float32)
    conv0 = rng.standard_normal((B, conv_dim, ck)).astype(np.float32)
    for b in range(B):
        st.upload(0, b, S=S0[b], conv_state=conv0[b])
    T = n_tok + 2
    qkv = rng.standard_normal((B, T, conv_dim)).astype(np.float32)
    z = rng.standard_normal((B, T, H * dv)).astype(np.float32)
    bb = rng.standard_normal((B, T, H)).astype(np.float32)
    aa = rng.standard_normal((B, T, H)).astype(np.float32)
    out = st.prefill_core(0, qkv[:, :n_tok], z[:, :n_tok], bb[:, :n_tok], aa[:, :n_tok])
    nxt = [st.core(0, qkv[:, t], z[:, t], bb[:, t], aa[:, t]) for t in range(n_tok, T)]
    for b in range(B):
        S, conv = S0[b].copy(), conv0[b].copy()
        ref = np.stack([orc.deltanet_core(qkv[b, t], z[b, t], bb[b, t], aa[b, t], conv, S, **w) for t in range(T)])
        assert rel_l2(out[b], ref[:n_tok]) <= REL, b
        ref16 = orc.deltanet_core_bf16_rule(qkv[b, :n_tok], z[b, :n_tok], bb[b, :n_tok], aa[b, :n_tok],
                                            conv0[b].copy(), S0[b].copy(), **w)
        assert np.all(np.abs(out[b] - ref16) <= ABS + 1e-2 * np.abs(ref16)), b
        got = np.stack([o[b] for o in nxt])
        assert rel_l2(got, ref[n_tok:]) <= REL, b
        Sg, cg = st.download(0, b)
        assert rel_l2(Sg, S) <= REL and np.max(np.abs(Sg - S)) <= ABS, b
        assert np.array_equal(cg, conv), b  # the window holds the raw inputs: exact


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
