"""Multi-GPU host logic on the CPU: the (sequence, head) partition, and two gloo ranks that each run
their shard of the DeltaNet recurrence (the oracle's restatement of src/eif_qwen35.c:594-639) and
reassemble the outputs with the all-gather.  The result must equal one process running the whole batch
bit for bit: heads and sequences share nothing, so splitting them changes no arithmetic."""
import os
import socket
import sys
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _shard_mod():
    import __graft_entry__
    return __graft_entry__.load_package().shard


@pytest.mark.parametrize("B,H,world", [(256, 16, 1), (256, 16, 3), (256, 16, 8), (4, 16, 8), (1, 16, 4),
                                       (8, 12, 8), (5, 4, 2), (2, 6, 6)])
def test_partition_covers_every_unit_once(B, H, world):
    sh = _shard_mod()
    seen = np.zeros((B, H), np.int32)
    for s in sh.all_shards(B, H, world):
        assert s.nb >= 1 and s.nh >= 1
        seen[s.b0:s.b0 + s.nb, s.h0:s.h0 + s.nh] += 1
    assert np.all(seen == 1)
    sizes = [s.units for s in sh.all_shards(B, H, world)]
    assert max(sizes) - min(sizes) <= H  # balanced to within one sequence


@pytest.mark.parametrize("B,H,world", [(3, 16, 4), (2, 5, 4), (4, 16, 6)])
def test_partition_refuses_uneven_head_split(B, H, world):
    with pytest.raises(ValueError):
        _shard_mod().shard(B, H, world, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, inputs, out_path):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import __graft_entry__
    from oracle import oracle as orc
    sh = __graft_entry__.load_package().shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    q, k, v, beta, g, S0, qs = inputs
    B, T, H, dv = v.shape
    s = sh.shard(B, H, world, rank)
    hs = slice(s.h0, s.h0 + s.nh)
    local = np.zeros((s.nb, T, s.nh, dv), np.float32)
    for i, b in enumerate(range(s.b0, s.b0 + s.nb)):
        S = np.ascontiguousarray(S0[b, hs])
        for t in range(T):
            local[i, t] = orc.deltanet_rule(S, np.ascontiguousarray(q[b, t, hs]).ravel(),
                                            np.ascontiguousarray(k[b, t, hs]).ravel(),
                                            np.ascontiguousarray(v[b, t, hs]).ravel(),
                                            np.ascontiguousarray(beta[b, t, hs]), np.ascontiguousarray(g[b, t, hs]),
                                            qs).reshape(s.nh, dv)
    full = sh.gather_outputs(dist, torch.from_numpy(local), B, H, world)
    slowest = sh.max_over_ranks(dist, float(10 + rank))
    if rank == 0:
        np.save(out_path, full.numpy())
        np.save(out_path + ".max.npy", np.array([slowest]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("B,H", [(4, 4), (1, 4), (3, 2)])
def test_two_gloo_ranks_match_one_process(orc, B, H):
    import torch.multiprocessing as mp
    rng = np.random.default_rng(B * 10 + H)
    T, dk, dv = 3, 16, 16
    qk = rng.standard_normal((2, B, T, H, dk)).astype(np.float32)
    qk /= np.sqrt((qk * qk).sum(-1, keepdims=True)).astype(np.float32)
    q, k = qk[0], qk[1]
    v = rng.standard_normal((B, T, H, dv)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(rng.standard_normal((B, T, H))))).astype(np.float32)
    S0 = (0.02 * rng.standard_normal((B, H, dk, dv))).astype(np.float32)
    qs = 1.0 / np.sqrt(dk)
    want = np.zeros((B, T, H, dv), np.float32)
    for b in range(B):
        S = S0[b].copy()
        for t in range(T):
            want[b, t] = orc.deltanet_rule(S, q[b, t].ravel(), k[b, t].ravel(), v[b, t].ravel(), beta[b, t], g[b, t],
                                           qs).reshape(H, dv)
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "full.npy")
        mp.spawn(_worker, args=(2, _free_port(), (q, k, v, beta, g, S0, qs), out), nprocs=2, join=True)
        got = np.load(out)
        slowest = float(np.load(out + ".max.npy")[0])
    assert np.array_equal(got, want)
    assert slowest == 11.0
