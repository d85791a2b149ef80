"""Multi-GPU partition of the token-mixing path: one process per GPU, no collective on the data path.

Every sequence's KV cache and DeltaNet state are independent of every other sequence's, and within a
sequence every head's state is independent of the others (the head loops of src/eif_qwen35.c:600 and
:753-771 share nothing), so ranks split the work by (sequence, head) units and each rank's
eif_cuda_* calls see an ordinary smaller problem.  The only collective is optional: an all-gather that
reassembles a layer's output on every rank for a caller that needs the whole batch on one device (for
instance to feed a replicated projection); it runs over torch.distributed (NCCL on GPUs, gloo in the
CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    """The rectangle of (sequence, head) units one rank owns: sequences [b0, b0 + nb), heads [h0, h0 + nh)."""
    b0: int
    nb: int
    h0: int
    nh: int

    @property
    def units(self) -> int:
        return self.nb * self.nh


def shard(global_batch: int, n_heads: int, world: int, rank: int) -> Shard:
    """Partition global_batch x n_heads units over `world` ranks.

    world <= global_batch: by sequence, contiguous, the first (global_batch % world) ranks one sequence
    more; every rank keeps all heads.  world > global_batch: each sequence is split by heads over
    world / global_batch ranks, which must divide both world and n_heads (raises ValueError otherwise).
    """
    if global_batch < 1 or n_heads < 1 or world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad partition request: batch {global_batch}, heads {n_heads}, world {world}, rank {rank}")
    if world <= global_batch:
        base, extra = divmod(global_batch, world)
        nb = base + (1 if rank < extra else 0)
        b0 = rank * base + min(rank, extra)
        return Shard(b0, nb, 0, n_heads)
    if world % global_batch or n_heads % (world // global_batch):
        raise ValueError(f"{world} ranks cannot split batch {global_batch} x {n_heads} heads evenly")
    per_seq = world // global_batch
    nh = n_heads // per_seq
    return Shard(rank // per_seq, 1, (rank % per_seq) * nh, nh)


def all_shards(global_batch: int, n_heads: int, world: int) -> list[Shard]:
    return [shard(global_batch, n_heads, world, r) for r in range(world)]


def max_over_ranks(dist, value: float, device=None) -> float:
    """The slowest rank's number (timings are reported as the max over ranks)."""
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def gather_outputs(dist, local, global_batch: int, n_heads: int, world: int):
    """Reassemble every rank's output into the global tensor, on every rank.

    `local` is this rank's output [nb, *mid, nh, d]: its sequences first, then any middle axes (tokens,
    for a prefill), then its heads and the head dimension.  The result is [global_batch, *mid, n_heads, d].
    Pieces are padded to the largest shard for the all-gather and placed by their Shard rectangles.
    """
    import torch
    shards = all_shards(global_batch, n_heads, world)
    nb_max = max(s.nb for s in shards)
    nh_max = max(s.nh for s in shards)
    mid = tuple(local.shape[1:-2])
    d = local.shape[-1]
    pad = local.new_zeros((nb_max, *mid, nh_max, d))
    pad[:local.shape[0], ..., :local.shape[-2], :] = local
    pieces = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(pieces, pad)
    out = local.new_empty((global_batch, *mid, n_heads, d))
    for s, piece in zip(shards, pieces):
        out[s.b0:s.b0 + s.nb, ..., s.h0:s.h0 + s.nh, :] = piece[:s.nb, ..., :s.nh, :]
    return out
