"""Benchmark of the token-mixing hot path on B200 (BASELINE config 5 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Default workload "qwen35_hybrid_decode": one decode step of a Qwen3.5-like
24-layer token-mixer stack -- 18 Gated DeltaNet layers (16 heads, d_k = d_v = 128, fp32 state) and 6
gated full-attention layers (8 Q / 2 KV heads, head_dim 256, bf16 KV cache, sigmoid output gate and
SubLN) in the engine's order (3 DeltaNet, 1 attention) x 6 -- for a decode batch of 256 sequences at
context 32768 (every sequence appends its token at row 32767 and attends over all 32768 rows).
Inputs are seeded synthetic tensors with the config's shapes and distributions (no model files).
Under torchrun the batch is split across ranks (256/N sequences each): fixed total work, "strong".

One JSON line on rank 0:
  value        tokens/s of the whole job, device-timed (CUDA events, max over ranks), inputs resident
  e2e          the same metric through the host-pointer C ABI calls (pinned host inputs copied in and
               outputs read back every layer of every step), wall-clock, max over ranks
  roofline     the dominant kernel (decode attention) against the measured HBM copy bandwidth
  cpu_baseline the reference's own C code on this box's host cores (rank 0, N=1), bounded sample
`--impl reference` times the reference's C code alone on the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# ---------------------------------------------------------------------------------------------------
# workload constants
# ---------------------------------------------------------------------------------------------------
N_LAYERS = 24
LAYER_TYPES = ["D", "D", "D", "A"] * 6  # Qwen3.5 layout: full attention every 4th layer
DN_H, DN_D = 16, 128
CONV_K = 4
DN_CONV = 3 * DN_H * DN_D  # conv channels: q, k, v
AT_HQ, AT_HKV, AT_D = 8, 2, 256
CTX = 32768
BATCH = 256
METRIC = "attn+DeltaNet tokens/s (24-layer Qwen3.5-like token-mixer decode step)"
UNIT = "tokens/s"


# DRAM traffic of each roofline kernel per algorithmic byte, from one ncu capture of a smaller case of the same
# kernel (dram__bytes_read.sum + dram__bytes_write.sum over the algorithmic bytes of that launch; the summaries
# under profiles/ give the commands).  The bench scales it to its own launch by the units processed, which is
# valid where traffic grows in proportion to the units (every kernel here streams each unit's bytes once).
# ncu flushes L2 before a captured launch, so a kernel whose writes still fit in L2 when it ends shows fewer
# DRAM write bytes than it eventually causes (the recurrent rule's state, the prefill outputs).
_DRAM = "profiles/dram_traffic_bench_kernels.md"
TRAFFIC_PER_ALG_BYTE = {
    # config 5's attention layer at batch 8: 537,031,168 B read + 137,472 B written / 537,067,520 B algorithmic
    "attn_decode_tc_hd256": (537168640 / 537067520, _DRAM),
    # config 2 at full size: 137,945,600 B read + 61,187,840 B written / 234,881,024 B (q, K, V, o)
    "attn_prefill_tc": (199133440 / 234881024, _DRAM),
    # config 4 at batch 1, both kernels of the prefill (k is read by the solve and by the state walk):
    # 185,881,344 B / 137,363,456 B
    "deltanet_chunked": (185881344 / 137363456, _DRAM),
    # config 3, one rule step over 64 x 16 heads: 68,700,160 B read + 7,954,176 B written / 136,323,072 B
    "delta_rule": (76654336 / 136323072, _DRAM),
    # config 1's heads batched (256 sequences, ctx 4096), attention launch
    "attn_decode_f32": (1079984896 / 1073741824, _DRAM),
    "attn_decode_tc": (552377088 / 536870912, _DRAM),
    "attn_decode_i8": (291107584 / 285212672, _DRAM),
    # row f4 at one token (linear_kernel): the 8224 x 1024 2-bit launch read 2,178,304 B / 2,175,232 B algorithmic;
    # the INT8 LM head 255,299,072 B read + 4,149,248 B written / 256,270,336 B
    "linear_ternary2": (2178304 / 2175232, "profiles/linear_projection_decode.md"),
    "linear_int8_head": ((255299072 + 4149248) / 256270336, "profiles/linear_projection_decode.md"),
}


def traffic(kernel, alg_bytes):
    """(DRAM bytes per launch, where the figure comes from) for the roofline's `traffic` / `traffic_source`."""
    r = TRAFFIC_PER_ALG_BYTE.get(kernel)
    if r is None:
        return None, None
    return r[0] * alg_bytes, f"{r[1]}: ncu DRAM bytes of a smaller case, x {r[0]:.4f} per algorithmic byte"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def _once(self):
        """One synchronous reading (brackets timed regions shorter than the 200 ms period)."""
        try:
            r = subprocess.run(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
            self.lines.extend(ln.strip() for ln in r.stdout.splitlines() if ln.strip())
        except (FileNotFoundError, OSError, subprocess.TimeoutExpired):
            pass

    def start(self):
        self._once()
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self._once()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------------

class CudaArray:
    """A raw device allocation presented to torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


class Weights:
    """Random-init mixer weights of the stack (seeded; the same on every rank): per DeltaNet layer
    conv_w, dt_bias, A_log, norm_w; per attention layer q_norm, k_norm, sub_norm."""

    def __init__(self, seed=4242):
        rng = np.random.default_rng(seed)
        self.dn = [dict(conv_w=(0.5 * rng.standard_normal((DN_CONV, CONV_K))).astype(np.float32),
                        dt_bias=rng.standard_normal(DN_H).astype(np.float32),
                        A_log=(0.5 * rng.standard_normal(DN_H)).astype(np.float32),
                        norm_w=(1 + 0.1 * rng.standard_normal(DN_D)).astype(np.float32))
                   for _ in range(LAYER_TYPES.count("D"))]
        self.at = [dict(q_norm=(1 + 0.1 * rng.standard_normal(AT_D)).astype(np.float32),
                        k_norm=(1 + 0.1 * rng.standard_normal(AT_D)).astype(np.float32),
                        sub_norm=(1 + 0.1 * rng.standard_normal(AT_HQ * AT_D)).astype(np.float32))
                   for _ in range(LAYER_TYPES.count("A"))]


class Hybrid:
    """Device-resident state and per-layer inputs of the config-5 decode step for `B` sequences: every
    DeltaNet layer is the engine's whole deltanet_core (conv window, norms, gates, rule, gated RMSNorm),
    every attention layer fullatt_prep (norms, partial RoPE, KV append) + fullatt_attend (GQA over the
    cache, sigmoid gate, SubLN)."""

    def __init__(self, pkg, ctx, torch, B, seed, weights):
        self.pkg, self.ctx, self.torch, self.B = pkg, ctx, torch, B
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        n_att = LAYER_TYPES.count("A")
        n_dn = LAYER_TYPES.count("D")
        self.kv = pkg.KVCache(ctx, n_att, B, CTX, AT_HKV, AT_D, pkg.BF16)
        self.dn = pkg.DeltaState(ctx, n_dn, B, DN_H, DN_D, DN_D, CONV_K)
        for l, w in enumerate(weights.dn):
            self.dn.set_weights(l, **w)
        for l, w in enumerate(weights.at):
            self.kv.set_norms(l, w["q_norm"], w["k_norm"])
        # KV cache ~ N(0,1) bf16, S ~ N(0, 0.02), conv windows ~ N(0,1), filled through the library's pointers
        for l in range(n_att):
            for p in self.kv.layer_ptrs(l):
                t = torch.as_tensor(CudaArray(p, (B * CTX * AT_HKV * AT_D,), "<i2"), device=dev)
                t.view(torch.bfloat16).normal_(generator=gen)
        for l in range(n_dn):
            s, c = self.dn.layer_ptrs(l)
            torch.as_tensor(CudaArray(s, (B * DN_H * DN_D * DN_D,), "<f4"), device=dev).normal_(0, 0.02,
                                                                                              generator=gen)
            torch.as_tensor(CudaArray(c, (B * DN_CONV * CONV_K,), "<f4"), device=dev).normal_(generator=gen)

        def nrm(*shape):
            return torch.randn(*shape, device=dev, generator=gen)
        # per-layer projection outputs (the mixers' inputs), N(0,1)
        self.dn_in = [dict(qkv=nrm(B, DN_CONV), z=nrm(B, DN_H * DN_D), b=nrm(B, DN_H), a=nrm(B, DN_H))
                      for _ in range(n_dn)]
        self.at_in = [dict(qg=nrm(B, AT_HQ * 2 * AT_D), k=nrm(B, AT_HKV * AT_D), v=nrm(B, AT_HKV * AT_D))
                      for _ in range(n_att)]
        self.sub_norm = [torch.from_numpy(w["sub_norm"]).to(dev) for w in weights.at]
        self.pos = torch.full((B,), CTX - 1, dtype=torch.int32, device=dev)
        self.q = torch.empty(B, AT_HQ * AT_D, device=dev)
        self.gate = torch.empty(B, AT_HQ * AT_D, device=dev)
        self.out = torch.empty(B, AT_HQ * AT_D, device=dev)
        self.dn_out = torch.empty(B, DN_H * DN_D, device=dev)
        self.scale = 1.0 / math.sqrt(AT_D)

    def step(self, att_events=None):
        """One decode step through the `_dev` entry points, asynchronously on the context's stream."""
        a = d = 0
        for typ in LAYER_TYPES:
            if typ == "D":
                x = self.dn_in[d]
                self.dn.core_dev(d, x["qkv"].data_ptr(), x["z"].data_ptr(), x["b"].data_ptr(), x["a"].data_ptr(),
                                 self.dn_out.data_ptr())
                d += 1
            else:
                x = self.at_in[a]
                self.kv.fullatt_prep_dev(a, x["qg"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(),
                                         self.pos.data_ptr(), AT_HQ, self.q.data_ptr(), self.gate.data_ptr())
                if att_events is not None:
                    att_events[a][0].record()
                self.kv.attend_decode_dev(a, self.q.data_ptr(), self.pos.data_ptr(), CTX - 1, AT_HQ, self.scale,
                                          self.out.data_ptr(), gate_dev=self.gate.data_ptr(),
                                          subln=self.pkg.SUBLN_WEIGHT, sub_norm_dev=self.sub_norm[a].data_ptr())
                if att_events is not None:
                    att_events[a][1].record()
                a += 1


class HybridPipe:
    """End to end with the copies overlapped: every layer's inputs come from pinned host memory (H2D on one copy
    stream into that layer's own device input buffers), every layer's output goes back to pinned host memory (D2H
    on a second copy stream), and the compute stream runs the layers through the `_dev` entry points
    (eif_cuda_deltanet_core_dev, eif_cuda_fullatt_decode_dev) as soon as their inputs have landed.  One input
    buffer set per layer (~230 MB at batch 256) lets the copy stream run ahead through a run of short DeltaNet
    layers, whose 8.4 MB of inputs take longer over PCIe than their 0.12 ms kernels, while an attention layer
    computes.  A step ends when its last output is on the host."""

    LOOKAHEAD = 6  # layers whose input copies are issued ahead of the current kernel (more than a D-D-D-A run)

    def __init__(self, torch, hy: Hybrid, seed):
        self.torch, self.hy = torch, hy
        B, dev = hy.B, torch.device("cuda", torch.cuda.current_device())
        rng = np.random.default_rng(seed)

        def pinned(*shape, dtype=np.float32):
            return torch.from_numpy(rng.standard_normal(shape).astype(dtype)).pin_memory()
        self.h_dn = dict(qkv=pinned(B, DN_CONV), z=pinned(B, DN_H * DN_D), b=pinned(B, DN_H), a=pinned(B, DN_H))
        self.h_at = dict(qg=pinned(B, AT_HQ * 2 * AT_D), k=pinned(B, AT_HKV * AT_D), v=pinned(B, AT_HKV * AT_D))
        self.h_pos = torch.full((B,), CTX - 1, dtype=torch.int32).pin_memory()
        self.h_dn_out = torch.zeros(B, DN_H * DN_D).pin_memory()
        self.h_out = torch.zeros(B, AT_HQ * AT_D).pin_memory()
        n = len(LAYER_TYPES)
        self.d_in = [{k: torch.empty_like(v, device=dev) for k, v in (self.h_dn if typ == "D" else self.h_at).items()}
                     for typ in LAYER_TYPES]
        self.d_pos = [torch.empty_like(self.h_pos, device=dev) if typ == "A" else None for typ in LAYER_TYPES]
        self.d_out = [torch.empty(B, (DN_H * DN_D) if typ == "D" else (AT_HQ * AT_D), device=dev) for typ in LAYER_TYPES]
        self.cp_in, self.cp_out = torch.cuda.Stream(), torch.cuda.Stream()
        E = torch.cuda.Event
        self.ev_in, self.ev_done = [E() for _ in range(n)], [E() for _ in range(n)]
        self.h2d = self.d2h = 0
        for typ in LAYER_TYPES:
            if typ == "D":
                self.h2d += sum(t.numel() * 4 for t in self.h_dn.values())
                self.d2h += self.h_dn_out.numel() * 4
            else:
                self.h2d += sum(t.numel() * 4 for t in self.h_at.values()) + self.h_pos.numel() * 4
                self.d2h += self.h_out.numel() * 4

    def step(self):
        torch, hy = self.torch, self.hy
        comp = torch.cuda.current_stream()  # the library context's stream
        # the inputs, in layer order on the copy stream, issued LOOKAHEAD layers ahead of the kernels (a layer's
        # buffers are its own, and the previous step ended with everything complete), so the first kernels do not
        # wait for the host to issue every copy of the step
        n = len(LAYER_TYPES)

        def copy_in(i):
            with torch.cuda.stream(self.cp_in):
                for k, t in (self.h_dn if LAYER_TYPES[i] == "D" else self.h_at).items():
                    self.d_in[i][k].copy_(t, non_blocking=True)
                if LAYER_TYPES[i] == "A":
                    self.d_pos[i].copy_(self.h_pos, non_blocking=True)
                self.ev_in[i].record(self.cp_in)
        for i in range(min(self.LOOKAHEAD, n)):
            copy_in(i)
        a = d = 0
        for i, typ in enumerate(LAYER_TYPES):
            if i + self.LOOKAHEAD < n:
                copy_in(i + self.LOOKAHEAD)
            comp.wait_event(self.ev_in[i])
            x = self.d_in[i]
            if typ == "D":
                hy.dn.core_dev(d, x["qkv"].data_ptr(), x["z"].data_ptr(), x["b"].data_ptr(), x["a"].data_ptr(),
                               self.d_out[i].data_ptr())
                d += 1
                out_h = self.h_dn_out
            else:
                hy.kv.fullatt_decode_dev(a, x["qg"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(),
                                         self.d_pos[i].data_ptr(), CTX - 1, AT_HQ, hy.scale, self.d_out[i].data_ptr(),
                                         subln=hy.pkg.SUBLN_WEIGHT, sub_norm_dev=hy.sub_norm[a].data_ptr())
                a += 1
                out_h = self.h_out
            self.ev_done[i].record(comp)
            self.cp_out.wait_event(self.ev_done[i])
            with torch.cuda.stream(self.cp_out):
                out_h.copy_(self.d_out[i], non_blocking=True)
        self.cp_out.synchronize()  # the step's results are on the host
        comp.synchronize()


class HybridHost:
    """Pinned host inputs / outputs for the end-to-end (host-pointer ABI) measurement."""

    def __init__(self, torch, B, seed, weights):
        rng = np.random.default_rng(seed)
        self._keep = []

        def pinned(a, dtype=np.float32):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype)).pin_memory()
            self._keep.append(t)
            return t.numpy()

        self.h = dict(qkv=pinned(rng.standard_normal((B, DN_CONV))), z=pinned(rng.standard_normal((B, DN_H * DN_D))),
                      b=pinned(rng.standard_normal((B, DN_H))), a=pinned(rng.standard_normal((B, DN_H))),
                      qg=pinned(rng.standard_normal((B, AT_HQ * 2 * AT_D))),
                      k=pinned(rng.standard_normal((B, AT_HKV * AT_D))),
                      v=pinned(rng.standard_normal((B, AT_HKV * AT_D))))
        self.sub_norm = [pinned(w["sub_norm"]) for w in weights.at]
        self.pos = pinned(np.full(B, CTX - 1), np.int32)
        # the results land in pinned host arrays too (an engine keeps its activations in such buffers)
        self.dn_out = pinned(np.zeros((B, DN_H * DN_D)))
        self.out = pinned(np.zeros((B, AT_HQ * AT_D)))
        h = self.h
        self.h2d = 0
        self.d2h = 0
        for typ in LAYER_TYPES:
            if typ == "D":
                self.h2d += h["qkv"].nbytes + h["z"].nbytes + h["b"].nbytes + h["a"].nbytes
                self.d2h += B * DN_H * DN_D * 4
            else:
                # fullatt_decode (prep + attention in one call): qg, k, v, pos, sub_norm in; out out
                self.h2d += h["qg"].nbytes + h["k"].nbytes + h["v"].nbytes + self.pos.nbytes + self.sub_norm[0].nbytes
                self.d2h += B * AT_HQ * AT_D * 4

    def step(self, hy: Hybrid):
        a = d = 0
        h = self.h
        for typ in LAYER_TYPES:
            if typ == "D":
                hy.dn.core(d, h["qkv"], h["z"], h["b"], h["a"], out=self.dn_out)
                d += 1
            else:
                hy.kv.fullatt_decode(a, h["qg"], h["k"], h["v"], self.pos, AT_HQ, hy.scale, subln=hy.pkg.SUBLN_WEIGHT,
                                     sub_norm=self.sub_norm[a], out=self.out)
                a += 1


def attn_layer_bytes(B):
    """Algorithmic HBM bytes of one decode-attention launch: the K and V rows read once, q and gate read,
    out written (fp32)."""
    kv = 2 * B * CTX * AT_HKV * AT_D * 2
    io = 3 * B * AT_HQ * AT_D * 4
    return kv + io


def deltanet_layer_bytes(B):
    """Algorithmic HBM bytes of one deltanet_core launch: S and the conv windows read + written, the
    projection outputs (qkv, z, b, a) read, the mixer output written."""
    state = 2 * B * DN_H * DN_D * DN_D * 4 + 2 * B * DN_CONV * CONV_K * 4
    io = B * (DN_CONV + DN_H * DN_D + 2 * DN_H + DN_H * DN_D) * 4
    return state + io


def run_ours(args, torch, dist, rank, world, local_rank):
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    GB = args.batch or BATCH
    B = pkg.shard.shard(GB, 1, world, rank).nb  # by sequence (layers differ in head count)
    ctx = pkg.Context(local_rank)
    # one explicit stream for the library's launches, the fills and the timing events
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    weights = Weights()
    hy = Hybrid(pkg, ctx, torch, B, seed=1234 + rank, weights=weights)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        hy.step()
    torch.cuda.synchronize()
    ctx.synchronize()

    n_att = LAYER_TYPES.count("A")
    # the attention launches' own times come from a separate pass: events recorded between the kernels of the
    # timed steps would break their programmatic (overlapped) launches
    n_att_steps = min(args.steps, 3)
    att_ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(n_att)]
              for _ in range(n_att_steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    launches0 = ctx.launch_count
    start.record()
    for s in range(args.steps):
        hy.step()
    end.record()
    torch.cuda.synchronize()
    launches = ctx.launch_count - launches0
    clk = clocks.stop()
    for s in range(n_att_steps):
        hy.step(att_ev[s])
    torch.cuda.synchronize()
    ctx.synchronize()  # surfaces any device-side error word
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    att_ms = float(np.mean([e[0].elapsed_time(e[1]) for st in att_ev for e in st]))
    ms_all = ms
    if dist:
        t = torch.tensor([ms, att_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_all, att_ms = float(t[0]), float(t[1])

    # the optional collective, timed on its own (not part of `value`): reassembling one attention layer's output
    # [batch, 8 heads, 256] fp32 on every rank with the NCCL all-gather of shard.gather_outputs, as a caller
    # feeding a replicated projection would
    gather = None
    if dist:
        loc = hy.out.view(B, AT_HQ, AT_D)
        for _ in range(3):
            pkg.shard.gather_outputs(dist, loc, GB, AT_HQ, world)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for _ in range(args.steps):
            pkg.shard.gather_outputs(dist, loc, GB, AT_HQ, world)
        g1.record()
        torch.cuda.synchronize()
        g_ms = pkg.shard.max_over_ranks(dist, g0.elapsed_time(g1) / args.steps, "cuda")
        g_bytes = GB * AT_HQ * AT_D * 4
        gather = {"op": "shard.gather_outputs: NCCL all-gather of one attention layer's output + placement",
                  "bytes_gathered": g_bytes, "ms_per_call": g_ms, "algbw_GBs": g_bytes / (g_ms * 1e-3) / 1e9,
                  "timed": "CUDA events on the collective's stream, max over ranks; not part of value"}

    # end to end: (1) through the `_dev` ABI with every layer's inputs copied from pinned host memory and its
    # output copied back, the copies overlapped with the neighbouring layers' kernels (the headline e2e); (2) through
    # the synchronous host-pointer ABI (H2D + D2H inside every call), reported beside it
    e2e = None
    if not args.no_e2e:
        pipe = HybridPipe(torch, hy, seed=77 + rank)
        pipe.step()  # warm
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            pipe.step()
        pipe_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / args.steps, "cuda")
        ctx.set_stream(None)
        host = HybridHost(torch, B, seed=99 + rank, weights=weights)
        host.step(hy)  # warm
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host.step(hy)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        if dist:
            t = torch.tensor([e2e_ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t[0])
        e2e = {"value": GB / (pipe_ms * 1e-3), "unit": UNIT, "ms_per_step": pipe_ms,
               "h2d_bytes_per_step": pipe.h2d * world, "d2h_bytes_per_step": pipe.d2h * world,
               "path": "C ABI _dev entry points (eif_cuda_deltanet_core_dev x 18, eif_cuda_fullatt_decode_dev x 6); "
                       "every layer's inputs H2D from pinned host memory and its output D2H on two copy streams, "
                       "overlapped with the neighbouring layers' kernels; the step ends with its last output on "
                       "the host",
               "host_calls": {"value": GB / (e2e_ms * 1e-3), "ms_per_step": e2e_ms,
                              "h2d_bytes_per_step": host.h2d * world, "d2h_bytes_per_step": host.d2h * world,
                              "path": "synchronous host-pointer C ABI (eif_cuda_deltanet_core x 18, "
                                      "eif_cuda_fullatt_decode x 6), copies inside every call"}}

    if rank != 0:
        return None
    hbm, _, src = peaks()
    bytes_att = attn_layer_bytes(B)
    achieved = bytes_att / (att_ms * 1e-3) / 1e9
    step_bytes = n_att * bytes_att + LAYER_TYPES.count("D") * deltanet_layer_bytes(B)
    line = {
        "metric": METRIC, "value": GB / (ms_all * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_all, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 math; bf16 KV, fp32 DeltaNet state", "data": "synthetic (seeded)",
        "config": {"workload": "qwen35_hybrid_decode (BASELINE configs[4])", "global_batch": GB, "ctx": CTX,
                   "layers": "18 DeltaNet (16h, d128, fp32 S) + 6 gated attention (8q/2kv, hd256, bf16 KV)",
                   "per_gpu_batch": B, "parallelism": f"batch-sharded x{world}, no collective",
                   "l2": "inputs larger than L2 (17.2 GB KV per attention layer, 268 MB S per DeltaNet layer)",
                   "step_hbm_bytes": step_bytes},
        "e2e": e2e,
        "roofline": {"kernel": "decode attention (split-K kernel + chunk combine), one attention layer",
                     "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": src, "algorithmic_bytes_per_launch": bytes_att, "ms_per_launch": att_ms,
                     "traffic": traffic("attn_decode_tc_hd256", bytes_att)[0],
                     "traffic_source": traffic("attn_decode_tc_hd256", bytes_att)[1]},
        "step_hbm_frac": world * step_bytes / (ms_all * 1e-3) / 1e9 / (hbm * world),
        "gather": gather,
        "gpu_launches": launches,
        "clocks": clk,
    }
    return line


# ---------------------------------------------------------------------------------------------------
# the reference's C code on the host cores
# ---------------------------------------------------------------------------------------------------

def cpu_reference(n_seq_rounds, threads=None, per_round_cap_s=None):
    """Time the reference's own deltanet_core x 18 and fullatt_prep + fullatt_attend x 6 (fp32 KV at ctx 32768, the only
    KV dtype of its Qwen3.5 engine) for one decode step of independent sequences, one sequence per host
    thread (the reference has no batch dimension; a batch is a loop over engine states).
    Returns (tokens_per_s, cores, kind, sample description)."""
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc

    kind = "reference" if orc.ref_available() else "port"
    ncpu = threads or len(os.sched_getaffinity(0))
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 64 << 30
    kv_bytes = 6 * 2 * CTX * AT_HKV * AT_D * 4
    workers = max(1, min(ncpu, int(avail * 0.5 // (kv_bytes + (20 << 20)))))
    rng = np.random.default_rng(77)
    block = rng.standard_normal((4096, AT_HKV * AT_D)).astype(np.float32)
    W = Weights()
    x = dict(qkv=rng.standard_normal(DN_CONV).astype(np.float32), z=rng.standard_normal(DN_H * DN_D).astype(
        np.float32), b=rng.standard_normal(DN_H).astype(np.float32), a=rng.standard_normal(DN_H).astype(np.float32),
             qg=rng.standard_normal(AT_HQ * 2 * AT_D).astype(np.float32),
             k=rng.standard_normal(AT_HKV * AT_D).astype(np.float32),
             v=rng.standard_normal(AT_HKV * AT_D).astype(np.float32))
    lib = orc.ref() if kind == "reference" else None

    class Seq:
        def __init__(self):
            self.kc = [np.tile(block, (CTX // 4096, 1)) for _ in range(6)]
            self.vc = [np.tile(block[::-1].copy(), (CTX // 4096, 1)) for _ in range(6)]
            self.S = [(0.02 * block.ravel()[:DN_H * DN_D * DN_D].reshape(DN_H, DN_D, DN_D)).copy() for _ in range(18)]
            self.conv = [np.zeros((DN_CONV, CONV_K), np.float32) for _ in range(18)]

        def step(self):
            # each mixer exactly as the engine calls it: deltanet_core; fullatt_prep then fullatt_attend
            a = d = 0
            for typ in LAYER_TYPES:
                if typ == "D":
                    orc.deltanet_core(x["qkv"], x["z"], x["b"], x["a"], self.conv[d], self.S[d], lib=lib, **W.dn[d])
                    d += 1
                else:
                    w = W.at[a]
                    q, g, _ = orc.fullatt_prep(x["qg"], x["k"], x["v"], w["q_norm"], w["k_norm"], self.kc[a],
                                               self.vc[a], CTX - 1, AT_HQ, AT_HKV, AT_D, lib=lib)
                    if kind == "reference":
                        orc.ref_fullatt_attend(q, g, self.kc[a], self.vc[a], w["sub_norm"], 0, CTX - 1, AT_HQ,
                                               AT_HKV, AT_D)
                    else:
                        o = orc.attend_decode(q, self.kc[a], self.vc[a], CTX - 1, AT_HQ, AT_HKV, AT_D, 1 / 16.0,
                                              gate=g)
                        orc.subln(o, w["sub_norm"], 2)
                    a += 1

    if kind == "reference":
        orc.ref().ref_set_threads(1)
    seqs = [Seq() for _ in range(workers)]
    pool = ThreadPoolExecutor(max_workers=workers)
    list(pool.map(lambda s: s.step(), seqs))  # warm (page in)
    times = []
    for _ in range(n_seq_rounds):
        t0 = time.perf_counter()
        list(pool.map(lambda s: s.step(), seqs))
        times.append(time.perf_counter() - t0)
        if per_round_cap_s and sum(times) > per_round_cap_s:
            break
    pool.shutdown()
    t = float(np.median(times))
    sample = (f"{workers} sequences x 1 decode step through the 24 mixers at ctx {CTX} (fp32 KV), one sequence "
              f"per host thread, median of {len(times)} rounds of {t:.3f} s; x{BATCH // workers if workers else 0} "
              f"rounds would cover the batch of {BATCH}")
    return workers / t, workers, kind, sample, t


def run_reference(args, rank):
    if rank != 0:
        return None
    warm = max(0, args.warmup)
    tps, cores, kind, sample, t = cpu_reference(max(1, args.steps) + warm, per_round_cap_s=240)
    return {"metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": BATCH / tps * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": "qwen35_hybrid_decode (BASELINE configs[4])", "global_batch": BATCH, "ctx": CTX,
                       "kv_dtype": "f32 (the reference's only Qwen3.5 KV dtype)"},
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PF_B, PF_S, PF_HQ, PF_HKV, PF_D = 8, 4096, 12, 2, 128


def prefill_flops(B, S):
    """Causal QK^T + PV FLOPs: 2 * B * Hq * D * S * (S + 1)."""
    return 2.0 * B * PF_HQ * PF_D * S * (S + 1)


def cpu_prefill_reference(seconds=20.0):
    """The reference's fullatt_attend per token (Qwen3.5 prefill_chunk's parallel loop over tokens,
    src/eif_qwen35.c:1122-1133; gate = +100 -> sigmoid 1, plain), one sequence of the config, tokens
    spread over the causal range, one token per host thread; scaled by FLOPs to the whole config."""
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    ncpu = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(5)
    kc = rng.standard_normal((PF_S, PF_HKV * PF_D)).astype(np.float32)
    vc = rng.standard_normal((PF_S, PF_HKV * PF_D)).astype(np.float32)
    q = rng.standard_normal(PF_HQ * PF_D).astype(np.float32)
    gate = np.full(PF_HQ * PF_D, 100.0, np.float32)
    kind = "reference" if orc.ref_available() else "port"

    def one(t):
        if kind == "reference":
            orc.ref_fullatt_attend(q, gate, kc, vc, None, 1, t, PF_HQ, PF_HKV, PF_D)
        else:
            orc.attend_decode(q, kc, vc, t, PF_HQ, PF_HKV, PF_D, 0.0884)
        return t

    positions = list(range(PF_S - 1, -1, -PF_S // 256))
    pool = ThreadPoolExecutor(max_workers=ncpu)
    done, t0 = [], time.perf_counter()
    while time.perf_counter() - t0 < seconds:  # cycle over the spread of positions for the time budget
        for i in range(0, len(positions), ncpu):
            done += list(pool.map(one, positions[i:i + ncpu]))
    el = time.perf_counter() - t0
    pool.shutdown()
    flops_done = sum(4.0 * PF_HQ * PF_D * (t + 1) for t in done)
    tps = PF_B * PF_S / (el * prefill_flops(PF_B, PF_S) / flops_done)
    return tps, ncpu, kind, (f"{len(done)} query tokens of one sequence (256 positions spread over the causal "
                             f"range, repeated), one token per host thread, {el:.1f} s; scaled by FLOPs to "
                             f"{PF_B} x {PF_S}")


_CPU_MEMO = {}


def cpu_chunked_reference(seconds=10.0):
    """Memoised: the recurrent and the chunked workloads share this measurement within one run."""
    if seconds not in _CPU_MEMO:
        _CPU_MEMO[seconds] = _cpu_chunked_reference(seconds)
    return _CPU_MEMO[seconds]


def _cpu_chunked_reference(seconds):
    """What the engine's prefill_chunk runs for a DeltaNet layer: the reference's deltanet_core once per
    token (src/eif_qwen35.c:1104-1106; conv window, norms, gates, the rule, gated RMSNorm), 16 heads of
    d 128 from a zero state, one sequence per host thread for the time budget.  Returns tokens/s of all
    threads together (the rule, config 4's work, is the bulk of each call)."""
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    ncpu = len(os.sched_getaffinity(0))
    kind = "reference" if orc.ref_available() else "port"
    lib = orc.ref() if kind == "reference" else None
    if kind == "reference":
        orc.ref().ref_set_threads(1)
    W = Weights().dn[0]
    rng = np.random.default_rng(6)
    xs = [dict(qkv=rng.standard_normal(DN_CONV).astype(np.float32), z=rng.standard_normal(DN_H * DN_D).astype(
        np.float32), b=rng.standard_normal(DN_H).astype(np.float32), a=rng.standard_normal(DN_H).astype(np.float32))
          for _ in range(16)]

    def run(_):
        S = np.zeros((DN_H, DN_D, DN_D), np.float32)
        conv = np.zeros((DN_CONV, CONV_K), np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            x = xs[n % len(xs)]
            orc.deltanet_core(x["qkv"], x["z"], x["b"], x["a"], conv, S, lib=lib, **W)
            n += 1
        return n, time.perf_counter() - t0

    pool = ThreadPoolExecutor(max_workers=ncpu)
    res = list(pool.map(run, range(ncpu)))
    pool.shutdown()
    tokens = sum(n for n, _ in res)
    el = max(t for _, t in res)
    return tokens / el, ncpu, kind, (f"{tokens} tokens of deltanet_core (16 heads, d 128), one sequence per host "
                                     f"thread, {el:.1f} s")


def run_prefill(args, torch, dist, rank, world, local_rank):
    """causal prefill, batch 8 x 4096 tokens, 12 q / 2 kv heads, head_dim 128, bf16."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    # (sequence, kv-head group) units: past 8 ranks a sequence's two kv groups go to different ranks
    GBP = args.batch or PF_B  # global batch (a smaller one only for profiling captures)
    sh = pkg.shard.shard(GBP, PF_HKV, world, rank)
    B, hkv = sh.nb, sh.nh
    hq = hkv * (PF_HQ // PF_HKV)
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(11 + rank)
    kv = pkg.KVCache(ctx, 1, B, PF_S, hkv, PF_D, pkg.BF16)
    for p in kv.layer_ptrs(0):
        torch.as_tensor(CudaArray(p, (B * PF_S * hkv * PF_D,), "<i2"), device=dev).view(torch.bfloat16).normal_(
            generator=gen)
    q = torch.randn(B, PF_S, hq * PF_D, device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(PF_D)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > L2: evicts q / K / V between launches
    for _ in range(args.warmup):
        kv.attend_prefill_dev(0, q.data_ptr(), PF_S, 0, hq, scale, out.data_ptr())
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    l0 = ctx.launch_count
    for s in range(args.steps):
        flush.zero_()
        ev[s][0].record()
        kv.attend_prefill_dev(0, q.data_ptr(), PF_S, 0, hq, scale, out.data_ptr())
        ev[s][1].record()
    torch.cuda.synchronize()
    launches = ctx.launch_count - l0
    clk = clocks.stop()
    ctx.synchronize()
    ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    # e2e through the host-pointer ABI: fp32 q from pinned host memory, fp32 output read back
    e2e_ms = None
    qh = torch.randn(B, PF_S, hq * PF_D, generator=torch.Generator().manual_seed(3)).pin_memory().numpy()
    if not args.no_e2e:
        ctx.set_stream(None)
        kv.attend_prefill(0, qh, PF_S, 0, hq, scale)
        t0 = time.perf_counter()
        for _ in range(max(1, args.steps // 4)):
            kv.attend_prefill(0, qh, PF_S, 0, hq, scale)
        e2e_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / max(1, args.steps // 4), "cuda")
    if rank != 0:
        return None
    _, tflops_peak, src = peaks()
    flops = prefill_flops(B, PF_S) * hq / PF_HQ  # this rank's launch
    pf_bytes = B * PF_S * (2 * hq + 2 * hkv) * PF_D * 2  # q, o (bf16) and the K / V rows, each once
    ach = flops / (ms * 1e-3) / 1e12
    GB = GBP
    line = {"metric": "causal prefill attention tokens/s (BASELINE configs[1])", "value": GB * PF_S / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 in, fp32 accumulate, bf16 out", "data": "synthetic (seeded)",
            "config": {"workload": "gqa_causal_prefill (BASELINE configs[1])", "global_batch": GB, "seq_len": PF_S,
                       "heads": "12 q / 2 kv", "head_dim": PF_D, "l2": "256 MiB flush between launches",
                       "parallelism": f"(sequence, kv head) units over {world} rank(s), no collective"},
            "e2e": None if e2e_ms is None else {
                "value": GB * PF_S / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": qh.nbytes * world, "d2h_bytes_per_step": qh.nbytes * world,
                "path": "host-pointer C ABI eif_cuda_attend_prefill (fp32 in/out)"},
            "roofline": {"kernel": "attn_prefill_tc_kernel", "bound": "tensor", "achieved": ach,
                         "peak": tflops_peak, "unit": "TFLOP/s", "frac": ach / tflops_peak, "peak_source": src,
                         "algorithmic_flops_per_launch": flops,
                         "traffic": traffic("attn_prefill_tc", pf_bytes)[0],
                         "traffic_source": traffic("attn_prefill_tc", pf_bytes)[1]},
            "gpu_launches": launches, "clocks": clk}
    if world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample = cpu_prefill_reference()
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}
    return line


CK_B, CK_T, CK_H, CK_D = 4, 8192, 16, 128


def run_chunked(args, torch, dist, rank, world, local_rank):
    """chunked DeltaNet prefill, batch 4 x 8192 tokens, 16 heads, d 128, bf16 q/k/v,
    zero initial state (reset before every timed launch, outside the events)."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    GBC = args.batch or CK_B  # global batch (a smaller one only for profiling captures)
    sh = pkg.shard.shard(GBC, CK_H, world, rank)  # (sequence, head) units; past 4 ranks heads split
    B, H = sh.nb, sh.nh
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(21 + rank)
    qk = torch.randn(2, B, CK_T, H, CK_D, device=dev, generator=gen)
    qk = (qk / torch.sqrt((qk * qk).sum(-1, keepdim=True) + 1e-12)).to(torch.bfloat16)
    q, k = qk[0].contiguous(), qk[1].contiguous()
    v = torch.randn(B, CK_T, H, CK_D, device=dev, generator=gen).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(B, CK_T, H, device=dev, generator=gen))
    g = -torch.nn.functional.softplus(torch.randn(B, CK_T, H, device=dev, generator=gen))
    o = torch.empty_like(v)
    st = pkg.DeltaState(ctx, 1, B, H, CK_D, CK_D)
    s_ptr, _ = st.layer_ptrs(0)
    S = torch.as_tensor(CudaArray(s_ptr, (B * H * CK_D * CK_D,), "<f4"), device=dev)
    qs = 1.0 / math.sqrt(CK_D)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def launch():
        st.prefill_dev(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), g.data_ptr(), CK_T, qs,
                       o.data_ptr())

    for _ in range(args.warmup):
        S.zero_()
        launch()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    l0 = ctx.launch_count
    for s in range(args.steps):
        S.zero_()
        flush.zero_()
        ev[s][0].record()
        launch()
        ev[s][1].record()
    torch.cuda.synchronize()
    launches = ctx.launch_count - l0
    clk = clocks.stop()
    ctx.synchronize()
    ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    # e2e through the host-pointer entry: fp32 q / k / v / beta / g from pinned host memory, fp32 o read back
    e2e = None
    if not args.no_e2e:
        def pinned(t_):
            return t_.float().cpu().pin_memory()
        hq, hk, hv, hb, hg = (pinned(x) for x in (q, k, v, beta, g))
        ho = torch.empty(B, CK_T, H, CK_D).pin_memory()
        ctx.set_stream(None)
        reps = max(1, args.steps // 4)
        st.reset()
        st.prefill(0, hq.numpy(), hk.numpy(), hv.numpy(), hb.numpy(), hg.numpy(), qs, out=ho.numpy())  # warm
        t0 = time.perf_counter()
        for _ in range(reps):
            st.reset()
            st.prefill(0, hq.numpy(), hk.numpy(), hv.numpy(), hb.numpy(), hg.numpy(), qs, out=ho.numpy())
        e2e_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / reps, "cuda")
        nb = sum(x.numel() * 4 for x in (hq, hk, hv, hb, hg))
        e2e = {"value": GBC * CK_T / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": nb * world, "d2h_bytes_per_step": ho.numel() * 4 * world,
               "path": "host-pointer C ABI eif_cuda_deltanet_prefill (fp32 in/out; state reset included)"}
    if rank != 0:
        return None
    hbm, _, src = peaks()
    GB = GBC
    # this rank's launch: q, k, v, o (bf16) + beta, g per token-head, S read and written once
    bytes_alg = B * CK_T * H * (3 * CK_D * 2 + 2 * 4 + CK_D * 2) + 2 * B * H * CK_D * CK_D * 4
    ach = bytes_alg / (ms * 1e-3) / 1e9
    flops_rec = 4.0 * CK_D * CK_D * GB * CK_T * CK_H
    line = {"metric": "chunked DeltaNet prefill tokens/s (BASELINE configs[3])", "value": GB * CK_T / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 q/k/v/o, fp32 state and accumulate", "data": "synthetic (seeded)",
            "config": {"workload": "deltanet_chunked_prefill (BASELINE configs[3])", "global_batch": GB,
                       "seq_len": CK_T, "heads": CK_H, "head_dim": CK_D, "chunk": 64,
                       "l2": "256 MiB flush between launches",
                       "parallelism": f"(sequence, head) units over {world} rank(s), no collective"},
            "roofline": {"kernel": "deltanet_chunked_kernel", "bound": "hbm", "achieved": ach, "peak": hbm,
                         "unit": "GB/s", "frac": ach / hbm, "peak_source": src, "algorithmic_bytes_per_launch":
                             bytes_alg, "recurrent_equivalent_tflops": flops_rec / (ms * 1e-3) / 1e12,
                         "traffic": traffic("deltanet_chunked", bytes_alg)[0],
                         "traffic_source": traffic("deltanet_chunked", bytes_alg)[1]},
            "gpu_launches": launches, "clocks": clk}
    if e2e is not None:
        line["e2e"] = e2e
    if world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample = cpu_chunked_reference()
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}
    return line


RC_B, RC_H, RC_D, RC_STEPS, RC_NIN = 64, 16, 128, 1024, 16  # BASELINE configs[2]; RC_NIN input sets, cycled
RC_LAYERS = 2  # states alternated step by step: 2 x 64 MiB > L2, so every step streams its state from HBM


def run_recurrent(args, torch, dist, rank, world, local_rank):
    """the Gated DeltaNet delta rule over 64 sequences x 16 heads, d_k = d_v = 128, fp32
    state ~ N(0, 0.02), 1024 sequential decode steps (one bench step = the 1024 steps): q, k ~ N(0,1)
    L2-normalised per head, v ~ N(0,1), beta = sigmoid(N(0,1)), log-decay g = -softplus(N(0,1)) (alpha = e^g),
    q_scale = 1/sqrt(d_k).  RC_NIN seeded input sets are cycled over the steps.  The state of one layer
    (64 MiB) would stay in the 126 MB L2 from one step to the next; the engine interleaves layers, so its
    state goes back to HBM every step (BASELINE's configs[2] note): the steps alternate between RC_LAYERS
    layers' states, and each bench step is 1024 rule steps (512 per layer)."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    GB = args.batch or RC_B
    sh = pkg.shard.shard(GB, RC_H, world, rank)  # (sequence, head) units
    B, H = sh.nb, sh.nh
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(31 + rank)
    st = pkg.DeltaState(ctx, RC_LAYERS, B, H, RC_D, RC_D, 0)
    for layer in range(RC_LAYERS):
        s_ptr, _ = st.layer_ptrs(layer)
        torch.as_tensor(CudaArray(s_ptr, (B * H * RC_D * RC_D,), "<f4"), device=dev).normal_(0, 0.02, generator=gen)

    def l2n(x):
        return x / x.norm(dim=-1, keepdim=True)
    ins = []
    for _ in range(RC_NIN):
        q = l2n(torch.randn(B, H, RC_D, device=dev, generator=gen)).reshape(B, H * RC_D).contiguous()
        k = l2n(torch.randn(B, H, RC_D, device=dev, generator=gen)).reshape(B, H * RC_D).contiguous()
        v = torch.randn(B, H * RC_D, device=dev, generator=gen)
        beta = torch.sigmoid(torch.randn(B, H, device=dev, generator=gen))
        g = -torch.nn.functional.softplus(torch.randn(B, H, device=dev, generator=gen))
        ins.append((q, k, v, beta, g))
    o = torch.empty(B, H * RC_D, device=dev)
    q_scale = 1.0 / math.sqrt(RC_D)

    def rule(i):
        q, k, v, beta, g = ins[i % RC_NIN]
        st.step_dev(i % RC_LAYERS, q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(), g.data_ptr(), q_scale,
                    o.data_ptr())

    for _ in range(args.warmup):
        for i in range(RC_STEPS):
            rule(i)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    l0 = ctx.launch_count
    for s_ in range(args.steps):
        ev[s_][0].record()
        for i in range(RC_STEPS):
            rule(i)
        ev[s_][1].record()
    torch.cuda.synchronize()
    launches = ctx.launch_count - l0
    clk = clocks.stop()
    ctx.synchronize()
    ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    ms = pkg.shard.max_over_ranks(dist, ms, "cuda")
    launch_ms = ms / RC_STEPS  # the timed region is the 1024 rule launches back to back, nothing else
    # e2e through the host-pointer ABI: every step copies q / k / v / beta / g from pinned host memory and
    # reads o back (the state stays on the device, as the engine's does)
    hin = [tuple(x.cpu().pin_memory().numpy() for x in ins[i]) for i in range(RC_NIN)]
    oh = torch.empty(B, H * RC_D).pin_memory().numpy()
    e2e_ms = None
    if not args.no_e2e:
        ctx.set_stream(None)
        st.step(0, *hin[0], q_scale, out=oh)
        t0 = time.perf_counter()
        for i in range(RC_STEPS):
            st.step(i % RC_LAYERS, *hin[i % RC_NIN], q_scale, out=oh)
        e2e_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3, "cuda")
    if rank != 0:
        return None
    hbm, _, src = peaks()
    sbytes = 2.0 * B * H * RC_D * RC_D * 4
    io_bytes = 4.0 * B * H * RC_D * 4 + 2.0 * B * H * 4
    ach = (sbytes + io_bytes) / (launch_ms * 1e-3) / 1e9
    h2d = sum(x.nbytes for x in hin[0]) * world
    d2h = oh.nbytes * world
    line = {"metric": "Gated DeltaNet recurrent decode tokens/s (BASELINE configs[2], 1024 sequential steps)",
            "value": GB * RC_STEPS / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": {"workload": "deltanet_recurrent_decode (BASELINE configs[2])", "global_batch": GB,
                       "heads": RC_H, "d_k": RC_D, "d_v": RC_D, "steps_per_bench_step": RC_STEPS,
                       "l2": f"state streamed from HBM every step ({RC_LAYERS} layers' states alternated, as "
                             "the engine interleaves layers); inputs cycled",
                       "parallelism": f"(sequence, head) units over {world} rank(s), no collective"},
            "e2e": None if e2e_ms is None else {
                "value": GB * RC_STEPS / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d * RC_STEPS, "d2h_bytes_per_step": d2h * RC_STEPS,
                "path": "host-pointer C ABI eif_cuda_deltanet_step (pinned), 1024 calls"},
            "roofline": {"kernel": "delta_rule_kernel", "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                         "frac": ach / hbm, "peak_source": src, "algorithmic_bytes_per_launch": sbytes + io_bytes,
                         "launch_ms": launch_ms, "traffic": traffic("delta_rule", sbytes + io_bytes)[0],
                         "traffic_source": traffic("delta_rule", sbytes + io_bytes)[1]},
            "gpu_launches": launches, "clocks": clk}
    if world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample = cpu_chunked_reference()
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind,
                                "sample": sample + " (the engine runs config 3's rule inside deltanet_core)"}
    return line


DC_HQ, DC_HKV, DC_D, DC_THETA = 14, 2, 64, 1e6  # BASELINE configs[0]'s heads (Qwen2.5-0.5B), NeoX RoPE
DC_B, DC_CTX = 256, 4096  # the batched variant; configs[0] itself is --batch 1 --ctx 512 --kv f32
KV_ELT = {"f32": 4, "bf16": 2, "int8": 1}
# --heads qwen35: the Qwen3.5 full-attention shape (8 q / 2 kv heads, head_dim 256), one attention mixer per step
Q5_HQ, Q5_HKV, Q5_D = AT_HQ, AT_HKV, AT_D


def decode_bytes(B, L, hkv, kv, D=DC_D):
    """Algorithmic bytes of one decode-attention launch: K and V rows [0, L) of every (sequence, kv head),
    plus the per-(row, kv head) K and V scales of an INT8 cache (q and out are < 0.1 %)."""
    b = 2.0 * B * hkv * L * D * KV_ELT[kv]
    if kv == "int8":
        b += 2.0 * B * hkv * L * 4
    return b


def cpu_decode_reference(kv_name, L, seconds=10.0):
    """The reference's own tinyllm decode step at position L-1 (tinyllm_forward_embedding_ex on a one-layer fp32
    model whose attention is observable, oracle/ref_shim.c: RoPE, the cache write -- quantised for an INT8
    cache, src/eif_tinyllm.c:509-553 -- and the head loop :555-656 over a pre-filled cache), one sequence per
    host thread for the time budget.  A bf16 cache is timed as the reference's fp32 cache (it has no bf16).
    Without the reference build: the restatement's attention loop (fp32 / INT8) alone."""
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    ncpu = len(os.sched_getaffinity(0))
    kind = "reference" if orc.ref_available() else "port"
    kv_type = 1 if kv_name == "int8" else 0
    if kind == "reference":
        orc.ref().ref_set_threads(1)

        def run(_):
            t1 = orc.ref_tinyllm_decode_time(DC_HQ, DC_HKV, DC_D, L, DC_THETA, kv_type, L - 1, 3) / 3
            n = max(3, int(seconds / max(t1, 1e-6)))
            return n, orc.ref_tinyllm_decode_time(DC_HQ, DC_HKV, DC_D, L, DC_THETA, kv_type, L - 1, n)
        what = ("the reference's tinyllm forward (one fp32 layer; its zero q/k/v and identity o projections add "
                "dim^2 matvecs to each step)")
    else:
        rng = np.random.default_rng(8)
        kv_dim = DC_HKV * DC_D
        q = rng.standard_normal(DC_HQ * DC_D).astype(np.float32)
        kc = rng.standard_normal((L, kv_dim)).astype(np.float32)
        vc = rng.standard_normal((L, kv_dim)).astype(np.float32)
        kq, ks = orc.kv_quantize(kc, DC_HKV, DC_D) if kv_type else (None, None)
        vq, vs = orc.kv_quantize(vc, DC_HKV, DC_D) if kv_type else (None, None)

        def run(_):
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < seconds:
                if kv_type:
                    orc.attend_decode_i8(q, kq, ks, vq, vs, L - 1, DC_HQ, DC_HKV, DC_D, 0.125)
                else:
                    orc.attend_decode(q, kc, vc, L - 1, DC_HQ, DC_HKV, DC_D, 0.125)
                n += 1
            return n, time.perf_counter() - t0
        what = "the restatement's attention loop"
    pool = ThreadPoolExecutor(max_workers=ncpu)
    res = list(pool.map(run, range(ncpu)))
    pool.shutdown()
    tokens = sum(n for n, _ in res)
    el = max(t for _, t in res)
    return tokens / el, ncpu, kind, (f"{tokens} decode steps at ctx {L} through {what}, "
                                     f"{'int8 codes + scales' if kv_type else 'fp32'} cache, one sequence per "
                                     f"host thread, {el:.1f} s")


def run_decode(args, torch, dist, rank, world, local_rank):
    """tinyllm GQA decode at BASELINE configs[0]'s head shape (14 q / 2 kv heads, head_dim 64, NeoX RoPE
    theta 1e6), batched: one decode step of one attention layer for `--batch` sequences at context `--ctx`
    over an fp32, bf16 or INT8 (`--kv`) cache -- eif_cuda_decode_step: RoPE of the new q and k, the (plain or
    quantised) cache write and attention over rows [0, ctx) in one call.  The roofline times the attention
    alone (attend_decode_dev on the same rows).
    `--heads qwen35`: the Qwen3.5 full-attention shape (8 q / 2 kv heads, head_dim 256, fp32 or bf16 cache) and
    its whole attention mixer per step -- eif_cuda_fullatt_decode_dev: q / k norms, partial RoPE, the cache
    write, attention with the sigmoid gate and SubLN."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    kv_name = args.kv
    q35 = getattr(args, "heads", "qwen2") == "qwen35"
    HQ, HKV, D = (Q5_HQ, Q5_HKV, Q5_D) if q35 else (DC_HQ, DC_HKV, DC_D)
    GB, L = args.batch or DC_B, args.ctx or DC_CTX
    sh = pkg.shard.shard(GB, HKV, world, rank)  # (sequence, kv group) units
    B, hkv = sh.nb, sh.nh
    hq = hkv * (HQ // HKV)
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local_rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(21 + rank)
    dt = {"f32": pkg.F32, "bf16": pkg.BF16, "int8": pkg.INT8}[kv_name]
    kv = pkg.KVCache(ctx, 1, B, L, hkv, D, dt)
    kv.set_rope(DC_THETA)
    if q35:
        w = Weights().at[0]
        kv.set_norms(0, w["q_norm"], w["k_norm"])
        sub = torch.from_numpy(w["sub_norm"][:hq * D]).to(dev)
    n_el = B * L * hkv * D
    for p in kv.layer_ptrs(0):  # cache ~ N(0,1) (fp32 / bf16) or uniform codes with scales ~ U(0.005, 0.03)
        if kv_name == "f32":
            torch.as_tensor(CudaArray(p, (n_el,), "<f4"), device=dev).normal_(generator=gen)
        elif kv_name == "bf16":
            torch.as_tensor(CudaArray(p, (n_el,), "<i2"), device=dev).view(torch.bfloat16).normal_(generator=gen)
        else:
            t = torch.as_tensor(CudaArray(p, (n_el,), "|i1"), device=dev)
            t.copy_(torch.randint(-127, 128, (n_el,), device=dev, generator=gen, dtype=torch.int8))
    if kv_name == "int8":  # head-major scales, rows padded to a multiple of 64
        for p in kv.layer_scales(0):
            torch.as_tensor(CudaArray(p, (B * hkv * ((L + 63) // 64 * 64),), "<f4"), device=dev).uniform_(
                0.005, 0.03, generator=gen)
    q = torch.randn(B, hq * D * (2 if q35 else 1), device=dev, generator=gen)  # Qwen3.5: [q | gate] per head
    k = torch.randn(B, hkv * D, device=dev, generator=gen)
    v = torch.randn(B, hkv * D, device=dev, generator=gen)
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    q_rot = torch.empty(B, hq * D, device=dev)
    gate = torch.empty(B, hq * D, device=dev)
    out = torch.empty(B, hq * D, device=dev)
    scale = 1.0 / math.sqrt(D)
    bytes_alg = decode_bytes(B, L, hkv, kv_name, D)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if bytes_alg < (1 << 30) else None

    def step():
        if q35:
            kv.fullatt_decode_dev(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), L - 1, hq, scale,
                                  out.data_ptr(), subln=pkg.SUBLN_WEIGHT, sub_norm_dev=sub.data_ptr())
        else:
            kv.decode_step_dev(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), L - 1, hq, scale,
                               out.data_ptr())

    def attend():
        if q35:
            kv.attend_decode_dev(0, q_rot.data_ptr(), pos.data_ptr(), L - 1, hq, scale, out.data_ptr(),
                                 gate_dev=gate.data_ptr(), subln=pkg.SUBLN_WEIGHT, sub_norm_dev=sub.data_ptr())
        else:
            kv.attend_decode_dev(0, q_rot.data_ptr(), pos.data_ptr(), L - 1, hq, scale, out.data_ptr())

    if q35:
        kv.fullatt_prep_dev(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), hq, q_rot.data_ptr(),
                            gate.data_ptr())
    else:
        kv.rope_append_dev(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), hq, q_rot.data_ptr())
    for _ in range(args.warmup):
        step()
        attend()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    l0 = ctx.launch_count
    for s in range(args.steps):
        if flush is not None:
            flush.zero_()  # caches smaller than 1 GiB: evict them from L2 between steps
        ev[s][0].record()
        step()
        ev[s][1].record()
    torch.cuda.synchronize()
    launches = ctx.launch_count - l0
    for s in range(args.steps):  # the attention alone, for the roofline
        if flush is not None:
            flush.zero_()
        ev[s][2].record()
        attend()
        ev[s][3].record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ctx.synchronize()
    ms = float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))
    att_ms = float(np.mean([e[2].elapsed_time(e[3]) for e in ev]))
    ms = pkg.shard.max_over_ranks(dist, ms, "cuda")
    # e2e through the host-pointer ABI: pinned fp32 q / k / v / pos in, the output back
    hg = torch.Generator().manual_seed(5)
    qh = torch.randn(B, hq * D * (2 if q35 else 1), generator=hg).pin_memory().numpy()
    kh = torch.randn(B, hkv * D, generator=hg).pin_memory().numpy()
    vh = torch.randn(B, hkv * D, generator=hg).pin_memory().numpy()
    subh = sub.cpu().pin_memory().numpy() if q35 else None
    ph = torch.full((B,), L - 1, dtype=torch.int32).pin_memory().numpy()
    oh = torch.empty(B, hq * D).pin_memory().numpy()

    def e2e_call():
        if q35:
            kv.fullatt_decode(0, qh, kh, vh, ph, hq, scale, subln=pkg.SUBLN_WEIGHT, sub_norm=subh, out=oh)
        else:
            kv.decode_step(0, qh, kh, vh, ph, hq, scale, out=oh)
    e2e_ms = None
    if not args.no_e2e:
        ctx.set_stream(None)
        n_e2e = max(3, args.steps) * (20 if bytes_alg < (64 << 20) else 1)  # short steps: enough of them to time
        for _ in range(3):
            e2e_call()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            e2e_call()
        e2e_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / n_e2e, "cuda")
    if rank != 0:
        return None
    hbm, _, src = peaks()
    ach = bytes_alg / (att_ms * 1e-3) / 1e9
    dec_kernel = {"bf16": "attn_decode_tc", "int8": "attn_decode_i8"}.get(kv_name, "attn_decode_f32")
    h2d = (qh.nbytes + kh.nbytes + vh.nbytes + ph.nbytes) * world
    d2h = oh.nbytes * world
    cfg_name = "BASELINE configs[0] exactly" if (GB, L, kv_name, q35) == (1, 512, "f32", False) else \
        "BASELINE configs[4]'s attention heads" if q35 else "BASELINE configs[0]'s heads, batched"
    metric = ("Qwen3.5 attention mixer decode tokens/s (one layer: fullatt_prep + gated attention + SubLN)" if q35
              else "tinyllm GQA decode tokens/s (one attention layer: RoPE + cache write + attention)")
    line = {"metric": metric,
            "value": GB / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 arithmetic over a " + kv_name + " cache", "data": "synthetic (seeded)",
            "config": {"workload": f"{'qwen35_attention' if q35 else 'tinyllm'}_decode ({cfg_name})",
                       "global_batch": GB, "ctx": L, "heads": f"{HQ} q / {HKV} kv", "head_dim": D,
                       "kv_dtype": kv_name,
                       "l2": "256 MiB flush between steps" if flush is not None else "cache > L2",
                       "parallelism": f"(sequence, kv group) units over {world} rank(s), no collective"},
            "e2e": None if e2e_ms is None else {
                "value": GB / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "host-pointer C ABI " + ("eif_cuda_fullatt_decode" if q35 else "eif_cuda_decode_step") +
                        " (pinned)"},
            "step_path": "fullatt_prep + split-K decode + combine" if q35 else
                         "one launch (attn_decode_step_kernel, a cluster per (sequence, kv head))"
                         if launches == args.steps else "rope_append_kernel + split-K decode + combine",
            "roofline": {"kernel": dec_kernel + "_kernel + combine", "bound": "hbm", "achieved": ach,
                         "peak": hbm,
                         "unit": "GB/s", "frac": ach / hbm, "peak_source": src,
                         "algorithmic_bytes_per_launch": bytes_alg, "attention_ms": att_ms,
                         "traffic": traffic(dec_kernel, bytes_alg)[0] if GB > 1 and not q35 else None,
                         "traffic_source": traffic(dec_kernel, bytes_alg)[1] if GB > 1 and not q35 else None},
            "gpu_launches": launches, "clocks": clk}
    if world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample = cpu_qwen35_attention_reference(L) if q35 else cpu_decode_reference(kv_name, L)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}
    return line


def cpu_qwen35_attention_reference(L, seconds=10.0):
    """The reference's fullatt_prep + fullatt_attend (src/eif_qwen35.c:699-790) of one token at position L-1
    over its fp32 cache (its only Qwen3.5 KV type), one sequence per host thread for the time budget."""
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    ncpu = len(os.sched_getaffinity(0))
    kind = "reference" if orc.ref_available() else "port"
    lib = orc.ref() if kind == "reference" else None
    if lib is not None:
        lib.ref_set_threads(1)
    w = Weights().at[0]
    rng = np.random.default_rng(9)
    qg = rng.standard_normal(Q5_HQ * 2 * Q5_D).astype(np.float32)
    k = rng.standard_normal(Q5_HKV * Q5_D).astype(np.float32)
    v = rng.standard_normal(Q5_HKV * Q5_D).astype(np.float32)
    block = rng.standard_normal((min(L, 4096), Q5_HKV * Q5_D)).astype(np.float32)

    def run(_):
        kc = np.tile(block, ((L + len(block) - 1) // len(block), 1))[:L].copy()
        vc = kc[::-1].copy()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            q, g, _ = orc.fullatt_prep(qg, k, v, w["q_norm"], w["k_norm"], kc, vc, L - 1, Q5_HQ, Q5_HKV, Q5_D, lib=lib)
            if lib is not None:
                orc.ref_fullatt_attend(q, g, kc, vc, w["sub_norm"], 0, L - 1, Q5_HQ, Q5_HKV, Q5_D)
            else:
                orc.subln(orc.attend_decode(q, kc, vc, L - 1, Q5_HQ, Q5_HKV, Q5_D, 1 / 16.0, gate=g), w["sub_norm"], 2)
            n += 1
        return n, time.perf_counter() - t0

    pool = ThreadPoolExecutor(max_workers=ncpu)
    res = list(pool.map(run, range(ncpu)))
    pool.shutdown()
    tokens = sum(n for n, _ in res)
    el = max(t for _, t in res)
    return tokens / el, ncpu, kind, (f"{tokens} tokens of fullatt_prep + fullatt_attend at ctx {L} (fp32 cache), one "
                                     f"sequence per host thread, {el:.1f} s")


# --workload projection: the quantised projections of one Qwen3.5-0.8B decode step (the reference's own model
# config, include/eif_qwen35.h:58-72): dim 1024, FFN 3584, 24 layers (DeltaNet x 3, attention) x 6, 16 x 128
# DeltaNet heads, 8 / 2 heads of 256 with the output gate, vocabulary 248320.  The projections that read the same
# input are stacked by rows into one matrix (DeltaNet qkv + z + b + a, attention q + k + v, FFN gate + up), so a
# step is 4 launches a layer plus the INT8 LM head (int8_gemv, the default tied embedding).
PJ_DIM, PJ_HID, PJ_VOCAB = 1024, 3584, 248320


def projection_step_shapes(qt=2):
    """(rows, cols, quant_type) of the launches of one decode step, in the engine's order."""
    out = []
    for typ in LAYER_TYPES:
        if typ == "A":  # q with its gate, k, v; o_proj
            out += [(2 * AT_HQ * AT_D + 2 * AT_HKV * AT_D, PJ_DIM, qt), (PJ_DIM, AT_HQ * AT_D, qt)]
        else:  # in_proj_qkv, in_proj_z, in_proj_b, in_proj_a; out_proj
            out += [(DN_CONV + DN_H * DN_D + 2 * DN_H, PJ_DIM, qt), (PJ_DIM, DN_H * DN_D, qt)]
        out += [(2 * PJ_HID, PJ_DIM, qt), (PJ_DIM, PJ_HID, qt)]  # FFN gate + up; down
    out.append((PJ_VOCAB, PJ_DIM, 4))
    return out


def _packed_bytes(rows, cols, qt):
    base = qt & 0xFF
    return rows * {0: 4 * cols, 1: (cols + 1) // 2, 2: (cols + 3) // 4, 3: (cols + 4) // 5}.get(base, cols)


def _linear_alg_bytes(rows, cols, qt, n):
    """Algorithmic bytes of one launch: the packed weights and scales once, n input and output vectors."""
    base, group = qt & 0xFF, qt >> 8
    n_sc = 0 if base == 0 else rows * (cols // group if group else 1)
    return _packed_bytes(rows, cols, qt) + 4 * n_sc + 4 * n * (cols + rows)


def cpu_projection_reference(shapes, n, seconds=10.0):
    """The reference's linear_gemv / linear_gemm / int8_gemv (oracle/_ref) over the step's projections with all
    host threads (its OpenMP loops), on random weight bytes; the port where the reference build is absent."""
    sys.path.insert(0, ROOT)
    from oracle import oracle as orc
    rng = np.random.default_rng(7)
    mats = []
    for rows, cols, qt in shapes:
        W = rng.integers(0, 256, _packed_bytes(rows, cols, qt), dtype=np.uint8)
        sc = None if (qt & 0xFF) == 0 else (0.01 + rng.random(rows)).astype(np.float32)
        mats.append((W, sc, rng.standard_normal((n, cols)).astype(np.float32), rows, cols, qt))
    use_ref = orc.ref_available()
    ncpu = os.cpu_count() or 1
    if use_ref:
        orc.ref().ref_set_threads(ncpu)
    steps, t_total = 0, 0.0
    while t_total < seconds:
        for W, sc, x, rows, cols, qt in mats:
            if use_ref:
                t_total += orc.ref_linear_time(W, sc, x, rows, cols, qt, 1)
            else:
                t0 = time.perf_counter()
                orc.linear(W, sc, x, rows, cols, qt)
                t_total += time.perf_counter() - t0
        steps += 1
    kind = "reference" if use_ref else "port"
    return n * steps / t_total, (ncpu if use_ref else 1), kind, (
        f"{steps} decode steps' projections ({len(shapes)} launches each, batch {n}), {t_total:.1f} s")


def run_projection(args, torch, dist, rank, world, local_rank):
    """Row f4: every projection of a Qwen3.5-0.8B decode step on the GPU (2-bit ternary weights with a scale a
    row, the INT8 LM head), `--batch` tokens a rank (default 1), replayed as one CUDA graph of the 97 launches.
    Weights: random bytes (every byte is a valid code of each format), ~380 MB > L2, so each step streams them
    from HBM.  Roofline: the ternary launches together (the dominant kernel), from a graph of those alone, and
    the LM head from its own launches."""
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    torch.cuda.set_device(local_rank)
    n = args.batch or 1
    shapes = projection_step_shapes()
    ctx = pkg.Context(local_rank)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    dev = torch.device("cuda", local_rank)
    rng = np.random.default_rng(11)
    lins, xs, outs = [], [], []
    for rows, cols, qt in shapes:
        W = rng.integers(0, 256, _packed_bytes(rows, cols, qt), dtype=np.uint8)
        sc = (0.01 + rng.random(rows)).astype(np.float32)
        lins.append(pkg.Linear(ctx, qt, rows, cols, W, sc))
        xs.append(torch.randn(n, cols, device=dev))
        outs.append(torch.empty(n, rows, device=dev))
    tern = [i for i, (_, _, qt) in enumerate(shapes) if qt != 4]
    head = len(shapes) - 1

    def launch(idx):
        for i in idx:
            lins[i].forward_dev(xs[i].data_ptr(), n, outs[i].data_ptr())

    every = list(range(len(shapes)))
    for _ in range(args.warmup):
        launch(every)
    torch.cuda.synchronize()
    graphs = {}
    for key, idx in (("step", every), ("ternary", tern)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch(idx)
        graphs[key] = g
    torch.cuda.synchronize()

    def timed(fn, k):
        ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in range(k)]
        for j in range(k):
            ev[j][0].record()
            fn()
            ev[j][1].record()
        torch.cuda.synchronize()
        return float(np.mean([e[0].elapsed_time(e[1]) for e in ev]))

    for _ in range(args.warmup):
        graphs["step"].replay()
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    ms = timed(graphs["step"].replay, args.steps)
    clk = clocks.stop()
    ms = pkg.shard.max_over_ranks(dist, ms, "cuda")
    tern_ms = pkg.shard.max_over_ranks(dist, timed(graphs["ternary"].replay, args.steps), "cuda")
    head_ms = pkg.shard.max_over_ranks(dist, timed(lambda: launch([head]), args.steps), "cuda")
    # e2e: each step copies the token's input from pinned host memory, runs the step's graph and reads the logits
    # back (the hidden states between projections stay on the device, as a device-resident decode step's do)
    e2e_ms = None
    xh = torch.randn(n, PJ_DIM).pin_memory()
    lh = torch.empty(n, PJ_VOCAB).pin_memory()
    if not args.no_e2e:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            xs[0].copy_(xh, non_blocking=True)
            graphs["step"].replay()
            lh.copy_(outs[head], non_blocking=True)
            stream.synchronize()
        e2e_ms = pkg.shard.max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / args.steps, "cuda")
    for g in graphs.values():
        del g
    graphs.clear()
    for lin in lins:
        lin.free()
    if rank != 0:
        return None
    hbm, _, src = peaks()
    tern_bytes = sum(_linear_alg_bytes(*shapes[i], n) for i in tern)
    head_bytes = _linear_alg_bytes(*shapes[head], n)
    step_bytes = tern_bytes + head_bytes
    ach = tern_bytes / (tern_ms * 1e-3) / 1e9
    head_ach = head_bytes / (head_ms * 1e-3) / 1e9
    kname = "linear_mma_kernel" if n >= 4 else "linear_kernel"  # the library's choice: tensor cores from 4 tokens
    # DRAM bytes per algorithmic byte were captured for the one-token kernel only
    tr, tr_src = traffic("linear_ternary2", tern_bytes) if n < 4 else (None, None)
    htr, htr_src = traffic("linear_int8_head", head_bytes) if n < 4 else (None, None)
    line = {"metric": "projection tokens/s (every quantised projection of a Qwen3.5-0.8B decode step)",
            "value": n * world / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weight bytes and inputs)",
            "config": {"workload": "projection (row f4): Qwen3.5-0.8B decode-step projections", "tokens_per_rank": n,
                       "launches_per_step": len(shapes), "weights": "2-bit ternary, a scale a row; INT8 LM head",
                       "weight_bytes_per_step": sum(_packed_bytes(*s) for s in shapes),
                       "l2": "weights (~380 MB) > L2: every step streams them from HBM",
                       "graph": "the step's launches replayed as one CUDA graph",
                       "parallelism": f"tokens over {world} rank(s), weights replicated, no collective"},
            "step_hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / hbm,
            "e2e": None if e2e_ms is None else {
                "value": n * world / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": xh.numel() * 4 * world, "d2h_bytes_per_step": lh.numel() * 4 * world,
                "path": "pinned input copied in, the step's eif_cuda_linear_forward_dev graph, logits copied out"},
            "roofline": {"kernel": f"{kname} (2-bit ternary, the 96 layer launches)", "bound": "hbm",
                         "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm, "peak_source": src,
                         "algorithmic_bytes_per_launch": tern_bytes / len(tern), "launch_ms": tern_ms / len(tern),
                         "traffic": None if tr is None else tr / len(tern), "traffic_source": tr_src},
            "lm_head": {"kernel": f"{kname} (INT8, 248320 x 1024)", "achieved": head_ach, "frac": head_ach / hbm,
                        "launch_ms": head_ms, "algorithmic_bytes": head_bytes, "traffic": htr,
                        "traffic_source": htr_src},
            "gpu_launches": len(shapes) * args.steps, "clocks": clk}
    if world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample = cpu_projection_reference(shapes, n)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample}
    return line


WORKLOADS = [  # (key, workload, overrides): BASELINE configs[0..3], config 1's heads batched per cache type, f4
    ("config1_decode", "decode", dict(batch=1, ctx=512, kv="f32")),
    ("config2_prefill", "prefill", {}),
    ("config3_recurrent", "recurrent", {}),
    ("config4_chunked", "chunked", {}),
    ("decode_batched_f32", "decode", dict(batch=256, ctx=4096, kv="f32")),
    ("decode_batched_bf16", "decode", dict(batch=256, ctx=4096, kv="bf16")),
    ("decode_batched_int8", "decode", dict(batch=256, ctx=4096, kv="int8")),
    # the Qwen3.5 attention mixer on the reference's own fp32 cache and on bf16 (config 5's heads)
    ("qwen35_attention_f32", "decode", dict(batch=64, ctx=32768, kv="f32", heads="qwen35")),
    ("qwen35_attention_bf16", "decode", dict(batch=64, ctx=32768, kv="bf16", heads="qwen35")),
    # row f4: every projection of a Qwen3.5-0.8B decode step, one token and sixteen
    ("projection_decode_b1", "projection", dict(batch=1)),
    ("projection_decode_b16", "projection", dict(batch=16)),
]
_KEEP = ("metric", "value", "unit", "ms_per_step", "dtype", "config", "roofline", "e2e", "cpu_baseline", "gpu_launches",
         "clocks", "step_path", "lm_head", "step_hbm_frac")


def run_workloads(args, torch, local_rank):
    """The other BASELINE configs on the same GPU after the headline, each through its own workload function
    (same timing rules: warm-up, events on the library's stream, L2 flush or inputs > L2), one compact entry
    each for the `workloads` object of the headline line."""
    import gc
    out = {}
    for key, wl, over in WORKLOADS:
        a = argparse.Namespace(**vars(args))
        a.workload, a.batch, a.ctx, a.kv = wl, over.get("batch"), over.get("ctx"), over.get("kv", "f32")
        a.heads = over.get("heads", "qwen2")
        fn = {"prefill": run_prefill, "chunked": run_chunked, "decode": run_decode, "recurrent": run_recurrent,
              "projection": run_projection}[wl]
        line = fn(a, torch, None, 0, 1, local_rank)
        out[key] = {k: line[k] for k in _KEEP if k in line}
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="hybrid",
                    choices=["hybrid", "prefill", "chunked", "decode", "recurrent", "projection"],
                    help="hybrid = BASELINE configs[4] (the headline); prefill = configs[1]; chunked = configs[3]; "
                         "recurrent = configs[2]; decode = configs[0]'s tinyllm heads, batched (--kv f32 | bf16 | "
                         "int8, --ctx); projection = the quantised projections of a Qwen3.5-0.8B decode step "
                         "(--batch tokens, default 1)")
    ap.add_argument("--kv", default="f32", choices=["f32", "bf16", "int8"], help="decode workload: cache dtype")
    ap.add_argument("--ctx", type=int, default=None, help="decode workload: context length (default 4096)")
    ap.add_argument("--heads", default="qwen2", choices=["qwen2", "qwen35"],
                    help="decode workload: 14 q / 2 kv heads at head_dim 64 (the tinyllm decode step), or the "
                         "Qwen3.5 attention mixer at 8 q / 2 kv, head_dim 256")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-pointer end-to-end leg (profiling runs)")
    ap.add_argument("--no-workloads", action="store_true",
                    help="hybrid at N=1: skip the other configs' entries (the `workloads` object)")
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch (default: the workload's config: 256 hybrid, 8 prefill, 4 chunked)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank)
        if line:
            print(json.dumps(line), flush=True)
        return

    import torch
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        dist = tdist
    if args.workload in ("prefill", "chunked", "decode", "recurrent", "projection"):
        run = {"prefill": run_prefill, "chunked": run_chunked, "decode": run_decode,
               "recurrent": run_recurrent, "projection": run_projection}[args.workload]
        line = run(args, torch, dist, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    line = run_ours(args, torch, dist, rank, world, local_rank)
    if line is not None and world == 1 and not args.no_cpu_baseline:
        tps, cores, kind, sample, _ = cpu_reference(3, per_round_cap_s=30)
        line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample}
    if line is not None and world == 1 and not args.no_workloads and args.batch is None:
        import gc
        gc.collect()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        line["workloads"] = run_workloads(args, torch, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
