"""BASELINE config 5 in its own regime: the 24-layer Qwen3.5-like token-mixer stack at decode batch 256 and
context 32768 over a bf16 KV cache -- the workload bench.py times for its headline number -- with sampled
sequences replayed on the reference's own C code (oracle/_ref, compiled from the reference's sources; the C
restatement, pinned to it, where that build is absent).

* At this shape the decode-attention split is one unsplit item per (sequence, kv head) (read back through
  eif_cuda_attend_decode_plan): the regime of the benchmark's attention launches.
* Two decode steps through all 24 mixers in the engine's order, (DeltaNet x 3, attention) x 6: step 1 at row
  32766 through fullatt_prep_dev + attend_decode_dev (the benchmark's calls), step 2 at row 32767 through the
  one-call fullatt_decode_dev.  For two sampled sequences every layer's output, and after both steps every
  S, conv window and written KV row, is compared with the reference run from the same state: deltanet_core
  (src/eif_qwen35.c:546-656), fullatt_prep (:699-737) and fullatt_attend (:741-790) on an fp32 cache holding
  the same bf16 rows, each new row rounded to bf16 as the device cache stores it.
  Tolerance: rel-L2 <= 1e-5 (the fp32 decode / recurrent bound); the new cache rows within one bf16 ulp per
  element (the device rounds its own fp32 row, so a value on a rounding boundary may go either way).
"""
import math

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5
LAYERS = ["D", "D", "D", "A"] * 6
H, DK, CK = 16, 128, 4
CONV = 3 * H * DK
HQ, HKV, HD = 8, 2, 256
CTX, B = 32768, 256
SAMPLE = (0, 201)
N_ATT, N_DN = LAYERS.count("A"), LAYERS.count("D")


class _DevArray:
    """A raw device allocation seen by torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (n,), "typestr": typestr, "version": 3,
                                         "strides": None}


@pytest.fixture(scope="module")
def stack(pkg, ctx):
    import torch
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    need = N_ATT * 2 * B * CTX * HKV * HD * 2 + N_DN * B * (H * DK * DK + CONV * CK) * 4
    free = torch.cuda.mem_get_info()[0]
    assert free > need + (4 << 30), f"config 5 needs {need / 1e9:.1f} GB of device memory, {free / 1e9:.1f} GB free"
    rng = np.random.default_rng(55)
    w_dn = [dict(conv_w=(0.5 * rng.standard_normal((CONV, CK))).astype(np.float32),
                 dt_bias=rng.standard_normal(H).astype(np.float32),
                 A_log=(0.5 * rng.standard_normal(H)).astype(np.float32),
                 norm_w=(1 + 0.1 * rng.standard_normal(DK)).astype(np.float32)) for _ in range(N_DN)]
    w_at = [dict(q_norm=(1 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
                 k_norm=(1 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
                 sub_norm=(1 + 0.1 * rng.standard_normal(HQ * HD)).astype(np.float32)) for _ in range(N_ATT)]
    kv = pkg.KVCache(ctx, N_ATT, B, CTX, HKV, HD, pkg.BF16)
    dn = pkg.DeltaState(ctx, N_DN, B, H, DK, DK, CK)
    for l, w in enumerate(w_dn):
        dn.set_weights(l, **w)
    for l, w in enumerate(w_at):
        kv.set_norms(l, w["q_norm"], w["k_norm"])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    # the cache ~ N(0, 1) in bf16, S ~ N(0, 0.02), conv windows ~ N(0, 1), written through the library's pointers
    for l in range(N_ATT):
        for p in kv.layer_ptrs(l):
            torch.as_tensor(_DevArray(p, B * CTX * HKV * HD, "<i2"), device="cuda").view(torch.bfloat16).normal_(
                generator=gen)
    for l in range(N_DN):
        s, c = dn.layer_ptrs(l)
        torch.as_tensor(_DevArray(s, B * H * DK * DK, "<f4"), device="cuda").normal_(0, 0.02, generator=gen)
        torch.as_tensor(_DevArray(c, B * CONV * CK, "<f4"), device="cuda").normal_(generator=gen)
    torch.cuda.synchronize()
    yield dict(kv=kv, dn=dn, w_dn=w_dn, w_at=w_at)
    kv.free()
    dn.free()
    torch.cuda.empty_cache()


def test_config5_attention_split_is_unsplit(stack):
    """Every attention layer of the stack decodes with one 32768-key item per (sequence, kv head)."""
    for l in range(N_ATT):
        for max_pos in (CTX - 2, CTX - 1):
            n_chunks, chunk_keys, _ = stack["kv"].decode_plan(l, HQ, max_pos)
            assert n_chunks == 1 and chunk_keys >= max_pos + 1, (l, n_chunks, chunk_keys)


def test_config5_two_steps_sampled_vs_reference(pkg, ctx, orc, stack):
    import torch
    kv, dn, w_dn, w_at = stack["kv"], stack["dn"], stack["w_dn"], stack["w_at"]
    lib = orc.ref() if orc.ref_available() else None
    rng = np.random.default_rng(56)

    def nrm(*shape):
        return rng.standard_normal(shape, dtype=np.float32)

    steps = [dict(pos=CTX - 2, dn=[dict(qkv=nrm(B, CONV), z=nrm(B, H * DK), b=nrm(B, H), a=nrm(B, H))
                                  for _ in range(N_DN)],
                  at=[dict(qg=nrm(B, HQ * 2 * HD), k=nrm(B, HKV * HD), v=nrm(B, HKV * HD)) for _ in range(N_ATT)])
             for _ in range(2)]
    steps[1]["pos"] = CTX - 1

    # the sampled sequences' state before the steps, as the reference's engine would hold it
    host = {b: dict(S=[], conv=[], kc=[], vc=[]) for b in SAMPLE}
    for b in SAMPLE:
        for l in range(N_DN):
            S, c = dn.download(l, b)
            host[b]["S"].append(S)
            host[b]["conv"].append(c)
        for l in range(N_ATT):
            kc, vc = kv.download(l, b, 0, CTX)
            host[b]["kc"].append(kc)
            host[b]["vc"].append(vc)

    # the device: two steps over the whole batch, every layer's output kept
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    sub_norm = [dev(w["sub_norm"]) for w in w_at]
    q_buf = torch.empty(B, HQ * HD, device="cuda")
    g_buf = torch.empty(B, HQ * HD, device="cuda")
    scale = 1.0 / math.sqrt(HD)
    gpu_out = []
    for si, st in enumerate(steps):
        pos = torch.full((B,), st["pos"], dtype=torch.int32, device="cuda")
        outs = []
        d = a = 0
        for typ in LAYERS:
            if typ == "D":
                x = {k: dev(v) for k, v in st["dn"][d].items()}
                o = torch.empty(B, H * DK, device="cuda")
                torch.cuda.synchronize()
                dn.core_dev(d, x["qkv"].data_ptr(), x["z"].data_ptr(), x["b"].data_ptr(), x["a"].data_ptr(),
                            o.data_ptr())
                d += 1
            else:
                x = {k: dev(v) for k, v in st["at"][a].items()}
                o = torch.empty(B, HQ * HD, device="cuda")
                torch.cuda.synchronize()
                if si == 0:
                    kv.fullatt_prep_dev(a, x["qg"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(), pos.data_ptr(),
                                        HQ, q_buf.data_ptr(), g_buf.data_ptr())
                    kv.attend_decode_dev(a, q_buf.data_ptr(), pos.data_ptr(), st["pos"], HQ, scale, o.data_ptr(),
                                         gate_dev=g_buf.data_ptr(), subln=pkg.SUBLN_WEIGHT,
                                         sub_norm_dev=sub_norm[a].data_ptr())
                else:
                    kv.fullatt_decode_dev(a, x["qg"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(),
                                          pos.data_ptr(), st["pos"], HQ, scale, o.data_ptr(), subln=pkg.SUBLN_WEIGHT,
                                          sub_norm_dev=sub_norm[a].data_ptr())
                a += 1
            ctx.synchronize()
            outs.append(o.cpu().numpy())
        gpu_out.append(outs)

    # the reference, sequence by sequence, from the same state
    for b in SAMPLE:
        hs = host[b]
        for si, st in enumerate(steps):
            p = st["pos"]
            d = a = 0
            for li, typ in enumerate(LAYERS):
                if typ == "D":
                    x = st["dn"][d]
                    ref = orc.deltanet_core(x["qkv"][b], x["z"][b], x["b"][b], x["a"][b], hs["conv"][d], hs["S"][d],
                                            lib=lib, **w_dn[d])
                    d += 1
                else:
                    x, w = st["at"][a], w_at[a]
                    kc, vc = hs["kc"][a], hs["vc"][a]
                    q, g, _ = orc.fullatt_prep(x["qg"][b], x["k"][b], x["v"][b], w["q_norm"], w["k_norm"], kc, vc,
                                               p, HQ, HKV, HD, lib=lib)
                    kc[p] = orc.round_bf16(kc[p])
                    vc[p] = orc.round_bf16(vc[p])
                    if lib is not None:
                        ref = orc.ref_fullatt_attend(q, g, kc, vc, w["sub_norm"], 0, p, HQ, HKV, HD)
                    else:
                        ref = orc.subln(orc.attend_decode(q, kc, vc, p, HQ, HKV, HD, scale, gate=g), w["sub_norm"], 2)
                    a += 1
                err = rel_l2(gpu_out[si][li][b], ref)
                assert err <= TOL, (b, si, li, typ, err)
        # state after both steps
        for l in range(N_DN):
            S, c = dn.download(l, b)
            assert rel_l2(S, hs["S"][l]) <= TOL, (b, "S", l)
            assert rel_l2(c, hs["conv"][l]) <= TOL, (b, "conv", l)
        for l in range(N_ATT):
            kr, vr = kv.download(l, b, CTX - 2, 2)
            for got, want in ((kr, hs["kc"][l][CTX - 2:]), (vr, hs["vc"][l][CTX - 2:])):
                assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 1e-30), (b, "kv row", l)
