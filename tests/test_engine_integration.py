"""The engines themselves on the GPU (row f1): bitllm.c's Qwen3.5 and tinyllm engines, patched at their token-mixer
call sites by bitllm.c_b200/engine/bitllm_cuda.patch, run synthetic models once on the host (as the reference
does) and once attached to the GPU, through their public APIs (qwen35_prefill / qwen35_forward / qwen35_reset,
tinyllm_forward_batch_embeddings / tinyllm_forward_embedding); the logits are compared (tests/c_engine/
engine_forward.c).  The patch only inserts lines, each under #ifdef BITLLM_CUDA, so the engine source stays the
reference's; unattached, the patched engines give the host logits exactly.

Logit tolerances (rel-L2 over the vocabulary), with what one B200 measured:
* fp32 paths (fp32 KV cache; Qwen3.5 prefill with deltanet_core per token): Qwen3.5 1e-4 (measured <= 1.1e-5
  over 24 layers; the same bound with the projections -- linear_gemv / linear_gemm / int8_gemv -- on the GPU too,
  `-proj`), tinyllm 1e-5 (measured <= 5e-7, fp32 and INT8 caches);
* bf16 paths (the chunked DeltaNet prefill's bf16 q / k / v, or a bf16 KV cache): 6e-2 (measured <= 4.5e-2 for
  Qwen3.5, whose 18 DeltaNet layers each carry a ~2e-3 input rounding into the residual stream; 1e-3 for
  tinyllm's bf16 cache).  The per-mixer prefill tolerance (rel-L2 <= 1e-2) is checked in the kernel tests."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE = os.path.join(ROOT, "bitllm.c_b200", "engine")
BIN = os.path.join(ROOT, "_build", "engine", "engine_forward")
PATCH = os.path.join(ENGINE, "bitllm_cuda.patch")
REF = os.environ.get("BITLLM_REF_DIR", "/root/reference")

CASES = [("qwen35", "f32", "tokenwise", 1e-4), ("qwen35", "f32", "chunked", 6e-2), ("qwen35", "bf16", "chunked", 6e-2),
         ("tinyllm", "f32", None, 1e-5), ("tinyllm", "int8", None, 1e-5), ("tinyllm", "bf16", None, 6e-2),
         # the Qwen3.5 projections (INT4 linears, the INT8 tied head) on the GPU as well (row f4)
         ("qwen35", "f32", "tokenwise-proj", 1e-4), ("qwen35", "f32", "chunked-proj", 6e-2)]


def _binary(build=True):
    """The test program built by build() (bitllm.c_b200/engine/Makefile).  The CPU tests build it here when the
    bitllm.c source tree is present; the GPU tests only run what was built (the tree is not on a GPU box)."""
    if build and not os.path.exists(BIN) and os.path.isdir(os.path.join(REF, "src")):
        subprocess.run(["make", "-s", "-C", ENGINE, f"REF={REF}"], check=True)
    if not os.path.exists(BIN):
        pytest.skip("engine_forward not built (needs the bitllm.c source tree: BITLLM_REF_DIR)")
    return BIN


def _run(args, host_only, tmp_path):
    env = dict(os.environ, OMP_NUM_THREADS="1")
    if host_only:
        env["ENGINE_FORWARD_HOST_ONLY"] = "1"
    r = subprocess.run([_binary(build=host_only)] + [str(a) for a in args], cwd=tmp_path, env=env,
                       capture_output=True, text=True, timeout=600)
    print(r.stdout + r.stderr)
    return r


def test_patch_only_inserts_guarded_lines():
    """Every hunk of the engine patch adds lines and removes none, and every added block is guarded."""
    lines = open(PATCH).read().splitlines()
    added = [ln[1:] for ln in lines if ln.startswith("+") and not ln.startswith("+++")]
    assert added and not any(ln.startswith("-") and not ln.startswith("---") for ln in lines)
    depth = 0
    for ln in added:
        if ln.startswith("#if"):
            assert "BITLLM_CUDA" in ln, ln
            depth += 1
        elif ln.startswith("#endif"):
            depth -= 1
        else:
            assert depth == 1, ln  # code lines only inside a BITLLM_CUDA block
    assert depth == 0


@pytest.mark.parametrize("case", CASES[:1] + CASES[3:5], ids=lambda c: "-".join(str(x) for x in c[:3] if x))
def test_unattached_engines_match_host(case, tmp_path):
    """The patched engines with no GPU attached are the reference engines: bit-identical logits (CPU only)."""
    eng, kv, mode, _ = case
    args = [eng, kv] + ([mode] if mode else []) + [0]
    assert _run(args, True, tmp_path).returncode == 0


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(str(x) for x in c[:3] if x))
def test_engine_on_gpu_matches_host(case, tmp_path):
    eng, kv, mode, tol = case
    args = [eng, kv] + ([mode] if mode else []) + [tol]
    r = _run(args, False, tmp_path)
    assert r.returncode == 0, r.stdout + r.stderr
