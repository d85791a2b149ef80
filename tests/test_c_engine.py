"""A C99 program makes the engine's calls through include/eif_cuda.h (tests/c_engine/engine_calls.c): the
tinyllm decode step over fp32 and INT8 caches and the DeltaNet delta rule, each checked against plain C
loops restating the reference arithmetic.  The CPU test compiles it with -std=c99 -Werror against the header
and links it with libeif_cuda.so (no GPU: the program reports no device and exits 0); the GPU test runs it."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_engine", "engine_calls.c")
LIBDIR = os.path.join(ROOT, "bitllm.c_b200")


def build(pkg, tmp_path):
    if not shutil.which("gcc"):
        pytest.skip("gcc not found")
    exe = str(tmp_path / "engine_calls")
    subprocess.run(["gcc", "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    SRC, "-o", exe, "-L", LIBDIR, "-leif_cuda", "-Wl,-rpath," + LIBDIR, "-lm"], check=True)
    return exe


def test_c99_engine_builds_and_links(pkg, tmp_path):
    exe = build(pkg, tmp_path)
    env = dict(os.environ, BITLLM_NO_CUDA="1")
    r = subprocess.run([exe], capture_output=True, text=True, env=env, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "no CUDA device" in r.stdout


@pytest.mark.gpu
def test_c99_engine_runs(pkg, tmp_path):
    exe = build(pkg, tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("OK")
