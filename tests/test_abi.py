"""The C ABI library without a GPU: it loads, exports every entry point include/eif_cuda.h declares,
and refuses cleanly (no CPU fallback) when no device is usable."""
import ctypes
import os
import subprocess
import sys

import pytest


def test_library_exports_header(pkg):
    L = pkg.lib()
    names = pkg.header_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_exports_are_only_the_abi(pkg):
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    ours = {n for n in exported if n.startswith("eif_cuda_")}
    assert ours == set(pkg.header_functions())


def test_no_cuda_env_refuses(pkg, tmp_path):
    code = ("import sys; sys.path.insert(0, %r); import __graft_entry__ as g; p = g.load_package();"
            "import ctypes; h = ctypes.c_void_p(); print(p.device_count(), p.lib().eif_cuda_init(ctypes.byref(h), 0))"
            % os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env = dict(os.environ, BITLLM_NO_CUDA="1")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["0", "-5"]  # no devices, EIF_STATUS_NOT_SUPPORTED


def test_null_arguments_rejected(pkg):
    L = pkg.lib()
    assert L.eif_cuda_init(None, 0) == -2
    assert L.eif_cuda_synchronize(None) == -2
    assert L.eif_cuda_kv_alloc(None, 1, 1, 1, 1, 64, 0, None) == -2
    assert L.eif_cuda_delta_alloc(None, 1, 1, 1, 64, 64, 0, None) == -2
    assert L.eif_cuda_attend_decode(None, None, 0, None, None, 1, 1.0, None, 0, None, None) == -2
    assert L.eif_cuda_deltanet_step(None, None, 0, None, None, None, None, None, 1.0, None) == -2
    assert L.eif_cuda_last_error(None) == b"no context"


@pytest.mark.skipif("__import__('torch').cuda.is_available()", reason="checks the no-GPU path")
def test_init_without_gpu_is_not_supported(pkg):
    h = ctypes.c_void_p()
    assert pkg.lib().eif_cuda_init(ctypes.byref(h), 0) == -5
    with pytest.raises(pkg.EifCudaError) as e:
        pkg.Context(0)
    assert e.value.name == "NOT_SUPPORTED"
