"""B200-native token-mixing hot path of bitllm.c: GQA attention over the KV cache and the Gated
DeltaNet state update, with the quantised projections either side of them, behind the C ABI of
include/eif_cuda.h (libeif_cuda.so, built in-tree by build.py).  This package is the Python host mirror of that ABI; a C99 engine calls it directly.

The directory name contains a dot, so load it by path (``__graft_entry__.load_package()`` does):

    spec = importlib.util.spec_from_file_location(
        "bitllm_c_b200", "bitllm.c_b200/__init__.py", submodule_search_locations=["bitllm.c_b200"])
"""
from .eif_cuda import (BF16, F32, INT8, SUBLN_NONE, SUBLN_RMS, SUBLN_WEIGHT, STATUS, Context, DeltaState,  # noqa: F401
                       EifCudaError, KVCache, Linear, W_F32, W_INT4, W_INT8, W_TERNARY2, W_TERNARY_DENSE,
                       device_count, header_functions, lib, LIB_PATH, packed_row_bytes)
from .build import build  # noqa: F401
from . import shard  # noqa: F401
