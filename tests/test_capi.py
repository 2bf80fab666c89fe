"""CPU: the C-ABI library builds, loads and exports every declared entry point.

No compute calls are made here (no GPU in this container); argument
validation paths that return before touching the device are exercised.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def declared_symbols() -> list[str]:
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(HEADER_DIR, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(mi_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from minference import _native, build

    build.build()
    return _native.lib()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("mi_stream_fwd", "mi_block_pool_topk", "mi_block_sparse_fwd", "mi_vs_estimate",
              "mi_vs_sparse_fwd", "mi_version", "mi_get_device_error"):
        assert s in syms


def test_every_declared_symbol_is_exported(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in include/ but not exported"


def test_version(lib):
    from minference import _native

    assert "sm_100a" in _native.version()


def test_workspace_sizes_monotone(lib):
    a = lib.mi_vs_sparse_fwd_workspace_size(1, 32, 16384)
    b = lib.mi_vs_sparse_fwd_workspace_size(1, 32, 32768)
    assert 0 < a < b
    assert lib.mi_block_sparse_fwd_workspace_size(1, 32, 16384, 100) > 0
    assert lib.mi_vs_estimate_workspace_size(1, 1, 4096) >= 64 * 4096 * 2
    assert lib.mi_block_pool_topk_workspace_size(1, 2, 1024, 1024, 96) == 2 * 2 * 16 * 96 * 4


def test_argument_validation_without_device(lib):
    """Bad dtypes / shapes are rejected before any CUDA call."""
    from minference import _native

    t = _native.mi_tensor4(0, 0, 0, 0, 1)
    assert lib.mi_stream_fwd(t, t, t, t, 1, 1, 16, 16, 96, 7, 0, 8, 1.0, None) == 2
    assert lib.mi_stream_fwd(t, t, t, t, 1, 1, 16, 16, 80, 1, 0, 8, 1.0, None) == 1
    assert lib.mi_stream_fwd(t, t, t, t, 1, 1, 32, 16, 96, 1, 0, 8, 1.0, None) == 1
    # empty problems are a no-op
    assert lib.mi_stream_fwd(t, t, t, t, 0, 1, 16, 16, 96, 1, 0, 8, 1.0, None) == 0
    assert lib.mi_block_sparse_fwd(t, t, t, t, 1, 1, 128, 96, 1, None, 0, 1.0, None, 0, None) == 1
    assert lib.mi_vs_estimate(t, t, 1, 1, 128, 96, 1, 200, 50, 0.1, None, None, None, 0, None) == 1
    assert lib.mi_vs_sparse_fwd(t, t, t, t, 1, 1, 128, 96, 1, None, 1, None, 1, 1.0, None, 0,
                                None) == 3
    # dense: causal rows need keys; more than MI_MAX_REPLICAS output replicas
    # or mismatched head tables are refused before any launch
    assert lib.mi_dense_fwd(t, t, t, t, 1, 1, 32, 16, 96, 1, 1, 1.0, None) == 1
    assert lib.mi_dense_fwd(t, t, t, t, 1, 1, 16, 16, 96, 5, 1, 1.0, None) == 2
    import ctypes

    arr = (ctypes.c_void_p * 8)(*([16] * 8))
    o = _native.mi_tensor4(0, 0, 0, 0, 1, None, 0, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)), 8)
    assert lib.mi_dense_fwd(t, t, t, o, 1, 1, 16, 16, 96, 1, 1, 1.0, None) == 1
    hq = _native.mi_tensor4(0, 0, 0, 0, 1, 64, 4, None, 0)
    assert lib.mi_dense_fwd(hq, t, t, t, 1, 1, 16, 16, 96, 1, 1, 1.0, None) == 1
    assert lib.mi_block_sparse_fwd_rows(t, t, t, t, 1, 1, 1000, 96, 1, None, 4, 1.0, 100, 500,
                                        None, 0, None) == 1  # row window not tile aligned


def test_ops_refuse_cpu_tensors():
    import torch

    from minference import ops

    q = torch.zeros(1, 1, 64, 96, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.streaming_forward(q, q, q, 4, 16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.block_sparse_attention(q, q, q, 2)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.vertical_and_slash(q, q, q, 30, 50)
