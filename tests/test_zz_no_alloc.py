"""The allocation-free block selector, checked against the regular one.

mi_block_pool_topk_noalloc is for callers that cannot allocate device memory
at call time -- e.g. code being recorded into a CUDA graph, or an engine
that has handed the whole device heap to its own pool -- so it keeps its
scratch in a fixed 32 MiB array inside the library instead of taking a
workspace.  This test calls it through the C ABI twice in a row (the second
call runs on scratch the first one left behind) and requires the same block
indices as mi_block_pool_topk with a freshly allocated workspace, and that
sizes beyond the built-in scratch are refused with MI_ERR_SCRATCH_LIMIT.

The file name sorts last so that a `-x` run reaches it only after every
other test has run.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, H, S, D, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    k = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    u = torch.randn(B, H, S, 4, generator=g)
    w = torch.randn(B, H, 4, D, generator=g) / math.sqrt(4 * D)
    k = k + 2.0 * (u @ w)
    return q.to(dtype).to(device), k.to(dtype).to(device)


def _bind(lib, name, argtypes):
    fn = getattr(lib, name)
    fn.argtypes = argtypes
    fn.restype = ctypes.c_int
    return fn


@pytest.fixture(scope="module")
def capi(cuda):
    from minference import _native

    lib = _native.lib()
    T4, I64, I, F, P = (_native.mi_tensor4, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                        ctypes.c_void_p)
    noalloc = _bind(lib, "mi_block_pool_topk_noalloc",
                    [T4, T4, I64, I64, I64, I64, I64, I, I64, I, F, P, P])
    lib.mi_block_pool_topk_noalloc_limit.restype = ctypes.c_size_t
    return _native, lib, noalloc


@pytest.mark.parametrize("case", [(1, 8, 4096, 96, torch.bfloat16, 100, 0),
                                  (2, 4, 3000, 64, torch.float16, 7, 1)])
def test_noalloc_matches_workspace_version_twice(capi, cuda, case):
    _native, lib, noalloc = capi
    B, H, S, D, dt, topk, force = case
    nb = -(-S // 64)
    kk = min(topk, nb)
    scale = (64 if D <= 64 else 128) ** -0.5
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call in range(2):
        q, k = _inputs(B, H, S, D, dt, 17 + call, cuda)
        ref = torch.empty(B, H, nb, kk, dtype=torch.int64, device=cuda)
        ws = _native.workspace(lib.mi_block_pool_topk_workspace_size(B, H, S, S, D), cuda)
        rc = lib.mi_block_pool_topk(_native.t4(q), _native.t4(k), B, H, S, S, D,
                                    _native.dtype_code(q), topk, force, scale, ref.data_ptr(),
                                    ws.data_ptr(), ws.numel(), stream)
        assert rc == 0
        got = torch.full_like(ref, -1)
        rc = noalloc(_native.t4(q), _native.t4(k), B, H, S, S, D, _native.dtype_code(q), topk,
                     force, scale, got.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {call}: no-alloc selection differs"


def test_noalloc_rejects_sizes_beyond_scratch(capi, cuda):
    _native, lib, noalloc = capi
    limit = lib.mi_block_pool_topk_noalloc_limit()
    B, H, D = 1, 64, 128
    S = 65536  # pooled q (32 MiB) + pooled k^T (32 MiB) = 64 MiB > 32 MiB
    assert lib.mi_block_pool_topk_workspace_size(B, H, S, S, D) > limit
    t = _native.mi_tensor4(0, 0, 0, 0, 1)
    rc = noalloc(t, t, B, H, S, S, D, 1, 10, 0, 0.1, None, None)
    assert rc == 7  # MI_ERR_SCRATCH_LIMIT, before any device work


def test_noalloc_reports_bad_shapes_as_shape_errors(capi, cuda):
    """Negative or overflowing sizes are argument errors (MI_ERR_SHAPE), not
    scratch-limit refusals."""
    _native, lib, noalloc = capi
    t = _native.mi_tensor4(0, 0, 0, 0, 1)
    assert noalloc(t, t, 1, -4, 1024, 1024, 96, 1, 10, 0, 0.1, None, None) == 1
    assert noalloc(t, t, -1, 4, 1024, 1024, 96, 1, 10, 0, 0.1, None, None) == 1
    assert noalloc(t, t, 1 << 40, 1 << 20, 1 << 30, 1 << 30, 96, 1, 10, 0, 0.1, None, None) == 1
    assert lib.mi_block_pool_topk_workspace_size(1, -4, 1024, 1024, 96) == 2 ** 64 - 1
