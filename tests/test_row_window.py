"""Query-row windows (``rows=``): a window of whole 128-row tiles computes
exactly the rows the full call computes there, bit for bit, and leaves the
other rows of the output untouched.  This is what lets one head's query tiles
be split over several GPUs."""

from __future__ import annotations

import pytest
import torch

from _util import gen_qkv

pytestmark = pytest.mark.gpu

WINDOWS = [(0, 256), (384, 1024), (1536, 2000), (0, 2000), (640, 640)]


def _check(full, fn, S):
    for r0, r1 in WINDOWS:
        sentinel = torch.full_like(full, 7.0)
        got = fn(sentinel, (r0, r1))
        assert torch.equal(got[:, :, r0:r1], full[:, :, r0:r1]), (r0, r1)
        assert (got[:, :, :r0] == 7.0).all() and (got[:, :, r1:] == 7.0).all(), (r0, r1)


def test_rows_block_sparse(cuda):
    from minference import ops

    S = 2000
    q, k, v = gen_qkv(1, 3, S, 96, torch.bfloat16, 1, lowrank=2.0, device=cuda)
    idx = ops.select_block_sparse_topk_indices(q, k, 5)
    full = ops.block_sparse_attention_from_indices(q, k, v, idx)
    _check(full, lambda o, rw: ops.block_sparse_attention_from_indices(q, k, v, idx, out=o,
                                                                      rows=rw), S)


def test_rows_vertical_slash(cuda):
    from minference import ops

    S = 2000
    q, k, v = gen_qkv(1, 3, S, 96, torch.bfloat16, 2, sinks=8, device=cuda)
    vi, si = ops.vertical_and_slash_estimate(q, k, 100, 200)
    full = ops.vertical_slash_sparse_attention(q, k, v, vi, si)
    _check(full, lambda o, rw: ops.vertical_slash_sparse_attention(q, k, v, vi, si, out=o,
                                                                   rows=rw), S)


def test_rows_stream_and_dense(cuda):
    from minference import ops

    S = 2000
    q, k, v = gen_qkv(1, 2, S, 96, torch.float16, 3, device=cuda)
    full = ops.streaming_forward(q, k, v, 64, 256)
    _check(full, lambda o, rw: ops.streaming_forward(q, k, v, 64, 256, out=o, rows=rw), S)
    full = ops.dense_attention(q, k, v)
    _check(full, lambda o, rw: ops.dense_attention(q, k, v, out=o, rows=rw), S)


def test_rows_rejects_unaligned(cuda):
    from minference import ops

    q, k, v = gen_qkv(1, 1, 512, 96, torch.bfloat16, 4, device=cuda)
    with pytest.raises(ValueError):
        ops.dense_attention(q, k, v, rows=(100, 256))
    with pytest.raises(ValueError):
        ops.streaming_forward(q, k, v, 16, 64, rows=(0, 300))
