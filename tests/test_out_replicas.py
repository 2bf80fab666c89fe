"""Output replicas: every output tile is also stored, by the kernel that
computes it, into each replica view (same strides, another buffer).  Across
GPUs the replicas are the peers' buffers opened through CUDA IPC, which is
how a head-sharded layer's output reaches every GPU without an all-gather;
here, on one GPU, they are other local buffers, and must equal the output
bit for bit."""

from __future__ import annotations

import pytest
import torch

from _util import gen_qkv

pytestmark = pytest.mark.gpu


def _bufs(like, n):
    return [torch.full_like(like, 3.0) for _ in range(n)]


@pytest.mark.parametrize("heads", [None, [3, 1]])
def test_replicas_all_ops(cuda, heads):
    from minference import ops

    H, S = 4, 1000
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, 7, lowrank=2.0, sinks=8, device=cuda)
    cases = [
        lambda o, r: ops.streaming_forward(q, k, v, 64, 256, out=o, heads=heads, out_replicas=r),
        lambda o, r: ops.dense_attention(q, k, v, out=o, heads=heads, out_replicas=r),
        lambda o, r: ops.block_sparse_attention(q, k, v, 5, out=o, heads=heads, out_replicas=r),
        lambda o, r: ops.vertical_and_slash(q, k, v, 100, 200, out=o, heads=heads,
                                            out_replicas=r),
    ]
    for fn in cases:
        out = torch.full_like(q, 3.0)
        reps = _bufs(q, 3)
        fn(out, [r.data_ptr() for r in reps])
        torch.cuda.synchronize()
        for r in reps:
            assert torch.equal(r, out)
        plain = fn(torch.full_like(q, 3.0), None)
        assert torch.equal(plain, out)


def test_replicas_of_a_view(cuda):
    """A replica address is the address of the output view's element 0 in the
    other buffer (here: the second half of a wider buffer)."""
    from minference import ops

    q, k, v = gen_qkv(1, 2, 512, 96, torch.bfloat16, 2, device=cuda)
    big = torch.zeros(2, 1, 2, 512, 96, dtype=torch.bfloat16, device=cuda)
    out = ops.dense_attention(q, k, v, out=big[0], out_replicas=[big[1].data_ptr()])
    torch.cuda.synchronize()
    assert torch.equal(big[0], big[1]) and torch.equal(out, big[0])
    with pytest.raises(ValueError):
        ops.dense_attention(q, k, v, out=big[0], out_replicas=[big[1].data_ptr()] * 8)
