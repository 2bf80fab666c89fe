"""NCCL path of minference.sharding.gather_o_proj on one GPU (world size 1).

The overlapped path (all-gather of sequence chunks on a side stream, o_proj
GEMM of each chunk on the current stream once it has arrived) must equal
o_proj of the head-ordered output.  Multi-rank numerics of the same function
are covered with gloo ranks in test_sharding_gloo.py.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_gather_o_proj_nccl_single_rank(cuda):
    import torch.distributed as dist

    from minference.sharding import gather_o_proj, o_proj_input_permutation

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=cuda)
    try:
        torch.manual_seed(5)
        B, S, H, D, hidden = 1, 1000, 6, 96, 256
        head_map = [[3, 0, 5, 1, 4, 2]]  # one rank, permuted head order
        heads = torch.randn(B, S, H, D, device=cuda, dtype=torch.bfloat16)
        W = torch.randn(hidden, H * D, device=cuda, dtype=torch.bfloat16) / 24
        local = heads[:, :, head_map[0]]
        wp = W[:, o_proj_input_permutation(head_map, D).to(cuda)]
        got = gather_o_proj(local, wp, chunks=4)
        want = torch.nn.functional.linear(heads.reshape(B, S, H * D), W)
        torch.cuda.synchronize()
        assert got.shape == (B, S, hidden)
        assert (got.float() - want.float()).abs().max().item() < 0.05
    finally:
        dist.destroy_process_group()
