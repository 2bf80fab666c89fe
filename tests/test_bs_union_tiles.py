"""block_sparse union tiles (MI_BS_SPLIT=0, kept for comparison with the
default split tiles) still compute the same attention.

The switch is read once per process, so the union path runs in a child
process; its output is compared with the default (split) path here, within
the fp16/bf16 tolerance the parity tests use (the two kernels rescale at
different points of the online softmax)."""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import math, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from minference import ops
g = torch.Generator().manual_seed(21)
q, k, v = [(torch.randn(1, 3, 2048, 96, generator=g) / math.sqrt(96)).bfloat16().cuda() for _ in range(3)]
out = ops.block_sparse_attention(q, k, v, 6)
np.save(sys.argv[2], out.float().cpu().numpy())
"""


def test_union_tiles_match_split_tiles(cuda, tmp_path):
    import math

    from minference import ops

    dst = str(tmp_path / "union.npy")
    env = dict(os.environ, MI_BS_SPLIT="0")
    subprocess.run([sys.executable, "-c", CHILD, os.path.join(ROOT, "minference-npu_b200"), dst],
                   env=env, check=True, timeout=300)
    g = torch.Generator().manual_seed(21)
    q, k, v = [(torch.randn(1, 3, 2048, 96, generator=g) / math.sqrt(96)).bfloat16().to(cuda)
               for _ in range(3)]
    split = ops.block_sparse_attention(q, k, v, 6).float().cpu().numpy()
    union = np.load(dst)
    assert np.abs(split - union).max() < 2e-3
