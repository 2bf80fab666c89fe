"""minference.host_pipeline: layer attention from pinned host q/k/v, with the
copies pipelined against the attention, equals the ops on device-resident
inputs (bit for bit: same kernels, same inputs)."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_layer_attention_from_host_matches_device(cuda):
    from minference.host_pipeline import layer_attention_from_host
    from minference.modules.minference_forward import _run_pattern, group_heads

    torch.manual_seed(11)
    B, H, S, D = 1, 7, 1536, 96
    q, k, v = [(torch.randn(B, H, S, D) / math.sqrt(D)).bfloat16() for _ in range(3)]
    pattern = {0: ("vertical_and_slash", 100, 200, 1), 1: ("block_sparse", 3, 0, 1),
               2: ("vertical_and_slash", 100, 200, 1), 3: ("block_sparse", 3, 0, 1),
               4: ("stream_llm", 64, 128, 1), 5: ("vertical_and_slash", 100, 200, 1),
               6: ("dense", 0, 0, 1)}
    groups = group_heads(pattern, H)
    pin = [t.pin_memory() for t in (q, k, v)]
    out = torch.empty(B, H, S, D, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):  # second call reuses the cached device buffers
        out.zero_()
        layer_attention_from_host(*pin, out, groups, cuda, chunk_heads=2)
        torch.cuda.synchronize()
        qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
        for key, heads in groups:
            idx = torch.tensor(heads, device=cuda)
            ref = _run_pattern(key, qd.index_select(1, idx), kd.index_select(1, idx),
                               vd.index_select(1, idx)).cpu()
            assert torch.equal(out[:, heads], ref), key


def test_layer_attention_from_host_rejects_pageable(cuda):
    from minference.host_pipeline import layer_attention_from_host

    x = torch.zeros(1, 2, 128, 96, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        layer_attention_from_host(x, x, x, x, [(("dense",), [0, 1])], cuda)
