"""Helpers shared by the tests (fixtures, fp32 references on sampled rows)."""

from __future__ import annotations

import math
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


def from_bits(arr: np.ndarray, is_bf16, device="cpu") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(arr).astype(np.int16))
    return t.view(torch.bfloat16 if int(is_bf16) else torch.float16).to(device)


def gen_qkv(B, H, S, D, dtype, seed, lowrank=0.0, sinks=0, device="cpu"):
    """Q,K,V ~ N(0,1)/sqrt(D); optional seeded rank-4 bias on K
    and K rows at `sinks` random positions scaled x4 (config 2)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    k = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    v = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    if lowrank:
        u = torch.randn(B, H, S, 4, generator=g)
        w = torch.randn(B, H, 4, D, generator=g) / math.sqrt(4 * D)
        k = k + lowrank * (u @ w)
    if sinks:
        for b in range(B):
            for h in range(H):
                pos = torch.randperm(S, generator=g)[:sinks]
                k[b, h, pos] *= 4.0
    return q.to(dtype).to(device), k.to(dtype).to(device), v.to(dtype).to(device)


def ref_rows(q, k, v, rows, visible_fn, scale):
    """fp32 attention for query `rows` of one head (torch, on q's device).

    visible_fn(rows) -> bool [len(rows), S_k] visible sets."""
    qf = q[rows].float()
    logits = (qf @ k.float().T) * scale
    vis = torch.as_tensor(visible_fn(rows), device=q.device)
    logits = logits.masked_fill(~vis, float("-inf"))
    p = torch.softmax(logits, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    return p @ v.float()


def assert_topk_equivalent(mine, ref, scores, rtol=1e-6, what=""):
    """Index sets equal, except for elements whose reference score ties with the
    k-th selected score (the reference's torch.topk order among ties is
    unspecified)."""
    mine = set(int(x) for x in mine)
    ref = set(int(x) for x in ref)
    if mine == ref:
        return
    diff = mine ^ ref
    kth = min(scores[i] for i in ref)
    for i in diff:
        s = scores[i]
        close = (s == kth) or (np.isfinite(s) and np.isfinite(kth) and abs(s - kth) <= rtol * max(abs(kth), 1e-30))
        assert close, f"{what}: index {i} (score {s}) differs from reference, k-th score {kth}"
