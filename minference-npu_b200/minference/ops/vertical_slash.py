"""vertical_and_slash pattern: top-k key columns plus top-k diagonals.

Drop-ins for the estimator ``_vertical_and_slash_kernel`` (MInference-NPU
minference/modules/minference_forward.py:140-167) and the attention
``vertical_slash_sparse_attention`` (minference/ops/vertical_slash_kernel_npu.py:518).
The attention follows the reference's direct mask (:255-369) at every
sequence length; the reference's own entry point switches to dense causal
attention above 16384 tokens (:582-592), which is not reproduced here.
"""

from __future__ import annotations

import math

import torch

from .. import _native
from ._common import (check_qkv, default_softmax_scale, head_table, kernel_dim, prepare,
                      replica_ptrs, row_window)
from ._common import output as _common_out

__all__ = [
    "vertical_slash_sparse_attention",
    "vertical_and_slash_estimate",
    "vertical_and_slash",
    "convert_vertical_slash_indexes",
]

LAST_Q = 64


def vertical_and_slash_estimate(q: torch.Tensor, k: torch.Tensor, vertical_size: int,
                                slash_size: int, heads=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(v_idx int32 [B,H,nv] ascending, s_idx int32 [B,H,ns] descending) from the
    last 64 queries; ``heads`` selects heads of q/k (one launch per kernel)."""
    _native.require_cuda(q, k)
    B, _, S, D = q.shape
    tbl, H = head_table(heads, q)
    nv = min(S, max(int(vertical_size), 30))
    ns = min(S, max(int(slash_size), 50))
    dk = kernel_dim(D)
    logit_scale = 1.0 / math.sqrt(D)  # the estimator uses the unpadded head dim
    qp, kp = prepare(q, dk), prepare(k, dk)
    v_idx = torch.empty((B, H, nv), dtype=torch.int32, device=q.device)
    s_idx = torch.empty((B, H, ns), dtype=torch.int32, device=q.device)
    if H == 0:
        return v_idx, s_idx
    ws = _native.workspace(_native.lib().mi_vs_estimate_workspace_size(B, H, S), q.device)
    with torch.cuda.device(q.device):
        rc = _native.lib().mi_vs_estimate(
            _native.t4(qp, tbl), _native.t4(kp, tbl), B, H, S, dk, _native.dtype_code(q), nv, ns,
            logit_scale, v_idx.data_ptr(), s_idx.data_ptr(), ws.data_ptr(), ws.numel(),
            _native.stream_ptr(q.device),
        )
    _native.check(rc, "mi_vs_estimate")
    return v_idx, s_idx


def vertical_slash_sparse_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                    v_idx: torch.Tensor, s_idx: torch.Tensor,
                                    block_size_M: int = 64, block_size_N: int = 64,
                                    softmax_scale: float | None = None, *,
                                    out: torch.Tensor | None = None,
                                    rows: tuple[int, int] | None = None,
                                    heads=None, out_replicas=None) -> torch.Tensor:
    """Vertical-slash causal attention; same signature as the reference op.

    ``rows=(begin, end)`` computes only those query rows (whole 128-row tiles,
    the end may be S); the other rows of the output are left as they are.
    ``heads`` runs only those heads in one launch (v_idx / s_idx then have
    ``len(heads)`` heads, in that order) and writes them in place."""
    check_qkv(query, key, value)
    if block_size_M != 64 or block_size_N != 64:
        raise NotImplementedError("block_size_M/N must be 64")
    B, Hf, S, D = query.shape
    tbl, H = head_table(heads, query)
    assert key.shape[2] == S, (
        f"vertical_slash_sparse_attention supports full prefill only (S_q == S_k); "
        f"got S_q={S}, S_k={key.shape[2]}"
    )
    scale = default_softmax_scale(D) if softmax_scale is None else float(softmax_scale)
    r0, r1 = row_window(rows, S)
    dk = kernel_dim(D)
    vi = v_idx.to(device=query.device, dtype=torch.int32).reshape(B, H, -1).contiguous()
    si = s_idx.to(device=query.device, dtype=torch.int32).reshape(B, H, -1).contiguous()
    qp, kp, vp = prepare(query, dk), prepare(key, dk), prepare(value, dk)
    out = _common_out(out, (B, Hf, S, dk), query, zero=tbl is not None)
    if H == 0:
        return out[..., :D] if dk != D else out
    ws = _native.workspace(_native.lib().mi_vs_sparse_fwd_workspace_size(B, H, S), query.device)
    with torch.cuda.device(query.device):
        rc = _native.lib().mi_vs_sparse_fwd_rows(
            _native.t4(qp, tbl), _native.t4(kp, tbl), _native.t4(vp, tbl),
            _native.t4(out, tbl, replica_ptrs(out_replicas, out, D, dk)), B, H, S, dk,
            _native.dtype_code(query), vi.data_ptr(), vi.shape[-1], si.data_ptr(), si.shape[-1],
            scale, r0, r1, ws.data_ptr(), ws.numel(), _native.stream_ptr(query.device),
        )
    _native.check(rc, "mi_vs_sparse_fwd_rows")
    return out[..., :D] if dk != D else out


def vertical_and_slash(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, vertical_size: int,
                       slash_size: int, *, out: torch.Tensor | None = None,
                       rows: tuple[int, int] | None = None, heads=None,
                       out_replicas=None) -> torch.Tensor:
    """Estimate indices from the last 64 queries, then run the sparse attention."""
    v_idx, s_idx = vertical_and_slash_estimate(q, k, vertical_size, slash_size, heads=heads)
    return vertical_slash_sparse_attention(q, k, v, v_idx, s_idx, out=out, rows=rows,
                                           heads=heads, out_replicas=out_replicas)


def convert_vertical_slash_indexes(seqlens: torch.Tensor, vertical_indexes: torch.Tensor,
                                   slash_indexes: torch.Tensor, context_size: int,
                                   block_size_M: int = 64, block_size_N: int = 64,
                                   causal: bool = True):
    """Legacy four-array index format of upstream MInference.

    Same signature and results as the reference's CPU port
    (MInference-NPU minference/backend_npu/cuda_shim.py:147-236), computed on
    the GPU (one thread per query block): returns ``(block_count [B,H,R],
    block_offset [B,H,R,NNZ_S], column_count [B,H,R], column_index
    [B,H,R,NNZ_V])`` as int32 CUDA tensors, R = ceil(context_size / 64)."""
    if block_size_M != 64 or block_size_N != 64:
        raise AssertionError("block_size_M / block_size_N must be 64")
    if not causal:
        raise NotImplementedError("only causal=True is supported")
    dev = slash_indexes.device
    _native.require_cuda(slash_indexes)
    B, H, ns = slash_indexes.shape
    nv = vertical_indexes.shape[2]
    vi = vertical_indexes.to(device=dev, dtype=torch.int32).contiguous()
    si = slash_indexes.to(device=dev, dtype=torch.int32).contiguous()
    sl = seqlens.to(device=dev, dtype=torch.int32).contiguous()
    R = -(-int(context_size) // 64)
    bc = torch.empty((B, H, R), dtype=torch.int32, device=dev)
    bo = torch.empty((B, H, R, ns), dtype=torch.int32, device=dev)
    cc = torch.empty((B, H, R), dtype=torch.int32, device=dev)
    ci = torch.empty((B, H, R, nv), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        rc = _native.lib().mi_vs_convert_indexes(
            sl.data_ptr(), vi.data_ptr(), nv, si.data_ptr(), ns, B, H, int(context_size),
            bc.data_ptr(), bo.data_ptr(), cc.data_ptr(), ci.data_ptr(), _native.stream_ptr(dev),
        )
    _native.check(rc, "mi_vs_convert_indexes")
    return bc, bo, cc, ci
