"""block_sparse pattern: top-k 64x64 key blocks per 64-row query block.

Drop-in for ``block_sparse_attention`` (MInference-NPU
minference/ops/block_sparse_kernel_npu.py:609-709) and its selector
``_select_block_sparse_topk_indices`` (:230-263).  The selector mean-pools Q
and K per 64-token block, scores the pooled blocks, masks future blocks and
keeps the top-k per query block (ties resolved towards the lower block
index); attention then runs over the selected blocks AND per-token causal
(:266-348).
"""

from __future__ import annotations

import torch

from .. import _native
from ._common import (check_qkv, default_softmax_scale, head_table, kernel_dim, prepare,
                      reference_padded_dim, replica_ptrs, row_window)
from ._common import output as _common_out

__all__ = [
    "block_sparse_attention",
    "block_sparse_attention_from_indices",
    "select_block_sparse_topk_indices",
]

_DEFAULT_BLOCK_SIZE = 64


def select_block_sparse_topk_indices(q: torch.Tensor, k: torch.Tensor, topk_blocks: int,
                                     block_size: int = _DEFAULT_BLOCK_SIZE,
                                     force_sink_diag: bool = False,
                                     score_scale: float | None = None,
                                     heads=None) -> torch.Tensor:
    """Selected key blocks ``[B,H,ceil(S_q/64),min(topk,ceil(S_k/64))]`` int64, ascending.

    ``score_scale`` defaults to ``padded_D ** -0.5`` as in the reference, where
    the op pads D before selecting.  ``force_sink_diag`` always keeps block 0
    and the diagonal block (counted inside topk).  ``heads`` selects heads of
    q/k (one launch); the result then has ``len(heads)`` heads, in that order."""
    if block_size != _DEFAULT_BLOCK_SIZE:
        raise NotImplementedError("block_size must be 64")
    _native.require_cuda(q, k)
    B, _, S_q, D = q.shape
    S_k = k.shape[2]
    tbl, H = head_table(heads, q)
    if score_scale is None:
        score_scale = reference_padded_dim(D) ** -0.5
    topk = max(1, int(topk_blocks))
    nbq, nbk = -(-S_q // 64), -(-S_k // 64)
    kk = min(topk, nbk)
    out = torch.empty((B, H, nbq, kk), dtype=torch.int64, device=q.device)
    if H == 0:
        return out
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    ws_n = _native.lib().mi_block_pool_topk_workspace_size(B, H, S_q, S_k, D)
    ws = _native.workspace(ws_n, q.device)
    with torch.cuda.device(q.device):
        rc = _native.lib().mi_block_pool_topk(
            _native.t4(q, tbl), _native.t4(k, tbl), B, H, S_q, S_k, D, _native.dtype_code(q), topk,
            int(bool(force_sink_diag)), float(score_scale), out.data_ptr(), ws.data_ptr(),
            ws.numel(), _native.stream_ptr(q.device),
        )
    _native.check(rc, "mi_block_pool_topk")
    return out


def block_sparse_attention_from_indices(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                        block_idx: torch.Tensor,
                                        softmax_scale: float | None = None, *,
                                        out: torch.Tensor | None = None,
                                        rows: tuple[int, int] | None = None,
                                        heads=None, out_replicas=None) -> torch.Tensor:
    """Block-sparse causal attention over given key blocks ``[B,H,ceil(S/64),topk]``.

    ``rows=(begin, end)`` computes only those query rows (whole 128-row tiles,
    the end may be S); the other rows of the output are left as they are.
    ``heads`` runs only those heads of q/k/v/out in one launch (``block_idx``
    then has ``len(heads)`` heads, in that order) and writes them in place."""
    check_qkv(q, k, v)
    B, Hf, S, D = q.shape
    if k.shape[2] != S:
        raise NotImplementedError("block_sparse attention needs S_q == S_k (full prefill)")
    tbl, H = head_table(heads, q)
    scale = default_softmax_scale(D) if softmax_scale is None else float(softmax_scale)
    dk = kernel_dim(D)
    idx = block_idx.to(device=q.device, dtype=torch.int64).contiguous()
    if idx.dim() != 4 or idx.shape[:3] != (B, H, -(-S // 64)):
        raise ValueError(f"block_idx must be [B,H,ceil(S/64),topk], got {tuple(idx.shape)}")
    topk = idx.shape[-1]
    r0, r1 = row_window(rows, S)
    qp, kp, vp = prepare(q, dk), prepare(k, dk), prepare(v, dk)
    out = _common_out(out, (B, Hf, S, dk), q, zero=tbl is not None)
    if H == 0:
        return out[..., :D] if dk != D else out
    ws = _native.workspace(_native.lib().mi_block_sparse_fwd_workspace_size(B, H, S, topk), q.device)
    with torch.cuda.device(q.device):
        rc = _native.lib().mi_block_sparse_fwd_rows(
            _native.t4(qp, tbl), _native.t4(kp, tbl), _native.t4(vp, tbl),
            _native.t4(out, tbl, replica_ptrs(out_replicas, out, D, dk)), B, H, S, dk,
            _native.dtype_code(q), idx.data_ptr(), topk, scale, r0, r1, ws.data_ptr(), ws.numel(),
            _native.stream_ptr(q.device),
        )
    _native.check(rc, "mi_block_sparse_fwd_rows")
    return out[..., :D] if dk != D else out


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, topk_blocks: int,
                           block_size: int = _DEFAULT_BLOCK_SIZE, *,
                           out: torch.Tensor | None = None,
                           rows: tuple[int, int] | None = None, heads=None,
                           out_replicas=None) -> torch.Tensor:
    """Block-sparse causal attention; same signature and semantics as the reference."""
    check_qkv(q, k, v)
    topk = max(1, int(topk_blocks))
    idx = select_block_sparse_topk_indices(q, k, topk, block_size, heads=heads)
    return block_sparse_attention_from_indices(q, k, v, idx, out=out, rows=rows, heads=heads,
                                               out_replicas=out_replicas)
