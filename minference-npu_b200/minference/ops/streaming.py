"""stream_llm (attention sink + sliding window) and dense causal attention.

Drop-in for ``streaming_forward`` (MInference-NPU
minference/ops/streaming_kernel_npu.py:349-397) and ``dense_attention``
(minference/backend_npu/attention.py:192).  A query at absolute position
``i = S_k - S_q + row`` sees keys ``j <= i`` with ``j < n_init`` or
``j > i - n_local`` (visible set of streaming_kernel_npu.py:131-136).  The
reference runs a band FA, a sink FA and an eager LSE merge (:233-341); here
one sm_100a kernel walks the sink blocks and then the band blocks inside a
single online softmax, so the merge is implicit.  Dense attention runs on the
same kernel with the window covering every key (``mi_dense_fwd``).
"""

from __future__ import annotations

import math

import torch

from .. import _native
from ._common import (check_qkv, default_softmax_scale, head_table, kernel_dim, prepare,
                      replica_ptrs, row_window)
from ._common import output as _common_out

__all__ = ["streaming_forward", "dense_attention"]


def _launch(q, k, v, n_init: int, n_local: int, scale: float,
            out: torch.Tensor | None = None, heads=None, out_replicas=None) -> torch.Tensor:
    check_qkv(q, k, v)
    B, H, S_q, D = q.shape
    S_k = k.shape[2]
    if S_q > S_k:
        raise ValueError(f"S_q={S_q} > S_k={S_k}: rows without any visible key")
    tbl, G = head_table(heads, q)
    dk = kernel_dim(D)
    qp, kp, vp = prepare(q, dk), prepare(k, dk), prepare(v, dk)
    out = _common_out(out, (B, H, S_q, dk), q, zero=tbl is not None)
    if G:
        with torch.cuda.device(q.device):
            rc = _native.lib().mi_stream_fwd(
                _native.t4(qp, tbl), _native.t4(kp, tbl), _native.t4(vp, tbl),
                _native.t4(out, tbl, replica_ptrs(out_replicas, out, D, dk)), B, G, S_q, S_k,
                dk, _native.dtype_code(q), int(n_init),
                int(n_local), float(scale), _native.stream_ptr(q.device),
            )
        _native.check(rc, "mi_stream_fwd")
    return out[..., :D] if dk != D else out


def _window(q, k, v, out, rows):
    """Restrict a causal problem to query rows [r0, r1): with bottom-right
    alignment, rows r0.. of a full prefill are the last r1 - r0 rows of the
    problem whose keys end at r1 (keys past a row are never visible)."""
    S = q.shape[2]
    if k.shape[2] != S:
        raise NotImplementedError("rows= needs S_q == S_k (full prefill)")
    r0, r1 = row_window(rows, S)
    if out is None:
        out = torch.zeros_like(q)
    return q[:, :, r0:r1], k[:, :, :r1], v[:, :, :r1], out, out[:, :, r0:r1]


def streaming_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_init: int,
                      n_local: int, *, out: torch.Tensor | None = None,
                      rows: tuple[int, int] | None = None, heads=None,
                      out_replicas=None) -> torch.Tensor:
    """Sink + sliding-window causal attention on BNSD ``[B,H,S,D]`` inputs.

    ``rows=(begin, end)`` (full prefill only) computes only those query rows
    (whole 128-row tiles, the end may be S); other output rows are left as
    they are.  ``heads`` (indices into the head dimension) runs only those
    heads, in one launch, writing them in place into ``out`` (the other heads
    are left as they are; a new output is zero there).  ``out_replicas``
    (with ``out``) are addresses of the same view in other buffers -- e.g. the
    peers' copies of the layer output -- that every output tile is also
    written to.

    Same signature and result as the reference.  The reference zero-pads D to
    the next supported head dim before anything else (streaming_kernel_npu.py:
    377-381), so both the sparse path (:114) and the ``k_len <= n_local``
    short-circuit to dense causal attention (:386-390) take their default
    scale from the padded dim: 1/sqrt(128) at D=96.
    """
    n_init = max(0, int(n_init))
    n_local = int(n_local)
    scale = default_softmax_scale(q.shape[-1])
    if rows is not None:
        if out_replicas:
            raise NotImplementedError("rows= with output replicas")
        qw, kw, vw, full, ow = _window(q, k, v, out, rows)
        if qw.shape[2]:
            if k.shape[2] <= n_local:  # the short-circuit is decided on the whole sequence
                dense_attention(qw, kw, vw, scale=scale, causal=True, out=ow, heads=heads)
            else:
                _launch(qw, kw, vw, n_init, n_local, scale, ow, heads)
        return full
    if k.shape[2] <= n_local:
        return dense_attention(q, k, v, scale=scale, causal=True, out=out, heads=heads,
                               out_replicas=out_replicas)
    return _launch(q, k, v, n_init, n_local, scale, out, heads, out_replicas)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                    scale: float | None = None, causal: bool = True,
                    out: torch.Tensor | None = None,
                    rows: tuple[int, int] | None = None, heads=None,
                    out_replicas=None) -> torch.Tensor:
    """Dense attention on BNSD ``[B,H,S,D]`` inputs (MInference-NPU
    minference/backend_npu/attention.py:192-211): ``scale`` defaults to
    ``1/sqrt(D)`` of the unpadded head dim; ``causal`` masks bottom-right
    aligned (row r sees keys ``j <= S_k - S_q + r``), otherwise every row sees
    every key.  Output has q's shape, dtype and device; ``out`` (optional) is a
    caller-owned ``[B,H,S_q,D]`` view written in place.  ``rows`` and ``heads``
    restrict the call as in ``streaming_forward``."""
    if rows is not None:
        if out_replicas:
            raise NotImplementedError("rows= with output replicas")
        if not causal:
            raise NotImplementedError("rows= is for causal prefill")
        qw, kw, vw, full, ow = _window(q, k, v, out, rows)
        if qw.shape[2]:
            dense_attention(qw, kw, vw, scale=scale, causal=True, out=ow, heads=heads)
        return full
    check_qkv(q, k, v)
    B, H, S_q, D = q.shape
    S_k = k.shape[2]
    if causal and S_q > S_k:
        raise ValueError(f"S_q={S_q} > S_k={S_k}: causal rows without any visible key")
    tbl, G = head_table(heads, q)
    sc = 1.0 / math.sqrt(D) if scale is None else float(scale)
    dk = kernel_dim(D)
    qp, kp, vp = prepare(q, dk), prepare(k, dk), prepare(v, dk)
    out = _common_out(out, (B, H, S_q, dk), q, zero=tbl is not None)
    if G:
        with torch.cuda.device(q.device):
            rc = _native.lib().mi_dense_fwd(
                _native.t4(qp, tbl), _native.t4(kp, tbl), _native.t4(vp, tbl),
                _native.t4(out, tbl, replica_ptrs(out_replicas, out, D, dk)), B, G, S_q, S_k,
                dk, _native.dtype_code(q), 1 if causal else 0, sc,
                _native.stream_ptr(q.device),
            )
        _native.check(rc, "mi_dense_fwd")
    return out[..., :D] if dk != D else out
