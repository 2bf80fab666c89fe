"""stream_llm (attention sink + sliding window) and dense causal attention.

Drop-in for ``streaming_forward`` (MInference-NPU
minference/ops/streaming_kernel_npu.py:349-397) and ``dense_attention``
(minference/backend_npu/attention.py:192).  A query at absolute position
``i = S_k - S_q + row`` sees keys ``j <= i`` with ``j < n_init`` or
``j > i - n_local`` (visible set of streaming_kernel_npu.py:131-136).  The
reference runs a band FA, a sink FA and an eager LSE merge (:233-341); here
one sm_100a kernel walks the sink blocks and then the band blocks inside a
single online softmax, so the merge is implicit.
"""

from __future__ import annotations

import torch

from .. import _native
from ._common import check_qkv, default_softmax_scale, kernel_dim, prepare
from ._common import output as _common_out

__all__ = ["streaming_forward", "dense_attention"]


def _launch(q, k, v, n_init: int, n_local: int, softmax_scale: float | None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    check_qkv(q, k, v)
    B, H, S_q, D = q.shape
    S_k = k.shape[2]
    if S_q > S_k:
        raise ValueError(f"S_q={S_q} > S_k={S_k}: rows without any visible key")
    scale = default_softmax_scale(D) if softmax_scale is None else float(softmax_scale)
    dk = kernel_dim(D)
    qp, kp, vp = prepare(q, dk), prepare(k, dk), prepare(v, dk)
    out = _common_out(out, (B, H, S_q, dk), q)
    with torch.cuda.device(q.device):
        rc = _native.lib().mi_stream_fwd(
            _native.t4(qp), _native.t4(kp), _native.t4(vp), _native.t4(out), B, H, S_q, S_k, dk,
            _native.dtype_code(q), int(n_init), int(n_local), scale, _native.stream_ptr(q.device),
        )
    _native.check(rc, "mi_stream_fwd")
    return out[..., :D] if dk != D else out


def streaming_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, n_init: int,
                      n_local: int, *, out: torch.Tensor | None = None) -> torch.Tensor:
    """Sink + sliding-window causal attention on BNSD ``[B,H,S,D]`` inputs.

    Same signature and result as the reference; ``k_len <= n_local`` is dense
    causal attention, which the same kernel computes (window covers all keys).
    """
    n_init = max(0, int(n_init))
    n_local = int(n_local)
    if k.shape[2] <= n_local:
        return dense_attention(q, k, v, causal=True, out=out)
    return _launch(q, k, v, n_init, n_local, None, out)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                    softmax_scale: float | None = None, *,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense causal attention (the stream kernel with an unbounded window)."""
    if not causal:
        raise NotImplementedError("only causal prefill attention is implemented")
    return _launch(q, k, v, 0, k.shape[2] + 1, softmax_scale, out)
