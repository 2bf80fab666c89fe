"""Dense attention entry points of the reference's backend module
(MInference-NPU minference/backend_npu/attention.py:192-293), on the sm_100a
kernel behind ``mi_dense_fwd``.

* ``dense_attention(q, k, v, *, scale=None, causal=True)``: prefill / fallback
  attention; ``scale`` defaults to ``1/sqrt(D)`` of the unpadded head dim.
* ``prefill_dense``: the same call under the reference's prefill name.
* ``decode_dense(q, k_cache, v_cache, *, scale=None)``: ``q_len == 1`` over the
  whole cache (not causal: the single row sees every cached key).
* ``is_npu_available``: kept under the reference's name; true when the
  sm_100 library and a CUDA device are usable, the condition under which the
  functions above run.

Inputs are BNSD ``[B, H, S, D]`` with the same head count for q and k/v
(``repeat_kv`` already applied), fp16 or bf16, on a CUDA device; there is no
CPU path.
"""

from __future__ import annotations

import torch

from ..ops.streaming import dense_attention

__all__ = ["dense_attention", "prefill_dense", "decode_dense", "is_npu_available"]


def prefill_dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                  scale: float | None = None, causal: bool = True) -> torch.Tensor:
    """Prefill dense attention; identical to ``dense_attention`` (reference :258-271)."""
    return dense_attention(q, k, v, scale=scale, causal=causal)


def decode_dense(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                 scale: float | None = None) -> torch.Tensor:
    """One decode step: ``q`` ``[B,H,1,D]`` against ``[B,H,S_kv,D]`` caches (reference :274-293)."""
    return dense_attention(q, k_cache, v_cache, scale=scale, causal=False)


def is_npu_available() -> bool:
    if not torch.cuda.is_available():
        return False
    try:
        from .. import _native

        _native.lib()
    except Exception:  # noqa: BLE001 - any load failure means "not available"
        return False
    return torch.cuda.get_device_capability()[0] == 10
