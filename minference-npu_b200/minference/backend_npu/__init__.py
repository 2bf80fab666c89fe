"""Reference module path kept for drop-in imports (MInference-NPU
minference/backend_npu/): dense attention and the legacy index converter,
here running on the sm_100a kernels."""

from ..ops.streaming import dense_attention
from .cuda_shim import convert_vertical_slash_indexes


def decode_dense(q, k, v):
    """q_len == 1 attention over the whole cache (reference attention.py:274)."""
    return dense_attention(q, k, v, causal=True)


__all__ = ["dense_attention", "decode_dense", "convert_vertical_slash_indexes"]
