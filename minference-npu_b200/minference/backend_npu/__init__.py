"""Reference module path kept for drop-in imports (MInference-NPU
minference/backend_npu/): dense / prefill / decode attention and the legacy
index converter, here running on the sm_100a kernels."""

from .attention import decode_dense, dense_attention, is_npu_available, prefill_dense
from .cuda_shim import convert_vertical_slash_indexes

__all__ = [
    "dense_attention",
    "decode_dense",
    "is_npu_available",
    "prefill_dense",
    "convert_vertical_slash_indexes",
]
