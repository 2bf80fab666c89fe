"""minference (B200 build): dynamic sparse prefill attention on sm_100a.

Drop-in for the MInference-NPU package API: ``MInference(attn_type, ...)(model)``,
``minference_patch``, ``patch_hf``, the per-head pattern JSON and the three
sparse ops, with the device work done by hand-written sm_100a CUDA kernels
(``libminference_b200.so``, C ABI in ``include/minference_b200.h``).
"""

from .ops import (
    block_sparse_attention,
    dense_attention,
    streaming_forward,
    vertical_slash_sparse_attention,
)
from .version import VERSION as __version__

__all__ = [
    "MInference",
    "MInferenceConfig",
    "minference_patch",
    "patch_hf",
    "block_sparse_attention",
    "dense_attention",
    "streaming_forward",
    "vertical_slash_sparse_attention",
]


def __getattr__(name):
    # The HF-facing layer imports transformers; load it lazily.
    if name == "MInference":
        from .models_patch import MInference

        return MInference
    if name == "MInferenceConfig":
        from .minference_configuration import MInferenceConfig

        return MInferenceConfig
    if name in ("minference_patch", "patch_hf"):
        from . import patch

        return getattr(patch, name)
    raise AttributeError(name)
