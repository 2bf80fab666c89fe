"""Sparse prefill attention ops (sm_100a CUDA behind the C ABI)."""

from .block_sparse import (
    block_sparse_attention,
    block_sparse_attention_from_indices,
    select_block_sparse_topk_indices,
)
from .streaming import dense_attention, streaming_forward
from .vertical_slash import (
    convert_vertical_slash_indexes,
    vertical_and_slash,
    vertical_and_slash_estimate,
    vertical_slash_sparse_attention,
)

__all__ = [
    "block_sparse_attention",
    "block_sparse_attention_from_indices",
    "select_block_sparse_topk_indices",
    "dense_attention",
    "streaming_forward",
    "vertical_and_slash",
    "vertical_and_slash_estimate",
    "vertical_slash_sparse_attention",
    "convert_vertical_slash_indexes",
]
