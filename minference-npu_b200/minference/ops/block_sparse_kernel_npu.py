"""Reference module name kept for drop-in imports; see block_sparse.py."""
from .block_sparse import (  # noqa: F401
    block_sparse_attention,
    block_sparse_attention_from_indices,
    select_block_sparse_topk_indices,
)

_select_block_sparse_topk_indices = select_block_sparse_topk_indices

__all__ = ["block_sparse_attention"]
