"""Reference module name kept for drop-in imports; see vertical_slash.py."""
from .vertical_slash import vertical_slash_sparse_attention  # noqa: F401

__all__ = ["vertical_slash_sparse_attention"]
