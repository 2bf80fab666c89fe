"""Reference module name kept for drop-in imports; see streaming.py."""
from .streaming import dense_attention, streaming_forward  # noqa: F401

__all__ = ["streaming_forward"]
