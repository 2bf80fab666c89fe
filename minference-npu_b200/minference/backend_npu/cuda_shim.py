"""Reference module path kept for drop-in imports; see ops/vertical_slash.py."""

from ..ops.vertical_slash import convert_vertical_slash_indexes

__all__ = ["convert_vertical_slash_indexes"]
