"""SRNL recurrence on B200 (mirror of models/srnl_core/__init__.py)."""

from .chunk import MAX_CHUNK, SUPPORTED_HEAD_DIMS, srnl_normalized_query, srnl_raw_query
from .lines import srnl_long_chunk, srnl_variable_lines

__all__ = [
    "MAX_CHUNK", "SUPPORTED_HEAD_DIMS", "srnl_normalized_query", "srnl_raw_query",
    "srnl_long_chunk", "srnl_variable_lines",
]
