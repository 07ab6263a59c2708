"""B200-native sparse-mask attention (drop-in for the reference's ``python`` package)."""

from .sparse_attention import (
    SparseAttentionFunction,
    pack_mask,
    sparse_attention,
    sparse_attention_func,
)
from .streaming import sparse_attention_from_host

__all__ = ["sparse_attention", "sparse_attention_func", "pack_mask", "SparseAttentionFunction",
           "sparse_attention_from_host"]
