"""Alias of the reference module ``python.fa2``: the autograd op."""

from tilelang_fa2_4d_mask import flash_attention_with_4d_mask

__all__ = ["flash_attention_with_4d_mask"]
