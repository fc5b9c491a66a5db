"""Alias of the reference module ``python.modeling_attention``: the wrappers."""

from tilelang_fa2_4d_mask import tilelang_attention_forward, tilelang_flash_attention

__all__ = ["tilelang_flash_attention", "tilelang_attention_forward"]
