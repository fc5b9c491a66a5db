"""Import-compatible alias of the reference's ``python`` package
(python/__init__.py of the reference): same three public names."""

from tilelang_fa2_4d_mask import (
    flash_attention_with_4d_mask,
    tilelang_attention_forward,
    tilelang_flash_attention,
)

__all__ = [
    "flash_attention_with_4d_mask",
    "tilelang_attention_forward",
    "tilelang_flash_attention",
]
