"""B200-native (sm_100a) FlashAttention-2 forward/backward with an optional 4D
bool mask and fp32 score: the drop-in implementation behind the import paths
``tilelang_fa2_4d_mask`` and ``python`` of the reference project.

The directory name is not a Python identifier, so the package is loaded under
the module name ``fa2_with_4d_mask_b200`` by ``tilelang_fa2_4d_mask/__init__.py``.
"""

from .fa2 import causal_mode, flash_attention_with_4d_mask
from .modeling_attention import tilelang_attention_forward, tilelang_flash_attention

__all__ = [
    "flash_attention_with_4d_mask",
    "tilelang_attention_forward",
    "tilelang_flash_attention",
    "causal_mode",
]
