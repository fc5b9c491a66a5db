"""Import-compatible entry point (the reference's package name).

Loads the implementation package from the ``fa2-with-4d-mask_b200`` directory
next to this one under the module name ``fa2_with_4d_mask_b200`` and re-exports
the reference's public names (tilelang_fa2_4d_mask/__init__.py:3-10 of the
reference).
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

IMPL_NAME = "fa2_with_4d_mask_b200"
IMPL_DIR = Path(__file__).resolve().parent.parent / "fa2-with-4d-mask_b200"


def load_impl():
    """Returns the implementation package, importing it on first use."""
    mod = sys.modules.get(IMPL_NAME)
    if mod is not None:
        return mod
    spec = importlib.util.spec_from_file_location(
        IMPL_NAME, IMPL_DIR / "__init__.py", submodule_search_locations=[str(IMPL_DIR)]
    )
    mod = importlib.util.module_from_spec(spec)
    sys.modules[IMPL_NAME] = mod
    try:
        spec.loader.exec_module(mod)
    except BaseException:
        sys.modules.pop(IMPL_NAME, None)
        raise
    return mod


_impl = load_impl()
flash_attention_with_4d_mask = _impl.flash_attention_with_4d_mask
tilelang_attention_forward = _impl.tilelang_attention_forward
tilelang_flash_attention = _impl.tilelang_flash_attention

__all__ = [
    "flash_attention_with_4d_mask",
    "tilelang_attention_forward",
    "tilelang_flash_attention",
]
