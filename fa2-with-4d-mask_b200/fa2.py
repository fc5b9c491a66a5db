"""Autograd op ``flash_attention_with_4d_mask`` over the sm_100a C ABI.

Drop-in for the reference op ``_flash_attention_with_4d_mask``
(python/fa2.py:437-558): same positional signature
``(Q, K, V, Mask, Score, scale, is_causal, use_atomic_backward, bhsd_input)``,
output in the input layout, nine gradients (dQ, dK, dV and six ``None``).
One optional tenth positional argument, ``causal_align`` ("top_left", the
reference's semantics, or "bottom_right"), selects where the causal diagonal
sits when Tq != Tk.

Differences that do not change results: BHSD inputs are passed to the kernels as
strided views instead of contiguous copies (a copy is made only when the strides
cannot be described by a TMA tensor map), and all three gradients come back in the
input dtype (the reference returns dQ in fp32 and lets autograd cast it,
python/fa2.py:556).  ``use_atomic_backward`` is accepted for compatibility; both
values run the same backward, in which dK/dV are summed over the GQA group inside
the kernel and dQ is accumulated in fp32.

A bool mask is first prepared once (``fa4d_mask_prepare``): a block map (each
128 x 128 block EMPTY, PARTIAL or FULL) that the forward and backward kernels use
to skip EMPTY blocks and the mask reads of FULL ones, and the mask as packed bits
that the kernels read instead of the bytes.  The preparation is cached per mask
tensor (identity of the tensor or of the tensor it views, plus its version
counter), so a mask shared by every layer of a model is scanned once while it is
unchanged.
"""

from __future__ import annotations

import weakref
from typing import Optional

import torch

from . import _lib

_CAUSAL_ALIGN = {"top_left": _lib.CAUSAL_TOP_LEFT, "bottom_right": _lib.CAUSAL_BOTTOM_RIGHT}


def causal_mode(is_causal: bool, causal_align: str = "top_left") -> int:
    """Maps (is_causal, causal_align) to the C ABI's causal enum."""
    if not is_causal:
        return _lib.CAUSAL_NONE
    try:
        return _CAUSAL_ALIGN[causal_align]
    except KeyError:
        raise ValueError(f"unsupported causal_align: {causal_align}") from None


class _BlockMapCache:
    """Block maps of recently used masks.  An entry is reused only while the tensor
    it was computed from (or the tensor that view points into) is alive and its
    version counter is unchanged; any in-place write through autograd-visible
    views bumps that counter."""

    def __init__(self, capacity: int = 8):
        self.capacity = capacity
        self._entries: list = []

    @staticmethod
    def _key(mask: torch.Tensor) -> tuple:
        return (mask.data_ptr(), tuple(mask.shape), tuple(mask.stride()), mask.dtype, mask.device, mask._version)

    def get(self, mask: torch.Tensor) -> "_lib.PreparedMask":
        owner = mask._base if mask._base is not None else mask
        key = self._key(mask)
        for i, (ref, k, bm) in enumerate(self._entries):
            if k == key and ref() is owner:
                if i:
                    self._entries.insert(0, self._entries.pop(i))
                return bm
        bm = _lib.mask_prepare(mask)
        self._entries.insert(0, (weakref.ref(owner), key, bm))
        del self._entries[self.capacity :]
        return bm

    def clear(self) -> None:
        self._entries.clear()


_block_maps = _BlockMapCache()


def clear_block_map_cache() -> None:
    """Drops every cached mask preparation (e.g. after writing a mask in place
    through a path that does not bump its version counter)."""
    _block_maps.clear()


def _fwd_views(Q, K, V, bhsd_input):
    if bhsd_input:
        Q, K, V = Q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2)
    return _lib.as_tma(Q), _lib.as_tma(K), _lib.as_tma(V)


class _flash_attention_with_4d_mask(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx,
        Q: torch.Tensor,
        K: torch.Tensor,
        V: torch.Tensor,
        Mask: Optional[torch.Tensor] = None,
        Score: Optional[torch.Tensor] = None,
        scale: Optional[float] = None,
        is_causal: Optional[bool] = False,
        use_atomic_backward: Optional[bool] = True,
        bhsd_input: Optional[bool] = True,
        causal_align: str = "top_left",
    ):
        assert Q.dim() == 4 and K.dim() == 4 and V.dim() == 4
        if not Q.is_cuda:
            raise RuntimeError("flash_attention_with_4d_mask runs on CUDA (sm_100a) tensors only")
        q, k, v = _fwd_views(Q, K, V, bhsd_input)
        B, Tq, Hq, D = q.shape
        if scale is None:
            scale = D ** -0.5
        mode = causal_mode(bool(is_causal), causal_align)
        mask = _lib.prepare_bias(Mask, torch.bool) if Mask is not None else None
        score = _lib.prepare_bias(Score, torch.float32) if Score is not None else None
        blocks = _block_maps.get(mask) if mask is not None else None
        O, LSE = _lib.forward(q, k, v, mask, score, float(scale), mode, blocks=blocks)
        ctx.save_for_backward(q, k, v, O, LSE, mask, score)
        ctx.blocks = blocks
        ctx.scale = float(scale)
        ctx.mode = mode
        ctx.use_atomic_backward = use_atomic_backward
        ctx.bhsd_input = bhsd_input
        return O.transpose(1, 2) if bhsd_input else O

    @staticmethod
    def backward(ctx, dO: torch.Tensor):
        q, k, v, O, LSE, mask, score = ctx.saved_tensors
        if ctx.bhsd_input:
            dO = dO.transpose(1, 2)
        dO = _lib.as_tma(dO)
        dQ, dK, dV = _lib.backward(dO, q, k, v, O, LSE, mask, score, ctx.scale, ctx.mode, blocks=ctx.blocks)
        if ctx.bhsd_input:
            dQ, dK, dV = dQ.transpose(1, 2), dK.transpose(1, 2), dV.transpose(1, 2)
        return dQ, dK, dV, None, None, None, None, None, None, None


flash_attention_with_4d_mask = _flash_attention_with_4d_mask.apply

__all__ = ["flash_attention_with_4d_mask", "causal_mode", "clear_block_map_cache"]
