"""Autograd op ``flash_attention_with_4d_mask`` over the sm_100a C ABI.

Drop-in for the reference op ``_flash_attention_with_4d_mask``
(python/fa2.py:437-558): same positional signature
``(Q, K, V, Mask, Score, scale, is_causal, use_atomic_backward, bhsd_input)``,
output in the input layout, nine gradients (dQ, dK, dV and six ``None``).
One optional tenth positional argument, ``causal_align`` ("top_left", the
reference's semantics, or "bottom_right"), selects where the causal diagonal
sits when Tq != Tk.  An optional eleventh, ``doc_ids``, describes packed sequences
without a mask tensor: per-token document ids ([B or 1, T] for self-attention, or a
(doc_q, doc_k) pair); query q keeps key k iff their ids are equal and not negative,
and query rows with a negative id (padding) produce zeros.

Differences that do not change results: BHSD inputs are passed to the kernels as
strided views instead of contiguous copies (a copy is made only when the strides
cannot be described by a TMA tensor map), and all three gradients come back in the
input dtype (the reference returns dQ in fp32 and lets autograd cast it,
python/fa2.py:556).  dK/dV are summed over the GQA group inside the kernel (no dK/dV
atomics or per-head buffers for either setting).  ``use_atomic_backward=True`` (the
default) accumulates dQ with fp32 additions in arrival order, like the reference's
atomic kernel; ``False`` selects the bit-reproducible backward, where a separate pass
computes dQ for each query tile by walking the key tiles in a fixed order.

A bool mask is first prepared once (``fa4d_mask_prepare``): a block map (each
128 x 128 block EMPTY, PARTIAL or FULL) that the forward and backward kernels use
to skip EMPTY blocks and the mask reads of FULL ones, and the mask as packed bits
that the kernels read instead of the bytes.  The preparation is cached per mask
tensor (identity of the tensor or of the tensor it views, plus its version
counter), so a mask shared by every layer of a model is scanned once while it is
unchanged.
"""

from __future__ import annotations

import os
import weakref
from typing import Optional

import torch

from . import _lib

_CAUSAL_ALIGN = {"top_left": _lib.CAUSAL_TOP_LEFT, "bottom_right": _lib.CAUSAL_BOTTOM_RIGHT}

# FA4D_CHECK_STATUS=1 makes every backward synchronise and read the device status word
# (bounded waits that gave up), raising instead of returning garbage gradients.  Off by
# default: the read costs a host synchronisation per call.
_CHECK_STATUS = os.environ.get("FA4D_CHECK_STATUS", "0") not in ("", "0")


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
    def _key(t: torch.Tensor) -> tuple:
        return (t.data_ptr(), tuple(t.shape), tuple(t.stride()), t.dtype, t.device, t._version)

    def _lookup(self, tensors: tuple, extra, build):
        owners = tuple(t._base if t._base is not None else t for t in tensors)
        key = (tuple(self._key(t) for t in tensors), extra)
        for i, (refs, k, val) in enumerate(self._entries):
            if k == key and all(r() is o for r, o in zip(refs, owners)):
                if i:
                    self._entries.insert(0, self._entries.pop(i))
                return val
        val = build()
        self._entries.insert(0, (tuple(weakref.ref(o) for o in owners), key, val))
        del self._entries[self.capacity :]
        return val

    def get(self, mask: torch.Tensor) -> "_lib.PreparedMask":
        return self._lookup((mask,), None, lambda: _lib.mask_prepare(mask))

    def get_docs(self, doc_q: torch.Tensor, doc_k: torch.Tensor, batch: int) -> "_lib.PreparedMask":
        return self._lookup((doc_q, doc_k), batch, lambda: _lib.mask_prepare_docs(doc_q, doc_k, batch))

    def clear(self) -> None:
        self._entries.clear()


_block_maps = _BlockMapCache()


def clear_block_map_cache() -> None:
    """Drops every cached mask preparation (e.g. after writing a mask in place
    through a path that does not bump its version counter)."""
    _block_maps.clear()


def _doc_ids(doc_ids, B: int, Tq: int, Tk: int, device) -> tuple:
    """(doc_q [B|1, Tq], doc_k [B|1, Tk]) int32 on `device` from a [B|1, T] tensor
    (self-attention, Tq == Tk) or a (doc_q, doc_k) pair."""
    if isinstance(doc_ids, (tuple, list)):
        if len(doc_ids) != 2:
            raise ValueError("doc_ids must be a tensor or a (doc_q, doc_k) pair")
        dq, dk = doc_ids
    else:
        if Tq != Tk:
            raise ValueError("doc_ids as one tensor needs Tq == Tk; pass (doc_q, doc_k)")
        dq = dk = doc_ids
    out = []
    for t, T, name in ((dq, Tq, "doc_q"), (dk, Tk, "doc_k")):
        if not isinstance(t, torch.Tensor) or t.dim() != 2 or t.shape[1] != T or t.shape[0] not in (1, B):
            raise ValueError(f"{name} must be an integer tensor of shape [B or 1, {T}]")
        if t.dtype.is_floating_point or t.dtype == torch.bool:
            raise ValueError(f"{name} must be an integer tensor")
        out.append(t.to(device=device, dtype=torch.int32))
    return out[0], out[1]


def _fwd_views(Q, K, V, bhsd_input):
    if bhsd_input:
        Q, K, V = Q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2)
    return _lib.as_tma(Q), _lib.as_tma(K), _lib.as_tma(V)


def _check_inputs(Q, K, V, Mask, Score, bhsd_input) -> None:
    """Rejects inputs the kernels would index out of bounds.  The C ABI takes Tq, Tk,
    Hq and Hk from Q and K and trusts the strides of everything else, so a mask, score
    or V of another shape must be refused here.  The reference rejects the same cases
    through its kernels' typed tensor signatures (python/fa2.py:38-44) and its
    wrapper's checks (python/modeling_attention.py:21-59)."""
    for name, x in (("Q", Q), ("K", K), ("V", V)):
        if not isinstance(x, torch.Tensor) or x.dim() != 4:
            raise ValueError(f"{name} must be a rank-4 tensor")
    if Q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"Q must be fp16 or bf16, got {Q.dtype}")
    if K.dtype != Q.dtype or V.dtype != Q.dtype:
        raise ValueError("Q, K and V must have the same dtype")
    if tuple(K.shape) != tuple(V.shape):
        raise ValueError(f"K and V must have the same shape, got {tuple(K.shape)} and {tuple(V.shape)}")
    if bhsd_input:
        B, Hq, Tq, D = Q.shape
        Bk, Hk, Tk, Dk = K.shape
    else:
        B, Tq, Hq, D = Q.shape
        Bk, Tk, Hk, Dk = K.shape
    if Bk != B:
        raise ValueError("Q, K and V must have the same batch size")
    if Dk != D:
        raise ValueError("Q, K and V must have the same head dimension")
    if Hk == 0 or Hq % Hk != 0:
        raise ValueError(f"query heads ({Hq}) must be divisible by key/value heads ({Hk})")
    for name, x, is_mask in (("Mask", Mask, True), ("Score", Score, False)):
        if x is None:
            continue
        if not isinstance(x, torch.Tensor) or x.dim() != 4:
            raise ValueError(f"{name} must have shape [B or 1, Hq or 1, Tq, Tk]")
        if is_mask and x.dtype not in (torch.bool, torch.uint8):
            raise ValueError("Mask must be a bool tensor with True for valid entries")
        if not is_mask and not torch.is_floating_point(x):
            raise ValueError("Score must be a floating-point tensor")
        if tuple(x.shape[-2:]) != (Tq, Tk):
            raise ValueError(f"{name} has trailing shape {tuple(x.shape[-2:])}, expected {(Tq, Tk)}")
        if x.shape[0] not in (1, B):
            raise ValueError(f"{name} batch dimension must be 1 or {B}")
        if x.shape[1] not in (1, Hq):
            raise ValueError(f"{name} head dimension must be 1 or {Hq}")
        if x.device != Q.device:
            raise ValueError(f"{name} must be on {Q.device}, got {x.device}")


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
        doc_ids=None,
    ):
        _check_inputs(Q, K, V, Mask, Score, bhsd_input)
        if not Q.is_cuda:
            raise RuntimeError("flash_attention_with_4d_mask runs on CUDA (sm_100a) tensors only")
        q, k, v = _fwd_views(Q, K, V, bhsd_input)
        B, Tq, Hq, D = q.shape
        if scale is None:
            scale = D ** -0.5
        mode = causal_mode(bool(is_causal), causal_align)
        mask = _lib.prepare_bias(Mask, torch.bool) if Mask is not None else None
        score = _lib.prepare_bias(Score, torch.float32) if Score is not None else None
        if doc_ids is not None:
            if mask is not None:
                raise ValueError("doc_ids cannot be combined with a bool mask")
            doc_q, doc_k = _doc_ids(doc_ids, B, Tq, k.shape[1], q.device)
            blocks = _block_maps.get_docs(doc_q, doc_k, B)
        else:
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
        dQ, dK, dV = _lib.backward(dO, q, k, v, O, LSE, mask, score, ctx.scale, ctx.mode, blocks=ctx.blocks,
                                   deterministic=ctx.use_atomic_backward is False)
        if _CHECK_STATUS:
            # Opt-in: synchronise and raise if any kernel since the last check gave up a
            # bounded wait (its outputs are then garbage).
            bits = _lib.device_status(q.device)
            if bits:
                raise RuntimeError(f"an attention kernel gave up a bounded wait (device status {bits:#x})")
        if ctx.bhsd_input:
            dQ, dK, dV = dQ.transpose(1, 2), dK.transpose(1, 2), dV.transpose(1, 2)
        return dQ, dK, dV, None, None, None, None, None, None, None, None


flash_attention_with_4d_mask = _flash_attention_with_4d_mask.apply

__all__ = ["flash_attention_with_4d_mask", "causal_mode", "clear_block_map_cache"]
