"""User-facing wrappers: ``tilelang_flash_attention`` and the HF-style adapter
``tilelang_attention_forward``.

Same names, arguments, defaults, validation and error messages as the
reference wrapper (python/modeling_attention.py:21-192), so model code that calls
the reference switches by changing the import.  Semantics kept verbatim:

* mask / score / attention_mask are ``[B or 1, Hq or 1, Tq, Tk]``;
* a bool ``attention_mask`` is AND-ed into ``mask``; a float one is converted to
  fp32, divided by ``scale`` when ``attention_mask_is_scaled`` (default True) and
  added into ``score`` (python/modeling_attention.py:125-135);
* ``score`` is added to ``Q K^T`` before scaling.

One deliberate difference: a broadcast ``[B|1, 1, Tq, Tk]`` mask or score is handed
to the kernel as a stride-0 view instead of being materialised to
``[B, Hq, Tq, Tk]`` (the reference's ``expand().contiguous()``,
python/modeling_attention.py:57-59); the values read are identical.

Extra keywords (not in the reference): ``causal_align`` = "top_left" (default,
the reference's ``q >= k``) or "bottom_right" (``k <= q + Tk - Tq``); ``doc_ids``,
per-token document ids of packed sequences ([B or 1, T], or a (doc_q, doc_k) pair)
used instead of a block-diagonal bool mask — the reference header advertises packed /
right-padded inputs (python/fa2.py:1) but supports them only through a dense mask.
"""

from __future__ import annotations

from typing import Literal, Optional

import torch

from .fa2 import flash_attention_with_4d_mask

Layout = Literal["bhsd", "bshd"]


def _shape_from_layout(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, layout: Layout):
    """Validates rank/shape agreement; returns (B, Hq, Tq, Tk, D).
    Checks and messages follow python/modeling_attention.py:21-45."""
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise ValueError("query, key, and value must be rank-4 tensors")
    if layout == "bhsd":
        b, hq, tq, d = query.shape
        bk, hk, tk, dk = key.shape
        bv, hv, tv, dv = value.shape
    elif layout == "bshd":
        b, tq, hq, d = query.shape
        bk, tk, hk, dk = key.shape
        bv, tv, hv, dv = value.shape
    else:
        raise ValueError(f"unsupported layout: {layout}")
    if bk != b or bv != b:
        raise ValueError("query, key, and value must have the same batch size")
    if tk != tv:
        raise ValueError("key and value must have the same sequence length")
    if hk != hv:
        raise ValueError("key and value must have the same number of heads")
    if dk != d or dv != d:
        raise ValueError("query, key, and value must have the same head dimension")
    if hq % hk != 0:
        raise ValueError(f"query heads ({hq}) must be divisible by key/value heads ({hk})")
    return b, hq, tq, tk, d


def _expand_4d(x: torch.Tensor, *, batch: int, heads: int, seqlen_q: int, seqlen_k: int, name: str) -> torch.Tensor:
    """Validates a [B|1, H|1, Tq, Tk] tensor and returns a broadcast *view*
    (python/modeling_attention.py:48-59 validates the same and then materialises)."""
    if x.dim() != 4:
        raise ValueError(f"{name} must have shape [B, H or 1, Tq, Tk]")
    if x.shape[-2:] != (seqlen_q, seqlen_k):
        raise ValueError(f"{name} has trailing shape {tuple(x.shape[-2:])}, expected {(seqlen_q, seqlen_k)}")
    if x.shape[0] not in (1, batch):
        raise ValueError(f"{name} batch dimension must be 1 or {batch}")
    if x.shape[1] not in (1, heads):
        raise ValueError(f"{name} head dimension must be 1 or {heads}")
    if x.stride(-1) != 1:
        x = x.contiguous()
    if x.shape[0] != batch or x.shape[1] != heads:
        x = x.expand(batch, heads, seqlen_q, seqlen_k)
    return x


def _merge_masks(lhs: Optional[torch.Tensor], rhs: torch.Tensor) -> torch.Tensor:
    return rhs if lhs is None else (lhs & rhs)


def _merge_scores(lhs: Optional[torch.Tensor], rhs: torch.Tensor) -> torch.Tensor:
    return rhs if lhs is None else (lhs + rhs)


def tilelang_flash_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    attention_mask: Optional[torch.Tensor] = None,
    mask: Optional[torch.Tensor] = None,
    score: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    is_causal: bool = False,
    layout: Layout = "bhsd",
    attention_mask_is_scaled: bool = True,
    use_atomic_backward: bool = True,
    causal_align: str = "top_left",
    doc_ids=None,
) -> torch.Tensor:
    """FlashAttention-2 on B200 with an optional 4D bool mask and fp32 score.

    Args:
        query/key/value: rank-4 fp16/bf16 tensors, BHSD ``[B, H, T, D]`` by default or
            BSHD ``[B, T, H, D]`` with ``layout="bshd"``; ``Hq % Hk == 0`` (GQA/MQA).
        attention_mask: optional ``[B, Hq or 1, Tq, Tk]`` bool mask (True keeps) or
            additive float mask on scaled logits.
        mask: optional explicit bool mask, True keeps.
        score: optional float score added to ``Q K^T`` before ``scale``.
        scale: softmax scale, ``head_dim ** -0.5`` by default.
        is_causal: causal attention without a materialised mask.
        attention_mask_is_scaled: divide a float ``attention_mask`` by ``scale``.
        use_atomic_backward: True (default) accumulates dQ with fp32 additions in
            arrival order; False gives a bit-reproducible backward.
        causal_align: "top_left" (reference semantics) or "bottom_right".
        doc_ids: optional per-token document ids (int) of packed sequences, [B or 1,
            T] or a (doc_q, doc_k) pair; keeps (q, k) with equal, non-negative ids.
            Cannot be combined with a bool mask; a float ``attention_mask`` / score
            still adds.  Rows with a negative id are padding and produce zeros.

    Returns:
        The attention output in the input layout.
    """
    batch, heads_q, seqlen_q, seqlen_k, head_dim = _shape_from_layout(query, key, value, layout)
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"TileLang attention expects fp16 or bf16 inputs, got {query.dtype}")
    if key.dtype != query.dtype or value.dtype != query.dtype:
        raise ValueError("query, key, and value must have the same dtype")
    if scale is None:
        scale = head_dim ** -0.5
    scale = float(scale)

    if mask is not None:
        if mask.dtype != torch.bool:
            raise ValueError("mask must be a bool tensor with True for valid entries")
        mask = _expand_4d(mask, batch=batch, heads=heads_q, seqlen_q=seqlen_q, seqlen_k=seqlen_k, name="mask")

    if score is not None:
        if not torch.is_floating_point(score):
            raise ValueError("score must be a floating-point tensor")
        score = _expand_4d(
            score.to(device=query.device, dtype=torch.float32),
            batch=batch, heads=heads_q, seqlen_q=seqlen_q, seqlen_k=seqlen_k, name="score",
        )

    if attention_mask is not None:
        attention_mask = _expand_4d(
            attention_mask.to(device=query.device),
            batch=batch, heads=heads_q, seqlen_q=seqlen_q, seqlen_k=seqlen_k, name="attention_mask",
        )
        if attention_mask.dtype == torch.bool:
            mask = _merge_masks(mask, attention_mask)
        elif torch.is_floating_point(attention_mask):
            additive = attention_mask.to(dtype=torch.float32)
            if attention_mask_is_scaled:
                additive = additive / scale
            score = _merge_scores(score, additive)
        else:
            raise ValueError("attention_mask must be bool or floating point")

    return flash_attention_with_4d_mask(
        query,
        key,
        value,
        mask,
        score,
        scale,
        bool(is_causal),
        bool(use_atomic_backward),
        layout == "bhsd",
        causal_align,
        doc_ids,
    )


def tilelang_attention_forward(
    module,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: Optional[torch.Tensor],
    scaling: float,
    dropout: float = 0.0,
    **kwargs,
) -> tuple:
    """HuggingFace-style attention adapter: BHSD in, ``(attn_output, None)`` out.

    Follows python/modeling_attention.py:150-192: dropout must be 0; keyword
    ``layout/mask/score/use_atomic_backward/attention_mask_is_scaled/is_causal``
    are honoured (plus ``causal_align``); ``is_causal`` defaults to
    ``attention_mask is None and module.is_causal`` (True when unset).
    """
    if dropout not in (0, 0.0, None):
        raise ValueError("TileLang FA2 wrapper does not implement attention dropout")

    layout = kwargs.pop("layout", "bhsd")
    mask = kwargs.pop("mask", None)
    score = kwargs.pop("score", None)
    use_atomic_backward = kwargs.pop("use_atomic_backward", True)
    attention_mask_is_scaled = kwargs.pop("attention_mask_is_scaled", True)
    causal_align = kwargs.pop("causal_align", "top_left")
    doc_ids = kwargs.pop("doc_ids", None)
    is_causal = kwargs.pop("is_causal", None)
    if is_causal is None:
        is_causal = attention_mask is None and bool(getattr(module, "is_causal", True))

    out = tilelang_flash_attention(
        query,
        key,
        value,
        attention_mask=attention_mask,
        mask=mask,
        score=score,
        scale=scaling,
        is_causal=bool(is_causal),
        layout=layout,
        attention_mask_is_scaled=attention_mask_is_scaled,
        use_atomic_backward=use_atomic_backward,
        causal_align=causal_align,
        doc_ids=doc_ids,
    )
    return out, None


__all__ = ["tilelang_flash_attention", "tilelang_attention_forward"]
