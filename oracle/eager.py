"""ORACLE — test infrastructure only.

CPU restatement, in fp32 PyTorch eager math, of the reference project's own
correctness oracle ``eager_ref`` (benchmark/precision_check.py:133-180) and of the
mask/score merging its user wrapper performs before the kernel
(python/modeling_attention.py:48-67 and 115-135).  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may use this
module, and only as the checker or the timed CPU baseline; the product path
(the ``fa2-with-4d-mask_b200`` package) never imports it.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
``eager_ref`` (and the reference wrapper's merge helpers) on seeded inputs and
stores the results in ``tests/golden/*.npz``; ``tests/test_oracle.py`` checks this
restatement against those fixtures.
"""

from __future__ import annotations

from typing import Optional

import torch


def attention_ref(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    mask: Optional[torch.Tensor],
    score: Optional[torch.Tensor],
    *,
    scale: float,
    is_causal: bool,
    causal_offset: int = 0,
    ref_block: int = 128,
) -> torch.Tensor:
    """Attention in fp32 on BHSD tensors; returns fp32 ``[B, Hq, Tq, D]``.

    Follows benchmark/precision_check.py:133-180 step by step:
    GQA by repeat_interleave of K/V over the head axis (:147-150); logits =
    einsum(Q, K) (:158) plus ``score`` *before* scaling (:159-161); ``* scale``
    (:161); causal keeps ``q_idx + causal_offset >= k_idx`` (:164-167, where the
    reference has offset 0, i.e. top-left alignment); AND with ``mask`` (:168-170);
    ``masked_fill(-inf)`` and softmax over keys (:171-174); probs @ V (:175).  Query
    rows are processed in blocks of ``ref_block`` (:177-179).  Unlike the reference,
    the result is returned in fp32 (it casts to the input dtype at :179-180) so
    tests can measure the kernel's own rounding.
    """
    B, Hq, Tq, D = q.shape
    Hk = k.shape[1]
    Tk = k.shape[2]
    assert Hq % Hk == 0, f"Hq={Hq} must be divisible by Hk={Hk}"
    groups = Hq // Hk
    if groups != 1:
        k = k.repeat_interleave(groups, dim=1)
        v = v.repeat_interleave(groups, dim=1)
    qf, kf, vf = q.float(), k.float(), v.float()

    def block(q0: int, q1: int) -> torch.Tensor:
        logits = torch.einsum("bhqd,bhkd->bhqk", qf[:, :, q0:q1, :], kf)
        if score is not None:
            logits = logits + score[:, :, q0:q1, :].float()
        logits = logits * scale
        valid = None
        if is_causal:
            qi = torch.arange(q0, q1, device=q.device)[:, None]
            ki = torch.arange(Tk, device=q.device)[None, :]
            valid = (qi + causal_offset >= ki).view(1, 1, q1 - q0, Tk)
        if mask is not None:
            m = mask[:, :, q0:q1, :]
            valid = m if valid is None else (valid & m)
        if valid is not None:
            logits = logits.masked_fill(~valid, float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        return torch.einsum("bhqk,bhkd->bhqd", probs, vf)

    if ref_block and 0 < ref_block < Tq:
        return torch.cat([block(s, min(s + ref_block, Tq)) for s in range(0, Tq, ref_block)], dim=2)
    return block(0, Tq)


def attention_ref_grads(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    dout: torch.Tensor,
    mask: Optional[torch.Tensor],
    score: Optional[torch.Tensor],
    *,
    scale: float,
    is_causal: bool,
    causal_offset: int = 0,
    ref_block: int = 128,
):
    """(out, dQ, dK, dV) in fp32, backward by autograd through ``attention_ref``
    exactly as the reference's backward check does (precision_check.py:297-304)."""
    qr = q.detach().float().clone().requires_grad_(True)
    kr = k.detach().float().clone().requires_grad_(True)
    vr = v.detach().float().clone().requires_grad_(True)
    out = attention_ref(qr, kr, vr, mask, score, scale=scale, is_causal=is_causal,
                        causal_offset=causal_offset, ref_block=ref_block)
    out.backward(dout.float())
    return out.detach(), qr.grad, kr.grad, vr.grad


def expand_4d(x: torch.Tensor, batch: int, heads: int, seqlen_q: int, seqlen_k: int) -> torch.Tensor:
    """Broadcast to ``[B, Hq, Tq, Tk]`` (python/modeling_attention.py:57-59)."""
    return x.expand(batch, heads, seqlen_q, seqlen_k).contiguous()


def merge_wrapper_inputs(
    *,
    batch: int,
    heads: int,
    seqlen_q: int,
    seqlen_k: int,
    scale: float,
    mask: Optional[torch.Tensor] = None,
    score: Optional[torch.Tensor] = None,
    attention_mask: Optional[torch.Tensor] = None,
    attention_mask_is_scaled: bool = True,
):
    """(mask, score) as the reference wrapper hands them to its kernel
    (python/modeling_attention.py:115-135): bool attention_mask AND-ed into mask,
    float attention_mask converted to fp32, divided by ``scale`` when
    ``attention_mask_is_scaled`` and added into score."""
    if mask is not None:
        mask = expand_4d(mask, batch, heads, seqlen_q, seqlen_k)
    if score is not None:
        score = expand_4d(score.to(torch.float32), batch, heads, seqlen_q, seqlen_k)
    if attention_mask is not None:
        am = expand_4d(attention_mask, batch, heads, seqlen_q, seqlen_k)
        if am.dtype == torch.bool:
            mask = am if mask is None else (mask & am)
        else:
            add = am.to(torch.float32)
            if attention_mask_is_scaled:
                add = add / scale
            score = add if score is None else (score + add)
    return mask, score


def bottom_right_mask(Tq: int, Tk: int) -> torch.Tensor:
    """Bool ``[1, 1, Tq, Tk]`` keeping ``k <= q + (Tk - Tq)``: the explicit mask that
    gives ``eager_ref`` bottom-right-aligned causal semantics."""
    qi = torch.arange(Tq)[:, None]
    ki = torch.arange(Tk)[None, :]
    return (ki <= qi + (Tk - Tq)).view(1, 1, Tq, Tk)
