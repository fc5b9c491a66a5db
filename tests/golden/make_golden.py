"""Generates tests/golden/*.npz from the reference project itself.

Runs only where the reference source tree is available (its path is given with
--reference).  For every case it calls the reference's own user wrapper
``tilelang_flash_attention`` (python/modeling_attention.py:70-147) with the kernel
call replaced by the reference's own correctness oracle ``eager_ref``
(benchmark/precision_check.py:133-180, fp32 math), so the fixture pins both the
wrapper's mask/score merging and the oracle's attention math.  Gradients come from
autograd through ``eager_ref``, as the reference's backward check does
(precision_check.py:297-304).

Stored per case: sizes and flags, the inputs (q/k/v/dout as bf16 bit patterns in
[B, T, H, D] storage order; mask/score/attention_mask as given to the wrapper) and
fp32 expected out/dq/dk/dv in BHSD order.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CASES = [
    dict(name="gqa_noncausal_tail", B=1, Tq=100, Tk=100, Hq=4, Hk=2, D=64),
    dict(name="gqa_causal_tail", B=1, Tq=100, Tk=100, Hq=4, Hk=2, D=64, is_causal=True),
    dict(name="mask_rect_d128", B=2, Tq=40, Tk=136, Hq=2, Hk=1, D=128, mask="random_full"),
    dict(name="score_and_bcast_mask", B=1, Tq=72, Tk=144, Hq=2, Hk=2, D=64, score="randn_full", mask="random_h1"),
    dict(name="attn_float_scaled_causal", B=1, Tq=130, Tk=130, Hq=2, Hk=1, D=64, attention_mask="float_h1",
         is_causal=True, attention_mask_is_scaled=True),
    dict(name="attn_float_unscaled_bshd", B=1, Tq=80, Tk=96, Hq=2, Hk=2, D=64, attention_mask="float_full",
         attention_mask_is_scaled=False, layout="bshd"),
    dict(name="attn_bool_and_mask", B=1, Tq=100, Tk=100, Hq=2, Hk=1, D=64, attention_mask="bool_b1h1",
         mask="random_full"),
    dict(name="bottom_right_rect", B=1, Tq=64, Tk=200, Hq=2, Hk=1, D=64, bottom_right=True),
    dict(name="mqa_causal_d128", B=1, Tq=72, Tk=72, Hq=3, Hk=1, D=128, is_causal=True),
    dict(name="score_causal_d96", B=1, Tq=80, Tk=136, Hq=2, Hk=1, D=96, is_causal=True, score="randn_full",
         mask="random_h1"),
]


def _bits(x: torch.Tensor) -> np.ndarray:
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_case(c: dict, eager_ref, wrapper_mod) -> dict:
    B, Tq, Tk, Hq, Hk, D = c["B"], c["Tq"], c["Tk"], c["Hq"], c["Hk"], c["D"]
    layout = c.get("layout", "bhsd")
    is_causal = c.get("is_causal", False)
    scale = D ** -0.5
    g = torch.Generator().manual_seed(1234 + sum(map(ord, c["name"])))
    # storage [B, T, H, D], bf16
    q_s = torch.randn((B, Tq, Hq, D), generator=g).to(torch.bfloat16)
    k_s = torch.randn((B, Tk, Hk, D), generator=g).to(torch.bfloat16)
    v_s = torch.randn((B, Tk, Hk, D), generator=g).to(torch.bfloat16)
    do_s = torch.randn((B, Tq, Hq, D), generator=g).to(torch.bfloat16)

    def rand_mask(b, h, keep=0.75):
        m = torch.rand((b, h, Tq, Tk), generator=g) < keep
        qi = torch.arange(Tq)
        m[:, :, qi, torch.clamp(qi, max=Tk - 1)] = True
        return m

    mask = score = attn = None
    if c.get("mask") == "random_full":
        mask = rand_mask(B, Hq)
    elif c.get("mask") == "random_h1":
        mask = rand_mask(B, 1)
    if c.get("score") == "randn_full":
        score = torch.randn((B, Hq, Tq, Tk), generator=g) * 0.5
    am = c.get("attention_mask")
    if am == "float_h1":
        attn = torch.randn((B, 1, Tq, Tk), generator=g) * 0.7
    elif am == "float_full":
        attn = torch.randn((B, Hq, Tq, Tk), generator=g) * 0.7
    elif am == "bool_b1h1":
        attn = rand_mask(1, 1, keep=0.8)
    if c.get("bottom_right"):
        qi = torch.arange(Tq)[:, None]
        ki = torch.arange(Tk)[None, :]
        mask = (ki <= qi + (Tk - Tq)).view(1, 1, Tq, Tk).expand(B, 1, Tq, Tk).contiguous()

    to_layout = (lambda x: x.transpose(1, 2)) if layout == "bhsd" else (lambda x: x)
    # fp32 leaves holding exactly the bf16 values, so gradients stay in fp32.
    qf = to_layout(q_s.float()).detach().requires_grad_(True)
    kf = to_layout(k_s.float()).detach().requires_grad_(True)
    vf = to_layout(v_s.float()).detach().requires_grad_(True)

    # The reference wrapper (which validates bf16 inputs and merges mask/score) with
    # its kernel call replaced by its own eager oracle, evaluated on the fp32 leaves.
    def fake_kernel(Q, K, V, Mask, Score, sc, causal, atomic, bhsd_input):
        Qe, Ke, Ve = (qf, kf, vf) if bhsd_input else (qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2))
        out = eager_ref(Qe, Ke, Ve, Mask, Score, scale=sc, is_causal=causal, ref_block=0)
        return out if bhsd_input else out.transpose(1, 2)

    orig = wrapper_mod.flash_attention_with_4d_mask
    wrapper_mod.flash_attention_with_4d_mask = fake_kernel
    try:
        out = wrapper_mod.tilelang_flash_attention(
            to_layout(q_s), to_layout(k_s), to_layout(v_s), attention_mask=attn, mask=mask, score=score,
            scale=scale, is_causal=is_causal,
            layout=layout, attention_mask_is_scaled=c.get("attention_mask_is_scaled", True),
        )
        out.backward(to_layout(do_s.float()))
    finally:
        wrapper_mod.flash_attention_with_4d_mask = orig
    to_bhsd = (lambda x: x) if layout == "bhsd" else (lambda x: x.transpose(1, 2))
    meta = dict(c, scale=scale, layout=layout, is_causal=is_causal,
                causal_align="bottom_right" if c.get("bottom_right") else "top_left")
    rec = {
        "meta": np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8),
        "q": _bits(q_s), "k": _bits(k_s), "v": _bits(v_s), "dout": _bits(do_s),
        "out": to_bhsd(out.detach()).contiguous().numpy().astype(np.float32),
        "dq": to_bhsd(qf.grad).contiguous().numpy().astype(np.float32),
        "dk": to_bhsd(kf.grad).contiguous().numpy().astype(np.float32),
        "dv": to_bhsd(vf.grad).contiguous().numpy().astype(np.float32),
    }
    if mask is not None and not c.get("bottom_right"):
        rec["mask"] = mask.numpy().astype(np.uint8)
    if score is not None:
        rec["score"] = score.numpy().astype(np.float32)
    if attn is not None:
        rec["attention_mask"] = attn.numpy().astype(np.uint8 if attn.dtype == torch.bool else np.float32)
        rec["attention_mask_is_bool"] = np.array([attn.dtype == torch.bool])
    return rec


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, help="reference source tree (the project's checkout)")
    ap.add_argument("--only", nargs="*", help="write only these cases (each case has its own seed)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from benchmark.precision_check import eager_ref  # noqa: E402  (reference oracle)
    import python.modeling_attention as wrapper_mod  # noqa: E402  (reference wrapper)

    ref_root = Path(args.reference).resolve()
    for mod in (wrapper_mod, sys.modules["benchmark.precision_check"]):
        if ref_root not in Path(mod.__file__).resolve().parents:
            raise SystemExit(f"{mod.__name__} was imported from {mod.__file__}, not from {ref_root}")

    torch.manual_seed(0)
    for c in CASES:
        if args.only and c["name"] not in args.only:
            continue
        rec = make_case(c, eager_ref, wrapper_mod)
        path = HERE / f"{c['name']}.npz"
        np.savez_compressed(path, **rec)
        print(f"{path.name}: {path.stat().st_size / 1024:.1f} KiB")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
