"""CPU: the oracle restatement reproduces the reference's own eager oracle and
wrapper semantics, as recorded in tests/golden by make_golden.py."""

from __future__ import annotations

import pytest
import torch

from conftest import golden_names, load_golden
from oracle import inputs as I
from oracle.eager import attention_ref, attention_ref_grads, bottom_right_mask, merge_wrapper_inputs

# Both sides are fp32 eager math; only summation order differs.
ATOL = 2e-5


def _oracle_inputs(rec):
    m = rec["meta"]
    B, Tq, Tk, Hq = m["B"], m["Tq"], m["Tk"], m["Hq"]
    mask, score = merge_wrapper_inputs(
        batch=B, heads=Hq, seqlen_q=Tq, seqlen_k=Tk, scale=m["scale"],
        mask=rec.get("mask"), score=rec.get("score"), attention_mask=rec.get("attention_mask"),
        attention_mask_is_scaled=m.get("attention_mask_is_scaled", True),
    )
    off = Tk - Tq if m["causal_align"] == "bottom_right" else 0
    is_causal = m["is_causal"] or m["causal_align"] == "bottom_right"
    return mask, score, is_causal, off


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(name):
    rec = load_golden(name)
    mask, score, is_causal, off = _oracle_inputs(rec)
    out, dq, dk, dv = attention_ref_grads(
        rec["q"], rec["k"], rec["v"], rec["dout"], mask, score,
        scale=rec["meta"]["scale"], is_causal=is_causal, causal_offset=off,
    )
    for got, key in ((out, "out"), (dq, "dq"), (dk, "dk"), (dv, "dv")):
        torch.testing.assert_close(got, rec[key], atol=ATOL, rtol=1e-4, msg=f"{name}:{key}")


def test_golden_set_covers_the_semantics():
    metas = [load_golden(n)["meta"] for n in golden_names()]
    assert any(m["is_causal"] and m["causal_align"] == "top_left" for m in metas)
    assert any(m["causal_align"] == "bottom_right" for m in metas)
    assert any(m.get("mask") for m in metas)
    assert any(m.get("score") for m in metas)
    assert any(m.get("attention_mask", "").startswith("float") and m.get("attention_mask_is_scaled") for m in metas)
    assert any(m.get("attention_mask", "").startswith("float") and not m.get("attention_mask_is_scaled", True)
               for m in metas)
    assert any(m.get("attention_mask", "").startswith("bool") for m in metas)
    assert any(m["layout"] == "bshd" for m in metas)
    assert any(m["Tq"] != m["Tk"] for m in metas)
    assert any(m["Tq"] % 128 for m in metas)
    assert {m["D"] for m in metas} >= {64, 96, 128}
    assert any(m["Hq"] > m["Hk"] for m in metas) and any(m["Hk"] == 1 and m["Hq"] > 1 for m in metas)


def test_bottom_right_mask_is_explicit_offset_causal():
    q = torch.randn(1, 2, 5, 8)
    k = torch.randn(1, 2, 9, 8)
    v = torch.randn(1, 2, 9, 8)
    a = attention_ref(q, k, v, bottom_right_mask(5, 9), None, scale=0.3, is_causal=False)
    b = attention_ref(q, k, v, None, None, scale=0.3, is_causal=True, causal_offset=4)
    torch.testing.assert_close(a, b)


def test_row_blocking_does_not_change_results():
    q, k, v = torch.randn(1, 2, 300, 16), torch.randn(1, 1, 200, 16), torch.randn(1, 1, 200, 16)
    a = attention_ref(q, k, v, None, None, scale=0.25, is_causal=True, ref_block=0)
    b = attention_ref(q, k, v, None, None, scale=0.25, is_causal=True, ref_block=64)
    torch.testing.assert_close(a, b)


def test_fully_masked_row_is_nan_like_softmax():
    q, k, v = torch.randn(1, 1, 4, 8), torch.randn(1, 1, 6, 8), torch.randn(1, 1, 6, 8)
    mask = torch.ones(1, 1, 4, 6, dtype=torch.bool)
    mask[0, 0, 2] = False
    out = attention_ref(q, k, v, mask, None, scale=1.0, is_causal=False)
    assert torch.isnan(out[0, 0, 2]).all() and not torch.isnan(out[0, 0, [0, 1, 3]]).any()


def test_doc_mask_matches_block_diagonal_construction():
    """The document-id mask equals the packed-document mask built block by block."""
    ids = I.packed_doc_ids(2, 300, min_len=40, max_len=90, pad=20, seed=9)
    m = I.doc_mask(ids, ids)
    ref = torch.zeros(2, 1, 300, 300, dtype=torch.bool)
    for b in range(2):
        for d in ids[b].unique().tolist():
            if d < 0:
                continue
            idx = (ids[b] == d).nonzero().flatten()
            ref[b, 0, idx.min() : idx.max() + 1, idx.min() : idx.max() + 1] = True
    assert torch.equal(m, ref)
    assert not m[:, :, 280:].any() and not m[:, :, :, 280:].any()
