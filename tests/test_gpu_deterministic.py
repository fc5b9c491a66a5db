"""GPU: the bit-reproducible backward (use_atomic_backward=False).  dQ comes from a
separate pass in which each query tile walks its key tiles in a fixed order, so two
runs give identical bits; results match the fp32 oracle like the default path."""

from __future__ import annotations

import pytest
import torch

from conftest import rel_err
from oracle import inputs as I
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle, run_api  # noqa: F401

pytestmark = pytest.mark.gpu


def _twice(q, k, v, do, **kw):
    a = run_api(q, k, v, do, use_atomic_backward=False, **kw)
    b = run_api(q, k, v, do, use_atomic_backward=False, **kw)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    return a


@pytest.mark.parametrize("causal", [False, True])
def test_deterministic_gqa(causal):
    q, k, v, do = I.qkv(1, 1024, 1024, 8, 2, 128, seed=81)
    got = _twice(q, k, v, do, is_causal=causal)
    check(got, oracle(q, k, v, do, causal=causal), f"det c={causal}")


@pytest.mark.parametrize("Tq,Tk,D", [(77, 77, 64), (129, 300, 128), (300, 129, 64)])
def test_deterministic_ragged(Tq, Tk, D):
    q, k, v, do = I.qkv(2, Tq, Tk, 4, 2, D, seed=Tq + Tk)
    check(_twice(q, k, v, do), oracle(q, k, v, do, device="cpu"), f"det {Tq}x{Tk}")


def test_deterministic_mask_score_and_docs():
    B, T, H, D = 1, 512, 4, 128
    q, k, v, do = I.qkv(B, T, T, H, H, D, seed=82)
    mask = I.random_mask(B, H, T, T, 0.8, seed=83)
    score = I.alibi_score(B, H, T, T, seed=84)
    check(_twice(q, k, v, do, mask=mask.to(DEV), score=score.to(DEV)), oracle(q, k, v, do, mask=mask, score=score),
          "det mask+score")
    ids = I.packed_doc_ids(B, T, min_len=100, max_len=200, seed=85)
    check(_twice(q, k, v, do, doc_ids=ids.to(DEV), is_causal=True),
          oracle(q, k, v, do, mask=I.doc_mask(ids, ids), causal=True), "det docs")


def test_deterministic_matches_default_path():
    q, k, v, do = I.qkv(1, 768, 768, 4, 4, 64, seed=86)
    a = run_api(q, k, v, do, use_atomic_backward=False)
    b = run_api(q, k, v, do, use_atomic_backward=True)
    assert torch.equal(a[0], b[0])
    for x, y in zip(a[1:], b[1:]):
        assert rel_err(x.float(), y.float()) < 1e-2
