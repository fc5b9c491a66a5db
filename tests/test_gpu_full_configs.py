"""GPU parity at the exact benchmark shapes of configurations 3, 4 and 5, and the
HF-style adapter on the device.

Each full-size problem runs whole on the kernels; the oracle (fp32) then checks
independent slices of it: a (batch element, KV-head group) unit of the output and
gradients depends only on that unit's Q/K/V/dO and mask/score slices, so checking a
slice against the oracle on the same slice is exact.  The mask and score semantics
follow the reference kernel (python/fa2.py:87-114 forward, :242-280 backward) and its
wrapper (python/modeling_attention.py:115-135, :150-192).
"""

from __future__ import annotations

import pytest
import torch

import tilelang_fa2_4d_mask as api
from gpu_cases import DEV, check, oracle, run_api
from oracle import inputs as I
from oracle.eager import merge_wrapper_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fp32_oracle_and_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    from fa2_with_4d_mask_b200 import _lib

    assert _lib.device_status(DEV) == 0, "a kernel gave up a bounded wait"
    torch.cuda.empty_cache()


def _slice(got, b, hs, ks):
    out, dq, dk, dv = got
    return out[b:b + 1, hs], dq[b:b + 1, hs], dk[b:b + 1, ks], dv[b:b + 1, ks]


def test_config3_full_size_packed_documents():
    """B=2, T=4096, Hq=32, Hk=8, D=128, bf16, one [2, 1, T, T] block-diagonal causal mask
    over seeded documents of length U[128, 1024]; checked on (batch 0, KV group 0) and
    (batch 1, KV group 5)."""
    B, T, Hq, Hk, D = 2, 4096, 32, 8, 128
    q, k, v, do = I.qkv(B, T, T, Hq, Hk, D, seed=31)
    mask = I.packed_doc_mask(B, T, min_len=128, max_len=1024, seed=32)
    got = run_api(q, k, v, do, mask=mask.to(DEV))
    for b, g in ((0, 0), (1, 5)):
        hs, ks = slice(4 * g, 4 * g + 4), slice(g, g + 1)
        ref = oracle(q[b:b + 1, hs], k[b:b + 1, ks], v[b:b + 1, ks], do[b:b + 1, hs], mask=mask[b:b + 1])
        check(_slice(got, b, hs, ks), ref, f"cfg3 full b={b} kv={g}")
    assert all(torch.isfinite(x).all() for x in got)


@pytest.fixture(scope="module")
def cfg4_inputs():
    B, T, H, D = 1, 4096, 16, 128
    q, k, v, do = I.qkv(B, T, T, H, H, D, seed=33)
    bias = I.alibi_score(B, H, T, T, seed=34)
    mask = I.random_mask(B, H, T, T, 0.9, seed=35)
    return q, k, v, do, bias, mask


@pytest.mark.parametrize("spelling", ["score", "attention_mask_scaled"])
def test_config4_full_size_score_and_mask(cfg4_inputs, spelling):
    """B=1, T=4096, Hq=Hk=16, D=128: fp32 ALiBi bias 2^(-8(h+1)/16)(k-q) + N(0, 0.5^2)
    and a per-head Bernoulli(0.9) bool mask with the diagonal kept; the bias given as
    ``score`` or as a float ``attention_mask = bias * scale`` with
    attention_mask_is_scaled=True (the wrapper divides it by scale).  Checked on
    heads 3 and 12."""
    q, k, v, do, bias, mask = cfg4_inputs
    D = q.shape[-1]
    if spelling == "score":
        got = run_api(q, k, v, do, score=bias.to(DEV), mask=mask.to(DEV))
    else:
        am = (bias.to(DEV) * D ** -0.5)
        got = run_api(q, k, v, do, attention_mask=am, mask=mask.to(DEV), attention_mask_is_scaled=True)
        del am
    for h in (3, 12):
        hs = slice(h, h + 1)
        ref = oracle(q[:, hs], k[:, hs], v[:, hs], do[:, hs], mask=mask[:, hs], score=bias[:, hs])
        check(_slice(got, 0, hs, hs), ref, f"cfg4 full {spelling} h={h}")
    assert all(torch.isfinite(x).all() for x in got)


@pytest.mark.parametrize("atomic", [True, False])
def test_config5_full_size_mqa_bshd_bottom_right(atomic):
    """B=16, Tq=1024, Tk=4096, Hq=64, Hk=1, D=64, bf16, layout bshd, causal with the
    diagonal bottom-right aligned (k <= q + Tk - Tq), both backward modes.  Each batch
    element is one unit (all 64 query heads share the single KV head); checked on
    batch elements 5 and 12."""
    B, Tq, Tk, Hq, Hk, D = 16, 1024, 4096, 64, 1, 64
    q, k, v, do = I.qkv(B, Tq, Tk, Hq, Hk, D, seed=36)
    got = run_api(q, k, v, do, layout="bshd", is_causal=True, causal_align="bottom_right",
                  use_atomic_backward=atomic)
    for b in (5, 12):
        ref = oracle(q[b:b + 1], k[b:b + 1], v[b:b + 1], do[b:b + 1], causal=True, offset=Tk - Tq)
        check(_slice(got, b, slice(None), slice(None)), ref, f"cfg5 full atomic={atomic} b={b}")
    assert all(torch.isfinite(x).all() for x in got)


class _Module:
    def __init__(self, is_causal=None):
        if is_causal is not None:
            self.is_causal = is_causal


def _hf(module, q, k, v, do, attention_mask, scaling, **kw):
    """(out, dq, dk, dv) through tilelang_attention_forward, BHSD in and out."""
    qg, kg, vg = (x.detach().to(DEV).requires_grad_(True) for x in (q, k, v))
    out, aux = api.tilelang_attention_forward(module, qg, kg, vg, attention_mask, scaling, **kw)
    assert aux is None
    out.backward(do.to(DEV))
    return out.detach(), qg.grad, kg.grad, vg.grad


def test_hf_adapter_causal_default_and_masks():
    """tilelang_attention_forward (python/modeling_attention.py:150-192) on the device:
    * no attention_mask and a module without ``is_causal`` -> causal (the default);
    * no attention_mask and ``module.is_causal = False`` -> non-causal;
    * an HF-style float additive mask (0 / finfo(bf16).min, causal pattern) -> not
      causal by default; the mask is divided by ``scaling`` and added (scaled form);
    * a bool attention_mask -> non-causal, AND-ed into the keep flags."""
    B, T, Hq, Hk, D = 2, 512, 8, 2, 64
    q, k, v, do = I.qkv(B, T, T, Hq, Hk, D, seed=37)
    scaling = D ** -0.5

    got = _hf(_Module(), q, k, v, do, None, scaling)
    check(got, oracle(q, k, v, do, causal=True), "hf default causal")

    got = _hf(_Module(is_causal=False), q, k, v, do, None, scaling)
    check(got, oracle(q, k, v, do, causal=False), "hf module non-causal")

    keep = torch.ones(T, T, dtype=torch.bool).tril()
    neg = torch.finfo(torch.bfloat16).min
    additive = torch.zeros(B, 1, T, T, dtype=torch.bfloat16).masked_fill(~keep, neg)
    got = _hf(_Module(is_causal=True), q, k, v, do, additive.to(DEV), scaling)
    m, s = merge_wrapper_inputs(batch=B, heads=Hq, seqlen_q=T, seqlen_k=T, scale=scaling, attention_mask=additive)
    check(got, oracle(q, k, v, do, mask=m, score=s), "hf float attention_mask")

    bool_mask = I.random_mask(B, 1, T, T, 0.8, seed=38)
    got = _hf(_Module(is_causal=True), q, k, v, do, bool_mask.to(DEV), scaling)
    check(got, oracle(q, k, v, do, mask=bool_mask.expand(B, Hq, T, T)), "hf bool attention_mask")
