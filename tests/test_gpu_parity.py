"""GPU parity: the sm_100a kernels, called through the public API (and so through
the C ABI), against the reference-generated golden fixtures and the oracle on the
benchmark configurations.  Tolerances and the error record: tests/gpu_cases.py.
"""

from __future__ import annotations

import pytest
import torch

from conftest import golden_names, load_golden, out_err, rel_err
from gpu_cases import DEV, O_MAX, O_MEAN, check, oracle, run_api  # noqa: F401  (re-exported to other GPU tests)
from oracle import inputs as I
from oracle.eager import bottom_right_mask

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fp32_oracle_and_status():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    from fa2_with_4d_mask_b200 import _lib

    assert _lib.device_status(DEV) == 0, "a kernel gave up a bounded wait"


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", golden_names())
def test_golden(name):
    rec = load_golden(name)
    m = rec["meta"]
    kw = dict(scale=m["scale"], is_causal=m["is_causal"] or m["causal_align"] == "bottom_right",
              causal_align=m["causal_align"], attention_mask_is_scaled=m.get("attention_mask_is_scaled", True))
    for key in ("mask", "score", "attention_mask"):
        if key in rec:
            kw[key] = rec[key].to(DEV)
    got = run_api(rec["q"], rec["k"], rec["v"], rec["dout"], layout=m["layout"], **kw)
    check(got, (rec["out"], rec["dq"], rec["dk"], rec["dv"]), name)


# ---------------------------------------------------------------- benchmark configs
def test_config1_small_gqa_causal():
    q, k, v, do = I.qkv(1, 512, 512, 8, 2, 64, seed=11)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True, device="cpu"), "cfg1")


@pytest.mark.parametrize("causal", [False, True])
def test_config2_shape_at_t1024(causal):
    q, k, v, do = I.qkv(1, 1024, 1024, 32, 8, 128, seed=12)
    check(run_api(q, k, v, do, is_causal=causal), oracle(q, k, v, do, causal=causal), f"cfg2-1k c={causal}")


@pytest.mark.parametrize("causal", [False, True])
def test_config2_full_size_one_kv_group(causal):
    """T=8192, Hq=32, Hk=8: full problem on the kernel, checked on KV group 3
    (query heads 12..15) — groups are independent, so the slice is exact."""
    q, k, v, do = I.qkv(1, 8192, 8192, 32, 8, 128, seed=13)
    out, dq, dk, dv = run_api(q, k, v, do, is_causal=causal)
    hs = slice(12, 16)
    ref = oracle(q[:, hs], k[:, 3:4], v[:, 3:4], do[:, hs], causal=causal)
    check((out[:, hs], dq[:, hs], dk[:, 3:4], dv[:, 3:4]), ref, f"cfg2-8k c={causal}")
    assert torch.isfinite(out).all() and torch.isfinite(dq).all() and torch.isfinite(dk).all()


@pytest.mark.parametrize("case", ["no_causal", "causal", "random_mask"])
def test_reference_precision_check_cases(case):
    """The reference's own correctness run (benchmark/precision_check.sh): B=1, T=8191
    (not a tile multiple), Hq=32, Hk=8, D=128, bf16, forward and backward, cases
    no_causal / causal / random_mask.  The random mask is Bernoulli(0.75) with the
    (q, min(q, Tk-1)) entry kept (precision_check.py:110-117) and comes with an fp32
    score of N(0, 0.1^2) (precision_check.py:128-129); both are drawn on the device, per
    head.  Checked on KV group 3 (query heads 12..15) against the fp32 oracle."""
    T = 8191
    q, k, v, do = I.qkv(1, T, T, 32, 8, 128, seed=21)
    kw, ref_kw = {}, {}
    if case == "causal":
        kw, ref_kw = dict(is_causal=True), dict(causal=True)
    elif case == "random_mask":
        g = torch.Generator(device=DEV)
        g.manual_seed(22)
        mask = torch.rand((1, 32, T, T), generator=g, device=DEV) < 0.75
        qi = torch.arange(T, device=DEV)
        mask[:, :, qi, qi] = True
        score = 0.1 * torch.randn((1, 32, T, T), generator=g, device=DEV)
        kw = dict(mask=mask, score=score)
        ref_kw = dict(mask=mask[:, 12:16], score=score[:, 12:16])
    out, dq, dk, dv = run_api(q, k, v, do, **kw)
    del kw
    hs = slice(12, 16)
    ref = oracle(q[:, hs], k[:, 3:4], v[:, 3:4], do[:, hs], **ref_kw)
    check((out[:, hs], dq[:, hs], dk[:, 3:4], dv[:, 3:4]), ref, f"precision_check {case}")
    assert torch.isfinite(out).all() and torch.isfinite(dq).all() and torch.isfinite(dk).all()


def test_config3_packed_documents():
    B, T = 1, 2048
    q, k, v, do = I.qkv(B, T, T, 8, 2, 128, seed=14)
    mask = I.packed_doc_mask(B, T, min_len=128, max_len=1024, seed=5)
    got = run_api(q, k, v, do, mask=mask.to(DEV))
    check(got, oracle(q, k, v, do, mask=mask), "cfg3")


def test_config4_alibi_score_and_mask_both_spellings():
    B, T, H, D = 1, 1024, 4, 128
    q, k, v, do = I.qkv(B, T, T, H, H, D, seed=15)
    bias = I.alibi_score(B, H, T, T, seed=6)
    mask = I.random_mask(B, H, T, T, 0.9, seed=7)
    ref = oracle(q, k, v, do, mask=mask, score=bias)
    a = run_api(q, k, v, do, score=bias.to(DEV), mask=mask.to(DEV))
    check(a, ref, "cfg4 score")
    scale = D ** -0.5
    b = run_api(q, k, v, do, attention_mask=(bias * scale).to(DEV), mask=mask.to(DEV), attention_mask_is_scaled=True)
    check(b, ref, "cfg4 attention_mask scaled")


@pytest.mark.parametrize("atomic", [True, False])
def test_config5_mqa_bshd_bottom_right(atomic):
    B, Tq, Tk, Hq, Hk, D = 2, 256, 1024, 64, 1, 64
    q, k, v, do = I.qkv(B, Tq, Tk, Hq, Hk, D, seed=16)
    got = run_api(q, k, v, do, layout="bshd", is_causal=True, causal_align="bottom_right",
                  use_atomic_backward=atomic)
    check(got, oracle(q, k, v, do, causal=True, offset=Tk - Tq), "cfg5")


# ---------------------------------------------------------------- edge cases
@pytest.mark.parametrize("T", [1, 17, 127, 129, 255])
@pytest.mark.parametrize("causal", [False, True])
def test_odd_lengths(T, causal):
    q, k, v, do = I.qkv(1, T, T, 2, 1, 64, seed=T)
    check(run_api(q, k, v, do, is_causal=causal), oracle(q, k, v, do, causal=causal, device="cpu"), f"T={T}")


@pytest.mark.parametrize("Tq,Tk", [(100, 300), (300, 100), (1, 257)])
def test_rectangular(Tq, Tk):
    q, k, v, do = I.qkv(1, Tq, Tk, 4, 2, 128, seed=Tq + Tk)
    check(run_api(q, k, v, do), oracle(q, k, v, do, device="cpu"), f"{Tq}x{Tk}")


def test_fp16():
    q, k, v, do = I.qkv(1, 384, 384, 4, 1, 128, seed=21, dtype=torch.float16)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True, device="cpu"), "fp16")


def test_bhsd_contiguous_storage_and_strided_views():
    q, k, v, do = I.qkv(1, 200, 200, 4, 2, 64, seed=22)
    ref = oracle(q, k, v, do, device="cpu")
    check(run_api(q.contiguous(), k.contiguous(), v.contiguous(), do), ref, "bhsd-contiguous")
    big = torch.randn(1, 200, 6, 64).to(torch.bfloat16)
    big[:, :, 1:5] = q.transpose(1, 2)
    check(run_api(big[:, :, 1:5].transpose(1, 2), k, v, do), ref, "head-sliced view")


def test_unaligned_mask_and_score_rows_use_scalar_loads():
    B, T, H = 2, 77, 2
    q, k, v, do = I.qkv(B, T, T, H, H, 64, seed=23)
    mask = I.random_mask(1, 1, T, T, 0.7, seed=8)
    score = torch.randn(B, H, T, T) * 0.3
    check(run_api(q, k, v, do, mask=mask.to(DEV), score=score.to(DEV)),
          oracle(q, k, v, do, mask=mask.expand(B, H, T, T), score=score, device="cpu"), "unaligned")


def test_first_key_tiles_fully_masked():
    """Rows whose first key tiles are all masked (later documents of a packed
    batch) must not produce NaN."""
    T = 512
    q, k, v, do = I.qkv(1, T, T, 2, 1, 64, seed=24)
    mask = torch.zeros(1, 1, T, T, dtype=torch.bool)
    mask[..., 300:, 300:] = True
    mask[..., :300, :300] = True
    got = run_api(q, k, v, do, mask=mask.to(DEV))
    assert torch.isfinite(got[0]).all()
    check(got, oracle(q, k, v, do, mask=mask, device="cpu"), "late docs")


def test_deterministic_forward_and_dkdv():
    q, k, v, do = I.qkv(1, 1024, 1024, 8, 2, 128, seed=25)
    a = run_api(q, k, v, do, is_causal=True)
    b = run_api(q, k, v, do, is_causal=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
    assert rel_err(a[1], b[1]) < 1e-2


def test_bottom_right_equals_explicit_mask():
    q, k, v, do = I.qkv(1, 96, 320, 2, 1, 128, seed=26)
    a = run_api(q, k, v, do, is_causal=True, causal_align="bottom_right")
    b = run_api(q, k, v, do, mask=bottom_right_mask(96, 320).to(DEV))
    assert out_err(a[0], b[0].float())[0] <= 1e-2
    assert rel_err(a[1], b[1]) < 1e-2
