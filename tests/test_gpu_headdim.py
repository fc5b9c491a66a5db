"""GPU: head dims 96 and 256 against the oracle, through the public API.

D = 96 runs the D = 128 kernels on tiles whose columns 96..127 the tensor maps fill
with zeros; only the first 96 columns of O, dQ, dK and dV are stored.  The cases cover
each kernel variant that this reaches (dense, causal, GQA, bool mask + fp32 score,
document ids, the split-group and deterministic backward, fp16, BSHD with bottom-right
causal), plus a direct check that nothing is written past column 96 of each output row.

D = 256 runs its own kernels: the forward with one 128-row query slot per CTA, the
backward with a cluster of two CTAs per key tile (one computing S^T, P and dV, the
other dP^T, dS and dK, P crossing through distributed shared memory), and the dQ pass
(used in both backward modes at this head dim) walking each key tile in two 64-key
halves.  The same variants are covered; the deterministic backward is also checked to
repeat bit for bit.

The last test runs head dims 64, 128 and 256 on inputs whose row maxima grow past the
forward's lazy-rescale threshold at every key tile.
"""

from __future__ import annotations

import pytest
import torch

from oracle import inputs as I
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle, run_api  # noqa: F401

from fa2_with_4d_mask_b200 import _lib

pytestmark = pytest.mark.gpu

D = 96


@pytest.mark.parametrize("causal", [False, True])
def test_dense_gqa_odd_length(causal):
    q, k, v, do = I.qkv(2, 333, 333, 8, 2, D, seed=90)
    check(run_api(q, k, v, do, is_causal=causal), oracle(q, k, v, do, causal=causal, device="cpu"), f"D96 c={causal}")


def test_longer_sequence_causal():
    q, k, v, do = I.qkv(1, 2048, 2048, 8, 2, D, seed=91)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True), "D96 T2048")


def test_mask_and_score():
    B, T, H = 1, 640, 4
    q, k, v, do = I.qkv(B, T, T, H, H, D, seed=92)
    mask = I.random_mask(B, H, T, T, 0.9, seed=93)
    score = I.alibi_score(B, H, T, T, seed=94)
    got = run_api(q, k, v, do, mask=mask.to(DEV), score=score.to(DEV))
    check(got, oracle(q, k, v, do, mask=mask, score=score), "D96 mask+score")


def test_document_ids():
    B, T = 2, 768
    q, k, v, do = I.qkv(B, T, T, 4, 1, D, seed=95)
    ids = I.packed_doc_ids(B, T, min_len=100, max_len=300, seed=96)
    got = run_api(q, k, v, do, doc_ids=ids.to(DEV), is_causal=True)
    check(got, oracle(q, k, v, do, mask=I.doc_mask(ids, ids), causal=True), "D96 docs")


@pytest.mark.parametrize("atomic", [True, False])
def test_mqa_bshd_bottom_right_split_and_deterministic(atomic):
    """MQA with few key tiles takes the split-group backward (fp32 slices of width
    128); use_atomic_backward=False takes the deterministic dQ pass."""
    B, Tq, Tk, Hq, Hk = 2, 200, 384, 16, 1
    q, k, v, do = I.qkv(B, Tq, Tk, Hq, Hk, D, seed=97)
    got = run_api(q, k, v, do, layout="bshd", is_causal=True, causal_align="bottom_right",
                  use_atomic_backward=atomic)
    check(got, oracle(q, k, v, do, causal=True, offset=Tk - Tq), f"D96 mqa atomic={atomic}")


def test_fp16():
    q, k, v, do = I.qkv(1, 300, 300, 4, 2, D, seed=98, dtype=torch.float16)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True, device="cpu"), "D96 fp16")


@pytest.mark.parametrize("deterministic", [False, True])
def test_stores_stay_inside_the_head(deterministic):
    """O, dQ, dK and dV written into 96-column views of 128-column buffers: the kernels
    compute 128 columns, and columns 96..127 of every row must keep their sentinel."""
    B, T, Hq, Hk = 1, 300, 4, 2
    bhsd = I.qkv(B, T, T, Hq, Hk, D, seed=99)
    q, k, v, do = (x.transpose(1, 2).to(DEV) for x in bhsd)  # [B, T, H, D]
    sentinel = 7.0

    def wide(H):
        return torch.full((B, T, H, 128), sentinel, dtype=torch.bfloat16, device=DEV)

    o_w, dq_w, dk_w, dv_w = wide(Hq), wide(Hq), wide(Hk), wide(Hk)
    sc = D ** -0.5
    o, lse = _lib.forward(q, k, v, None, None, sc, _lib.CAUSAL_TOP_LEFT, out=o_w[..., :D])
    _lib.backward(do, q, k, v, o, lse, None, None, sc, _lib.CAUSAL_TOP_LEFT, deterministic=deterministic,
                  grads=(dq_w[..., :D], dk_w[..., :D], dv_w[..., :D]))
    torch.cuda.synchronize()
    for name, t in (("O", o_w), ("dQ", dq_w), ("dK", dk_w), ("dV", dv_w)):
        assert (t[..., D:] == sentinel).all(), f"{name} written past column {D}"
        assert torch.isfinite(t[..., :D]).all() and not (t[..., :D] == sentinel).all(), name
    ref = oracle(*bhsd, causal=True, device="cpu")
    got = tuple(t[..., :D].transpose(1, 2) for t in (o_w, dq_w, dk_w, dv_w))
    check(got, ref, "D96 strided outputs")


# ---------------------------------------------------------------- head dim 256
D256 = 256


def _fwd_only(q, k, v, layout="bhsd", **kw):
    """O from the public wrapper without autograd; q/k/v given BHSD."""
    from conftest import from_layout, to_layout
    import tilelang_fa2_4d_mask as api

    with torch.no_grad():
        out = api.tilelang_flash_attention(*(to_layout(x.to(DEV), layout) for x in (q, k, v)), layout=layout, **kw)
    return from_layout(out, layout)


def _check_out(out, ref, what):
    from conftest import out_err
    from test_gpu_parity import O_MAX, O_MEAN

    mx, mean = out_err(out, ref)
    bound = max(O_MEAN, 2.0 ** -8 * float(ref.float().abs().mean()))
    assert mx <= O_MAX and mean <= bound, f"{what} O max_abs={mx:.3e} mean_abs={mean:.3e}"


def _ref_out(q, k, v, mask=None, score=None, causal=False, offset=0):
    from oracle.eager import attention_ref

    return attention_ref(q.float(), k.float(), v.float(), mask, score, scale=q.shape[-1] ** -0.5, is_causal=causal,
                         causal_offset=offset)


@pytest.mark.parametrize("causal", [False, True])
def test_d256_forward_dense_gqa(causal):
    q, k, v, _ = I.qkv(2, 333, 333, 4, 2, D256, seed=100)
    _check_out(_fwd_only(q, k, v, is_causal=causal), _ref_out(q, k, v, causal=causal), f"D256 c={causal}")


def test_d256_forward_long_causal_and_fp16():
    q, k, v, _ = I.qkv(1, 1024, 1024, 8, 2, D256, seed=101)
    _check_out(_fwd_only(q, k, v, is_causal=True), _ref_out(q, k, v, causal=True), "D256 T1024")
    q, k, v, _ = I.qkv(1, 300, 300, 2, 1, D256, seed=102, dtype=torch.float16)
    _check_out(_fwd_only(q, k, v), _ref_out(q, k, v), "D256 fp16")


def test_d256_forward_mask_score_and_docs():
    B, T, H = 1, 640, 4
    q, k, v, _ = I.qkv(B, T, T, H, H, D256, seed=103)
    mask = I.random_mask(B, H, T, T, 0.9, seed=104)
    score = I.alibi_score(B, H, T, T, seed=105)
    _check_out(_fwd_only(q, k, v, mask=mask.to(DEV), score=score.to(DEV)), _ref_out(q, k, v, mask=mask, score=score),
               "D256 mask+score")
    ids = I.packed_doc_ids(B, T, min_len=100, max_len=300, seed=106)
    _check_out(_fwd_only(q, k, v, doc_ids=ids.to(DEV), is_causal=True),
               _ref_out(q, k, v, mask=I.doc_mask(ids, ids), causal=True), "D256 docs")


def test_d256_forward_bshd_bottom_right():
    Tq, Tk = 200, 384
    q, k, v, _ = I.qkv(2, Tq, Tk, 4, 1, D256, seed=107)
    out = _fwd_only(q, k, v, layout="bshd", is_causal=True, causal_align="bottom_right")
    _check_out(out, _ref_out(q, k, v, causal=True, offset=Tk - Tq), "D256 bshd bottom-right")


@pytest.mark.parametrize("causal", [False, True])
def test_d256_backward_dense_gqa_odd_length(causal):
    q, k, v, do = I.qkv(2, 333, 333, 4, 2, D256, seed=110)
    check(run_api(q, k, v, do, is_causal=causal), oracle(q, k, v, do, causal=causal, device="cpu"),
          f"D256 bwd c={causal}")


def test_d256_backward_longer_causal():
    q, k, v, do = I.qkv(1, 1024, 1024, 8, 2, D256, seed=111)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True), "D256 bwd T1024")


def test_d256_backward_mask_and_score():
    B, T, H = 1, 640, 4
    q, k, v, do = I.qkv(B, T, T, H, H, D256, seed=112)
    mask = I.random_mask(B, H, T, T, 0.9, seed=113)
    score = I.alibi_score(B, H, T, T, seed=114)
    got = run_api(q, k, v, do, mask=mask.to(DEV), score=score.to(DEV))
    check(got, oracle(q, k, v, do, mask=mask, score=score), "D256 bwd mask+score")


def test_d256_backward_document_ids():
    B, T = 2, 768
    q, k, v, do = I.qkv(B, T, T, 4, 1, D256, seed=115)
    ids = I.packed_doc_ids(B, T, min_len=100, max_len=300, seed=116)
    got = run_api(q, k, v, do, doc_ids=ids.to(DEV), is_causal=True)
    check(got, oracle(q, k, v, do, mask=I.doc_mask(ids, ids), causal=True), "D256 bwd docs")


def test_d256_backward_mqa_bshd_bottom_right_split():
    """MQA with few key tiles takes the split-group backward (fp32 slices of width 256,
    each CTA of a pair writing its half)."""
    B, Tq, Tk, Hq, Hk = 2, 200, 384, 16, 1
    assert _lib.load_library().fa4d_bwd_group_split(B, Tq, Tk, Hq, Hk, D256, _lib.CAUSAL_BOTTOM_RIGHT) > 1
    q, k, v, do = I.qkv(B, Tq, Tk, Hq, Hk, D256, seed=117)
    got = run_api(q, k, v, do, layout="bshd", is_causal=True, causal_align="bottom_right")
    check(got, oracle(q, k, v, do, causal=True, offset=Tk - Tq), "D256 bwd mqa split")


def test_d256_backward_fp16():
    q, k, v, do = I.qkv(1, 300, 300, 4, 2, D256, seed=118, dtype=torch.float16)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True, device="cpu"), "D256 bwd fp16")


@pytest.mark.parametrize("case", ["dense_causal", "mask_score", "bshd_bottom_right"])
def test_d256_deterministic_backward(case):
    """use_atomic_backward=False at D = 256: the dQ pass over 64-key halves (key
    bound, causal limit, mask words split per half, score), against the oracle and
    bit for bit against a second run."""
    if case == "dense_causal":
        q, k, v, do = I.qkv(2, 333, 333, 4, 2, D256, seed=119)
        kw, ref_kw = dict(is_causal=True), dict(causal=True)
    elif case == "mask_score":
        B, T, H = 1, 400, 2
        q, k, v, do = I.qkv(B, T, T, H, H, D256, seed=120)
        mask = I.random_mask(B, H, T, T, 0.85, seed=121)
        score = I.alibi_score(B, H, T, T, seed=122)
        kw, ref_kw = dict(mask=mask.to(DEV), score=score.to(DEV)), dict(mask=mask, score=score)
    else:
        Tq, Tk = 200, 320
        q, k, v, do = I.qkv(2, Tq, Tk, 8, 1, D256, seed=123)
        kw = dict(layout="bshd", is_causal=True, causal_align="bottom_right")
        ref_kw = dict(causal=True, offset=Tk - Tq)
    a = run_api(q, k, v, do, use_atomic_backward=False, **kw)
    b = run_api(q, k, v, do, use_atomic_backward=False, **kw)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    check(a, oracle(q, k, v, do, device="cpu", **ref_kw), f"D256 deterministic {case}")


@pytest.mark.parametrize("Tq,Tk,causal", [(1, 1, False), (17, 17, True), (1, 257, False), (130, 65, True)])
def test_d256_backward_tiny_and_rectangular(Tq, Tk, causal):
    """Sequences shorter than one 64-key half, a single query row, and Tq > Tk (rows
    that see only part of a tile), in both backward modes."""
    q, k, v, do = I.qkv(1, Tq, Tk, 2, 1, D256, seed=130 + Tq)
    ref = oracle(q, k, v, do, causal=causal, device="cpu")
    for atomic in (True, False):
        got = run_api(q, k, v, do, is_causal=causal, use_atomic_backward=atomic)
        check(got, ref, f"D256 Tq={Tq} Tk={Tk} c={causal} atomic={atomic}")


@pytest.mark.parametrize("T,H,causal", [(8192, 8, 0), (4096, 8, 1)])
def test_d256_backward_repeats_bitwise_at_size(T, H, causal):
    """The D = 256 backward is deterministic in both modes (dK, dV summed in tensor
    memory, dQ from the ordered pass): repeated runs on the same inputs must agree bit
    for bit.  At these sizes the key-tile clusters run many tiles each, which is where a
    hand-back of the received P^T buffer issued before the buffer had been read once
    let the next copy overwrite the first rows of a tile (dK differed from run to run)."""
    g = torch.Generator(device=DEV)
    g.manual_seed(140 + causal)
    mk = lambda: torch.randn((1, T, H, D256), generator=g, device=DEV).to(torch.bfloat16)
    q, k, v, do = mk(), mk(), mk(), mk()
    scale = D256 ** -0.5
    mode = _lib.CAUSAL_TOP_LEFT if causal else _lib.CAUSAL_NONE
    o, lse = _lib.forward(q, k, v, None, None, scale, mode)
    ref = _lib.backward(do, q, k, v, o, lse, None, None, scale, mode)
    for rep in range(3):
        got = _lib.backward(do, q, k, v, o, lse, None, None, scale, mode)
        for name, a, b in zip(("dQ", "dK", "dV"), got, ref):
            assert torch.equal(a, b), f"repeat {rep}: {name} differs"
    assert _lib.device_status(DEV) == 0


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("causal", [False, True])
def test_rescale_when_the_row_max_grows(d, causal):
    """Keys of key tile j scaled by 1 + 3j, so each row's maximum logit grows by far more
    than the forward's lazy-rescale threshold (2^8 in the exp2 domain) from one key tile
    to the next: the running O is rescaled at every tile.  At D = 256 the next tile's S
    is computed before the previous PV, and the rescale first waits for that PV."""
    q, k, v, do = I.qkv(1, 512, 512, 4, 1, d, seed=93)
    factor = (1.0 + 3.0 * (torch.arange(512) // 128).float()).view(1, 1, 512, 1)
    k.mul_(factor.to(k.dtype))  # k is a [B, H, T, D] view; scale its key rows in place
    check(run_api(q, k, v, do, is_causal=causal), oracle(q, k, v, do, causal=causal, device="cpu"),
          f"growing max D{d} c={causal}")
