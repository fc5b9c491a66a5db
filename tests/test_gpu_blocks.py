"""GPU: the mask pre-passes (fa4d_mask_blocks, fa4d_mask_prepare) against the
oracle's block classification and bit layouts, and block-sparse skipping plus
packed-bit mask reads in the forward and backward kernels.

Skipping an EMPTY block removes keys whose probabilities are exactly zero, and a
FULL block is processed like an unmasked one, so results with the block map must
equal results without it bit for bit (O, dK, dV; dQ is accumulated with fp32 adds
in arrival order and is compared by relative error)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import out_err, rel_err
from oracle import inputs as I
from oracle.blocks import EMPTY, FULL, PARTIAL, kb_order_ref, mask_bits_ref, mask_blocks_ref
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle, run_api  # noqa: F401

from fa2_with_4d_mask_b200 import _lib
import fa2_with_4d_mask_b200.fa2 as impl_fa2

pytestmark = pytest.mark.gpu


def _structured_mask(shape, seed):
    """Random mask whose 128 x 128 blocks are randomly all-False, all-True or mixed."""
    rng = np.random.default_rng(seed)
    m = rng.random(shape) < 0.5
    _, _, Tq, Tk = shape
    for i in range(0, Tq, 128):
        for j in range(0, Tk, 128):
            pick = rng.integers(3)
            if pick < 2:
                m[:, :, i : i + 128, j : j + 128] = bool(pick)
    return torch.from_numpy(m)


@pytest.mark.parametrize("shape", [(2, 3, 300, 520), (1, 2, 256, 512), (1, 1, 1, 1), (2, 1, 1000, 4096)])
def test_mask_blocks_match_oracle(shape):
    m = _structured_mask(shape, sum(shape))
    got = _lib.mask_blocks(m.to(DEV)).blocks.cpu().numpy()
    np.testing.assert_array_equal(got, mask_blocks_ref(m.numpy()))


def _check_prepared(mask_dev, ref_mask):
    pm = _lib.mask_prepare(mask_dev)
    np.testing.assert_array_equal(pm.blocks().cpu().numpy(), mask_blocks_ref(ref_mask))
    rw, cw = mask_bits_ref(ref_mask)
    np.testing.assert_array_equal(pm.row_bits().cpu().numpy(), rw)
    np.testing.assert_array_equal(pm.col_bits().cpu().numpy(), cw)
    # Key tiles by decreasing count of non-EMPTY query blocks, ties by index: the order
    # the backward launches its key tiles in.
    np.testing.assert_array_equal(pm.kb_order().cpu().numpy(), kb_order_ref(mask_blocks_ref(ref_mask)))
    return pm


@pytest.mark.parametrize("shape", [(2, 3, 300, 520), (1, 2, 256, 512), (1, 1, 1, 1), (2, 1, 1000, 4096)])
def test_mask_prepare_matches_oracle(shape):
    m = _structured_mask(shape, sum(shape) + 1)
    _check_prepared(m.to(DEV), m.numpy())


def test_mask_prepare_broadcast_uint8_and_unaligned_rows():
    T = 640
    base = I.packed_doc_mask(1, T, min_len=128, max_len=384, seed=31)
    pm = _check_prepared(base.to(DEV).expand(2, 4, T, T), base.numpy())
    assert (pm.Bm, pm.Hm) == (1, 1)
    _check_prepared((base.to(torch.uint8) * 9).to(DEV), base.numpy())
    wide = torch.zeros(1, 1, T, T + 3, dtype=torch.bool)
    wide[..., :T] = base
    _check_prepared(wide.to(DEV)[..., :T], base.numpy())
    odd = _structured_mask((1, 2, 77, 333), 5)
    _check_prepared(odd.to(DEV), odd.numpy())


def test_mask_blocks_broadcast_uint8_and_unaligned_rows():
    T = 640
    base = I.packed_doc_mask(1, T, min_len=128, max_len=384, seed=31)
    bm = _lib.mask_blocks(base.to(DEV).expand(2, 4, T, T))
    assert tuple(bm.blocks.shape) == (1, 1, 5, 5) and bm.strides == (0, 0)
    np.testing.assert_array_equal(bm.blocks.cpu().numpy(), mask_blocks_ref(base.numpy()))
    # Nonzero bytes other than 1 count as True.
    u8 = base.to(torch.uint8) * 9
    np.testing.assert_array_equal(_lib.mask_blocks(u8.to(DEV)).blocks.cpu().numpy(), mask_blocks_ref(base.numpy()))
    # Rows 3 bytes apart from 16-B alignment take the scalar path.
    wide = torch.zeros(1, 1, T, T + 3, dtype=torch.bool)
    wide[..., :T] = base
    view = wide.to(DEV)[..., :T]
    np.testing.assert_array_equal(_lib.mask_blocks(view).blocks.cpu().numpy(), mask_blocks_ref(base.numpy()))


def _raw(q, k, v, do, mask, score=None, causal=_lib.CAUSAL_NONE, blocks=None):
    """fwd + bwd through _lib on [B, T, H, D] device views."""
    t = lambda x: x.transpose(1, 2).to(DEV)
    qd, kd, vd, dod = t(q), t(k), t(v), t(do)
    D = q.shape[-1]
    o, lse = _lib.forward(qd, kd, vd, mask, score, D ** -0.5, causal, blocks=blocks)
    dq, dk, dv = _lib.backward(dod, qd, kd, vd, o, lse, mask, score, D ** -0.5, causal, blocks=blocks)
    return o, dq, dk, dv


@pytest.mark.parametrize("causal", [False, True])
def test_packed_documents_block_sparse(causal):
    B, T, Hq, Hk, D = 2, 1024, 4, 2, 128
    q, k, v, do = I.qkv(B, T, T, Hq, Hk, D, seed=32)
    mask = I.packed_doc_mask(B, T, min_len=128, max_len=512, seed=33)
    states = mask_blocks_ref(mask.numpy())
    assert (states == EMPTY).any() and (states == FULL).any() and (states == PARTIAL).any()
    got = run_api(q, k, v, do, mask=mask.to(DEV), is_causal=causal)
    check(got, oracle(q, k, v, do, mask=mask, causal=causal), f"packed docs c={causal}")


@pytest.mark.parametrize("causal", [_lib.CAUSAL_NONE, _lib.CAUSAL_TOP_LEFT])
def test_mask_paths_are_exact(causal):
    """Three ways to read one mask give bit-identical O, dK and dV: mask bytes with no
    map, mask bytes with the block map (EMPTY blocks skipped), and the prepared packed
    bits with the same map.  FULL blocks are demoted to PARTIAL here so every visited
    block takes the masked path; FULL blocks take the unmasked forward path, whose
    exponent arithmetic rounds differently (checked in test_full_blocks_equal_no_mask)."""
    B, T, Hq, Hk, D = 1, 896, 4, 1, 128
    q, k, v, do = I.qkv(B, T, T, Hq, Hk, D, seed=34)
    mask = I.packed_doc_mask(B, T, min_len=128, max_len=400, seed=35).to(DEV)
    bm = _lib.mask_blocks(mask)
    assert (bm.blocks == EMPTY).any()
    bm.blocks[bm.blocks == FULL] = PARTIAL
    pm = _lib.mask_prepare(mask)
    pm.blocks()[pm.blocks() == FULL] = PARTIAL
    a = _raw(q, k, v, do, mask, causal=causal, blocks=None)
    for blocks in (bm, pm):
        b = _raw(q, k, v, do, mask, causal=causal, blocks=blocks)
        assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
        assert rel_err(b[1].float(), a[1].float()) < 1e-2


def test_full_blocks_equal_no_mask():
    """An all-True mask makes every block FULL: the kernels then read no mask at all
    and give the unmasked results bit for bit (O, dK, dV)."""
    q, k, v, do = I.qkv(1, 512, 512, 4, 2, 128, seed=36)
    mask = torch.ones(1, 1, 512, 512, dtype=torch.bool, device=DEV)
    bm = _lib.mask_blocks(mask)
    assert (bm.blocks == FULL).all()
    a = _raw(q, k, v, do, None)
    for blocks in (bm, _lib.mask_prepare(mask)):
        b = _raw(q, k, v, do, mask, blocks=blocks)
        assert torch.equal(a[0], b[0]) and torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])


def test_per_head_block_sparse_mask_with_score():
    """Each head has its own mask (band, packed documents, all True, dense random),
    combined with an fp32 score: staged mask/score tiles plus per-head skipping."""
    B, T, H, D = 1, 768, 4, 64
    q, k, v, do = I.qkv(B, T, T, H, H, D, seed=37)
    idx = torch.arange(T)
    band = (idx.view(-1, 1) - idx.view(1, -1)).abs() < 100
    docs = I.packed_doc_mask(1, T, min_len=128, max_len=300, seed=38)[0, 0]
    dense = I.random_mask(1, 1, T, T, 0.6, seed=39)[0, 0]
    mask = torch.stack([band, docs, torch.ones(T, T, dtype=torch.bool), dense]).unsqueeze(0)
    score = I.alibi_score(B, H, T, T, seed=40)
    got = run_api(q, k, v, do, mask=mask.to(DEV), score=score.to(DEV))
    check(got, oracle(q, k, v, do, mask=mask, score=score), "per-head masks + score")


def test_fully_masked_query_block_forward():
    """Query rows with no True key at all give NaN, as softmax over all -inf does in
    the oracle; the other rows are unaffected.  (Gradients are not compared for such
    rows: the oracle's NaN probabilities reach every dK/dV entry, whereas the kernels
    never visit the EMPTY blocks.)"""
    T = 512
    q, k, v, do = I.qkv(1, T, T, 2, 1, 64, seed=41)
    mask = torch.ones(1, 1, T, T, dtype=torch.bool)
    mask[..., :128, :] = False
    out, _, _, _ = run_api(q, k, v, do, mask=mask.to(DEV))
    ref = oracle(q, k, v, do, mask=mask)[0]
    assert torch.isnan(out[:, :, :128]).all()
    mx, _ = out_err(out[:, :, 128:], ref[:, :, 128:])
    assert mx <= 2e-2


def test_block_map_is_cached_per_mask():
    q, k, v, do = I.qkv(1, 256, 256, 2, 1, 64, seed=42)
    mask = I.packed_doc_mask(1, 256, min_len=128, max_len=200, seed=43).to(DEV)
    impl_fa2.clear_block_map_cache()
    run_api(q, k, v, do, mask=mask)
    run_api(q, k, v, do, mask=mask)
    assert len(impl_fa2._block_maps._entries) == 1
    mask[..., 0, 0] = False  # in-place write: the next call rescans
    run_api(q, k, v, do, mask=mask)
    assert len(impl_fa2._block_maps._entries) == 2
