"""GPU: packed sequences given as per-token document ids (no mask tensor).

``fa4d_mask_prepare_docs`` must produce exactly the block map and bits the oracle
derives from the equivalent block-diagonal bool mask; attention with ``doc_ids``
must match the oracle run with that mask; padding tokens (id -1) attend to nothing,
produce zero output and contribute nothing to any gradient, so the valid tokens
match the oracle on the unpadded sequence."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import out_err, rel_err
from fa2_with_4d_mask_b200 import _lib
from oracle import inputs as I
from oracle.blocks import mask_bits_ref, mask_blocks_ref
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle, run_api  # noqa: F401

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,pad", [(2, 1000, 0), (1, 777, 90), (2, 256, 256)])
def test_prepare_docs_matches_oracle(B, T, pad):
    ids = I.packed_doc_ids(B, T, min_len=60, max_len=300, pad=pad, seed=B + T)
    pm = _lib.mask_prepare_docs(ids.to(DEV), ids.to(DEV), B)
    ref = I.doc_mask(ids, ids).numpy()
    np.testing.assert_array_equal(pm.blocks().cpu().numpy(), mask_blocks_ref(ref))
    rw, cw = mask_bits_ref(ref)
    np.testing.assert_array_equal(pm.row_bits().cpu().numpy(), rw)
    np.testing.assert_array_equal(pm.col_bits().cpu().numpy(), cw)


def test_prepare_docs_broadcast_row():
    ids = I.packed_doc_ids(1, 640, min_len=100, max_len=200, seed=3)
    pm = _lib.mask_prepare_docs(ids.to(DEV), ids.to(DEV), 3)
    ref = I.doc_mask(ids, ids).expand(3, 1, 640, 640).numpy()
    np.testing.assert_array_equal(pm.blocks().cpu().numpy(), mask_blocks_ref(ref))


@pytest.mark.parametrize("causal", [False, True])
def test_doc_ids_match_block_diagonal_mask(causal):
    B, T, Hq, Hk, D = 2, 1024, 4, 2, 128
    q, k, v, do = I.qkv(B, T, T, Hq, Hk, D, seed=71)
    ids = I.packed_doc_ids(B, T, min_len=128, max_len=512, seed=72)
    got = run_api(q, k, v, do, doc_ids=ids.to(DEV), is_causal=causal)
    check(got, oracle(q, k, v, do, mask=I.doc_mask(ids, ids), causal=causal), f"doc_ids c={causal}")


def test_doc_ids_with_padding():
    T, valid, Hq, Hk, D = 512, 400, 4, 1, 64
    q, k, v, do = I.qkv(1, T, T, Hq, Hk, D, seed=73)
    ids = I.packed_doc_ids(1, T, min_len=100, max_len=160, pad=T - valid, seed=74)
    out, dq, dk, dv = run_api(q, k, v, do, doc_ids=ids.to(DEV))
    # Padding rows: zero output, zero dQ; padding keys: zero dK, dV.
    assert (out[:, :, valid:] == 0).all() and (dq[:, :, valid:] == 0).all()
    assert (dk[:, :, valid:] == 0).all() and (dv[:, :, valid:] == 0).all()
    # Valid tokens: the oracle on the unpadded sequence.
    s = slice(0, valid)
    ref = oracle(q[:, :, s], k[:, :, s], v[:, :, s], do[:, :, s], mask=I.doc_mask(ids[:, s], ids[:, s]))
    check((out[:, :, s], dq[:, :, s], dk[:, :, s], dv[:, :, s]), ref, "doc_ids padded")


def test_doc_ids_reject_bool_mask():
    q, k, v, do = I.qkv(1, 128, 128, 2, 1, 64, seed=75)
    ids = torch.zeros(1, 128, dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="cannot be combined"):
        run_api(q, k, v, do, doc_ids=ids, mask=torch.ones(1, 1, 128, 128, dtype=torch.bool, device=DEV))
