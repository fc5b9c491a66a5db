"""CPU: the block-occupancy map — the oracle's classification against a direct
per-block loop, the sparsity of the packed-document workload, the key-tile launch
order a prepared mask carries, and the reuse rules of the op's per-mask map cache
(no device work)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import inputs as I
from oracle.blocks import EMPTY, FULL, ORDER_MAX_TILES, PARTIAL, empty_fraction, kb_order_ref, mask_blocks_ref

impl_fa2 = __import__("fa2_with_4d_mask_b200.fa2", fromlist=["x"])


def _loop_blocks(m: np.ndarray, block: int) -> np.ndarray:
    Bm, Hm, Tq, Tk = m.shape
    nqb, nkb = -(-Tq // block), -(-Tk // block)
    out = np.zeros((Bm, Hm, nqb, nkb), dtype=np.uint8)
    for b in range(Bm):
        for h in range(Hm):
            for i in range(nqb):
                for j in range(nkb):
                    t = m[b, h, i * block : (i + 1) * block, j * block : (j + 1) * block] != 0
                    out[b, h, i, j] = FULL if t.all() else (PARTIAL if t.any() else EMPTY)
    return out


@pytest.mark.parametrize("shape", [(1, 1, 5, 7), (2, 3, 130, 257), (1, 2, 256, 384)])
def test_oracle_matches_direct_loop(shape):
    rng = np.random.default_rng(sum(shape))
    # Block-structured values so all three states occur.
    m = rng.random(shape) < 0.5
    Bm, Hm, Tq, Tk = shape
    for i in range(0, Tq, 128):
        for j in range(0, Tk, 128):
            pick = rng.integers(3)
            if pick == 0:
                m[:, :, i : i + 128, j : j + 128] = False
            elif pick == 1:
                m[:, :, i : i + 128, j : j + 128] = True
    for block in (16, 128):
        np.testing.assert_array_equal(mask_blocks_ref(m, block), _loop_blocks(m, block))


def test_oracle_nonzero_bytes_are_true_and_edges_ignore_padding():
    m = np.full((1, 1, 200, 130), 7, dtype=np.uint8)
    b = mask_blocks_ref(m)
    assert b.shape == (1, 1, 2, 2) and (b == FULL).all()
    m[0, 0, 199, 129] = 0
    assert mask_blocks_ref(m)[0, 0, 1, 1] == PARTIAL


def test_packed_document_workload_is_mostly_empty_blocks():
    """The packed-document configuration (B=2, T=4096, documents of 128..1024) leaves
    close to 90% of the 128 x 128 blocks with no True element."""
    m = I.packed_doc_mask(2, 4096, min_len=128, max_len=1024, seed=5).numpy()
    assert empty_fraction(m) > 0.8


def test_block_map_cache_reuse_and_invalidation(monkeypatch):
    calls = []

    def fake(mask):
        calls.append(mask)
        return object()

    monkeypatch.setattr(impl_fa2._lib, "mask_prepare", fake)
    cache = impl_fa2._BlockMapCache(capacity=2)
    base = torch.zeros(1, 1, 8, 8, dtype=torch.bool)
    a = cache.get(base)
    assert cache.get(base) is a and len(calls) == 1
    # A fresh broadcast view of the same tensor reuses the entry of an identical view.
    v1 = base.expand(2, 4, 8, 8)
    m1 = cache.get(v1)
    assert cache.get(base.expand(2, 4, 8, 8)) is m1 and len(calls) == 2
    # An in-place write bumps the version counter: the map is recomputed.
    base[0, 0, 0, 0] = True
    assert cache.get(base) is not a and len(calls) == 3
    # Another tensor with equal shape is never mistaken for the first.
    other = torch.zeros(1, 1, 8, 8, dtype=torch.bool)
    cache.get(other)
    assert len(calls) == 4
    # Capacity bounds the number of entries.
    assert len(cache._entries) == 2
    cache.clear()
    cache.get(other)
    assert len(calls) == 5


def test_bits_oracle_layout():
    rng = np.random.default_rng(3)
    m = rng.random((1, 2, 70, 200)) < 0.5
    from oracle.blocks import mask_bits_ref

    rw, cw = mask_bits_ref(m)
    assert rw.shape == (1, 2, 2, 70, 4) and cw.shape == (1, 2, 2, 200, 2)
    for (h, q, k) in [(0, 0, 0), (1, 69, 199), (1, 33, 130), (0, 5, 127)]:
        word = rw[0, h, k // 128, q, (k % 128) // 32].view(np.uint32)
        assert bool((int(word) >> (k % 32)) & 1) == bool(m[0, h, q, k])
        word = cw[0, h, q // 64, k, (q % 64) // 32].view(np.uint32)
        assert bool((int(word) >> (q % 32)) & 1) == bool(m[0, h, q, k])
    # Flags past Tk / Tq are zero.
    assert (rw[0, :, 1, :, 3] == 0).all() and (cw[0, :, 1, :, 1] == 0).all()
    assert (rw[0, :, 1, :, 2].view(np.uint32) >> 8 == 0).all()


def test_kb_order_oracle_by_hand():
    """Live counts per key tile [2, 0, 3, 2] give ranks 2, 0, 3, 1 (ties by index)."""
    blocks = np.full((1, 1, 3, 4), EMPTY, dtype=np.uint8)
    blocks[0, 0, :2, 0] = PARTIAL
    blocks[0, 0, :, 2] = FULL
    blocks[0, 0, 1:, 3] = PARTIAL
    np.testing.assert_array_equal(kb_order_ref(blocks)[0, 0], [2, 0, 3, 1])
    # An all-EMPTY map keeps index order.
    np.testing.assert_array_equal(kb_order_ref(np.zeros((1, 1, 2, 5), np.uint8))[0, 0], np.arange(5))


def test_kb_order_oracle_rows_and_identity_past_limit():
    rng = np.random.default_rng(7)
    blocks = rng.integers(0, 3, size=(2, 3, 9, 40)).astype(np.uint8)
    got = kb_order_ref(blocks)
    live = (blocks != EMPTY).sum(axis=2)
    nkb = blocks.shape[-1]
    # The same order by a stable sort on one combined key.
    want = np.argsort(-live * (nkb + 1) + np.arange(nkb), axis=-1, kind="stable")
    np.testing.assert_array_equal(got, want)
    for i in range(2):
        for j in range(3):
            assert sorted(got[i, j]) == list(range(nkb))  # a permutation
            assert all(np.diff(live[i, j][got[i, j]]) <= 0)  # counts never rise with rank
    big = np.zeros((1, 2, 1, ORDER_MAX_TILES + 1), np.uint8)
    big[..., -1] = FULL
    np.testing.assert_array_equal(kb_order_ref(big), np.broadcast_to(np.arange(ORDER_MAX_TILES + 1), (1, 2, ORDER_MAX_TILES + 1)))


@pytest.mark.parametrize("dims", [(1, 1, 1, 1), (2, 3, 300, 520), (1, 16, 4096, 4096), (4, 1, 77, 4099)])
def test_prepared_views_match_the_library_layout(dims):
    """The Python views of a prepared-mask buffer (block map, row bits, column bits,
    key-tile order) sit in that order, do not overlap, start on 256-byte boundaries and
    end where the library's own size function says the buffer ends."""
    from fa2_with_4d_mask_b200 import _lib

    Bm, Hm, Tq, Tk = dims
    size = int(_lib.load_library().fa4d_mask_prepare_size(Bm, Hm, Tq, Tk))
    pm = _lib.PreparedMask(torch.empty(size, dtype=torch.uint8), Bm, Hm, Tq, Tk)
    views = [pm.blocks(), pm.row_bits(), pm.col_bits(), pm.kb_order()]
    nqb, nkb, nqt = -(-Tq // 128), -(-Tk // 128), -(-Tq // 64)
    assert [tuple(v.shape) for v in views] == [(Bm, Hm, nqb, nkb), (Bm, Hm, nkb, Tq, 4), (Bm, Hm, nqt, Tk, 2),
                                              (Bm, Hm, nkb)]
    base = pm.buffer.data_ptr()
    spans = [(v.data_ptr() - base, v.data_ptr() - base + v.numel() * v.element_size()) for v in views]
    assert spans[0][0] == 0
    for (s0, e0), (s1, _) in zip(spans, spans[1:]):
        assert s1 % 256 == 0 and s1 >= e0
    assert -(-spans[-1][1] // 256) * 256 == size
