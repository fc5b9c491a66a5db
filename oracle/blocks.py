"""ORACLE — test infrastructure only: CPU restatement of the block-occupancy map
the kernels use to skip work under a 4D bool mask.

The reference has no such map: its forward and backward visit every 128-key tile
and apply the mask per element (python/fa2.py:95-124 and :242-302), so skipping an
EMPTY block (no True element) must not change any result, and a FULL block (every
in-bounds element True) must behave exactly like an unmasked one.  This module
states the classification the GPU pre-pass must reproduce bit for bit, and the
fraction of blocks the packed-document workload leaves EMPTY.
"""

from __future__ import annotations

import numpy as np

BLOCK = 128
EMPTY, PARTIAL, FULL = 0, 1, 2


def mask_blocks_ref(mask, block: int = BLOCK) -> np.ndarray:
    """mask: [Bm, Hm, Tq, Tk] bool (or integer, nonzero = True).  Returns uint8
    [Bm, Hm, ceil(Tq/block), ceil(Tk/block)] with EMPTY / PARTIAL / FULL, judged on
    the in-bounds elements of each block only."""
    m = np.asarray(mask) != 0
    Bm, Hm, Tq, Tk = m.shape
    nqb, nkb = -(-Tq // block), -(-Tk // block)
    # Padding is False for "any" and True for "all", so it never changes a state.
    any_pad = np.zeros((Bm, Hm, nqb * block, nkb * block), dtype=bool)
    all_pad = np.ones_like(any_pad)
    any_pad[:, :, :Tq, :Tk] = m
    all_pad[:, :, :Tq, :Tk] = m
    shape = (Bm, Hm, nqb, block, nkb, block)
    has_any = any_pad.reshape(shape).any(axis=(3, 5))
    has_all = all_pad.reshape(shape).all(axis=(3, 5))
    out = np.full((Bm, Hm, nqb, nkb), PARTIAL, dtype=np.uint8)
    out[~has_any] = EMPTY
    out[has_all] = FULL
    return out


ORDER_MAX_TILES = 1024


def kb_order_ref(blocks: np.ndarray) -> np.ndarray:
    """The key-tile order a prepared mask stores for the backward's launch: for each
    (b, h) row of the block map [Bm, Hm, nqb, nkb], the key tiles sorted by decreasing
    count of non-EMPTY query blocks, ties by ascending key-tile index; the identity
    when nkb exceeds ORDER_MAX_TILES.  Returns int32 [Bm, Hm, nkb] with entry r = the
    key tile launched at rank r.  The order is this library's own launch schedule (the
    reference launches key tiles in index order, python/fa2.py:242-302); it changes no
    result, only which CTAs start first."""
    b = np.asarray(blocks)
    Bm, Hm, _, nkb = b.shape
    if nkb > ORDER_MAX_TILES:
        return np.broadcast_to(np.arange(nkb, dtype=np.int32), (Bm, Hm, nkb)).copy()
    live = (b != EMPTY).sum(axis=2)  # [Bm, Hm, nkb]
    out = np.empty((Bm, Hm, nkb), dtype=np.int32)
    for i in range(Bm):
        for j in range(Hm):
            out[i, j] = sorted(range(nkb), key=lambda kb: (-int(live[i, j, kb]), kb))
    return out


def empty_fraction(mask, block: int = BLOCK) -> float:
    """Share of blocks with no True element."""
    b = mask_blocks_ref(mask, block)
    return float((b == EMPTY).mean())


def _pack32(flags: np.ndarray) -> np.ndarray:
    """Packs the last axis (a multiple of 32 booleans) into int32 words, bit j of
    word w = flag 32*w + j."""
    f = flags.astype(np.uint64).reshape(*flags.shape[:-1], -1, 32)
    words = (f << np.arange(32, dtype=np.uint64)).sum(axis=-1)
    return words.astype(np.uint32).view(np.int32)


def mask_bits_ref(mask):
    """The packed-bit layouts of a prepared mask [Bm, Hm, Tq, Tk]:
    row bits [Bm, Hm, ceil(Tk/128), Tq, 4] (word w of (kt, q) = keys 128kt+32w+0..31)
    and column bits [Bm, Hm, ceil(Tq/64), Tk, 2] (word w of (qt, k) = queries
    64qt+32w+0..31), flags past Tk / Tq zero."""
    m = np.asarray(mask) != 0
    Bm, Hm, Tq, Tk = m.shape
    nkb, nqt = -(-Tk // BLOCK), -(-Tq // 64)
    rows = np.zeros((Bm, Hm, Tq, nkb * BLOCK), dtype=bool)
    rows[..., :Tk] = m
    rw = _pack32(rows).reshape(Bm, Hm, Tq, nkb, 4).transpose(0, 1, 3, 2, 4)
    cols = np.zeros((Bm, Hm, Tk, nqt * 64), dtype=bool)
    cols[..., :Tq] = m.transpose(0, 1, 3, 2)
    cw = _pack32(cols).reshape(Bm, Hm, Tk, nqt, 2).transpose(0, 1, 3, 2, 4)
    return np.ascontiguousarray(rw), np.ascontiguousarray(cw)
