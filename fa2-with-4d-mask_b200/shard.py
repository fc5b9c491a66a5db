"""Sharding of the attention path over ranks (one process per GPU).

The unit of work is one (batch element b, KV head hk) with its G = Hq / Hk query
heads.  O, LSE, dQ, dK and dV of a unit depend only on that unit's Q, K, V, dO and
the matching query-head slices of the mask and the score: the reference's mask and
score are indexed by (batch, query head) (python/fa2.py:43-44) and query head h
reads KV head h // G (python/fa2.py:36, 65).  Units are numbered b * Hk + hk and split
into contiguous ranges of balanced size over the ranks, so a rank's work is a few
(b, KV-head range) segments and the data path needs no exchange.  Collectives are
used only around it: a barrier, the maximum of the per-rank times, and gathering
results for verification.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch


def unit_range(B: int, Hk: int, rank: int, world: int) -> Tuple[int, int]:
    """Units [start, stop) of `rank` among B * Hk units; the first (B*Hk) % world
    ranks take one unit more than the others."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, rem = divmod(B * Hk, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


@dataclass(frozen=True)
class Segment:
    """KV heads [hk0, hk1) of batch element b, with their query heads."""

    b: int
    hk0: int
    hk1: int


def segments(B: int, Hk: int, rank: int, world: int) -> List[Segment]:
    """The rank's units as segments, one per batch element they touch."""
    start, stop = unit_range(B, Hk, rank, world)
    out: List[Segment] = []
    u = start
    while u < stop:
        b, hk = divmod(u, Hk)
        end = min(stop, (b + 1) * Hk)
        out.append(Segment(b, hk, end - b * Hk))
        u = end
    return out


def _head_dim(layout: str) -> int:
    if layout not in ("bhsd", "bshd"):
        raise ValueError(f"unsupported layout: {layout}")
    return 1 if layout == "bhsd" else 2


def _slice(x: torch.Tensor, b: int, h0: int, h1: int, hd: int) -> torch.Tensor:
    idx = [slice(None)] * x.dim()
    idx[0] = slice(b, b + 1)
    idx[hd] = slice(h0, h1)
    return x[tuple(idx)]


def _bias_slice(x: Optional[torch.Tensor], b: int, h0: int, h1: int) -> Optional[torch.Tensor]:
    """[B or 1, Hq or 1, Tq, Tk] mask / score: the segment's batch element and query
    heads; broadcast (size-1) dimensions stay broadcast."""
    if x is None:
        return None
    xb = x[b : b + 1] if x.shape[0] > 1 else x
    return xb[:, h0:h1] if xb.shape[1] > 1 else xb


def slice_inputs(
    seg: Segment,
    Hq: int,
    Hk: int,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    dout: Optional[torch.Tensor] = None,
    mask: Optional[torch.Tensor] = None,
    score: Optional[torch.Tensor] = None,
    layout: str = "bhsd",
) -> tuple:
    """Views of one segment's inputs: (q, k, v, dout, mask, score)."""
    G = Hq // Hk
    hd = _head_dim(layout)
    h0, h1 = seg.hk0 * G, seg.hk1 * G
    return (
        _slice(q, seg.b, h0, h1, hd),
        _slice(k, seg.b, seg.hk0, seg.hk1, hd),
        _slice(v, seg.b, seg.hk0, seg.hk1, hd),
        None if dout is None else _slice(dout, seg.b, h0, h1, hd),
        _bias_slice(mask, seg.b, h0, h1),
        _bias_slice(score, seg.b, h0, h1),
    )


def assemble(
    parts: Sequence[Tuple[Segment, Sequence[torch.Tensor]]],
    Hq: int,
    Hk: int,
    full: Sequence[torch.Tensor],
    kv_heads: Sequence[bool],
    layout: str = "bhsd",
) -> None:
    """Writes per-segment results into full-size tensors: `full[i]` receives tensor i
    of every part, on its query heads (or its KV heads where `kv_heads[i]`)."""
    G = Hq // Hk
    hd = _head_dim(layout)
    for seg, tensors in parts:
        for dst, src, kv in zip(full, tensors, kv_heads):
            h0, h1 = (seg.hk0, seg.hk1) if kv else (seg.hk0 * G, seg.hk1 * G)
            _slice(dst, seg.b, h0, h1, hd).copy_(src)


def max_over_ranks(value: float, dist=None, device: Optional[torch.device] = None) -> float:
    """The maximum of `value` over the ranks of the default process group (the value
    itself without one): the whole job takes as long as its slowest rank."""
    if dist is None or not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def max_units(B: int, Hk: int, world: int) -> int:
    """The most units any rank holds (ranks pad to this for an equal-size gather)."""
    return -(-(B * Hk) // world)


def _unit_views(tensors: Sequence[torch.Tensor], kv_heads: Sequence[bool], G: int, b: int, hk: int, hd: int):
    for t, kv in zip(tensors, kv_heads):
        h0, h1 = (hk, hk + 1) if kv else (hk * G, (hk + 1) * G)
        yield _slice(t, b, h0, h1, hd)


def pack_units(
    tensors: Sequence[torch.Tensor],
    kv_heads: Sequence[bool],
    B: int,
    Hq: int,
    Hk: int,
    rank: int,
    world: int,
    layout: str = "bhsd",
) -> torch.Tensor:
    """One flat buffer holding, unit by unit, the rank's pieces of full-size result
    tensors (each tensor's query heads of the unit, or its KV head where `kv_heads`),
    padded with zeros to max_units units so that every rank sends the same number of
    elements to an all-gather."""
    G = Hq // Hk
    hd = _head_dim(layout)
    start, stop = unit_range(B, Hk, rank, world)
    pieces = []
    for u in range(start, stop):
        b, hk = divmod(u, Hk)
        pieces.extend(v.reshape(-1) for v in _unit_views(tensors, kv_heads, G, b, hk, hd))
    per_unit = sum(t[0:1].numel() // t.shape[hd] * (1 if kv else G) for t, kv in zip(tensors, kv_heads))
    pad = (max_units(B, Hk, world) - (stop - start)) * per_unit
    ref = tensors[0]
    if pad:
        pieces.append(torch.zeros(pad, dtype=ref.dtype, device=ref.device))
    return torch.cat(pieces) if pieces else torch.zeros(0, dtype=ref.dtype, device=ref.device)


def unpack_units(
    gathered: torch.Tensor,
    tensors: Sequence[torch.Tensor],
    kv_heads: Sequence[bool],
    B: int,
    Hq: int,
    Hk: int,
    world: int,
    layout: str = "bhsd",
) -> None:
    """Inverse of pack_units over all ranks: `gathered` is the concatenation of every
    rank's buffer (rank order); each unit's pieces are written into `tensors`."""
    G = Hq // Hk
    hd = _head_dim(layout)
    per_rank = gathered.numel() // world
    for r in range(world):
        off = r * per_rank
        start, stop = unit_range(B, Hk, r, world)
        for u in range(start, stop):
            b, hk = divmod(u, Hk)
            for v in _unit_views(tensors, kv_heads, G, b, hk, hd):
                n = v.numel()
                v.copy_(gathered[off : off + n].view(v.shape))
                off += n


def gather_units(dist, tensors, kv_heads, B: int, Hq: int, Hk: int, layout: str = "bhsd") -> None:
    """All ranks exchange their units of `tensors` (full-size on every rank, each rank
    having filled its own units) so that every rank ends with all of them."""
    world, rank = dist.get_world_size(), dist.get_rank()
    mine = pack_units(tensors, kv_heads, B, Hq, Hk, rank, world, layout)
    if hasattr(dist, "all_gather_into_tensor") and mine.is_cuda:
        out = torch.empty(world * mine.numel(), dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(out, mine)
    else:
        chunks = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(chunks, mine)
        out = torch.cat(chunks)
    unpack_units(out, tensors, kv_heads, B, Hq, Hk, world, layout)
