"""Multi-rank host logic on CPU: the sharding of (batch, KV head) units over ranks, the
reassembly of per-rank results, the max-over-ranks timing, and what a rank sees when
another rank dies — with world_size-2 `gloo` process groups (no GPU)."""

from __future__ import annotations

import multiprocessing as mp
import queue
import socket

import pytest
import torch

import _dist_workers as W
from fa2_with_4d_mask_b200 import shard
from oracle import inputs as I
from oracle.eager import attention_ref_grads


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world, *args, timeout=120):
    """Runs target(rank, world, port, *args, q) in `world` spawned processes; returns
    what they put on the queue.  Stragglers are killed by their own PID."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    try:
        out.append(q.get(timeout=timeout))
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join(timeout=10)
    return out


@pytest.mark.parametrize("B,Hk,world", [(1, 8, 2), (2, 8, 8), (16, 1, 8), (3, 5, 4), (1, 1, 2), (2, 3, 7)])
def test_units_partition_contiguously_and_evenly(B, Hk, world):
    ranges = [shard.unit_range(B, Hk, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == B * Hk
    assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1
    units = []
    for r in range(world):
        for seg in shard.segments(B, Hk, r, world):
            assert 0 <= seg.hk0 < seg.hk1 <= Hk
            units += [seg.b * Hk + h for h in range(seg.hk0, seg.hk1)]
    assert units == list(range(B * Hk))


def test_benchmark_configs_shard_as_planned():
    """Config 2: 8 units, 1 per GPU at 8 GPUs; configs 3-5: 16 units, 2 per GPU."""
    assert [shard.unit_range(1, 8, r, 8) for r in range(8)] == [(r, r + 1) for r in range(8)]
    for B, Hk in ((2, 8), (1, 16), (16, 1)):
        assert all(shard.unit_range(B, Hk, r, 8)[1] - shard.unit_range(B, Hk, r, 8)[0] == 2 for r in range(8))


def test_sharded_oracle_reassembles_to_the_unsharded_result():
    """Two gloo ranks each compute only their units (GQA, per-head mask, broadcast
    score, causal); the gathered pieces equal the single-process result."""
    B, Tq, Hq, Hk, D = 2, 40, 6, 3, 16
    q, k, v, do = (x.float() for x in I.qkv(B, Tq, Tq, Hq, Hk, D, seed=70))
    mask = I.random_mask(B, Hq, Tq, Tq, 0.8, seed=71)
    score = torch.randn(B, 1, Tq, Tq, generator=torch.Generator().manual_seed(72))
    res = _run(W.sharded_oracle, 2, (q, k, v, do, mask, score), (B, Hq, Hk, True))
    assert res and res[0][0] == "ok", res
    _, gathered, slowest = res[0]
    assert slowest == 20.0  # max over ranks of 10 * (rank + 1)
    full = [torch.full_like(t, float("nan")) for t in (q, q, k, k)]  # out, dq, dk, dv
    shard.assemble([p for parts in gathered for p in parts], Hq, Hk, full, kv_heads=(False, False, True, True))
    ref = attention_ref_grads(q, k, v, do, mask, score, scale=D ** -0.5, is_causal=True)
    for name, got, want in zip(("out", "dq", "dk", "dv"), full, ref):
        assert torch.isfinite(got).all(), name
        torch.testing.assert_close(got, want.float(), rtol=1e-5, atol=1e-5, msg=name)


def test_a_dead_rank_makes_the_next_collective_fail_not_hang():
    res = _run(W.rank_dies, 2, timeout=90)
    assert res, "the surviving rank reported nothing"
    assert res[0][0] == "error", res


@pytest.mark.parametrize("shape,world", [((1, 6, 8, 4, 3), 2), ((3, 5, 6, 1, 2), 2), ((2, 4, 6, 3, 2), 3)])
def test_units_gathered_over_ranks_rebuild_the_full_results(shape, world):
    """The verification gather of the strong-scaling benchmark: each rank packs its
    units (uneven counts are padded), all ranks all-gather, every unit lands back."""
    res = _run(W.gathered_units, world, shape)
    assert res and res[0][0] == "ok", res
    assert res[0][1] is True


@pytest.mark.parametrize("B,Hq,Hk,world", [(1, 32, 8, 8), (16, 64, 1, 8), (3, 6, 3, 4), (2, 4, 1, 3)])
def test_unit_packing_round_trip(B, Hq, Hk, world):
    T, D = 3, 4
    full = [torch.randn(B, T, Hq, D), torch.randn(B, T, Hq, D), torch.randn(B, T, Hk, D)]
    kv = [False, False, True]
    bufs = [shard.pack_units(full, kv, B, Hq, Hk, r, world, "bshd") for r in range(world)]
    assert len({b.numel() for b in bufs}) == 1
    out = [torch.zeros_like(t) for t in full]
    shard.unpack_units(torch.cat(bufs), out, kv, B, Hq, Hk, world, "bshd")
    assert all(torch.equal(a, b) for a, b in zip(out, full))
