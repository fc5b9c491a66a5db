"""Worker bodies for the multi-process (gloo, CPU) tests; run in spawned processes."""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import tilelang_fa2_4d_mask  # noqa: E402,F401  (registers fa2_with_4d_mask_b200)
from fa2_with_4d_mask_b200 import shard  # noqa: E402
from oracle.eager import attention_ref_grads  # noqa: E402


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def sharded_oracle(rank, world, port, inputs, shape, out_q):
    """Each rank runs the fp32 oracle (forward + gradients) on its own units only; rank
    0 collects every rank's pieces and the max-over-ranks of a per-rank number."""
    try:
        _init(rank, world, port, 60)
        B, Hq, Hk, causal = shape
        q, k, v, do, mask, score = inputs
        parts = []
        for seg in shard.segments(B, Hk, rank, world):
            qs, ks, vs, ds, ms, ss = shard.slice_inputs(seg, Hq, Hk, q, k, v, do, mask, score)
            out = attention_ref_grads(qs, ks, vs, ds, ms, ss, scale=q.shape[-1] ** -0.5, is_causal=causal)
            parts.append((seg, [t.detach() for t in out]))
        gathered = [None] * world
        dist.all_gather_object(gathered, parts)
        slowest = shard.max_over_ranks(10.0 * (rank + 1), dist)
        if rank == 0:
            out_q.put(("ok", gathered, slowest))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the test, never swallowed silently
        out_q.put(("error", f"rank {rank}: {type(e).__name__}: {e}", None))


def rank_dies(rank, world, port, out_q):
    """Rank 1 exits between steps, before the next collective; rank 0 must get an
    error from that collective (peer gone or the group's short timeout), not hang."""
    _init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        out_q.put(("no error", None))
    except Exception as e:
        out_q.put(("error", type(e).__name__))


def gathered_units(rank, world, port, shape, out_q):
    """Each rank fills only its own units of full-size result tensors (the others stay
    NaN), then gather_units exchanges them; rank 0 reports what it ends with."""
    try:
        _init(rank, world, port, 60)
        B, T, Hq, Hk, D = shape
        g = torch.Generator().manual_seed(80)
        ref = [torch.randn(B, T, Hq, D, generator=g), torch.randn(B, T, Hk, D, generator=g)]
        kv = [False, True]
        local = [torch.full_like(t, float("nan")) for t in ref]
        G = Hq // Hk
        for seg in shard.segments(B, Hk, rank, world):
            for dst, src, is_kv in zip(local, ref, kv):
                h0, h1 = (seg.hk0, seg.hk1) if is_kv else (seg.hk0 * G, seg.hk1 * G)
                dst[seg.b : seg.b + 1, :, h0:h1].copy_(src[seg.b : seg.b + 1, :, h0:h1])
        shard.gather_units(dist, local, kv, B, Hq, Hk, layout="bshd")
        if rank == 0:
            out_q.put(("ok", all(torch.equal(a, b) for a, b in zip(local, ref)), None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        out_q.put(("error", f"rank {rank}: {type(e).__name__}: {e}", None))
