#!/usr/bin/env python
"""Benchmark of the attention hot path on B200: one JSON line on rank 0.

Workload (a "step"): one forward + backward of FlashAttention-2 at the reference's
headline configuration B=1, Tq=Tk=8192, Hq=32, Hk=8, D=128, bf16, non-causal, no
mask/score (synthetic N(0,1) inputs), per GPU.  Multi-GPU runs are weak-scaled:
rank r owns batch element r of a global batch of N (whole GQA groups, no data-path
collective); NCCL is used only for the barrier, the max-over-ranks timing and a
verification all-gather of per-rank output checksums outside the timed region.

``value`` is whole-job TFLOP/s under the reference's FLOP convention
(14 * B * Hq * Tq * Tk * D per fwd+bwd, benchmark/throughput_check.py:85-92) with
inputs resident in HBM; ``e2e`` is the same metric through the public API
(``tilelang_flash_attention`` + autograd) with pinned host inputs and outputs,
host<->device copies inside the timed region.  ``--impl reference`` times the
reference's own CPU path (its fp32 eager attention, restated in oracle/eager.py)
on the host cores.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
(torchrun for N > 1).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "attn fwd & fwd+bwd TFLOPS/B200 (bf16 T8192 Hq32 Hk8 D128), % tensor/HBM roof"
UNIT = "TFLOP/s"
B, T, HQ, HK, D = 1, 8192, 32, 8, 128
WORKLOAD = "cfg2: B1 Tq=Tk=8192 Hq32 Hk8 D128 bf16 non-causal, fwd+bwd per GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per launch of the backward main kernel at this workload,
# dram__bytes_read.sum + dram__bytes_write.sum from one ncu capture of this bench
# command, and the commit of the kernel code that capture measured.
NCU_BWD_MAIN_TRAFFIC = 545651712
NCU_BWD_MAIN_TRAFFIC_CODE = "369d887"
L2_FLUSH_BYTES = 256 << 20


def median_ms(pairs):
    """Median elapsed time (ms) of a list of (start, end) CUDA events."""
    return statistics.median(a.elapsed_time(b) for a, b in pairs)


def fwd_flops(b, hq, tq, tk, d, causal):
    return 4.0 * b * hq * tq * tk * d * (0.5 if causal else 1.0)


def fwd_bwd_flops(b, hq, tq, tk, d, causal):
    return 14.0 * b * hq * tq * tk * d * (0.5 if causal else 1.0)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling every 200 ms while the timed region runs."""

    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        self.proc = None
        self.out = None
        self.error = None
        props = torch.cuda.get_device_properties(device)
        self.bus = getattr(props, "pci_bus_id", None)
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.out, stderr=subprocess.STDOUT)
        except Exception as e:  # no nvidia-smi
            self.proc = None
            self.error = f"{type(e).__name__}: {e}"

    @staticmethod
    def _bus_of(field: str):
        try:  # "00000000:1B:00.0" -> 0x1B
            return int(field.split(":")[1], 16)
        except (IndexError, ValueError):
            return None

    def stop(self):
        if self.proc is None:
            return {"error": self.error or "nvidia-smi not started"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.flush()
        text = Path(self.out.name).read_text()
        os.unlink(self.out.name)
        rows = [[x.strip() for x in r.split(",")] for r in text.strip().splitlines() if r.strip()]
        buses = {self._bus_of(r[0]) for r in rows if len(r) >= 9}
        sm, mx, reasons = [], [], set()
        for r in rows:
            if len(r) < 9:
                continue
            if len(buses) > 1 and self.bus is not None and self._bus_of(r[0]) != self.bus:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"error": "no samples: " + text.strip()[:200]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- NUMA placement
def numa_bind(device: torch.device) -> dict:
    """Runs this process on the CPUs of the GPU's NUMA node, so that its pinned host
    buffers (allocated afterwards, first touch) sit next to the GPU's PCIe root."""
    props = torch.cuda.get_device_properties(device)
    bus = getattr(props, "pci_bus_id", None)
    dom = getattr(props, "pci_domain_id", 0) or 0
    dev_id = getattr(props, "pci_device_id", 0) or 0
    if bus is None:
        return {"applied": False, "why": "no PCI id"}
    try:
        node = int(Path(f"/sys/bus/pci/devices/{dom:04x}:{bus:02x}:{dev_id:02x}.0/numa_node").read_text())
        if node < 0:
            return {"applied": False, "why": "no NUMA node reported"}
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return {"applied": False, "node": node, "why": "no allowed CPU on the node"}
        os.sched_setaffinity(0, cpus)
        return {"applied": True, "node": node, "cpus": len(cpus)}
    except (OSError, ValueError) as e:
        return {"applied": False, "why": f"{type(e).__name__}"}


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    from fa2_with_4d_mask_b200 import _lib  # noqa: E402  (registered by the import below)
    return _run_ours(args, _lib)


def _run_ours(args, _lib):
    import tilelang_fa2_4d_mask as api
    from fa2_with_4d_mask_b200 import shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    numa = numa_bind(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist

        # NCCL writes its version banner to stdout at INFO/VERSION levels; keep stdout
        # to the one JSON line unless the caller asked for NCCL logs.
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks, peak_src = load_peaks()

    # Rank r owns batch element r of the global batch (weak scaling): with B = 1 per
    # rank, the rank's (batch, KV head) units are exactly that element's KV heads.
    (seg,) = shard.segments(world * B, HK, rank, world)
    assert (seg.b, seg.hk0, seg.hk1) == (rank * B, 0, HK)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + seg.b)
    mk = lambda shape: torch.randn(shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q = mk((B, T, HQ, D))
    k = mk((B, T, HK, D))
    v = mk((B, T, HK, D))
    do = mk((B, T, HQ, D))
    scale = D ** -0.5
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    ev = lambda: torch.cuda.Event(enable_timing=True)

    def measure(mode):
        """One causal mode of the workload: per-stage medians of eager launches with
        events around each stage, then the medians of `steps` graph replays of the
        whole step (fwd + the backward's launches) and of the forward alone, with L2
        flushed before each replay (outside its events)."""
        rec = {"fwd": [], "preprocess": [], "main": [], "dq_convert": [], "step": []}

        def step(timed, events=True):
            if not events:  # the step as captured into the CUDA graph
                o, lse = _lib.forward(q, k, v, None, None, scale, mode)
                _lib.backward(do, q, k, v, o, lse, None, None, scale, mode)
                return o
            e0, e1 = ev(), ev()
            e0.record(stream)
            o, lse = _lib.forward(q, k, v, None, None, scale, mode)
            e1.record(stream)
            marks = []

            def stage(name, launch):
                a, b = ev(), ev()
                a.record(stream)
                launch()
                b.record(stream)
                marks.append((name, a, b))

            _lib.backward(do, q, k, v, o, lse, None, None, scale, mode, stages=stage)
            if timed:
                rec["fwd"].append((e0, e1))
                for name, a, b in marks:
                    rec[name].append((a, b))
                rec["step"].append((e0, marks[-1][2]))
            return o

        for _ in range(args.warmup):
            step(False)
        torch.cuda.synchronize(dev)
        for _ in range(min(args.steps, 10)):
            flush.zero_()
            step(True)
        torch.cuda.synchronize(dev)
        # Graph replays, so host-side launch work cannot leave gaps between the kernels.
        graph, fgraph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            o = step(False, events=False)
        with torch.cuda.graph(fgraph):
            _lib.forward(q, k, v, None, None, scale, mode)
        for _ in range(args.warmup):
            graph.replay()
            fgraph.replay()
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        steps_ev, fwd_ev = [], []
        for g_, out_ in ((graph, steps_ev), (fgraph, fwd_ev)):
            for _ in range(args.steps):
                flush.zero_()  # L2 flush between steps, outside the step's events
                a, b = ev(), ev()
                a.record(stream)
                g_.replay()
                b.record(stream)
                out_.append((a, b))
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ms = {k2: median_ms(v2) for k2, v2 in rec.items()}
        ms["step_eager"] = ms.pop("step")
        ms["step"] = median_ms(steps_ev)
        ms["fwd_graph"] = median_ms(fwd_ev)
        del graph, fgraph
        return ms, o

    sampler = ClockSampler(dev) if rank == 0 else None  # started early: nvidia-smi needs ~0.5 s to begin
    ms, o = measure(_lib.CAUSAL_NONE)
    ms_causal, _ = measure(_lib.CAUSAL_TOP_LEFT)
    clocks = sampler.stop() if sampler else None

    t_step = shard.max_over_ranks(ms["step"], dist, dev)
    t_fwd = shard.max_over_ranks(ms["fwd_graph"], dist, dev)
    t_step_causal = shard.max_over_ranks(ms_causal["step"], dist, dev)
    t_fwd_causal = shard.max_over_ranks(ms_causal["fwd_graph"], dist, dev)
    if dist:
        # Verification only (outside the timed region): per-rank output checksums.
        chk = o.float().abs().sum().reshape(1)
        allchk = [torch.zeros_like(chk) for _ in range(world)]
        dist.all_gather(allchk, chk)
        if rank == 0 and not all(torch.isfinite(c).all() for c in allchk):
            raise SystemExit("non-finite output on some rank")
    per_rank = fwd_bwd_flops(B, HQ, T, T, D, False)
    value = world * per_rank / (t_step * 1e-3) / 1e12
    status = _lib.device_status(dev)
    # End-to-end leg on every rank (each rank its own host batch element), max over ranks.
    e2e = run_e2e(api, dev, args, dist, world) if args.e2e_steps > 0 else None
    copies = copy_leg(dev, dist, world) if args.e2e_steps > 0 else None
    strong = strong_leg(_lib, dev, dist, world, rank, min(args.steps, 20), args.warmup) if args.strong else None

    if rank != 0:
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return None

    bwd_main_flops = fwd_bwd_flops(B, HQ, T, T, D, False) - fwd_flops(B, HQ, T, T, D, False)
    main_tflops = bwd_main_flops / (ms["main"] * 1e-3) / 1e12
    fwd_tflops = fwd_flops(B, HQ, T, T, D, False) / (t_fwd * 1e-3) / 1e12
    peak = peaks["bf16_tflops"]
    c_fwd = fwd_flops(B, HQ, T, T, D, True) / (t_fwd_causal * 1e-3) / 1e12
    c_fb = fwd_bwd_flops(B, HQ, T, T, D, True) / (t_step_causal * 1e-3) / 1e12
    c_main = (fwd_bwd_flops(B, HQ, T, T, D, True) - fwd_flops(B, HQ, T, T, D, True)) / (ms_causal["main"] * 1e-3) / 1e12
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1) inputs, seeded per rank",
        "config": {
            "workload": WORKLOAD,
            "global_batch": world * B,
            "seq_len": T,
            "heads_q": HQ,
            "heads_kv": HK,
            "head_dim": D,
            "parallelism": f"dp{world} (batch shards, whole GQA groups per GPU, no data-path collective)",
            "l2": "flushed between steps (256 MiB write outside the step's events)",
        },
        "fwd_tflops": round(fwd_tflops, 2),
        "fwd_frac_of_peak": round(fwd_tflops / peak, 4),
        "fwd_bwd_frac_of_peak": round(value / world / peak, 4),
        "kernel_ms": {k2: round(v2, 4) for k2, v2 in ms.items() if k2 not in ("step", "step_eager")},
        "step_ms_eager_launches": round(ms["step_eager"], 4),
        # The same workload with top-left causal masking, measured the same way (graph
        # replays, L2 flushed, median of `steps`; FLOPs x0.5 by the convention).
        "causal": {
            "fwd_ms": round(t_fwd_causal, 4), "fwd_tflops": round(c_fwd, 2), "fwd_frac_of_peak": round(c_fwd / peak, 4),
            "fwd_bwd_ms": round(t_step_causal, 4), "fwd_bwd_tflops": round(world * c_fb, 2),
            "fwd_bwd_frac_of_peak": round(c_fb / peak, 4),
            "bwd_main_ms": round(ms_causal["main"], 4), "bwd_main_frac_of_peak": round(c_main / peak, 4),
            "kernel_ms": {k2: round(v2, 4) for k2, v2 in ms_causal.items() if k2 not in ("step", "step_eager")},
        },
        "timing": "median over `steps` of CUDA events around graph replays of the whole step (value) and of "
                  "the forward alone (fwd_tflops), L2 flushed before each replay; per-kernel times are medians "
                  "of 10 eager steps with events around each stage",
        # The same figures against the measured sustained GEMM peak: these loops run for
        # tens to hundreds of ms, and the forward alone slows by about 10% after its first
        # ~60 ms of back-to-back launches (eager and graph alike) under the power cap.
        "sustained_peak": {
            "peak": peaks["bf16_tflops_sustained"],
            "fwd_frac": round(fwd_tflops / peaks["bf16_tflops_sustained"], 4),
            "fwd_bwd_frac": round(value / world / peaks["bf16_tflops_sustained"], 4),
            "bwd_main_frac": round(main_tflops / peaks["bf16_tflops_sustained"], 4),
            "causal_fwd_frac": round(c_fwd / peaks["bf16_tflops_sustained"], 4),
            "causal_fwd_bwd_frac": round(c_fb / peaks["bf16_tflops_sustained"], 4),
        },
        "roofline": {
            "kernel": "bwd_kernel<128,bf16> (fa4d_bwd_main)",
            "bound": "tensor",
            "achieved": round(main_tflops, 2),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(main_tflops / peak, 4),
            "peak_source": f"{peak_src} bf16_tflops (burst, MEASURED_PEAKS.json)" if peak_src == "measured"
            else "fallback 1590 TFLOP/s",
            "algorithmic": "10*B*Hq*Tq*Tk*D FLOP per launch (bwd share of the 14x convention)",
            "traffic": NCU_BWD_MAIN_TRAFFIC,
            "traffic_source": f"ncu dram__bytes_read.sum + dram__bytes_write.sum, one capture of this command "
                              f"on kernel code {NCU_BWD_MAIN_TRAFFIC_CODE}",
        },
        # fwd, preprocess, main, dQ convert, plus the split-slice sum when the
        # backward's group split is on for this workload.
        "gpu_launches": (4 + (_lib.load_library().fa4d_bwd_group_split(B, T, T, HQ, HK, D, _lib.CAUSAL_NONE) > 1))
        * args.steps,
        "device_status": status,
        "clocks": clocks,
    }
    if args.extra and world == 1:
        line["extra"] = extra_measurements(_lib, dev, peaks)
        line["extra"]["library_context_cfg2"] = library_context(dev, peaks)
    if e2e is not None:
        line["e2e"] = e2e
    if copies is not None:
        line["host_copies"] = copies
    line["numa"] = numa
    if strong is not None:
        line["strong_scaling"] = strong
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


_FLUSH = {}


def time_fn(fn, iters=10, warm=3):
    """Median ms of `iters` calls of fn after `warm` untimed ones, CUDA events on the
    current stream, L2 flushed (a 256 MiB write) before each timed call."""
    dev = torch.cuda.current_device()
    if dev not in _FLUSH:
        _FLUSH[dev] = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush = _FLUSH[dev]
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return median_ms(evs)


def _dev_inputs(dev, b, tq, tk, hq, hk, d, seed):
    """Seeded N(0,1) bf16 BHSD views over [B, T, H, D] storage, generated on the device."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    mk = lambda t, h: torch.randn((b, t, h, d), generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)
    return mk(tq, hq), mk(tk, hk), mk(tk, hk), mk(tq, hq)


def _alibi_score(dev, b, h, tq, tk, seed=3):
    """fp32 [B, H, Tq, Tk] = 2^(-8(h+1)/H) * (k - q) + N(0, 0.5^2)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    slopes = torch.tensor([2.0 ** (-8.0 * (i + 1) / h) for i in range(h)], device=dev).view(1, h, 1, 1)
    rel = (torch.arange(tk, device=dev).view(1, 1, 1, tk) - torch.arange(tq, device=dev).view(1, 1, tq, 1)).float()
    return slopes * rel + 0.5 * torch.randn((b, h, tq, tk), generator=g, device=dev)


def _bernoulli_mask(dev, b, h, tq, tk, keep, seed=4):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    m = torch.rand((b, h, tq, tk), generator=g, device=dev) < keep
    i = torch.arange(min(tq, tk), device=dev)
    m[:, :, i, i] = True
    return m


def _packed_doc_mask(dev, b, t, lo=128, hi=1024, seed=2):
    """[B, 1, T, T]: causal inside seeded documents of length U[lo, hi], False across."""
    g = torch.Generator()
    g.manual_seed(seed)
    doc = torch.empty((b, t), dtype=torch.int32)
    for bi in range(b):
        s, n = 0, 0
        while s < t:
            ln = int(torch.randint(lo, hi + 1, (1,), generator=g))
            doc[bi, s:s + ln] = n
            s, n = s + ln, n + 1
    doc = doc.to(dev)
    same = doc[:, :, None] == doc[:, None, :]
    causal = torch.ones((t, t), dtype=torch.bool, device=dev).tril()
    return (same & causal).unsqueeze(1)


def extra_measurements(_lib, dev, peaks):
    """The other benchmark configurations, a few iterations each (context, not `value`)."""
    out = {}
    peak = peaks["bf16_tflops"]

    def fb(b, tq, tk, hq, hk, d, causal_mode, mask=None, score=None, iters=10, deterministic=False):
        """(fwd ms, bwd ms) with the mask prepared once beforehand (block map + packed bits,
        as the op caches it per mask); the preparation itself is timed by map_ms()."""
        q, k, v, do = (x.transpose(1, 2) for x in _dev_inputs(dev, b, tq, tk, hq, hk, d, seed=3))
        sc = d ** -0.5
        bm = _lib.mask_prepare(mask) if mask is not None else None
        tf = time_fn(lambda: _lib.forward(q, k, v, mask, score, sc, causal_mode, blocks=bm), iters)
        o, lse = _lib.forward(q, k, v, mask, score, sc, causal_mode, blocks=bm)
        tb = time_fn(lambda: _lib.backward(do, q, k, v, o, lse, mask, score, sc, causal_mode, blocks=bm,
                                           deterministic=deterministic), iters)
        return tf, tb

    hbm = peaks["hbm_gbs"]

    def map_ms(mask):
        return round(time_fn(lambda: _lib.mask_prepare(mask)), 4)

    def tensor_bytes(b, tq, tk, hq, hk, d):
        """(fwd, bwd) bytes of the dense tensors: fwd reads Q, K, V and writes O and LSE;
        bwd reads Q, K, V, O, dO, LSE and writes dQ, dK, dV (2-byte elements)."""
        qb, kb, lse = 2 * b * tq * hq * d, 2 * b * tk * hk * d, 4 * b * hq * tq
        return 2 * qb + 2 * kb + lse, 3 * qb + 2 * kb + lse + qb + 2 * kb

    tf, tb = fb(B, T, T, HQ, HK, D, _lib.CAUSAL_NONE, deterministic=True)
    fbf = fwd_bwd_flops(B, HQ, T, T, D, False)
    out["cfg2_deterministic_bwd"] = {"fwd_bwd_ms": round(tf + tb, 4), "bwd_ms": round(tb, 4),
                                     "fwd_bwd_tflops": round(fbf / (tf + tb) / 1e9, 1),
                                     "fwd_bwd_frac": round(fbf / (tf + tb) / 1e9 / peak, 4)}
    # cfg4: ALiBi-style fp32 score + Bernoulli(0.9) bool mask, MHA, non-causal (HBM-bound)
    b4, t4, h4 = 1, 4096, 16
    score = _alibi_score(dev, b4, h4, t4, t4)
    mask = _bernoulli_mask(dev, b4, h4, t4, t4, 0.9)
    tf, tb = fb(b4, t4, t4, h4, h4, D, _lib.CAUSAL_NONE, mask=mask, score=score)
    prep = map_ms(mask)
    tfw, tbw = tensor_bytes(b4, t4, t4, h4, h4, D)
    sm = score.numel() * 4 + mask.numel()
    bits = 2 * mask.numel() // 8  # the prepared row bits (forward) and column bits (backward)
    bytes_fwd = sm + tfw
    bytes_fb = 2 * sm + tfw + tbw
    moved_fwd = score.numel() * 4 + bits // 2 + tfw  # the forward reads the row bits, not the mask bytes
    out["cfg4_score_mask"] = {
        "fwd_ms": round(tf, 4), "fwd_bwd_ms": round(tf + tb, 4), "mask_prepare_ms": prep,
        "algorithmic_fwd_bytes": bytes_fwd, "algorithmic_fwd_bwd_bytes": bytes_fb,
        "fwd_gbs": round(bytes_fwd / tf / 1e6, 1),
        "fwd_frac_hbm": round(bytes_fwd / tf / 1e6 / hbm, 4),
        "fwd_bwd_frac_hbm": round(bytes_fb / (tf + tb) / 1e6 / hbm, 4),
        # Bytes the forward kernel actually moves (packed bits instead of mask bytes),
        # and the algorithmic fraction with one mask preparation charged to the call.
        "fwd_frac_hbm_bytes_moved": round(moved_fwd / tf / 1e6 / hbm, 4),
        "fwd_frac_hbm_with_prepare": round(bytes_fwd / (tf + prep) / 1e6 / hbm, 4),
        "fwd_bwd_frac_hbm_with_prepare": round(bytes_fb / (tf + tb + prep) / 1e6 / hbm, 4),
        "mask_prepare_frac_hbm": round((mask.numel() + bits) / prep / 1e6 / hbm, 4),
    }
    del score, mask
    # cfg3: packed-document [B,1,T,T] mask
    b3, t3 = 2, 4096
    mask = _packed_doc_mask(dev, b3, t3)
    mview = mask.expand(b3, HQ, t3, t3)
    tf, tb = fb(b3, t3, t3, HQ, HK, D, _lib.CAUSAL_NONE, mask=mview)
    prep = map_ms(mview)
    ff, fbf = fwd_flops(b3, HQ, t3, t3, D, False), fwd_bwd_flops(b3, HQ, t3, t3, D, False)
    counts = _lib.mask_blocks(mview).counts()
    live = (counts["partial"] + counts["full"]) / sum(counts.values())
    tfw, tbw = tensor_bytes(b3, t3, t3, HQ, HK, D)
    mbytes = mask.numel()  # the unexpanded [B, 1, T, T] mask, each element once
    out["cfg3_packed_docs"] = {"fwd_ms": round(tf, 4), "fwd_bwd_ms": round(tf + tb, 4),
                               "fwd_dense_equiv_tflops": round(ff / tf / 1e9, 1),
                               "fwd_bwd_dense_equiv_tflops": round(fbf / (tf + tb) / 1e9, 1),
                               "blocks": counts,
                               "fwd_live_block_tflops": round(live * ff / tf / 1e9, 1),
                               "fwd_bwd_live_block_tflops": round(live * fbf / (tf + tb) / 1e9, 1),
                               "fwd_live_block_frac_tensor": round(live * ff / tf / 1e9 / peak, 4),
                               "algorithmic_fwd_bytes": mbytes + tfw,
                               "algorithmic_fwd_bwd_bytes": 2 * mbytes + tfw + tbw,
                               "fwd_frac_hbm": round((mbytes + tfw) / tf / 1e6 / hbm, 4),
                               "fwd_bwd_frac_hbm": round((2 * mbytes + tfw + tbw) / (tf + tb) / 1e6 / hbm, 4),
                               "mask_prepare_ms": prep,
                               "mask_prepare_frac_hbm": round((mbytes + 2 * mbytes // 8) / prep / 1e6 / hbm, 4)}
    del mask, mview
    # cfg5: MQA, bshd, bottom-right causal, one GPU's shard of 16 (B=2)
    tf, tb = fb(2, 1024, 4096, 64, 1, 64, _lib.CAUSAL_BOTTOM_RIGHT)
    ff, fbf = fwd_flops(2, 64, 1024, 4096, 64, True), fwd_bwd_flops(2, 64, 1024, 4096, 64, True)
    tbd = fb(2, 1024, 4096, 64, 1, 64, _lib.CAUSAL_BOTTOM_RIGHT, deterministic=True)[1]
    # Bottom-right causal with Tq=1024 < Tk=4096 keeps 87.5% of the (q, k) pairs, not the
    # convention's 50%: the true work is 0.875 / 0.5 of the convention's FLOPs.
    true_fb = fbf * 0.875 / 0.5
    out["cfg5_mqa_shard_b2"] = {"fwd_ms": round(tf, 4), "fwd_bwd_ms": round(tf + tb, 4),
                                "fwd_bwd_tflops_convention": round(fbf / (tf + tb) / 1e9, 1),
                                "fwd_bwd_tflops_true_work": round(true_fb / (tf + tb) / 1e9, 1),
                                "fwd_bwd_frac_true_work": round(true_fb / (tf + tb) / 1e9 / peak, 4),
                                "fwd_bwd_ms_use_atomic_backward_false": round(tf + tbd, 4)}
    # Head dim 256 at config 2's shape (its own kernels: one-slot forward, column-split
    # backward and the ordered dQ pass)
    tf, tb = fb(B, T, T, HQ, HK, 256, _lib.CAUSAL_NONE, iters=5)
    ff, fbf = fwd_flops(B, HQ, T, T, 256, False), fwd_bwd_flops(B, HQ, T, T, 256, False)
    out["cfg2_shape_d256"] = {"fwd_ms": round(tf, 4), "fwd_tflops": round(ff / tf / 1e9, 1),
                              "fwd_bwd_ms": round(tf + tb, 4), "fwd_bwd_tflops": round(fbf / (tf + tb) / 1e9, 1),
                              "fwd_bwd_frac": round(fbf / (tf + tb) / 1e9 / peak, 4)}
    return out


def library_context(dev, peaks):
    """Context only (not this library's work): the same config-2 shape through torch's
    scaled_dot_product_attention (whatever backend torch picks on this GPU) and, when
    it loads and runs on this GPU, flash_attn 2.x — fwd and fwd+bwd, non-causal and
    causal, bf16, CUDA events, median of 20 after 3 warm-ups, L2 flushed before each."""
    out = {}
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    mk = lambda shape: torch.randn(shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q, k, v, do = mk((B, T, HQ, D)), mk((B, T, HK, D)), mk((B, T, HK, D)), mk((B, T, HQ, D))

    def measure(run_fwd, name):
        res = {}
        for causal in (False, True):
            c = 0.5 if causal else 1.0
            try:
                tf = time_fn(lambda: run_fwd(causal, False), 20)
                tfb = time_fn(lambda: run_fwd(causal, True), 20)
            except Exception as exc:  # context only: report and go on
                res["error"] = f"{type(exc).__name__}: {str(exc)[:160]}"
                break
            tag = "causal" if causal else "noncausal"
            res[f"{tag}_fwd_tflops"] = round(4.0 * B * HQ * T * T * D * c / tf / 1e9, 1)
            res[f"{tag}_fwd_bwd_tflops"] = round(14.0 * B * HQ * T * T * D * c / tfb / 1e9, 1)
        out[name] = res

    import torch.nn.functional as F

    qb, kb, vb, dob = (x.transpose(1, 2) for x in (q, k, v, do))

    def sdpa(causal, backward):
        if not backward:
            with torch.no_grad():
                return F.scaled_dot_product_attention(qb, kb, vb, is_causal=causal, enable_gqa=True)
        qq, kk, vv = (x.detach().requires_grad_(True) for x in (qb, kb, vb))
        F.scaled_dot_product_attention(qq, kk, vv, is_causal=causal, enable_gqa=True).backward(dob)

    measure(sdpa, "torch_sdpa")
    try:
        from flash_attn import flash_attn_func
    except Exception as exc:
        out["flash_attn"] = {"error": f"import failed: {type(exc).__name__}"}
    else:
        def fa(causal, backward):
            if not backward:
                with torch.no_grad():
                    return flash_attn_func(q, k, v, causal=causal)
            qq, kk, vv = (x.detach().requires_grad_(True) for x in (q, k, v))
            flash_attn_func(qq, kk, vv, causal=causal).backward(do)

        measure(fa, "flash_attn")
    return out


# Runs in a child process whose working directory is baseline/_ref (the reference
# installed unmodified, `pip install --target baseline/_ref`), so `python.fa2` is the
# reference's own TileLang op and nothing of this repository is importable there.
# Timed like the reference's benchmark (benchmark/throughput_check.py:206-256): fwd under
# no_grad, fwd+bwd as forward + backward with fresh leaves; here the median of 20 CUDA-event
# timings after 3 warm-ups (which include TileLang's JIT compilation), L2 flushed before each.
_TILELANG_CONTEXT = r"""
import json, statistics, sys, torch
from python.fa2 import flash_attention_with_4d_mask
B, T, HQ, HK, D = (int(x) for x in sys.argv[1:6])
dev = torch.device("cuda", 0)
g = torch.Generator(device=dev)
g.manual_seed(9)
mk = lambda h: torch.randn((B, T, h, D), generator=g, device=dev).to(torch.bfloat16).transpose(1, 2)
q, k, v, do = mk(HQ), mk(HK), mk(HK), mk(HQ)
flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
scale = D ** -0.5

def med(fn, iters=20, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(iters):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(); fn(); b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in evs)

out = {"tilelang": __import__("tilelang").__version__}
for causal in (False, True):
    c = 0.5 if causal else 1.0
    def fwd():
        with torch.no_grad():
            flash_attention_with_4d_mask(q, k, v, None, None, scale, causal, True, True)
    def fwd_bwd():
        qq, kk, vv = (x.detach().requires_grad_(True) for x in (q, k, v))
        flash_attention_with_4d_mask(qq, kk, vv, None, None, scale, causal, True, True).backward(do)
    tag = "causal" if causal else "noncausal"
    tf, tfb = med(fwd), med(fwd_bwd)
    out[tag + "_fwd_ms"] = round(tf, 4)
    out[tag + "_fwd_tflops"] = round(4.0 * B * HQ * T * T * D * c / tf / 1e9, 1)
    out[tag + "_fwd_bwd_ms"] = round(tfb, 4)
    out[tag + "_fwd_bwd_tflops"] = round(14.0 * B * HQ * T * T * D * c / tfb / 1e9, 1)
print("CONTEXT " + json.dumps(out), flush=True)
"""


def tilelang_context(dev, timeout_s=1500):
    """The reference's own TileLang kernels on this GPU at config 2 (context only)."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "python" / "fa2.py").exists():
        return {"error": "baseline/_ref not installed"}
    env = {k2: v2 for k2, v2 in os.environ.items() if k2 != "PYTHONPATH"}
    env["CUDA_VISIBLE_DEVICES"] = str(dev.index if dev.index is not None else 0)
    try:
        res = subprocess.run([sys.executable, "-c", _TILELANG_CONTEXT, str(B), str(T), str(HQ), str(HK), str(D)],
                             cwd=str(ref), env=env, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"error": f"timed out after {timeout_s} s"}
    for line in res.stdout.splitlines():
        if line.startswith("CONTEXT "):
            return json.loads(line[len("CONTEXT "):])
    tail = (res.stderr or res.stdout).strip().splitlines()[-3:]
    return {"error": f"exit {res.returncode}: " + " | ".join(tail)[:400]}


def run_context(args):
    """--impl context: library kernels on this GPU at config 2 (torch SDPA, flash_attn and
    the reference's TileLang kernels), one JSON line; context, not this library's work."""
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    peaks, _ = load_peaks()
    line = {"impl": "context", "config": {"workload": WORKLOAD}, "unit": UNIT}
    line.update(library_context(dev, peaks))
    line["reference_tilelang"] = tilelang_context(dev)
    return line


# Global problems of the strong-scaling leg: (name, B, Tq, Tk, Hq, Hk, D, causal mode).
STRONG = (
    ("cfg2", 1, 8192, 8192, 32, 8, 128, "none"),
    ("cfg5", 16, 1024, 4096, 64, 1, 64, "bottom_right"),
)


def _launch_slices(segs, Hk):
    """The rank's segments as launches: consecutive whole batch elements (every KV
    head) merge into one batch range; a partial element is its own launch.
    Returns (b0, b1, hk0, hk1) tuples."""
    out = []
    for s in segs:
        whole = s.hk0 == 0 and s.hk1 == Hk
        if whole and out and out[-1][2] == 0 and out[-1][3] == Hk and out[-1][1] == s.b:
            out[-1] = (out[-1][0], s.b + 1, 0, Hk)
        else:
            out.append((s.b, s.b + 1, s.hk0, s.hk1))
    return out


def strong_leg(_lib, dev, dist, world, rank, steps, warmup):
    """Fixed global problems split over the ranks by (batch, KV head) units, no exchange
    on the data path.  Each rank times its share (graph replays of fwd + bwd over its
    launches, L2 flushed, median), the step is the max over ranks; rank 0 also times the
    whole problem alone.  Outside the timed region every rank's O, dQ, dK, dV units are
    all-gathered and compared on rank 0 with its single-GPU result."""
    from fa2_with_4d_mask_b200 import shard

    modes = {"none": _lib.CAUSAL_NONE, "bottom_right": _lib.CAUSAL_BOTTOM_RIGHT}
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    res = {}
    for name, B_, Tq, Tk, Hq, Hk, D_, cm in STRONG:
        mode = modes[cm]
        G = Hq // Hk
        g = torch.Generator(device=dev)
        g.manual_seed(4242)
        mk = lambda t, h: torch.randn((B_, t, h, D_), generator=g, device=dev).to(torch.bfloat16)
        q, k, v, do = mk(Tq, Hq), mk(Tk, Hk), mk(Tk, Hk), mk(Tq, Hq)  # [B, T, H, D] storage
        sc = D_ ** -0.5

        def views_of(slices):
            return [(b0, hk0, hk1, q[b0:b1, :, hk0 * G:hk1 * G], k[b0:b1, :, hk0:hk1], v[b0:b1, :, hk0:hk1],
                     do[b0:b1, :, hk0 * G:hk1 * G]) for b0, b1, hk0, hk1 in slices]

        def step(views):
            outs = []
            for _, _, _, qs, ks, vs, ds in views:
                o, lse = _lib.forward(qs, ks, vs, None, None, sc, mode)
                outs.append((o, *_lib.backward(ds, qs, ks, vs, o, lse, None, None, sc, mode)))
            return outs

        def timed(views):
            for _ in range(warmup):
                step(views)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step(views)
            for _ in range(warmup):
                graph.replay()
            torch.cuda.synchronize(dev)
            evs = []
            for _ in range(steps):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                graph.replay()
                b.record(stream)
                evs.append((a, b))
            torch.cuda.synchronize(dev)
            del graph
            return median_ms(evs)

        mine = views_of(_launch_slices(shard.segments(B_, Hk, rank, world), Hk))
        if dist:
            dist.barrier()
        t_n = shard.max_over_ranks(timed(mine), dist, dev)
        # Verification, outside the timed region.
        nan = float("nan")
        full = [torch.full((B_, Tq, Hq, D_), nan, dtype=torch.bfloat16, device=dev),
                torch.full((B_, Tq, Hq, D_), nan, dtype=torch.bfloat16, device=dev),
                torch.full((B_, Tk, Hk, D_), nan, dtype=torch.bfloat16, device=dev),
                torch.full((B_, Tk, Hk, D_), nan, dtype=torch.bfloat16, device=dev)]
        for (b0, hk0, hk1, *_), outs in zip(mine, step(mine)):
            for dst, src, kv in zip(full, outs, (False, False, True, True)):
                h0, h1 = (hk0, hk1) if kv else (hk0 * G, hk1 * G)
                dst[b0:b0 + src.shape[0], :, h0:h1].copy_(src)
        if dist:
            shard.gather_units(dist, full, (False, False, True, True), B_, Hq, Hk, layout="bshd")
        entry = None
        if rank == 0:
            whole = views_of([(0, B_, 0, Hk)])
            t_1 = timed(whole)
            ref = step(whole)[0]
            rel = lambda a, r: float((a.float() - r.float()).norm() / r.float().norm())
            flops = fwd_bwd_flops(B_, Hq, Tq, Tk, D_, cm != "none")
            entry = {
                "global": f"B{B_} Tq{Tq} Tk{Tk} Hq{Hq} Hk{Hk} D{D_} bf16 causal={cm}",
                "units": B_ * Hk, "ranks": world, "ms": round(t_n, 4), "ms_1gpu": round(t_1, 4),
                "tflops": round(flops / t_n / 1e9, 1), "tflops_1gpu": round(flops / t_1 / 1e9, 1),
                "speedup": round(t_1 / t_n, 3), "efficiency": round(t_1 / (world * t_n), 4),
                "verified": {
                    "all_finite": bool(all(torch.isfinite(t.float()).all() for t in full)),
                    "o_bitwise_equal": bool(torch.equal(full[0], ref[0])),
                    "dq_rel": rel(full[1], ref[1]), "dk_rel": rel(full[2], ref[2]), "dv_rel": rel(full[3], ref[3]),
                    "how": "NCCL all_gather_into_tensor of every rank's O, dQ, dK, dV units, compared with the "
                           "whole problem run on rank 0",
                },
            }
            entry["verified"]["ok"] = (entry["verified"]["all_finite"] and entry["verified"]["o_bitwise_equal"]
                                       and max(entry["verified"][k2] for k2 in ("dq_rel", "dk_rel", "dv_rel")) < 1e-2)
        if dist:
            dist.barrier()
        del q, k, v, do, full
        if entry is not None:
            res[name] = entry
    return res if rank == 0 else None


def copy_leg(dev, dist, world, reps=5):
    """Host<->device bandwidth alone: each rank copies one e2e step's inputs (q, k, v,
    dO) from pinned host memory and its outputs (O, dQ, dK, dV) back, all ranks at
    once, timed with CUDA events (median of `reps`, max over ranks)."""
    from fa2_with_4d_mask_b200 import shard

    n_in = 2 * B * T * D * (2 * HQ + 2 * HK)
    h = torch.empty(n_in, dtype=torch.uint8).pin_memory()
    d = torch.empty(n_in, dtype=torch.uint8, device=dev)
    out = {}
    for name, dst, src in (("h2d", d, h), ("d2h", h, d)):
        dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize(dev)
        evs = []
        for _ in range(reps):
            if dist:
                dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            dst.copy_(src, non_blocking=True)
            b.record()
            torch.cuda.synchronize(dev)
            evs.append((a, b))
        ms = shard.max_over_ranks(median_ms(evs), dist, dev)
        out[name] = {"bytes_per_rank": n_in, "ms": round(ms, 4), "gbs_per_rank": round(n_in / ms / 1e6, 1),
                     "gbs_all_ranks": round(world * n_in / ms / 1e6, 1)}
    # Both directions at once, as the end-to-end step runs them (one step's inputs up and
    # the previous step's outputs down on two copy streams): the copy bound of that step.
    h2 = torch.empty(n_in, dtype=torch.uint8).pin_memory()
    d2 = torch.empty(n_in, dtype=torch.uint8, device=dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    evs = []
    for _ in range(reps):
        if dist:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        up.wait_event(a)
        down.wait_event(a)
        with torch.cuda.stream(up):
            d.copy_(h, non_blocking=True)
        with torch.cuda.stream(down):
            h2.copy_(d2, non_blocking=True)
        torch.cuda.current_stream(dev).wait_stream(up)
        torch.cuda.current_stream(dev).wait_stream(down)
        b.record()
        torch.cuda.synchronize(dev)
        evs.append((a, b))
    ms = shard.max_over_ranks(median_ms(evs), dist, dev)
    out["both"] = {"bytes_per_rank_each_way": n_in, "ms": round(ms, 4),
                   "gbs_per_rank_each_way": round(n_in / ms / 1e6, 1)}
    return out


def run_e2e(api, dev, args, dist=None, world=1):
    """Same metric through the public API with pinned host buffers, as a training input
    pipeline runs it: every step uploads its q/k/v/dO host->device, runs forward +
    autograd backward and downloads O, dQ, dK, dV device->host.  Uploads and downloads
    run on their own streams with two device/host buffer sets, so step i+1's upload
    and step i-1's download overlap step i's compute (PCIe is full duplex).  Every rank
    runs it on its own batch element; the step time is the max over ranks and the value
    is whole-job (all ranks' FLOPs)."""
    from fa2_with_4d_mask_b200 import shard

    g = torch.Generator()
    g.manual_seed(77)
    host = lambda shape: torch.randn(shape, generator=g).to(torch.bfloat16).pin_memory()
    shapes = ((B, T, HQ, D), (B, T, HK, D), (B, T, HK, D), (B, T, HQ, D))
    h_in = [[host(sh) for sh in shapes] for _ in range(2)]
    out_shapes = ((B, T, HQ, D), (B, T, HQ, D), (B, T, HK, D), (B, T, HK, D))  # O, dQ, dK, dV
    h_out = [[torch.empty(sh, dtype=torch.bfloat16).pin_memory() for sh in out_shapes] for _ in range(2)]
    d_in = [[torch.empty(sh, dtype=torch.bfloat16, device=dev) for sh in shapes] for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in h_in[0])
    d2h = sum(x.numel() * x.element_size() for x in h_out[0])
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    inputs_ready = [ev(), ev()]
    inputs_free = [None, None]  # compute finished reading buffer set b
    outputs_done = [None, None]  # download of host set b finished

    def step(i):
        b = i % 2
        with torch.cuda.stream(up):
            if inputs_free[b] is not None:
                up.wait_event(inputs_free[b])
            for dst, src in zip(d_in[b], h_in[b]):
                dst.copy_(src, non_blocking=True)
            inputs_ready[b].record(up)
        comp.wait_event(inputs_ready[b])
        qd, kd, vd, dod = d_in[b]
        q = qd.transpose(1, 2).requires_grad_(True)
        k = kd.transpose(1, 2).requires_grad_(True)
        v = vd.transpose(1, 2).requires_grad_(True)
        o = api.tilelang_flash_attention(q, k, v)
        o.backward(dod.transpose(1, 2))
        res = (o.detach(), q.grad, k.grad, v.grad)
        inputs_free[b] = ev()
        inputs_free[b].record(comp)
        with torch.cuda.stream(down):
            down.wait_stream(comp)
            for dst, src in zip(h_out[b], res):
                src.record_stream(down)
                dst.copy_(src.transpose(1, 2), non_blocking=True)
            outputs_done[b] = ev()
            outputs_done[b].record(down)

    def run(n):
        for i in range(n):
            step(i)

    run(4)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    try:
        free_gib = round(torch.cuda.mem_get_info(dev)[0] / 2**30, 1)
    except RuntimeError:
        free_gib = None
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(comp)
    up.wait_event(a)
    t0 = time.perf_counter()
    run(args.e2e_steps)
    # Host time to enqueue the steps: near ms_per_step means the leg was host-bound.
    host_ms = (time.perf_counter() - t0) * 1e3 / args.e2e_steps
    comp.wait_stream(up)
    comp.wait_stream(down)
    b.record(comp)
    torch.cuda.synchronize(dev)
    ms = shard.max_over_ranks(a.elapsed_time(b) / args.e2e_steps, dist, dev)
    return {"value": round(world * fwd_bwd_flops(B, HQ, T, T, D, False) / (ms * 1e-3) / 1e12, 2), "unit": UNIT,
            "ms_per_step": round(ms, 4), "h2d_bytes_per_step": world * h2d, "d2h_bytes_per_step": world * d2h,
            "host_enqueue_ms_per_step": round(host_ms, 4), "device_free_gib_at_start": free_gib,
            "path": "tilelang_flash_attention + autograd backward; each step uploads its pinned inputs and "
                    "downloads O, dQ, dK, dV on separate copy streams, double-buffered so copies of "
                    "neighbouring steps overlap compute"}


# --------------------------------------------------------------------------- CPU arms
def cpu_sample_step(hq_sample):
    """One fwd+bwd of the reference's eager fp32 attention on the host: query heads
    0..hq_sample-1 of the workload with their KV head (T=8192, D=128)."""
    from oracle import inputs as I
    from oracle.eager import attention_ref_grads

    hk_sample = max(1, hq_sample // (HQ // HK))
    q, k, v, do = I.qkv(1, T, T, hq_sample, hk_sample, D, seed=5)
    t0 = time.perf_counter()
    attention_ref_grads(q, k, v, do, None, None, scale=D ** -0.5, is_causal=False)
    return time.perf_counter() - t0, fwd_bwd_flops(1, hq_sample, T, T, D, False)


def cpu_baseline(args):
    torch.set_num_threads(os.cpu_count() or 1)
    cpu_sample_step(1)  # warm-up
    secs, flops = [], 0.0
    for _ in range(3):
        s, flops = cpu_sample_step(4)
        secs.append(s)
    s = statistics.median(secs)
    return {"value": round(flops / s / 1e12, 5), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": "oracle/eager.py (restated eager_ref, fp32) fwd+bwd on one GQA group "
                      "(4 query heads, 1 KV head) of the workload, median of 3 after 1 warm-up"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    for _ in range(args.warmup):
        cpu_sample_step(1)
    secs, flops = [], 0.0
    for _ in range(args.steps):
        s, flops = cpu_sample_step(1)
        secs.append(s)
    ms = 1e3 * sum(secs) / len(secs)
    value = flops / (ms * 1e-3) / 1e12
    sample = ("reference eager fp32 attention (oracle/eager.py restatement of "
              "benchmark/precision_check.py:133-180) fwd+bwd on query head 0 and its KV head of the workload "
              "(T=8192, D=128) per step, on the host cores")
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 5),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic N(0,1) inputs, seeded",
        "config": {"workload": WORKLOAD, "global_batch": world * B, "seq_len": T,
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference", "context"), default="ours")
    # End-to-end steps (default: --steps).  The first step's upload and the last step's
    # download have no neighbour to overlap, so too few steps overstate their cost.
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-extra", dest="extra", action="store_false")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong", dest="strong", action="store_false",
                    help="skip the strong-scaling leg (fixed global problems split over the ranks)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.e2e_steps is None:
        args.e2e_steps = args.steps
    if args.impl == "reference":
        line = run_reference(args)
    elif args.impl == "context":
        line = run_context(args)
    else:
        import tilelang_fa2_4d_mask  # noqa: F401  (registers fa2_with_4d_mask_b200)

        line = run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
