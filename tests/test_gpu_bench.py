"""GPU: a short run of the benchmark's own arm prints one line with the contract's keys
(roofline of the backward main kernel, end-to-end figure with the bytes it copies,
launch count, clock record) and a clean device status."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


def test_bench_line_contract():
    res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--steps", "3", "--warmup", "3", "--no-extra",
                          "--no-cpu-baseline", "--e2e-steps", "3"], capture_output=True, text=True, timeout=900,
                         cwd=ROOT)
    assert res.returncode == 0, res.stderr[-3000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    line = json.loads(lines[0])
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["device_status"] == 0
    assert line["higher_is_better"] is True and line["scaling"] == "weak" and line["dtype"] == "bf16"
    roof = line["roofline"]
    assert roof["bound"] == "tensor" and roof["unit"] == "TFLOP/s"
    assert roof["achieved"] > 0 and roof["peak"] > 0 and roof["frac"] == pytest.approx(roof["achieved"] / roof["peak"],
                                                                                           rel=1e-3)
    assert roof["traffic"] > 0
    e2e = line["e2e"]
    assert e2e["value"] > 0 and e2e["unit"] == line["unit"]
    # Every step uploads q, k, v, dO and downloads O, dQ, dK, dV (bf16).
    B, T, HQ, HK, D = 1, 8192, 32, 8, 128
    io = 2 * B * T * D * (2 * HQ + 2 * HK)
    assert e2e["h2d_bytes_per_step"] == io and e2e["d2h_bytes_per_step"] == io
    # Diagnostics of the e2e leg: host enqueue time per step and free device memory.
    assert e2e["host_enqueue_ms_per_step"] > 0 and "device_free_gib_at_start" in e2e
    # Four launches per step (forward, preprocess, main, convert) plus the slice sum
    # when the group split is on.
    assert line["gpu_launches"] in (4 * 3, 5 * 3)
    assert "sm_mhz" in line["clocks"] or "error" in line["clocks"]
    # Strong scaling on one GPU: the sharded run is the whole problem; the gathered
    # results match the single-GPU run.
    for name in ("cfg2", "cfg5"):
        st = line["strong_scaling"][name]
        assert st["ranks"] == 1 and st["ms"] > 0 and st["verified"]["ok"], st
    assert line["host_copies"]["h2d"]["gbs_per_rank"] > 0 and line["host_copies"]["d2h"]["gbs_per_rank"] > 0
    # The causal leg is measured like the headline and reports its own fractions.
    c = line["causal"]
    assert c["fwd_ms"] > 0 and c["fwd_bwd_ms"] > c["fwd_ms"]
    assert 0 < c["fwd_frac_of_peak"] < 2 and 0 < c["fwd_bwd_frac_of_peak"] < 2
