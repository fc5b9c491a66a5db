"""CPU: the benchmark's JSON contract, checked on its reference arm (the reference's
CPU attention path, which needs no GPU), and its argument checks."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _run(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    res = _run("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["higher_is_better"] is True and line["scaling"] == "weak" and line["vs_baseline"] is None
    assert line["config"]["workload"] == bench.WORKLOAD
    for key in ("dtype", "data"):
        assert isinstance(line[key], str) and line[key]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"] and cb["kind"] == "port"
    assert cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_warmup_below_three_is_rejected():
    res = _run("--warmup", "2", timeout=300)
    assert res.returncode == 2 and "--warmup must be >= 3" in res.stderr


@pytest.mark.parametrize("causal", [False, True])
def test_flop_convention(causal):
    """fwd = 4 B Hq Tq Tk D, fwd+bwd = 14 B Hq Tq Tk D, halved when causal
    (benchmark/throughput_check.py:85-92)."""
    f = 0.5 if causal else 1.0
    assert bench.fwd_flops(1, 32, 8192, 8192, 128, causal) == 4 * 32 * 8192 * 8192 * 128 * f
    assert bench.fwd_bwd_flops(1, 32, 8192, 8192, 128, causal) == 14 * 32 * 8192 * 8192 * 128 * f
