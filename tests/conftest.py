"""Shared pytest setup: the ``gpu`` marker, repo import paths and golden loaders."""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN_DIR = ROOT / "tests" / "golden"

# Registers the implementation package under the module name fa2_with_4d_mask_b200.
import tilelang_fa2_4d_mask  # noqa: E402,F401


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_names():
    return sorted(p.stem for p in GOLDEN_DIR.glob("*.npz"))


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)


def load_golden(name: str) -> dict:
    """Fixture as tensors: q/k/v/dout as BHSD bf16 views over [B, T, H, D] storage,
    optional mask/score/attention_mask, fp32 expected out/dq/dk/dv (BHSD)."""
    z = np.load(GOLDEN_DIR / f"{name}.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    rec = {"meta": meta}
    for key in ("q", "k", "v", "dout"):
        rec[key] = _bf16(z[key]).transpose(1, 2)
    for key in ("out", "dq", "dk", "dv"):
        rec[key] = torch.from_numpy(z[key])
    if "mask" in z:
        rec["mask"] = torch.from_numpy(z["mask"]).bool()
    if "score" in z:
        rec["score"] = torch.from_numpy(z["score"])
    if "attention_mask" in z:
        am = torch.from_numpy(z["attention_mask"])
        rec["attention_mask"] = am.bool() if bool(z["attention_mask_is_bool"][0]) else am
    return rec


def to_layout(x: torch.Tensor, layout: str) -> torch.Tensor:
    """BHSD tensor -> the layout a case's API call uses."""
    return x if layout == "bhsd" else x.transpose(1, 2)


def from_layout(x: torch.Tensor, layout: str) -> torch.Tensor:
    return x if layout == "bhsd" else x.transpose(1, 2)


def rel_err(a: torch.Tensor, ref: torch.Tensor) -> float:
    """||a - ref|| / ||ref|| in fp32 (the gradient tolerance's measure).  The
    denominator is floored at 1e-3 * sqrt(numel) so a gradient that is exactly zero
    in the oracle (e.g. dQ with a single key) is compared in absolute terms."""
    a = a.float()
    ref = ref.float().to(a.device)
    floor = 1e-3 * math.sqrt(ref.numel())
    return float((a - ref).norm() / ref.norm().clamp_min(floor))


def out_err(a: torch.Tensor, ref: torch.Tensor):
    """(max_abs, mean_abs) of a 16-bit output against the fp32 oracle rounded to
    the output dtype, as the reference's own check compares (eager_ref returns
    ``.to(q.dtype)``, benchmark/precision_check.py:179-180)."""
    r = ref.to(a.device).to(a.dtype).float()
    d = (a.float() - r).abs()
    return float(d.max()), float(d.mean())
