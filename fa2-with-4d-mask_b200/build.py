"""Builds libfa4d.so (the sm_100a kernels behind include/fa4d.h) in place.

The library is compiled with nvcc for ``sm_100a`` only and written next to this
file, so it travels with the source tree.  Objects go to ``_build/`` beside it.
Run ``python build.py`` (add ``--ptxas-info`` to print register / spill counts).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
LIB = HERE / "libfa4d.so"

SOURCES = ["fa4d_api.cu", "fa4d_fwd.cu", "fa4d_bwd.cu", "fa4d_bwd256.cu", "fa4d_mask.cu", "fa4d_dq.cu", "fa4d_dq256.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "fa4d.h"]


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


# Kernels that rebalance registers with setmaxnreg assume this exact allocation per
# thread at launch; fewer would make a setmaxnreg.inc wait forever.
LAUNCH_REGS = {"bwd_kernel": 128, "bwd256_kernel": 168, "fwd_kernel": 168}


def _check_launch_regs(src: Path, log: str) -> None:
    entry = None
    for line in log.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            entry = m.group(1)
            continue
        m = re.search(r"Used (\d+) registers", line)
        if m and entry:
            for name, regs in LAUNCH_REGS.items():
                if name in entry and int(m.group(1)) != regs:
                    raise RuntimeError(f"{src.name}: {entry} uses {m.group(1)} registers, expected {regs}")
            entry = None


def _compile(nvcc: str, src: Path, obj: Path, ptxas_info: bool) -> str:
    cmd = [nvcc, *ARCH, *CFLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj), "-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    _check_launch_regs(src, res.stdout + res.stderr)
    return res.stdout + res.stderr


def build(force: bool = False, ptxas_info: bool = False, jobs: int | None = None) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    deps = _deps()
    todo = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (src.stem + ".o")
        if force or ptxas_info or _stale(obj, [src, *deps]):
            todo.append((src, obj))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 1)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, ptxas_info) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    objs = [BUILD / (Path(n).stem + ".o") for n in SOURCES]
    if force or todo or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    if ptxas_info:
        for log in logs:
            sys.stdout.write(log)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    args = ap.parse_args()
    lib = build(force=args.force, ptxas_info=args.ptxas_info, jobs=args.jobs)
    print(lib)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
