"""CPU: the C-ABI library loads, exports every function include/fa4d.h declares,
its ctypes mirror matches the C struct layout (checked with a gcc-compiled probe),
and argument errors come back as status codes before any device work."""

from __future__ import annotations

import ctypes
import re
import shutil
import subprocess

import pytest
import torch

from conftest import ROOT
from fa2_with_4d_mask_b200 import _lib  # noqa: F401  (loaded through tilelang_fa2_4d_mask)

HEADER = ROOT / "include" / "fa4d.h"


def _declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa4d_\w+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = _lib.load_library()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} missing from libfa4d.so"
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS)
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
        exported = set(re.findall(r"\bT (fa4d_\w+)", out))
        assert exported == set(declared)


def test_abi_version():
    assert _lib.load_library().fa4d_abi_version() == _lib.ABI_VERSION == 2


def _c_layout(struct: str, fields):
    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("gcc not available")
    lines = [f'printf("%zu\\n", sizeof({struct}));']
    lines += [f'printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"fa4d.h\"\nint main(void){" + "".join(lines) + "return 0;}\n"
    import tempfile, os
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(src)
        subprocess.run([gcc, "-I", str(ROOT / "include"), c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("cls,cname", [(_lib.FwdArgs, "fa4d_fwd_args"), (_lib.BwdArgs, "fa4d_bwd_args")])
def test_ctypes_mirror_matches_c_layout(cls, cname):
    names = [f[0] for f in cls._fields_]
    size, offsets = _c_layout(cname, names)
    assert ctypes.sizeof(cls) == size
    assert [getattr(cls, n).offset for n in names] == offsets


def test_host_size_helpers():
    lib = _lib.load_library()
    assert lib.fa4d_lse_row_stride(1) == 128
    assert lib.fa4d_lse_row_stride(128) == 128
    assert lib.fa4d_lse_row_stride(8191) == 8192
    assert lib.fa4d_lse_row_stride(8193) == 8320
    dq = 1 * 8192 * 32 * 128 * 4
    delta = 1 * 32 * 8192 * 4
    assert lib.fa4d_bwd_workspace_size(1, 8192, 32, 128) == dq + delta
    assert lib.fa4d_bwd_workspace_size(1, 1, 1, 64) % 256 == 0
    # Head dim 96 computes at width 128: its dQ accumulator rows hold 128 floats.
    assert lib.fa4d_bwd_workspace_size(1, 8192, 32, 96) == lib.fa4d_bwd_workspace_size(1, 8192, 32, 128)
    # Head dim 256 has no dQ accumulator (the ordered dQ pass writes dQ): Delta only.
    assert lib.fa4d_bwd_workspace_size(1, 8192, 32, 256) == delta


def test_group_split_choices():
    """The backward's group split on a 148-SM B200 (also the host-side default when no
    device is visible): equal-work grids are split to fill the last wave, causal grids
    (balanced by the grid order) only when too small for the GPU."""
    lib = _lib.load_library()
    if torch.cuda.is_available() and torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("choices below are for 148 SMs")
    assert lib.fa4d_bwd_group_split(1, 8192, 8192, 32, 8, 128, _lib.CAUSAL_NONE) == 2  # 512 CTAs: 3.46 waves
    assert lib.fa4d_bwd_group_split(1, 8192, 8192, 32, 8, 128, _lib.CAUSAL_TOP_LEFT) == 1
    assert lib.fa4d_bwd_group_split(16, 1024, 4096, 64, 1, 64, _lib.CAUSAL_BOTTOM_RIGHT) == 2  # a band: equal work
    assert lib.fa4d_bwd_group_split(1, 512, 512, 8, 2, 64, _lib.CAUSAL_TOP_LEFT) == 4  # 8 CTAs
    assert lib.fa4d_bwd_group_split(1, 4096, 4096, 16, 16, 128, _lib.CAUSAL_NONE) == 1  # group of one
    assert lib.fa4d_bwd_group_split(1, 128, 128, 3, 2, 64, _lib.CAUSAL_NONE) == 0  # invalid
    # The workspace covers the largest split of any causal mode.
    base = lib.fa4d_bwd_workspace_size(1, 8192, 32, 128)
    assert lib.fa4d_bwd_workspace_size_ex(1, 8192, 8192, 32, 8, 128) > base
    # Head dim 256 runs a CTA pair per key tile: config 2's shape already makes 1024 CTAs
    # (6.92 waves), a small MQA grid (12 CTAs) splits 8 ways.  Its workspace is Delta plus
    # the two fp32 dK / dV slice sets, with no dQ accumulator.
    assert lib.fa4d_bwd_group_split(1, 8192, 8192, 32, 8, 256, _lib.CAUSAL_NONE) == 1
    assert lib.fa4d_bwd_group_split(2, 200, 384, 16, 1, 256, _lib.CAUSAL_BOTTOM_RIGHT) == 8
    delta = 2 * 16 * 256 * 4
    slices = 8 * 2 * 384 * 1 * 256 * 4
    assert lib.fa4d_bwd_workspace_size(2, 200, 16, 256) == delta
    assert lib.fa4d_bwd_workspace_size_ex(2, 200, 384, 16, 1, 256) == delta + 2 * slices


def _fwd_args(**kw):
    a = _lib.FwdArgs()
    a.q = a.k = a.v = a.o = a.lse = 0x1000
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = 1, 128, 128, 2, 1, 128
    a.dtype, a.causal, a.scale = _lib.FA4D_BF16, 0, 0.088
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize(
    "kw,code",
    [
        (dict(D=80), _lib.FA4D_ERR_UNSUPPORTED),
        (dict(D=512), _lib.FA4D_ERR_UNSUPPORTED),
        (dict(Hq=3, Hk=2), _lib.FA4D_ERR_INVALID),
        (dict(B=0), _lib.FA4D_ERR_INVALID),
        (dict(dtype=7), _lib.FA4D_ERR_INVALID),
        (dict(causal=5), _lib.FA4D_ERR_INVALID),
        (dict(q=None), _lib.FA4D_ERR_INVALID),
        (dict(scale=float("nan")), _lib.FA4D_ERR_INVALID),
    ],
)
def test_fwd_rejects_bad_arguments_without_device_work(kw, code):
    lib = _lib.load_library()
    rc = lib.fa4d_fwd(ctypes.byref(_fwd_args(**kw)), None)
    assert rc == code
    assert lib.fa4d_last_error()


def test_null_args_pointer():
    lib = _lib.load_library()
    assert lib.fa4d_fwd(None, None) == _lib.FA4D_ERR_INVALID
    assert lib.fa4d_bwd(None, None) == _lib.FA4D_ERR_INVALID


def test_bwd_rejects_bad_flag_and_small_workspace():
    lib = _lib.load_library()
    a = _lib.BwdArgs()
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.dq = a.dk = a.dv = 0x1000
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = 1, 128, 128, 2, 1, 128
    a.dtype, a.causal, a.scale = _lib.FA4D_BF16, 0, 0.088
    a.deterministic = 2
    assert lib.fa4d_bwd(ctypes.byref(a), None) == _lib.FA4D_ERR_INVALID
    a.deterministic = 0
    a.workspace, a.workspace_bytes = 0x1000, 16
    assert lib.fa4d_bwd(ctypes.byref(a), None) == _lib.FA4D_ERR_WORKSPACE
    # Head dim 256 is built for both backward modes: the call gets past the head-dim
    # checks and fails on the workspace.
    a.D = 256
    for det in (0, 1):
        a.deterministic = det
        assert lib.fa4d_bwd(ctypes.byref(a), None) == _lib.FA4D_ERR_WORKSPACE
