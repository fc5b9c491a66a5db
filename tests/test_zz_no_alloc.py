"""fa4d_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some hosts of this library own only the input and output buffers — a plugin or
FFI caller with no device allocator of its own, or a process whose device memory
is already reserved by another pool, where a fresh cudaMalloc fails and cudaFree
synchronises the device.  fa4d_bwd_noalloc serves them from a fixed scratch buffer
inside the library instead of a caller-provided workspace.  These tests call it
through the C ABI and compare its gradients with fa4d_bwd (caller-owned workspace)
on two different problems in a row, so anything the first call leaves in the shared
buffer would show up in the second.  This file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err
from fa2_with_4d_mask_b200 import _lib
from oracle import inputs as I

G_REL = 3e-2  # same gradient tolerance as the parity tests
I3 = ctypes.c_int64 * 3


def _args(q, k, v, o, lse, do, dq, dk, dv, mask, scale, causal, deterministic):
    a = _lib.BwdArgs()
    a.q, a.k, a.v, a.o, a.dout, a.lse = (t.data_ptr() for t in (q, k, v, o, do, lse))
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    for name, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", o), ("do_stride", do),
                    ("dq_stride", dq), ("dk_stride", dk), ("dv_stride", dv)):
        setattr(a, name, I3(t.stride(0), t.stride(1), t.stride(2)))
    if mask is not None:
        a.mask = mask.data_ptr()
        a.mask_stride = I3(0 if mask.shape[0] == 1 else mask.stride(0), 0 if mask.shape[1] == 1 else mask.stride(1),
                           mask.stride(2))
    B, Tq, Hq, D = q.shape
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = B, Tq, k.shape[1], Hq, k.shape[2], D
    a.dtype = _lib.FA4D_BF16 if q.dtype == torch.bfloat16 else _lib.FA4D_F16
    a.causal, a.scale, a.deterministic = causal, scale, deterministic
    return a


def _grads(entry, q, k, v, o, lse, do, mask, scale, causal, deterministic):
    lib = _lib.load_library()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = _args(q, k, v, o, lse, do, dq, dk, dv, mask, scale, causal, deterministic)
    ws = None
    if entry == "fa4d_bwd":
        B, Tq, Hq, D = q.shape
        a.workspace_bytes = lib.fa4d_bwd_workspace_size(B, Tq, Hq, D)
        ws = torch.empty(a.workspace_bytes, dtype=torch.uint8, device=q.device)
        a.workspace = ws.data_ptr()
    rc = getattr(lib, entry)(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream))
    assert rc == _lib.FA4D_OK, lib.fa4d_last_error()
    torch.cuda.synchronize(q.device)
    return dq, dk, dv


PROBLEMS = [
    # (B, Tq, Tk, Hq, Hk, D, causal mode, with mask, deterministic, dtype)
    (1, 1024, 1024, 8, 2, 128, _lib.CAUSAL_TOP_LEFT, False, 0, torch.bfloat16),
    (2, 300, 520, 4, 4, 64, _lib.CAUSAL_NONE, True, 0, torch.bfloat16),
    # The bit-reproducible backward: dQ from the ordered pass, which shares only the
    # Delta region of the buffer (no accumulator to clear).
    (1, 700, 900, 8, 2, 128, _lib.CAUSAL_BOTTOM_RIGHT, False, 1, torch.bfloat16),
    # Head dim 256: the scratch is Delta only, in both backward modes.
    (1, 384, 384, 4, 2, 256, _lib.CAUSAL_TOP_LEFT, False, 0, torch.bfloat16),
    (1, 256, 320, 2, 1, 256, _lib.CAUSAL_NONE, True, 1, torch.bfloat16),
    (2, 513, 513, 4, 1, 128, _lib.CAUSAL_TOP_LEFT, True, 0, torch.float16),
    # The first problem again, after every other one has left its contents behind.
    (1, 1024, 1024, 8, 2, 128, _lib.CAUSAL_TOP_LEFT, False, 0, torch.bfloat16),
]


@pytest.mark.gpu
def test_noalloc_matches_workspace_backward_on_two_calls_in_a_row():
    """Each problem is run through fa4d_bwd (caller workspace) and then fa4d_bwd_noalloc;
    consecutive noalloc calls reuse the one built-in buffer.  dK/dV never use atomics and
    must match bit for bit; so must dQ where it comes from the ordered pass
    (deterministic mode, or head dim 256 in either mode)."""
    dev = torch.device("cuda", 0)
    for i, (B, Tq, Tk, Hq, Hk, D, causal, with_mask, det, dtype) in enumerate(PROBLEMS):
        q, k, v, do = (x.to(dev).transpose(1, 2).contiguous()
                       for x in I.qkv(B, Tq, Tk, Hq, Hk, D, seed=40 + i, dtype=dtype))
        mask = I.random_mask(1, 1, Tq, Tk, 0.8, seed=9).to(dev) if with_mask else None
        scale = D ** -0.5
        o, lse = _lib.forward(q, k, v, mask, None, scale, causal)
        ref = _grads("fa4d_bwd", q, k, v, o, lse, do, mask, scale, causal, det)
        got = _grads("fa4d_bwd_noalloc", q, k, v, o, lse, do, mask, scale, causal, det)
        for name, g, r in zip(("dQ", "dK", "dV"), got, ref):
            assert torch.isfinite(g.float()).all(), f"call {i}: {name} not finite"
            e = rel_err(g, r)
            assert e <= G_REL, f"call {i}: {name} rel={e:.3e}"
        assert torch.equal(got[1], ref[1]) and torch.equal(got[2], ref[2]), f"call {i}: dK/dV differ"
        if det or D == 256:
            assert torch.equal(got[0], ref[0]), f"call {i}: ordered-pass dQ differs"
    assert _lib.device_status(dev) == 0


def test_noalloc_rejects_problems_larger_than_its_buffer():
    """A problem whose scratch exceeds the built-in buffer is refused up front (no device work)."""
    lib = _lib.load_library()
    a = _lib.BwdArgs()
    a.q = a.k = a.v = a.o = a.dout = a.lse = a.dq = a.dk = a.dv = 0x1000
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = 1, 8192, 8192, 32, 8, 128  # needs ~129 MiB
    a.dtype, a.causal, a.scale = _lib.FA4D_BF16, 0, 0.088
    assert lib.fa4d_bwd_noalloc(ctypes.byref(a), None) == _lib.FA4D_ERR_WORKSPACE
    assert b"built-in buffer" in lib.fa4d_last_error()
