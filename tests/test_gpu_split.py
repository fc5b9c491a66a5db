"""GPU: the backward's group split.  When one CTA per (key tile, KV head, batch) would
leave SMs idle (MQA here: 16 query heads on one KV head, 8 key tiles), the query-head
group is split over CTAs whose fp32 partial dK/dV are added in a fixed slice order:
results match the unsplit backward (same math, different summation grouping) and are
bit-identical from run to run."""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err
from fa2_with_4d_mask_b200 import _lib
from oracle import inputs as I
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle  # noqa: F401

pytestmark = pytest.mark.gpu


def _bwd(q, k, v, o, lse, do, scale, causal, split: bool):
    lib = _lib.load_library()
    B, Tq, Hq, D = q.shape
    Tk, Hk = k.shape[1], k.shape[2]
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = _lib.BwdArgs()
    a.q, a.k, a.v, a.o, a.dout, a.lse = (t.data_ptr() for t in (q, k, v, o, do, lse))
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    I3 = ctypes.c_int64 * 3
    for name, t in (("q_stride", q), ("k_stride", k), ("v_stride", v), ("o_stride", o), ("do_stride", do),
                    ("dq_stride", dq), ("dk_stride", dk), ("dv_stride", dv)):
        setattr(a, name, I3(t.stride(0), t.stride(1), t.stride(2)))
    a.B, a.Tq, a.Tk, a.Hq, a.Hk, a.D = B, Tq, Tk, Hq, Hk, D
    a.dtype, a.causal, a.scale = _lib.FA4D_BF16, causal, scale
    n = lib.fa4d_bwd_workspace_size_ex(B, Tq, Tk, Hq, Hk, D) if split else lib.fa4d_bwd_workspace_size(B, Tq, Hq, D)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    a.workspace, a.workspace_bytes = ws.data_ptr(), n
    assert lib.fa4d_bwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)) == 0
    torch.cuda.synchronize()
    return dq, dk, dv


@pytest.mark.parametrize("causal", [_lib.CAUSAL_NONE, _lib.CAUSAL_BOTTOM_RIGHT])
def test_group_split_matches_unsplit_and_is_deterministic(causal):
    lib = _lib.load_library()
    B, Tq, Tk, Hq, Hk, D = 2, 256, 1024, 16, 1, 64
    assert lib.fa4d_bwd_workspace_size_ex(B, Tq, Tk, Hq, Hk, D) > lib.fa4d_bwd_workspace_size(B, Tq, Hq, D)
    q, k, v, do = (x.transpose(1, 2).to(DEV) for x in I.qkv(B, Tq, Tk, Hq, Hk, D, seed=61))
    scale = D ** -0.5
    o, lse = _lib.forward(q, k, v, None, None, scale, causal)
    s1 = _bwd(q, k, v, o, lse, do, scale, causal, split=True)
    s2 = _bwd(q, k, v, o, lse, do, scale, causal, split=True)
    u = _bwd(q, k, v, o, lse, do, scale, causal, split=False)
    assert torch.equal(s1[1], s2[1]) and torch.equal(s1[2], s2[2])
    for g_split, g_plain in zip(s1, u):
        assert rel_err(g_split.float(), g_plain.float()) < 1e-2
    # And against the fp32 oracle, through the public API (which sizes for the split).
    qc, kc, vc, doc = I.qkv(B, Tq, Tk, Hq, Hk, D, seed=61)
    ref = oracle(qc, kc, vc, doc, causal=causal != _lib.CAUSAL_NONE, offset=Tk - Tq, device="cpu")
    dq, dk, dv = _lib.backward(do, q, k, v, o, lse, None, None, scale, causal)
    check((o.transpose(1, 2), dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)), ref, "split")
