"""GPU: the bounded-wait failure path, exercised without any fault.  A kernel waits on
an mbarrier that nothing completes, using the same wait routine as the attention
kernels with a ~1 ms limit; it must give up, set its bit in the device status word
and leave the context usable (an attention call afterwards still matches the oracle)."""

from __future__ import annotations

import pytest
import torch

from fa2_with_4d_mask_b200 import _lib
from oracle import inputs as I
from test_gpu_parity import DEV, _fp32_oracle_and_status, check, oracle, run_api  # noqa: F401

pytestmark = pytest.mark.gpu


def test_expired_wait_sets_status_and_context_survives():
    lib = _lib.load_library()
    assert _lib.device_status(DEV, clear=True) == 0
    stream = torch.cuda.current_stream(DEV).cuda_stream
    assert lib.fa4d_check_wait_timeout(DEV.index or 0, 2_000_000, stream) == 0
    status = _lib.device_status(DEV, clear=True)
    assert status == _lib.DEV_TIMEOUT_CHECK
    assert _lib.device_status(DEV, clear=False) == 0
    q, k, v, do = I.qkv(1, 256, 256, 2, 1, 64, seed=51)
    check(run_api(q, k, v, do, is_causal=True), oracle(q, k, v, do, causal=True, device="cpu"), "after timeout")


def test_wait_limit_is_validated():
    lib = _lib.load_library()
    assert lib.fa4d_check_wait_timeout(0, 0, None) == _lib.FA4D_ERR_INVALID
