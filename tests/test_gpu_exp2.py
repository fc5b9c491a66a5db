"""GPU: the polynomial exp2 used for part of the forward's exponentials stays within
its stated error bound of CUDA's exp2f over the argument range the kernel feeds it."""

from __future__ import annotations

import ctypes

import pytest
import torch

from fa2_with_4d_mask_b200 import _lib

pytestmark = pytest.mark.gpu

# Stated bound of the fitted degree-3 polynomial (7.5e-5) plus fp32 rounding of the
# Horner steps and of exp2f itself; half a bf16 ulp (the precision P is stored in)
# is 2^-9 = 1.95e-3.
BOUND = 1.0e-4


# The kernel feeds exp2 arguments s - m <= 8 of a softmax row whose sum is >= 1, so
# only values above ~2^-100 can matter; below 2^-120 the polynomial's exponent-field
# scaling produces denormal-range bit patterns (values under 1.2e-38).
@pytest.mark.parametrize("lo,hi", [(-30.0, 8.0), (-100.0, 0.0), (-1.0, 1.0)])
def test_exp2_polynomial_error_bound(lo, hi):
    n = 1 << 20
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    lib = _lib.load_library()
    rc = lib.fa4d_check_exp2(out.data_ptr(), n, lo, hi, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.fa4d_last_error()
    err = out.abs().max().item()
    assert err <= BOUND, f"max relative error {err:.3e} on [{lo}, {hi}]"
