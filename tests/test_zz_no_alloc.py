"""RMSNorm backward without a caller workspace (pmb_rms_norm_backward_noalloc).

Some callers of the library cannot allocate device memory for a call -- a
program binding the C ABI from another language with no device allocator of
its own, or a training loop that must not allocate mid-step because
cudaMalloc / cudaFree synchronise the device.  The no-allocation variant keeps
its scratch in a fixed array inside the library.  These tests call it through
the C ABI twice in a row on each case (the second call runs on the scratch the
first one left behind) and compare each result with pmb_rms_norm_backward
given a caller-allocated workspace, within the tolerances the other RMSNorm
tests use; two of the cases fill the array to its last element.

This file is collected last (tests/test_zz_*), so a run that stops at the
first failure has already run every other test.
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200 import _native as nat
from pymsst_b200.extension import ops, rms_norm_backward_into

TOL = {torch.float32: (2e-5, 2e-5), torch.bfloat16: (2e-2, 2e-2)}


def _noalloc(dy, saved, saved_is_input, inv, gamma, grad_x_dtype, grad_gamma_dtype):
    rows, dim = dy.numel() // dy.shape[-1], dy.shape[-1]
    gx = torch.empty(dy.shape, dtype=grad_x_dtype, device=dy.device)
    gg = torch.empty(dim, dtype=grad_gamma_dtype, device=dy.device)
    nat.call(
        "pmb_rms_norm_backward_noalloc", dy.data_ptr(), saved.data_ptr(), int(saved_is_input), inv.data_ptr(),
        gamma.data_ptr(), gx.data_ptr(), gg.data_ptr(), rows, dim, nat.dtype_code(dy.dtype), nat.dtype_code(gamma.dtype),
        nat.dtype_code(grad_x_dtype), nat.dtype_code(grad_gamma_dtype), nat.stream_handle(dy.device),
    )
    return gx, gg


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_version_twice(cuda_device):
    # (rows, dim, dtype, saved is the input).  The last two fill the scratch array exactly: dim 1024 with enough
    # rows for the largest backward grid (592 blocks), each block writing a full 1024-float partial row of
    # grad_gamma.
    cases = [(4096, 192, torch.bfloat16, True), (777, 384, torch.float32, False), (8192, 1024, torch.float32, False),
             (6000, 1024, torch.bfloat16, True)]
    for seed, (rows, dim, dtype, from_input) in enumerate(cases):
        g = torch.Generator().manual_seed(100 + seed)
        x = (torch.randn(rows, dim, generator=g) * 3).to(dtype).to(cuda_device)
        gamma = (torch.rand(dim, generator=g) + 0.5).to(cuda_device)
        dy = torch.randn(rows, dim, generator=g).to(dtype).to(cuda_device)
        if dtype == torch.float32:
            _, normed, inv = ops.rms_norm_forward(x, gamma)
        else:
            _, normed, inv = ops.rms_norm_forward_fp32_gamma(x, gamma)
        saved = x if from_input else normed
        ref_gx, ref_gg = rms_norm_backward_into(dy, saved, inv, gamma, saved_is_input=from_input, grad_x_dtype=dtype,
                                                grad_gamma_dtype=torch.float32)
        rtol, atol = TOL[dtype]
        for call in range(2):  # the second call runs on the scratch contents the first one left behind
            gx, gg = _noalloc(dy, saved, from_input, inv, gamma, dtype, torch.float32)
            torch.cuda.synchronize()
            msg = f"rows={rows} dim={dim} {dtype} call {call}"
            torch.testing.assert_close(gx.double().cpu(), ref_gx.double().cpu(), rtol=rtol, atol=atol,
                                       msg=lambda m: f"{msg}: {m}")
            torch.testing.assert_close(gg.double().cpu(), ref_gg.double().cpu(), rtol=1e-4, atol=1e-3,
                                       msg=lambda m: f"{msg}: {m}")


def test_noalloc_rejects_dims_beyond_its_scratch():
    lib = nat.library()
    status = lib.pmb_rms_norm_backward_noalloc(None, None, 0, None, None, None, None, 8, 4096, 0, 0, 0, 0, None)
    assert status == -5
    assert b"scratch limit of 1024" in lib.pmb_last_error()
