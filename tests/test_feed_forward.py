"""Feed-forward block on the tensor cores against a float64 reference of
Linear -> GELU(erf) -> Linear on the same bf16 inputs and fp32 parameters.

Tolerance: outputs and gradients within 2e-2 of their max magnitude (bf16
storage of the two linear outputs and the GELU output, fp32 accumulation);
bias gradients (long column sums) within 1e-2 relative.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from pymsst_b200 import _native as nat
from pymsst_b200.fused import FeedForwardFn

pytestmark = pytest.mark.gpu


def _close(got, exp, what, tol=2e-2):
    scale = float(exp.abs().max().clamp_min(1e-6))
    torch.testing.assert_close(got.detach().double().cpu(), exp.detach(), rtol=tol, atol=tol * scale,
                               msg=lambda m: f"{what}: {m}")


@pytest.mark.parametrize("rows,dim,hidden", [(1000, 192, 768), (130, 64, 256), (4100, 384, 1536), (77, 192, 768)])
def test_feed_forward_matches_float64(cuda_device, rows, dim, hidden):
    torch.manual_seed(rows + dim)
    x = torch.randn(rows, dim).to(torch.bfloat16)
    w1 = torch.randn(hidden, dim) / dim ** 0.5
    b1 = torch.randn(hidden) * 0.1
    w2 = torch.randn(dim, hidden) / hidden ** 0.5
    b2 = torch.randn(dim) * 0.1
    gy = torch.randn(rows, dim).to(torch.bfloat16)
    dev = [t.to(cuda_device).requires_grad_() for t in (x, w1, b1, w2, b2)]
    out = FeedForwardFn.apply(*dev)
    out.backward(gy.to(cuda_device))
    ref = [t.double().requires_grad_() for t in (x, w1, b1, w2, b2)]
    h = torch.nn.functional.linear(ref[0], ref[1].to(torch.bfloat16).double(), ref[2])
    y = torch.nn.functional.linear(torch.nn.functional.gelu(h), ref[3].to(torch.bfloat16).double(), ref[4])
    y.backward(gy.double())
    _close(out, y, "out")
    for name, got, exp in zip(("grad_x", "grad_w1", "grad_b1", "grad_w2", "grad_b2"), dev, ref):
        _close(got.grad, exp.grad, name)
    assert nat.library().pmb_umma_timeout(1) == 0


def test_feed_forward_matches_autocast_torch_path(cuda_device):
    """Same bf16 result as torch's autocast Linear -> GELU -> Linear (the unfused path) within bf16 rounding."""
    torch.manual_seed(3)
    rows, dim, hidden = 2048, 192, 768
    lin1 = torch.nn.Linear(dim, hidden).to(cuda_device)
    lin2 = torch.nn.Linear(hidden, dim).to(cuda_device)
    x = torch.randn(rows, dim, device=cuda_device).to(torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref = lin2(torch.nn.functional.gelu(lin1(x)))
    got = FeedForwardFn.apply(x, lin1.weight, lin1.bias, lin2.weight, lin2.bias)
    _close(got, ref.double().cpu(), "out", tol=2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_gelu_kernels_match_torch(cuda_device, dtype):
    """GELU forward / backward equal torch's erf GELU (one-ulp slack); bias sums match a float64 column sum
    of the stored gradient; pmb_column_sum matches a float64 column sum."""
    torch.manual_seed(11)
    rows, cols = 3001, 768
    x = (torch.randn(rows, cols, device=cuda_device) * 2).to(dtype)
    gy = torch.randn(rows, cols, device=cuda_device).to(dtype)
    st = nat.stream_handle(cuda_device)
    y = torch.empty_like(x)
    nat.call("pmb_gelu_forward", x.data_ptr(), y.data_ptr(), x.numel(), nat.dtype_code(dtype), st)
    ref = torch.nn.functional.gelu(x)
    ulp = {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 2 ** -22}[dtype]
    torch.testing.assert_close(y.float(), ref.float(), rtol=ulp, atol=1e-6)
    xr = x.detach().clone().requires_grad_()
    torch.nn.functional.gelu(xr).backward(gy)
    gx = torch.empty_like(x)
    gb = torch.empty(cols, device=cuda_device)
    wsb = nat.library().pmb_rows_pass_workspace_size(rows, cols)
    ws = nat.workspace(wsb, cuda_device)
    nat.call("pmb_gelu_backward", gy.data_ptr(), x.data_ptr(), gx.data_ptr(), rows, cols, gb.data_ptr(), 0,
             nat.dtype_code(dtype), ws.data_ptr(), wsb, st)
    torch.testing.assert_close(gx.float(), xr.grad.float(), rtol=ulp, atol=1e-6)
    torch.testing.assert_close(gb.double(), gx.double().sum(0), rtol=1e-5, atol=1e-4)
    cs = torch.empty(cols, device=cuda_device)
    nat.call("pmb_column_sum", gy.data_ptr(), rows, cols, cs.data_ptr(), 0, nat.dtype_code(dtype), ws.data_ptr(),
             wsb, st)
    torch.testing.assert_close(cs.double(), gy.double().sum(0), rtol=1e-5, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gelu_every_16bit_input(cuda_device, dtype):
    """Every finite 16-bit value through the 16-bit GELU path (logistic form of the normal CDF, csrc/gelu.cuh):
    forward and derivative within one unit in the last place of torch's erf GELU, equal for almost all."""
    x = torch.arange(0, 65536, dtype=torch.int32).to(torch.int16).view(dtype)
    x = x[torch.isfinite(x.float())]
    x = x[: x.numel() // 8 * 8].reshape(-1, 8).to(cuda_device)
    rows, cols = x.shape
    st = nat.stream_handle(cuda_device)
    ulp = {torch.bfloat16: 2 ** -8, torch.float16: 2 ** -11}[dtype]

    def check(got, want):
        got, want = got.float(), want.float()
        diff = (got - want).abs()
        assert bool((diff <= want.abs() * 2 * ulp + 1e-6).all()), float(diff.max())
        assert int((diff > 0).sum()) <= 0.01 * want.numel(), int((diff > 0).sum())

    y = torch.empty_like(x)
    nat.call("pmb_gelu_forward", x.data_ptr(), y.data_ptr(), x.numel(), nat.dtype_code(dtype), st)
    check(y, torch.nn.functional.gelu(x))
    xr = x.clone().requires_grad_()
    gy = torch.ones_like(x)
    torch.nn.functional.gelu(xr).backward(gy)
    gx = torch.empty_like(x)
    wsb = nat.library().pmb_rows_pass_workspace_size(rows, cols)
    ws = nat.workspace(wsb, cuda_device)
    nat.call("pmb_gelu_backward", gy.data_ptr(), x.data_ptr(), gx.data_ptr(), rows, cols, None, 0,
             nat.dtype_code(dtype), ws.data_ptr(), wsb, st)
    check(gx, xr.grad)

