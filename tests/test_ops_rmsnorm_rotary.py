"""RMSNorm and rotary kernels against the CPU oracle (reference formulas).

Tolerances: fp32 kernels vs a float64 oracle on the same inputs, 2e-5
relative; fp16/bf16 kernels vs the float64 oracle evaluated on the rounded
inputs, within a few output ulps (rtol 1e-2 / 2e-2).
"""
from __future__ import annotations

import pytest
import torch

from oracle import ops_ref
from pymsst_b200.extension import ops, rms_norm_backward_into

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 2e-5), torch.float16: (1e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


def _close(actual, expected, dtype, scale=1.0):
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(actual.double().cpu(), expected.double().cpu(), rtol=rtol, atol=atol * scale)


SHAPES = [(0, 192), (1, 192), (1000, 192), (777, 384), (33, 37), (5, 1536), (3, 7, 64)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_rms_norm_forward_backward(cuda_device, shape, dtype):
    x = (torch.randn(*shape) * 3).to(dtype)
    gamma = (torch.rand(shape[-1]) + 0.5).to(dtype)
    dy = torch.randn(*shape).to(dtype)
    out, normed, inv = ops.rms_norm_forward(x.to(cuda_device), gamma.to(cuda_device))
    r_out, r_normed, r_inv = ops_ref.rms_norm_forward(x.double(), gamma.double())
    _close(out, r_out, dtype)
    _close(normed, r_normed, dtype)
    torch.testing.assert_close(inv.double().cpu(), r_inv, rtol=1e-5, atol=0)

    gx, gg = ops.rms_norm_backward(dy.to(cuda_device), normed, inv, gamma.to(cuda_device))
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.double(), normed.double().cpu(), inv.double().cpu(), gamma.double())
    _close(gx, r_gx, dtype)
    rows = max(1, x.numel() // shape[-1])
    _close(gg, r_gg, dtype, scale=rows ** 0.5)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rms_norm_fp32_gamma_and_mixed(cuda_device, dtype):
    x = torch.randn(300, 192).to(dtype)
    gamma = torch.rand(192) + 0.5
    dy = torch.randn(300, 192)
    out, normed, inv = ops.rms_norm_forward_fp32_gamma(x.to(cuda_device), gamma.to(cuda_device))
    assert out.dtype == dtype and normed.dtype == dtype
    r_out, r_normed, _ = ops_ref.rms_norm_forward(x.double(), gamma.double())
    _close(out, r_out, dtype)
    gx, gg = ops.rms_norm_backward_fp32_gamma(dy.to(dtype).to(cuda_device), normed, inv, gamma.to(cuda_device))
    assert gg.dtype == torch.float32
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.to(dtype).double(), normed.double().cpu(), inv.double().cpu(), gamma.double())
    _close(gx, r_gx, dtype)
    torch.testing.assert_close(gg.double().cpu(), r_gg, rtol=1e-4, atol=1e-3)

    out, normed, inv = ops.rms_norm_forward_mixed(x.to(cuda_device), gamma.to(cuda_device))
    assert out.dtype == torch.float32 and normed.dtype == torch.float32
    _close(out, r_out, torch.float32)
    gx, gg = ops.rms_norm_backward_mixed(dy.to(cuda_device), normed, inv, gamma.to(cuda_device), x.to(cuda_device))
    assert gx.dtype == dtype and gg.dtype == torch.float32
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.double(), normed.double().cpu(), inv.double().cpu(), gamma.double())
    _close(gx, r_gx, dtype)
    torch.testing.assert_close(gg.double().cpu(), r_gg, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rms_norm_backward_from_saved_input(cuda_device, dtype):
    """The training path saves x (not normed) and recomputes normed in the backward."""
    x = torch.randn(4096, 192).to(dtype).to(cuda_device)
    gamma = (torch.rand(192) + 0.5).to(cuda_device)
    dy = torch.randn(4096, 192).to(dtype).to(cuda_device)
    _, normed32, inv = ops.rms_norm_forward_mixed(x, gamma) if dtype != torch.float32 else ops.rms_norm_forward(x, gamma)
    gx, gg = rms_norm_backward_into(dy, x, inv, gamma, saved_is_input=True, grad_x_dtype=dtype,
                                    grad_gamma_dtype=torch.float32)
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.double().cpu(), normed32.double().cpu(), inv.double().cpu(),
                                           gamma.double().cpu())
    _close(gx, r_gx, dtype)
    torch.testing.assert_close(gg.double().cpu(), r_gg, rtol=1e-4, atol=1e-2)


# bulk (rows of 192 / 384), vector (dim 1536 > the bulk limit) and generic (dim 37, unaligned) kernels
@pytest.mark.parametrize("rows,dim", [(4096, 192), (777, 384), (300, 1536), (65, 37)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rms_norm_backward_adds_the_residual_gradient(cuda_device, rows, dim, dtype):
    """pmb_rms_norm_backward_add: grad_x = RMSNorm'(dy) + grad_residual in the norm's own pass, against the
    float64 oracle's RMSNorm' plus the residual gradient (one 16-bit rounding of the sum)."""
    g = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, dim, generator=g).to(dtype).to(cuda_device)
    gamma = (torch.rand(dim, generator=g) + 0.5).to(cuda_device)
    dy = torch.randn(rows, dim, generator=g).to(dtype).to(cuda_device)
    res = torch.randn(rows, dim, generator=g).to(dtype).to(cuda_device)
    _, normed32, inv = ops.rms_norm_forward_mixed(x, gamma) if dtype != torch.float32 else ops.rms_norm_forward(x, gamma)
    gx, gg = rms_norm_backward_into(dy, x, inv, gamma, saved_is_input=True, grad_x_dtype=dtype,
                                    grad_gamma_dtype=torch.float32, grad_residual=res)
    plain, gg0 = rms_norm_backward_into(dy, x, inv, gamma, saved_is_input=True, grad_x_dtype=dtype,
                                        grad_gamma_dtype=torch.float32)
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.double().cpu(), normed32.double().cpu(), inv.double().cpu(),
                                           gamma.double().cpu())
    _close(gx, r_gx + res.double().cpu(), dtype, scale=float(res.abs().max()))
    # the gamma gradient does not see the residual (summed over a different grid: the same up to fp32 ordering)
    torch.testing.assert_close(gg, gg0, rtol=1e-5, atol=1e-5 * float(gg0.abs().max()))
    if dtype == torch.float32:
        torch.testing.assert_close(gx, plain + res, rtol=1e-6, atol=1e-6)


def test_rms_norm_residual_fn_matches_norm_plus_sum(cuda_device):
    """RMSNormResidualFn (y, x) used as a pre-norm residual block gives the gradients of RMSNormFn plus an
    autograd sum."""
    from pymsst_b200.fused import RMSNormFn, RMSNormResidualFn

    g = torch.Generator().manual_seed(11)
    x0 = torch.randn(2, 300, 192, generator=g).to(torch.bfloat16).to(cuda_device)
    gamma0 = (torch.rand(192, generator=g) + 0.5).to(cuda_device)
    w = torch.randn(192, 192, generator=g).to(torch.bfloat16).to(cuda_device) / 14

    def run(fused):
        x, gamma = x0.clone().requires_grad_(), gamma0.clone().requires_grad_()
        if fused:
            y, r = RMSNormResidualFn.apply(x, gamma)
        else:
            y, r = RMSNormFn.apply(x, gamma), x
        out = (y @ w) + r
        out.float().square().sum().backward()
        return out.detach(), x.grad, gamma.grad

    o1, gx1, gg1 = run(True)
    o2, gx2, gg2 = run(False)
    assert torch.equal(o1, o2)
    torch.testing.assert_close(gx1.float(), gx2.float(), rtol=1e-2, atol=1e-2 * float(gx2.abs().max()))
    torch.testing.assert_close(gg1, gg2, rtol=1e-5, atol=1e-5 * float(gg2.abs().max()))


def test_rms_norm_zero_rows_and_zero_vector(cuda_device):
    x = torch.zeros(3, 192, device=cuda_device)
    gamma = torch.ones(192, device=cuda_device)
    out, normed, inv = ops.rms_norm_forward(x, gamma)
    assert torch.all(out == 0)
    torch.testing.assert_close(inv.cpu(), torch.full((3,), 1e12), rtol=1e-6, atol=0)
    gx, gg = ops.rms_norm_backward(torch.zeros_like(x), normed, inv, gamma)
    assert torch.all(gx == 0) and torch.all(gg == 0)


@pytest.mark.parametrize("shape", [(2, 62, 8, 64), (1, 1024, 8, 64), (3, 5, 2, 6), (0, 4, 8, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_rotary_forward_backward(cuda_device, shape, dtype):
    b, n, h, d = shape
    t = torch.randn(shape).to(dtype)
    angles = torch.arange(n)[:, None].double() * torch.rand(d // 2).double()
    cos = angles.cos().to(dtype).reshape(1, n, 1, d // 2)
    sin = angles.sin().to(dtype).reshape(1, n, 1, d // 2)
    out = ops.rotary_forward(t.to(cuda_device), cos.to(cuda_device), sin.to(cuda_device))
    ref = ops_ref.rotary_forward(t.double(), cos.double(), sin.double())
    _close(out, ref, dtype)
    back = ops.rotary_backward(out, cos.to(cuda_device), sin.to(cuda_device))
    ref_back = ops_ref.rotary_backward(out.double().cpu(), cos.double(), sin.double())
    _close(back, ref_back, dtype)


def test_rejects_mismatched_arguments(cuda_device):
    x = torch.randn(4, 8, device=cuda_device)
    with pytest.raises(RuntimeError, match="gamma dimension must match"):
        ops.rms_norm_forward(x, torch.ones(7, device=cuda_device))
    with pytest.raises(RuntimeError, match="gamma dtype must match"):
        ops.rms_norm_forward(x, torch.ones(8, device=cuda_device, dtype=torch.float16))
    t = torch.randn(1, 4, 2, 6, device=cuda_device)
    c = torch.randn(1, 3, 1, 3, device=cuda_device)
    with pytest.raises(RuntimeError, match="cos sequence dimension must match t"):
        ops.rotary_forward(t, c, c)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dim", [4, 64, 192, 384, 1024, 1536])
@pytest.mark.parametrize("rows", [1, 5, 17, 300, 777, 5000])
def test_rms_norm_backward_stays_inside_workspace(cuda_device, rows, dim, dtype):
    """The grad_gamma partials fit the advertised workspace for every path:
    the exact size is followed by a sentinel region that must stay untouched."""
    from pymsst_b200 import _native as nat

    lib = nat.library()
    need = int(lib.pmb_rms_norm_backward_workspace_size(rows, dim))
    guard = 1 << 16
    buf = torch.full((need + guard,), 0xA5, dtype=torch.uint8, device=cuda_device)
    dy = torch.randn(rows, dim, device=cuda_device).to(dtype)
    normed = torch.randn(rows, dim, device=cuda_device).to(dtype)
    inv = torch.rand(rows, device=cuda_device) + 0.5
    gamma = (torch.rand(dim, device=cuda_device) + 0.5).to(dtype)
    gx = torch.empty_like(dy)
    gg = torch.empty(dim, dtype=dtype, device=cuda_device)
    code = nat.dtype_code(dtype)
    nat.call("pmb_rms_norm_backward", dy.data_ptr(), normed.data_ptr(), 0, inv.data_ptr(), gamma.data_ptr(),
             gx.data_ptr(), gg.data_ptr(), rows, dim, code, code, code, code, buf.data_ptr(), need,
             nat.stream_handle(cuda_device))
    assert bool((buf[need:] == 0xA5).all()), "backward wrote past the workspace"
    r_gx, r_gg = ops_ref.rms_norm_backward(dy.double().cpu(), normed.double().cpu(), inv.double().cpu(),
                                           gamma.double().cpu())
    _close(gx, r_gx, dtype)
    _close(gg, r_gg, dtype, scale=rows ** 0.5)
