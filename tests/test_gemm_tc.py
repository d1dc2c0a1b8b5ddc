"""tcgen05 GEMM engine against a float64 reference of the same 16-bit inputs.

Tolerance: fp32 accumulation of bf16/fp16 products; outputs compared with
rtol 2e-3 and an absolute floor of 2e-3 x sqrt(K) x the operand scale.
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _gemm(a, b, m, n, k, a_mn, b_mn, out_dtype, bias=None, act=0):
    c = torch.empty(m, n, dtype=out_dtype, device=a.device)
    nat.call("pmb_gemm_tc", a.data_ptr(), a.stride(0), int(a_mn), b.data_ptr(), b.stride(0), int(b_mn), c.data_ptr(),
             c.stride(0), nat.dtype_code(out_dtype), nat.ptr(bias), nat.dtype_code(bias.dtype) if bias is not None else 0,
             act, m, n, k, nat.dtype_code(a.dtype), nat.stream_handle(a.device))
    return c


def _padded(t, device):
    """Copy of a 2-D tensor whose row stride is rounded up to 8 elements
    (16 bytes), the alignment TMA needs; ragged shapes stay ragged."""
    ld = (t.shape[1] + 7) // 8 * 8
    store = torch.zeros(t.shape[0], ld, dtype=t.dtype)
    store[:, : t.shape[1]] = t
    return store.to(device)[:, : t.shape[1]]


# (4096, 1536, 192), (9000, 768, 192), (1000, 600, 72) and (300, 129, 40) run the resident-B schedule (K <= 192,
# 256-wide N blocks): N blocks that do not divide the 148-CTA grid, ragged M / N tails, K below one k-block
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (1000, 192, 768), (130, 70, 100), (4096, 1536, 192), (64, 8, 16),
                                   (9000, 768, 192), (1000, 600, 72), (300, 129, 40)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_tc_matches_reference(cuda_device, m, n, k, a_mn, b_mn, dtype):
    torch.manual_seed(m + n + k)
    A = torch.randn(m, k).to(dtype)
    B = torch.randn(n, k).to(dtype)
    ref = A.double() @ B.double().t()
    a = _padded(A.t() if a_mn else A, cuda_device)
    b = _padded(B.t() if b_mn else B, cuda_device)
    c = _gemm(a, b, m, n, k, a_mn, b_mn, torch.float32)
    tol = 2e-3 * max(1.0, k ** 0.5)
    torch.testing.assert_close(c.double().cpu(), ref, rtol=2e-3, atol=tol)
    assert nat.library().pmb_umma_timeout(1) == 0


def test_gemm_tc_bias_tanh_bf16_out(cuda_device):
    m, n, k = 300, 768, 192
    A = torch.randn(m, k).to(torch.bfloat16)
    B = (torch.randn(n, k) / k ** 0.5).to(torch.bfloat16)
    bias = torch.randn(n)
    ref = torch.tanh(A.double() @ B.double().t() + bias.double())
    c = _gemm(A.to(cuda_device), B.to(cuda_device), m, n, k, False, False, torch.bfloat16, bias=bias.to(cuda_device),
              act=1)
    torch.testing.assert_close(c.double().cpu(), ref, rtol=1e-2, atol=1e-2)


def test_gemm_tc_rejects_unaligned_stride(cuda_device):
    a = torch.randn(130, 100, device=cuda_device).to(torch.bfloat16)
    c = torch.empty(130, 130, device=cuda_device)
    st = nat.library().pmb_gemm_tc(a.data_ptr(), 100, 0, a.data_ptr(), 100, 0, c.data_ptr(), 130, 0, None, 0, 0,
                                   130, 130, 100, nat.dtype_code(a.dtype), nat.stream_handle(a.device))
    assert st == -4 and b"16-byte" in nat.library().pmb_last_error()


@pytest.mark.parametrize("m,n,k", [(1536, 192, 63984), (768, 192, 5000), (192, 768, 4100), (130, 70, 100),
                                   (64, 64, 64)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_tc_wgrad_split_k(cuda_device, m, n, k, out_dtype):
    """C = A^T B over K rows (split-K with fp32 partials) against float64."""
    torch.manual_seed(m * 7 + n + k)
    A = torch.randn(k, m).to(torch.bfloat16)
    B = torch.randn(k, n).to(torch.bfloat16)
    ref = A.double().t() @ B.double()
    a, b = _padded(A, cuda_device), _padded(B, cuda_device)
    c = torch.empty(m, n, dtype=out_dtype, device=cuda_device)
    wsb = nat.library().pmb_gemm_tc_wgrad_workspace_size(m, n, k)
    ws = nat.workspace(wsb, cuda_device)
    nat.call("pmb_gemm_tc_wgrad", a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), m, n, k, c.data_ptr(),
             c.stride(0), nat.dtype_code(out_dtype), nat.dtype_code(torch.bfloat16), ws.data_ptr(), wsb,
             nat.stream_handle(cuda_device))
    tol = 2e-3 * max(1.0, k ** 0.5)
    rtol = 2e-3 if out_dtype == torch.float32 else 1e-2
    torch.testing.assert_close(c.double().cpu(), ref, rtol=rtol, atol=tol)
    assert nat.library().pmb_umma_timeout(1) == 0
