"""Tensor-core MaskEstimator (bf16 / fp16) against the float64 oracle MLP.

Tolerance: bf16 activations and weights -> 2e-2 relative (per tensor, max
abs error over max abs value); fp16 -> 1e-2.
"""
from __future__ import annotations

import pytest
import torch

from oracle import roformer_ref
from pymsst_b200 import bands
from pymsst_b200.fused import MaskEstimatorTCFn
from pymsst_b200 import _native as nat

pytestmark = pytest.mark.gpu

BSR_WIDTHS = tuple(4 * n for n in bands.DEFAULT_FREQS_PER_BANDS)


def _rel(a, b):
    return float((a.double().cpu() - b.double().cpu()).abs().max() / b.double().abs().max().clamp_min(1e-12))


@pytest.mark.parametrize("widths,rows,dim,hidden_layers", [
    (BSR_WIDTHS, 260, 192, 1),
    ((12, 28, 8, 516, 130), 77, 64, 2),
    ((4, 4, 8), 5, 64, 0),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_mask_estimator_tc(cuda_device, widths, rows, dim, hidden_layers, dtype):
    torch.manual_seed(0)
    est = roformer_ref.MaskEstimator(dim, widths, hidden_layers, mlp_expansion_factor=4).double()
    x = torch.randn(rows, len(widths), dim, dtype=torch.float64)
    dy = torch.randn(rows, sum(widths), dtype=torch.float64)
    xr = x.clone().requires_grad_()
    ref = est(xr)
    ref.backward(dy)
    ref_grads = {n: p.grad.clone() for n, p in est.named_parameters()}

    dev = roformer_ref.MaskEstimator(dim, widths, hidden_layers, mlp_expansion_factor=4)
    dev.load_state_dict({k: v.float() for k, v in est.state_dict().items()})
    dev = dev.to(cuda_device)
    params = []
    for layer in range(hidden_layers + 1):
        lins = [net[0][2 * layer] for net in dev.to_freqs]
        params += [lin.weight for lin in lins] + [lin.bias for lin in lins]
    xd = x.to(dtype).to(cuda_device).requires_grad_()
    out = MaskEstimatorTCFn.apply(xd, widths, hidden_layers, dim * 4, *params)
    out.backward(dy.to(dtype).to(cuda_device))
    assert nat.library().pmb_umma_timeout(1) == 0
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-2
    assert _rel(out, ref) < tol
    assert _rel(xd.grad, xr.grad) < tol
    for n, p in dev.named_parameters():
        assert p.grad is not None, n
        assert _rel(p.grad, ref_grads[n]) < 3 * tol, n
