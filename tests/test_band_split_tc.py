"""BandSplit on the tcgen05 path against a float64 restatement of the
reference formula (per band: RMSNorm over the band's features, times gamma,
Linear with bias; fused_roformer.py:1265-1271).

Tolerance: bf16 outputs and parameter gradients within 2e-2 of their scale
(bf16 normalised features and bf16 W*gamma operands, fp32 accumulation).
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200 import _native as nat
from pymsst_b200.bands import DEFAULT_FREQS_PER_BANDS
from pymsst_b200.fused import BandSplitFn

pytestmark = pytest.mark.gpu


def _reference(x, widths, gammas, weights, biases):
    outs, off = [], 0
    for w, g, W, b in zip(widths, gammas, weights, biases):
        xb = x[:, off:off + w]
        off += w
        n = xb / xb.norm(dim=-1, keepdim=True).clamp_min(1e-12) * w ** 0.5
        outs.append((n * g) @ W.t() + b)
    return torch.stack(outs, dim=1)


@pytest.mark.parametrize("widths", [
    [2 * 2 * f for f in DEFAULT_FREQS_PER_BANDS],           # BS-RoFormer split bands (widths 8 .. 516)
    [4 * f for f in (3, 5, 7, 11, 13, 17, 19, 23, 29, 31)],  # ragged, offsets not 8-aligned
    [64] * 6,
])
@pytest.mark.parametrize("rows", [1032, 77])
def test_band_split_tc_matches_float64(cuda_device, widths, rows):
    torch.manual_seed(len(widths) + rows)
    D = 192
    total = sum(widths)
    x = torch.randn(rows, total).to(torch.bfloat16)
    gammas = [1 + 0.1 * torch.randn(w) for w in widths]
    weights = [torch.randn(D, w) / w ** 0.5 for w in widths]
    biases = [0.1 * torch.randn(D) for _ in widths]
    params = [p.to(cuda_device).requires_grad_() for p in (*gammas, *weights, *biases)]
    out = BandSplitFn.apply(x.to(cuda_device), list(widths), D, *params)
    gy = torch.randn(rows, len(widths), D).to(torch.bfloat16)
    out.backward(gy.to(cuda_device))
    ref_params = [p.detach().double().cpu().requires_grad_() for p in params]
    nb = len(widths)
    ref = _reference(x.double(), widths, ref_params[:nb], ref_params[nb:2 * nb], ref_params[2 * nb:])
    ref.backward(gy.double())

    def close(a, e, what):
        scale = float(e.abs().max().clamp_min(1e-6))
        torch.testing.assert_close(a.detach().double().cpu(), e.detach(), rtol=2e-2, atol=2e-2 * scale,
                                   msg=lambda m: f"{what}: {m}")

    close(out, ref, "out")
    for k, (p, r) in enumerate(zip(params, ref_params)):
        close(p.grad, r.grad, f"param {k}")
    assert nat.library().pmb_umma_timeout(1) == 0
