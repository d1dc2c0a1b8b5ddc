"""The graph trainer's 16-bit parameter mirror (``fused.lowp_weight``) on the host: it is served only inside the
trainer's own forward / backward scope, and every other call gets a fresh cast, so a mirror older than the
parameters can never reach a caller.  (The GPU side -- graph and eager training bit for bit equal with the
mirror -- is tests/test_model_parity.py::test_cuda_graph_trainer_matches_eager.)"""
from __future__ import annotations

import torch

from pymsst_b200.fused import OutProjFn, lowp_weight


def _mirrored(shape=(3, 4)):
    p = torch.nn.Parameter(torch.randn(*shape))
    live = [False]
    p._pmb_half = p.detach().to(torch.bfloat16).clone()
    p._pmb_half_live = live
    return p, live


def test_mirror_served_only_inside_the_scope():
    p, live = _mirrored()
    assert lowp_weight(p, torch.bfloat16).data_ptr() != p._pmb_half.data_ptr()  # outside: a cast
    live[0] = True
    assert lowp_weight(p, torch.bfloat16).data_ptr() == p._pmb_half.data_ptr()  # inside: the mirror
    assert lowp_weight(p, torch.float16).dtype == torch.float16  # another type: a cast
    live[0] = False
    with torch.no_grad():
        p.add_(1.0)  # an update the mirror has not seen
    torch.testing.assert_close(lowp_weight(p, torch.bfloat16), p.detach().to(torch.bfloat16), rtol=0, atol=0)


def test_plain_parameter_is_cast():
    p = torch.nn.Parameter(torch.randn(5))
    out = lowp_weight(p, torch.bfloat16)
    assert out.dtype == torch.bfloat16 and torch.equal(out, p.detach().to(torch.bfloat16))


def test_output_projection_matches_autograd_through_the_cast():
    """OutProjFn forms the products autograd forms for addmm(residual, gated, W.to(bf16).t()): outputs and all
    three gradients equal bit for bit."""
    g = torch.Generator().manual_seed(3)
    res = torch.randn(9, 6, generator=g).to(torch.bfloat16).requires_grad_()
    gated = torch.randn(9, 10, generator=g).to(torch.bfloat16).requires_grad_()
    w = torch.randn(6, 10, generator=g).requires_grad_()
    gy = torch.randn(9, 6, generator=g).to(torch.bfloat16)
    got = OutProjFn.apply(res, gated, w)
    got_g = torch.autograd.grad(got, (res, gated, w), gy)
    r2, g2, w2 = (t.detach().clone().requires_grad_() for t in (res, gated, w))
    want = torch.addmm(r2, g2, w2.to(torch.bfloat16).t())
    want_g = torch.autograd.grad(want, (r2, g2, w2), gy)
    assert torch.equal(got, want)
    for a, b in zip(got_g, want_g):
        assert a.dtype == b.dtype and torch.equal(a, b)
