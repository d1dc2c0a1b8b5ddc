"""Attention projection with the rotary embedding in the tensor-core GEMM
epilogue, against the unfused path (torch projection + split kernel) and a
float64 restatement of projection + rotation.

Tolerances: bf16 outputs compared at rtol/atol 2e-2 of the output scale
(rounding of the projection before rotation may differ in the last bit when
the fp32 accumulation order differs); gradients at 2e-2 of their scale.
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200 import _native as nat
from pymsst_b200.fused import QKVRotaryFn, rotary_tables

pytestmark = pytest.mark.gpu


def _rotate_ref(t, cos, sin):
    """Interleaved-pair rotation of t [..., n, dh] by cos/sin [n, dh/2] in float64."""
    e, o = t[..., 0::2], t[..., 1::2]
    out = torch.empty_like(t)
    out[..., 0::2] = e * cos - o * sin
    out[..., 1::2] = o * cos + e * sin
    return out


@pytest.mark.parametrize("b,n,d,heads,dh", [(8, 258, 192, 8, 64), (31, 62, 192, 8, 64), (3, 37, 64, 2, 32),
                                            (2, 100, 384, 8, 64)])
@pytest.mark.parametrize("rotate", [True, False])
def test_qkv_linear_rotary_matches_reference(cuda_device, b, n, d, heads, dh, rotate):
    torch.manual_seed(b * n + d)
    dt = torch.bfloat16
    x = torch.randn(b, n, d).to(dt)
    w = (torch.randn(3 * heads * dh, d) / d ** 0.5).to(dt)
    freqs = 1.0 / (10000 ** (torch.arange(0, dh, 2).float() / dh))
    cos, sin = rotary_tables(freqs.to(cuda_device), n, cuda_device) if rotate else (None, None)
    xd = x.to(cuda_device).requires_grad_()
    wd = w.float().to(cuda_device).requires_grad_()
    q, k, v = QKVRotaryFn.apply(xd, wd, cos, sin, None, None, heads)
    qkv = (x.double().reshape(b * n, d) @ w.double().t()).reshape(b, n, 3, heads, dh).permute(2, 0, 3, 1, 4)
    ref = [qkv[0], qkv[1], qkv[2]]
    if rotate:
        c64, s64 = cos.double().cpu(), sin.double().cpu()
        ref[0], ref[1] = _rotate_ref(ref[0], c64, s64), _rotate_ref(ref[1], c64, s64)
    for got, exp, name in zip((q, k, v), ref, "qkv"):
        scale = float(exp.abs().max())
        torch.testing.assert_close(got.double().cpu(), exp, rtol=2e-2, atol=2e-2 * scale, msg=lambda m: f"{name}: {m}")
    gq, gk, gv = (torch.randn_like(t) for t in (q, k, v))
    (q * gq + k * gk + v * gv).float().sum().backward()
    # float64 reference gradients through the same formulas
    x64 = x.double().requires_grad_()
    w64 = w.double().requires_grad_()
    p = (x64.reshape(b * n, d) @ w64.t()).reshape(b, n, 3, heads, dh).permute(2, 0, 3, 1, 4)
    r = [p[0], p[1], p[2]]
    if rotate:
        r[0], r[1] = _rotate_ref(r[0], c64, s64), _rotate_ref(r[1], c64, s64)
    (r[0] * gq.double().cpu() + r[1] * gk.double().cpu() + r[2] * gv.double().cpu()).sum().backward()
    for got, exp, name in ((xd.grad, x64.grad, "grad_x"), (wd.grad, w64.grad, "grad_w")):
        scale = float(exp.abs().max())
        torch.testing.assert_close(got.double().cpu(), exp, rtol=2e-2, atol=2e-2 * scale, msg=lambda m: f"{name}: {m}")
    assert nat.library().pmb_umma_timeout(1) == 0


def test_qkv_linear_rotary_matches_unfused_split(cuda_device):
    """Fused epilogue output equals the split kernel applied to the same bf16 projection, up to projection
    rounding (a one-ulp difference of the bf16 projection moves the rotated value by at most 2 ulps)."""
    torch.manual_seed(5)
    b, n, d, heads, dh = 4, 258, 192, 8, 64
    x = torch.randn(b * n, d, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(3 * heads * dh, d, device=cuda_device) / d ** 0.5).to(torch.bfloat16)
    freqs = 1.0 / (10000 ** (torch.arange(0, dh, 2, device=cuda_device).float() / dh))
    cos, sin = rotary_tables(freqs, n, cuda_device)
    planes = [torch.empty(b, n, heads, dh, dtype=torch.bfloat16, device=cuda_device) for _ in range(3)]
    st = nat.stream_handle(cuda_device)
    cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
    nat.call("pmb_qkv_linear_rotary_forward", x.data_ptr(), w.data_ptr(), cos_t.data_ptr(), sin_t.data_ptr(), b, n,
             d, heads, dh, planes[0].data_ptr(), planes[1].data_ptr(), planes[2].data_ptr(), 1, 2, 1, st)
    split = [torch.empty(b, heads, n, dh, dtype=torch.bfloat16, device=cuda_device) for _ in range(3)]
    qkv = (x.float() @ w.float().t()).to(torch.bfloat16)
    nat.call("pmb_qkv_rotary_split", qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), b, n, heads, dh,
             split[0].data_ptr(), split[1].data_ptr(), split[2].data_ptr(), 1, 2, 1, st)
    for i in range(3):
        a, e = planes[i].transpose(1, 2).float(), split[i].float()
        bad = ((a - e).abs() > 2 * 2 ** -7 * e.abs().clamp_min(1e-3) + 1e-3).float().mean().item()
        assert bad < 1e-3, f"output {i}: {bad:.2%} of values differ by more than 2 ulps"


@pytest.mark.parametrize("heads,dh", [(2, 32), (8, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_row_map_matches_permuted_input(cuda_device, dtype, heads, dh):
    """Rows ordered (outer, position, inner) with inner > 1 give the same q / k / v, gate output and input
    gradients as the permuted copy in plain (sequence, position) order: the axial transformer's time axis.
    8 heads of 64 run the streamed gate kernels, 2 heads of 32 the tiled ones."""
    from pymsst_b200.fused import AttentionGateFn

    torch.manual_seed(9)
    b, t, f, d = 2, 37, 6, 64
    x = torch.randn(b, t, f, d, device=cuda_device).to(dtype)
    w = (torch.randn(3 * heads * dh, d, device=cuda_device) / d ** 0.5)
    gw = torch.randn(heads, d, device=cuda_device) * 0.1
    gb = torch.randn(heads, device=cuda_device)
    freqs = 1.0 / (10000 ** (torch.arange(0, dh, 2, device=cuda_device).float() / dh))
    cos, sin = rotary_tables(freqs, t, cuda_device)
    ct, st = cos.t().contiguous(), sin.t().contiguous()

    def run(inp, inner):
        inp = inp.detach().requires_grad_()
        rows = inp.numel() // d
        q, k, v = QKVRotaryFn.apply(inp.reshape(rows // t, t, d), w, cos, sin, ct, st, heads, inner)
        attn = q * 0.5 + k * 0.25 + v  # any function of q, k, v in sequence order
        out = AttentionGateFn.apply(attn, inp.reshape(rows, d), gw, gb, inner)
        return inp, (q, k, v), out

    xp = x.permute(0, 2, 1, 3).contiguous()  # [b, f, t, d]: plain order, sequences (b, f)
    a_in, a_qkv, a_out = run(x, f)
    b_in, b_qkv, b_out = run(xp, 1)
    for u, v_ in zip(a_qkv, b_qkv):
        torch.testing.assert_close(u, v_, rtol=0, atol=0)
    torch.testing.assert_close(a_out.reshape(b, t, f, -1), b_out.reshape(b, f, t, -1).permute(0, 2, 1, 3),
                               rtol=0, atol=0)
    g = torch.randn_like(a_out)
    a_out.backward(g)
    b_out.backward(g.reshape(b, t, f, -1).permute(0, 2, 1, 3).reshape(b_out.shape))
    torch.testing.assert_close(a_in.grad, b_in.grad.permute(0, 2, 1, 3), rtol=1e-5, atol=1e-5)
