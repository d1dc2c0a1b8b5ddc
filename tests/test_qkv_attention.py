"""Projection + rotary + attention as one autograd Function (QKVAttentionFn): the attention backward writes the
projection gradient with dQ / dK rotated back (pmb_attention_backward_rotary), against the two-Function path
(QKVRotaryFn + AttentionFn, whose backward merges the three gradients with the inverse rotation) and a float64
restatement of projection, rotation and attention.

Tolerances: the forward is the same kernels on both paths (bit-identical); input / weight gradients differ from
the two-Function path only in where a 16-bit rounding happens (the fused path rotates the fp32 gradient before
rounding it once), so they are compared at 1e-2 of their scale, and against float64 at the 16-bit bar of the
attention tests (3e-2 of the scale).
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200 import _native as nat
from pymsst_b200.fused import AttentionFn, QKVAttentionFn, QKVAttentionGateFn, QKVRotaryFn, rotary_tables

pytestmark = pytest.mark.gpu


def _rotate_ref(t, cos, sin):
    e, o = t[..., 0::2], t[..., 1::2]
    out = torch.empty_like(t)
    out[..., 0::2] = e * cos - o * sin
    out[..., 1::2] = o * cos + e * sin
    return out


def _inputs(device, b, n, d, heads, seed, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, n, d, generator=g).to(dt)
    w = torch.randn(3 * heads * 64, d, generator=g) / d ** 0.5
    gy = torch.randn(b, heads, n, 64, generator=g).to(dt)
    freqs = 1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64))
    cos, sin = rotary_tables(freqs.to(device), n, device)
    return x.to(device), w.to(device), gy.to(device), cos, sin


def _grads(fn, x, w, gy):
    xr, wr = x.clone().requires_grad_(), w.clone().requires_grad_()
    o = fn(xr, wr)
    gx, gw = torch.autograd.grad(o, (xr, wr), gy)
    return o.detach(), gx, gw


# n = 62: two sequences per backward item; 100: one per item; 258: the long-sequence kernels (backend "pmb")
@pytest.mark.parametrize("b,n,d,heads", [(33, 62, 192, 8), (5, 100, 192, 8), (3, 258, 192, 8), (4, 62, 384, 8)])
@pytest.mark.parametrize("rotate", [True, False])
def test_qkv_attention_matches_two_function_path(cuda_device, b, n, d, heads, rotate):
    x, w, gy, cos, sin = _inputs(cuda_device, b, n, d, heads, seed=b * n + d)
    if not rotate:
        cos = sin = None

    def fused(xr, wr):
        return QKVAttentionFn.apply(xr, wr, cos, sin, None, None, heads)

    def split(xr, wr):
        q, k, v = QKVRotaryFn.apply(xr, wr, cos, sin, None, None, heads)
        return AttentionFn.apply(q, k, v)

    o1, gx1, gw1 = _grads(fused, x, w, gy)
    o2, gx2, gw2 = _grads(split, x, w, gy)
    assert torch.equal(o1, o2)
    for got, exp, name in ((gx1, gx2, "grad_x"), (gw1, gw2, "grad_w")):
        scale = float(exp.abs().max())
        torch.testing.assert_close(got.float(), exp.float(), rtol=1e-2, atol=1e-2 * scale,
                                   msg=lambda m: f"{name}: {m}")
    assert nat.library().pmb_umma_timeout(1) == 0


@pytest.mark.parametrize("b,n", [(9, 62), (2, 258)])
def test_qkv_attention_matches_float64(cuda_device, b, n):
    d, heads = 192, 8
    x, w, gy, cos, sin = _inputs(cuda_device, b, n, d, heads, seed=7 * n)
    o, gx, gw = _grads(lambda xr, wr: QKVAttentionFn.apply(xr, wr, cos, sin, None, None, heads), x, w, gy)
    x64 = x.double().cpu().requires_grad_()
    w64 = w.double().cpu().to(torch.bfloat16).double().requires_grad_()  # the kernels read W in bf16
    p = (x64.reshape(b * n, d) @ w64.t()).reshape(b, n, 3, heads, 64).permute(2, 0, 3, 1, 4)
    c64, s64 = cos.double().cpu(), sin.double().cpu()
    q, k, v = _rotate_ref(p[0], c64, s64), _rotate_ref(p[1], c64, s64), p[2]
    att = torch.softmax(q @ k.transpose(-1, -2) / 8.0, dim=-1) @ v
    att.backward(gy.double().cpu())
    for got, exp, name in ((o, att.detach(), "out"), (gx, x64.grad, "grad_x"), (gw, w64.grad, "grad_w")):
        scale = float(exp.abs().max())
        torch.testing.assert_close(got.double().cpu(), exp, rtol=3e-2, atol=3e-2 * scale,
                                   msg=lambda m: f"{name}: {m}")
    assert nat.library().pmb_umma_timeout(1) == 0


def test_rotary_backward_entry_matches_merge(cuda_device):
    """pmb_attention_backward_rotary into strided views of the projection gradient equals
    pmb_attention_backward followed by pmb_qkv_rotary_merge, up to the one rounding the merge adds."""
    from pymsst_b200.fused import _attn_strides, _bnhd_empty

    b, n, h = 17, 62, 8
    g = torch.Generator().manual_seed(3)
    q, k, v, go = (torch.randn(b, n, h, 64, generator=g).to(torch.bfloat16).to(cuda_device).transpose(1, 2)
                   for _ in range(4))
    freqs = 1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64))
    cos, sin = rotary_tables(freqs.to(cuda_device), n, cuda_device)
    st = nat.stream_handle(cuda_device)
    o = _bnhd_empty(b, h, n, 64, torch.bfloat16, cuda_device)
    lse = torch.empty(b * h, (n + 3) // 4 * 4, dtype=torch.float32, device=cuda_device)
    nat.call("pmb_attention_forward", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, n, h,
             64, nat.i64_array(_attn_strides(q, k, v, o)), 0.125, 2, st)
    wsb = int(nat.library().pmb_attention_backward_workspace_size(b, n, h))
    ws = nat.workspace(wsb, cuda_device)
    dq, dk, dv = (_bnhd_empty(b, h, n, 64, torch.bfloat16, cuda_device) for _ in range(3))
    nat.call("pmb_attention_backward", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), go.data_ptr(),
             lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, n, h, 64,
             nat.i64_array(_attn_strides(q, k, v, o, go, dq, dk, dv)), 0.125, 2, ws.data_ptr(), wsb, st)
    merged = torch.empty(b * n, 3 * h * 64, dtype=torch.bfloat16, device=cuda_device)
    sd = dq.stride()
    nat.call("pmb_qkv_rotary_merge", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), cos.data_ptr(), sin.data_ptr(), b,
             n, h, 64, merged.data_ptr(), 1, 2, sd[0], sd[1], sd[2], 1, st)
    direct = torch.empty_like(merged)
    parts = direct.view(b, n, 3, h, 64)
    views = [parts[:, :, i].transpose(1, 2) for i in range(3)]
    nat.call("pmb_attention_backward_rotary", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), go.data_ptr(),
             lse.data_ptr(), cos.data_ptr(), sin.data_ptr(), *(t.data_ptr() for t in views), b, n, h, 64,
             nat.i64_array(_attn_strides(q, k, v, o, go, *views)), 0.125, 2, ws.data_ptr(), wsb, st)
    torch.cuda.synchronize(cuda_device)
    # dV is the same rounding of the same value on both paths
    assert torch.equal(direct[:, 2 * h * 64:], merged[:, 2 * h * 64:])
    scale = float(merged.float().abs().max())
    torch.testing.assert_close(direct.float(), merged.float(), rtol=1e-2, atol=2e-2 * scale)
    assert nat.library().pmb_umma_timeout(1) == 0


# ------------------------------------------------------------------ head gate folded into the attention kernels
def _gate_params(device, d, heads, seed):
    g = torch.Generator().manual_seed(seed)
    wg = (torch.randn(heads, d, generator=g) / d ** 0.5).to(device)
    bg = (torch.randn(heads, generator=g) * 0.5).to(device)
    return wg, bg


@pytest.mark.parametrize("b,n,d,heads", [(33, 62, 192, 8), (6, 60, 384, 8), (5, 17, 192, 4)])
@pytest.mark.parametrize("rotate", [True, False])
def test_qkv_attention_gate_matches_separate_gate(cuda_device, b, n, d, heads, rotate):
    """QKVAttentionGateFn against QKVAttentionFn + AttentionGateFn on the same inputs.  The two compute the gate
    logits differently (a 16-bit GEMM as autocast does, against the gate kernel's fp32 dot products with the fp32
    weight), so outputs and gradients agree at the 16-bit bar (2e-2 of the scale)."""
    from pymsst_b200.fused import AttentionGateFn

    x, w, gy, cos, sin = _inputs(cuda_device, b, n, d, heads, seed=3 * b + n)
    wg, bg = _gate_params(cuda_device, d, heads, seed=n)
    gy = gy.transpose(1, 2).reshape(b * n, heads * 64)
    if not rotate:
        cos = sin = None

    def run(fused):
        xr, wr, wgr, bgr = (t.clone().requires_grad_() for t in (x, w, wg, bg))
        if fused:
            out = QKVAttentionGateFn.apply(xr, wr, cos, sin, None, None, heads, wgr, bgr)
        else:
            o = QKVAttentionFn.apply(xr, wr, cos, sin, None, None, heads)
            out = AttentionGateFn.apply(o, xr.reshape(b * n, d), wgr, bgr, 1)
        grads = torch.autograd.grad(out, (xr, wr, wgr, bgr), gy)
        return (out.detach(), *grads)

    got, exp = run(True), run(False)
    for a, e, name in zip(got, exp, ("out", "grad_x", "grad_w", "grad_w_gate", "grad_b_gate")):
        scale = float(e.abs().max())
        torch.testing.assert_close(a.float(), e.float(), rtol=2e-2, atol=2e-2 * scale, msg=lambda m: f"{name}: {m}")
    assert nat.library().pmb_umma_timeout(1) == 0


def test_qkv_attention_gate_matches_float64(cuda_device):
    from pymsst_b200.fused import QKVAttentionGateFn

    b, n, d, heads = 9, 62, 192, 8
    x, w, gy, cos, sin = _inputs(cuda_device, b, n, d, heads, seed=21)
    wg, bg = _gate_params(cuda_device, d, heads, seed=22)
    gy = gy.transpose(1, 2).reshape(b * n, heads * 64)
    xr, wr, wgr, bgr = (t.clone().requires_grad_() for t in (x, w, wg, bg))
    out = QKVAttentionGateFn.apply(xr, wr, cos, sin, None, None, heads, wgr, bgr)
    grads = torch.autograd.grad(out, (xr, wr, wgr, bgr), gy)
    # float64: the kernels read W, W_g and b_g in bf16
    x64 = x.double().cpu().requires_grad_()
    w64, wg64, bg64 = (t.double().cpu().to(torch.bfloat16).double().requires_grad_() for t in (w, wg, bg))
    p = (x64.reshape(b * n, d) @ w64.t()).reshape(b, n, 3, heads, 64).permute(2, 0, 3, 1, 4)
    c64, s64 = cos.double().cpu(), sin.double().cpu()
    q, k, v = _rotate_ref(p[0], c64, s64), _rotate_ref(p[1], c64, s64), p[2]
    att = torch.softmax(q @ k.transpose(-1, -2) / 8.0, dim=-1) @ v  # [b, h, n, 64]
    gate = torch.sigmoid(x64.reshape(b * n, d) @ wg64.t() + bg64)  # [b * n, h]
    ref = (att.transpose(1, 2).reshape(b * n, heads, 64) * gate[:, :, None]).reshape(b * n, heads * 64)
    rgrads = torch.autograd.grad(ref, (x64, w64, wg64, bg64), gy.double().cpu())
    for a, e, name in zip((out, *grads), (ref, *rgrads), ("out", "grad_x", "grad_w", "grad_w_gate", "grad_b_gate")):
        scale = float(e.abs().max())
        torch.testing.assert_close(a.double().cpu(), e.detach(), rtol=3e-2, atol=3e-2 * scale,
                                   msg=lambda m: f"{name}: {m}")
    assert nat.library().pmb_umma_timeout(1) == 0
