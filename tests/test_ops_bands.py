"""Band-wise kernels (BandSplit, grouped linear, MaskEstimator final, gate,
band gather / recombine) against the CPU oracle at model shapes.

Tolerances: fp32 kernels vs a float64 oracle, rtol 1e-4 with an absolute
floor of 1e-4 x the output scale (reductions of up to ~64K terms);
16-bit kernels vs the float64 oracle on the rounded inputs, 2e-2.
"""
from __future__ import annotations

import math

import pytest
import torch

from oracle import mel_ref, ops_ref
from pymsst_b200 import bands
from pymsst_b200 import extension as ext
from pymsst_b200.extension import ops

pytestmark = pytest.mark.gpu

BSR_WIDTHS = [4 * n for n in bands.DEFAULT_FREQS_PER_BANDS]


def _close(actual, expected, dtype, what=""):
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert actual.shape == expected.shape, f"{what}: shape {tuple(actual.shape)} vs {tuple(expected.shape)}"
    if expected.numel() == 0:
        return
    scale = max(1.0, float(expected.double().abs().max()))
    torch.testing.assert_close(actual.detach().double().cpu(), expected.double().cpu(), rtol=tol, atol=tol * scale,
                               msg=lambda m: f"{what}: {m}")


def _offsets(widths, device):
    return torch.tensor(ops_ref.offsets_from_widths(widths), dtype=torch.long, device=device)


@pytest.mark.parametrize("widths,rows,out_f", [(BSR_WIDTHS, 130, 192), ((3, 5, 2, 7), 5, 4), ((1, 1, 2), 3, 8),
                                               ((516,), 70, 33), (BSR_WIDTHS, 0, 192)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_band_split_ragged(cuda_device, widths, rows, out_f, dtype):
    total = sum(widths)
    x = (torch.randn(rows, total) * torch.rand(total) * 10).to(dtype)
    gammas = [(torch.rand(w) + 0.5).to(dtype) for w in widths]
    weights = [(torch.randn(out_f, w) / math.sqrt(w)).to(dtype) for w in widths]
    biases = [torch.randn(out_f).to(dtype) for _ in widths]
    dev = lambda ts: [t.to(cuda_device) for t in ts]  # noqa: E731
    out, normed, inv = ops.band_split_ragged_forward(x.to(cuda_device), dev(gammas), dev(weights), dev(biases),
                                                     list(widths), _offsets(widths, cuda_device))
    d64 = lambda ts: [t.double() for t in ts]  # noqa: E731
    r_out, r_normed, r_inv = ops_ref.band_split_ragged_forward(x.double(), d64(gammas), d64(weights), d64(biases),
                                                               widths)
    _close(out, r_out, dtype, "out")
    _close(normed, r_normed, dtype, "normed")
    if rows:
        torch.testing.assert_close(inv.double().cpu(), r_inv, rtol=1e-5, atol=0)
    dy = torch.randn(rows, len(widths), out_f).to(dtype)
    res = ops.band_split_ragged_backward(dy.to(cuda_device), normed, inv, dev(gammas), dev(weights), list(widths),
                                         _offsets(widths, cuda_device))
    ref = ops_ref.band_split_ragged_backward(dy.double(), normed.double().cpu(), inv.double().cpu(), d64(gammas),
                                             d64(weights), widths)
    assert len(res) == len(ref) == 1 + 3 * len(widths)
    for k, (a, e) in enumerate(zip(res, ref)):
        _close(a, e, dtype, f"grad[{k}]")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_band_split_grouped_strided(cuda_device, dtype):
    m, g, i, o = 37, 5, 12, 20
    big = torch.randn(m, g, 2 * i).to(dtype)
    x = big[:, :, ::2]  # feature stride 2
    gamma = (torch.rand(g, i) + 0.5).to(dtype)
    weight = (torch.randn(g, o, i) * 0.3).to(dtype)
    bias = torch.randn(g, o).to(dtype)
    out, normed, inv = ops.band_split_forward(big.to(cuda_device)[:, :, ::2], gamma.to(cuda_device),
                                              weight.to(cuda_device), bias.to(cuda_device))
    r_out, r_normed, r_inv = ops_ref.band_split_forward(x.double(), gamma.double(), weight.double(), bias.double())
    _close(out, r_out, dtype, "out")
    _close(normed, r_normed, dtype, "normed")
    dy = torch.randn(m, g, o).to(dtype)
    for fn in (ops.band_split_backward, ops.band_split_backward_v2, ops.band_split_backward_v3):
        res = fn(dy.to(cuda_device), normed, inv, gamma.to(cuda_device), weight.to(cuda_device), True)
        ref = ops_ref.band_split_backward(dy.double(), normed.double().cpu(), inv.double().cpu(), gamma.double(),
                                          weight.double(), True)
        for k, (a, e) in enumerate(zip(res, ref)):
            _close(a, e, dtype, f"{fn.__name__}[{k}]")
    res = ops.band_split_backward(dy.to(cuda_device), normed, inv, gamma.to(cuda_device), weight.to(cuda_device),
                                  False)
    assert res[3] is None


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_grouped_linear_forward_backward(cuda_device, act, dtype):
    m, g, i, o = 130, 62, 192, 768
    x = torch.randn(m, g, i).to(dtype)
    w = (torch.randn(g, o, i) / math.sqrt(i)).to(dtype)
    b = (torch.randn(g, o) * 0.1).to(dtype)
    xr, wr, br = (t.double().requires_grad_() for t in (x, w, b))
    ref = ops_ref.grouped_linear_forward(xr, wr, br)
    if act:
        ref = torch.tanh(ref)
    out = ops.grouped_linear_forward(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device)) if not act else \
        ext.grouped_linear_forward(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), activation=1)
    _close(out, ref, dtype, "out")
    dy = torch.randn(m, g, o).to(dtype)
    ref.backward(dy.double())
    gx, gw, gb = ext.grouped_linear_backward(dy.to(cuda_device), x.to(cuda_device), out, w.to(cuda_device),
                                             activation=act)
    # tanh' is evaluated from the stored (rounded) output; compare against the
    # oracle's exact derivative with the 16-bit tolerance.
    _close(gx, xr.grad, dtype, "grad_x")
    _close(gw, wr.grad, dtype, "grad_w")
    _close(gb, br.grad, dtype, "grad_b")


@pytest.mark.parametrize("widths,rows,hidden", [(BSR_WIDTHS, 130, 768), ((3, 4, 2, 5, 6), 4, 16), ((7,), 1, 9)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mask_estimator_final(cuda_device, widths, rows, hidden, dtype):
    nb = len(widths)
    x = torch.randn(rows, nb, hidden).to(dtype)
    weights = [(torch.randn(2 * w, hidden) / math.sqrt(hidden)).to(dtype) for w in widths]
    bias = (torch.randn(2 * sum(widths)) * 0.1).to(dtype)
    offs = _offsets(widths, cuda_device)
    out, pre, xs = ops.mask_estimator_final_direct_forward(x.to(cuda_device), [w.to(cuda_device) for w in weights],
                                                           bias.to(cuda_device), list(widths), offs)
    r_out, r_pre, _ = ops_ref.mask_estimator_final_forward(x.double(), [w.double() for w in weights], bias.double(),
                                                           widths)
    _close(out, r_out, dtype, "out")
    _close(pre, r_pre, dtype, "pre")
    dy = torch.randn(rows, sum(widths)).to(dtype)
    res = ops.mask_estimator_final_direct_backward(dy.to(cuda_device), xs, pre, [w.to(cuda_device) for w in weights],
                                                   list(widths), offs)
    ref = ops_ref.mask_estimator_final_backward(dy.double(), x.double(), pre.double().cpu(),
                                                [w.double() for w in weights], widths)
    for k, (a, e) in enumerate(zip(res, ref)):
        _close(a, e, dtype, f"grad[{k}]")


@pytest.mark.parametrize("layout", ["bhnd", "bnhd"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("bsz,heads,seq,dh,dim", [(6, 8, 62, 64, 192), (3, 4, 41, 32, 100), (2, 16, 33, 16, 64),
                                                  (5, 8, 258, 64, 384), (7, 8, 62, 64, 256)])
def test_attention_gate_strided_attention_layout(cuda_device, dtype, bsz, heads, seq, dh, dim, layout):
    """The gate reads the [batch, heads, seq, Dh] attention output in place, stored either as such ("bhnd") or as
    the [batch, seq, heads, Dh] planes the attention kernels write ("bnhd", heads contiguous).

    Shapes cover the warp-per-row kernels (bnhd, 16-bit, 8 heads x 64, dim <= 256), the streamed kernels (bnhd
    with dim 384: cp.async ring of 8-row tiles, partial last tile), the 32-row tiled kernels (bhnd, and bnhd with
    4 heads) and the row-wise fallback (dim 100 is not a multiple of the bf16 vector width)."""
    from pymsst_b200 import _native as nat

    rows = bsz * seq
    if layout == "bhnd":
        attn_bhnd = torch.randn(bsz, heads, seq, dh).to(dtype)
    else:
        attn_bhnd = torch.randn(bsz, seq, heads, dh).to(dtype).transpose(1, 2)
    x = torch.randn(rows, dim).to(dtype)
    w = (torch.randn(heads, dim) * 0.1).to(dtype)
    b = torch.randn(heads).to(dtype)
    attn_rows = attn_bhnd.permute(0, 2, 1, 3).reshape(rows, heads, dh)
    r_out, r_gate, _, _ = ops_ref.attention_gate_forward(attn_rows.double(), x.double(), w.double(), b.double())
    a_dev = attn_bhnd.to(cuda_device)  # keeps the layout's strides
    out = torch.empty(rows, heads * dh, dtype=dtype, device=cuda_device)
    gate = torch.empty(rows, heads, dtype=dtype, device=cuda_device)
    xd, wd, bd = x.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    nat.call("pmb_attention_gate_forward", a_dev.data_ptr(), seq, a_dev.stride(0), a_dev.stride(2), a_dev.stride(1),
             xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), rows, heads, dh, dim, out.data_ptr(), gate.data_ptr(),
             nat.dtype_code(dtype), nat.dtype_code(dtype), 1, nat.stream_handle(cuda_device))
    _close(out, r_out, dtype, "out")
    _close(gate, r_gate, dtype, "gate")
    dy = torch.randn(rows, heads * dh).to(dtype)
    grad_attn = torch.empty_like(a_dev)
    gx = torch.empty_like(xd)
    gw = torch.empty_like(wd)
    gb = torch.empty_like(bd)
    ws_bytes = nat.library().pmb_attention_gate_backward_workspace_size(rows, heads, dim)
    ws = nat.workspace(ws_bytes, cuda_device)
    dyd = dy.to(cuda_device)
    nat.call("pmb_attention_gate_backward", dyd.data_ptr(), a_dev.data_ptr(), seq, a_dev.stride(0), a_dev.stride(2),
             a_dev.stride(1), xd.data_ptr(), wd.data_ptr(), gate.data_ptr(), rows, heads, dh, dim,
             grad_attn.data_ptr(), gx.data_ptr(), gw.data_ptr(), gb.data_ptr(), nat.dtype_code(dtype),
             nat.dtype_code(dtype), ws.data_ptr(), ws_bytes, 1, nat.stream_handle(cuda_device))
    r = ops_ref.attention_gate_backward(dy.double(), attn_rows.double(), x.double(), w.double(),
                                        gate.double().cpu())
    _close(grad_attn.permute(0, 2, 1, 3).reshape(rows, heads, dh), r[0], dtype, "grad_attn")
    _close(gx, r[1], dtype, "grad_x")
    _close(gw, r[2], dtype, "grad_w")
    _close(gb, r[3], dtype, "grad_b")


@pytest.mark.parametrize("layout", ["mel", "split"])
def test_band_gather_and_recombine(cuda_device, layout):
    if layout == "mel":
        index = bands.mel_band_index(44100, 2048, 60, channels=2)
        ref_idx, *_ = mel_ref.mel_band_tables(44100, 2048, 60, stereo=True)
    else:
        index = bands.split_band_index(bands.DEFAULT_FREQS_PER_BANDS, channels=2)
        ref_idx = torch.arange(2050)
    tables = index.device_tables(cuda_device)
    b, t, n = 2, 13, 2
    stft = torch.randn(b, 2, 1025, t, 2)
    x = ext.band_gather(stft.to(cuda_device), tables)
    torch.testing.assert_close(x.cpu(), mel_ref.gather(stft, ref_idx), rtol=0, atol=0)
    gx = torch.randn_like(x)
    g_stft = ext.band_gather_backward(gx, tables, channels=2, freqs=1025)
    ref_stft = stft.double().requires_grad_()
    mel_ref.gather(ref_stft, ref_idx).backward(gx.double().cpu())
    torch.testing.assert_close(g_stft.double().cpu(), ref_stft.grad, rtol=1e-6, atol=1e-6)

    mask = torch.randn(b, n, t, index.pairs * 2)
    for multiply in (True, False):
        out = ext.band_recombine(mask.to(cuda_device), stft.to(cuda_device), tables, 2, 1025, multiply=multiply)
        m64 = mask.double().requires_grad_()
        ref = mel_ref.recombine(m64, stft.double(), ref_idx, multiply=multiply)
        torch.testing.assert_close(out.double().cpu(), ref, rtol=1e-5, atol=1e-5)
        gout = torch.randn_like(out)
        gm = ext.band_recombine_backward(gout, stft.to(cuda_device), tables, multiply=multiply)
        ref.backward(gout.double().cpu())
        torch.testing.assert_close(gm.double().cpu(), m64.grad, rtol=1e-5, atol=1e-5)
