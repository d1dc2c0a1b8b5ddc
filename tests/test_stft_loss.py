"""STFT framing of the multi-resolution STFT loss (STFTFramesFn / pmb_stft_frames_backward) against torch.stft.

The forward is torch.stft's own framing (reflect padding, unfold, window, real FFT), so spectra agree to fp32
rounding; the backward replaces torch's atomic index_add / reflection-pad backward with one overlap-add per
sample, so input gradients agree to fp32 summation-order differences (1e-5 relative to the largest).
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from pymsst_b200 import _native as nat

HOP = 147


def _window(win, n_fft, device):
    w = torch.hann_window(win, device=device)
    left = (n_fft - win) // 2
    return torch.nn.functional.pad(w, (left, n_fft - win - left)).contiguous()


@pytest.mark.gpu
@pytest.mark.parametrize("win", [4096, 2048, 1024, 512, 256])
@pytest.mark.parametrize("length", [131584, 5000, 1025])
def test_stft_frames_match_torch_stft(cuda_device, win, length):
    from pymsst_b200.fused import stft_loss_spectrum

    n_fft = max(win, 2048)
    if n_fft // 2 >= length:
        pytest.skip("reflect padding needs n_fft / 2 < length")
    g = torch.Generator().manual_seed(win + length)
    x = torch.randn(3, length, generator=g).to(cuda_device)
    t = torch.randn(3, length, generator=g).to(cuda_device)
    w_small = torch.hann_window(win, device=cuda_device)

    xa = x.clone().requires_grad_()
    ours = stft_loss_spectrum(xa, n_fft, HOP, _window(win, n_fft, cuda_device), False)
    ref_x = x.clone().requires_grad_()
    ref = torch.stft(ref_x, n_fft=n_fft, hop_length=HOP, win_length=win, window=w_small, return_complex=True)
    assert ours.shape == ref.transpose(1, 2).shape
    torch.testing.assert_close(ours, ref.transpose(1, 2), rtol=1e-5, atol=1e-4)

    target_ref = torch.stft(t, n_fft=n_fft, hop_length=HOP, win_length=win, window=w_small, return_complex=True)
    torch.nn.functional.l1_loss(ours, target_ref.transpose(1, 2)).backward()
    torch.nn.functional.l1_loss(ref, target_ref).backward()
    err = (xa.grad - ref_x.grad).abs().max() / ref_x.grad.abs().max()
    assert float(err) < 1e-5, float(err)


@pytest.mark.gpu
def test_stft_frames_backward_is_deterministic(cuda_device):
    from pymsst_b200.fused import stft_loss_spectrum

    x = torch.randn(2, 20000, device=cuda_device)
    grads = []
    for _ in range(2):
        xa = x.clone().requires_grad_()
        stft_loss_spectrum(xa, 4096, HOP, _window(4096, 4096, cuda_device), False).abs().sum().backward()
        grads.append(xa.grad)
    assert torch.equal(grads[0], grads[1])


# ------------------------------------------------------------- host side (CPU)
def _lib():
    try:
        return nat.library()
    except nat.FusedKernelUnavailable as e:  # pragma: no cover - library not built
        pytest.skip(str(e))


@pytest.mark.parametrize(
    "length, n_fft, frames, message",
    [(1000, 2048, 1, "reflect padding"), (10000, 2048, 5, "frame count")],
)
@pytest.mark.parametrize("entry", ["pmb_stft_frames_forward", "pmb_stft_frames_backward"])
def test_stft_frames_rejects_bad_shapes(entry, length, n_fft, frames, message):
    lib = _lib()
    st = getattr(lib, entry)(None, None, None, 1, length, n_fft, HOP, frames, None)
    assert st != 0 and message in lib.pmb_last_error().decode()


@pytest.mark.parametrize("n", [16, 17, 2048])
@pytest.mark.parametrize("norm", ["backward", "ortho", "forward"])
def test_real_fft_backward_matches_torch(n, norm):
    """RealFFTFn's backward (half-weighted inner bins through an inverse real FFT) equals torch's rfft backward
    (zero-padded complex FFT) in float64, for even and odd lengths and every normalisation."""
    from pymsst_b200.fused import RealFFTFn

    g = torch.Generator().manual_seed(n)
    x = torch.randn(3, 5, n, dtype=torch.float64, generator=g, requires_grad=True)
    gy = torch.randn(3, 5, n // 2 + 1, dtype=torch.complex128, generator=g)
    want, = torch.autograd.grad(torch.fft.rfft(x, norm=norm), x, gy)
    got, = torch.autograd.grad(RealFFTFn.apply(x, norm), x, gy)
    assert got.is_contiguous()
    torch.testing.assert_close(got, want, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("win", [4096, 2048, 256])
@pytest.mark.parametrize("normalized", [False, True])
def test_stft_l1_loss_matches_torch(cuda_device, win, normalized):
    """stft_l1_loss (framing kernels + rfft + SpectralL1Fn's one-pass mean and gradient) against
    F.l1_loss(torch.stft(recon), torch.stft(target)): value and the recon gradient to 1e-5 relative."""
    from pymsst_b200.fused import stft_l1_loss

    n_fft = max(win, 2048)
    g = torch.Generator().manual_seed(win + int(normalized))
    x = torch.randn(3, 9000, generator=g).to(cuda_device)
    t = torch.randn(3, 9000, generator=g).to(cuda_device)
    w = torch.hann_window(win, device=cuda_device)
    xa = x.clone().requires_grad_()
    ours = stft_l1_loss(xa, t, n_fft, HOP, _window(win, n_fft, cuda_device), normalized)
    (gx,) = torch.autograd.grad(ours, xa, torch.tensor(1.7, device=cuda_device))
    xb = x.clone().requires_grad_()
    kw = dict(n_fft=n_fft, hop_length=HOP, win_length=win, window=w, normalized=normalized, return_complex=True)
    ref = torch.nn.functional.l1_loss(torch.stft(xb, **kw), torch.stft(t, **kw))
    (gr,) = torch.autograd.grad(ref, xb, torch.tensor(1.7, device=cuda_device))
    torch.testing.assert_close(ours, ref, rtol=1e-5, atol=0)
    torch.testing.assert_close(gx, gr, rtol=1e-5, atol=1e-5 * float(gr.abs().max()))


@pytest.mark.gpu
def test_spectral_l1_zero_difference_and_odd_count(cuda_device):
    """Equal spectra give loss 0 and gradient 0 (torch's convention for |z| at 0); an odd element count takes the
    scalar tail of the vectorised sum."""
    from pymsst_b200.fused import SpectralL1Fn

    frames = torch.randn(3, 1, 2048, device=cuda_device).requires_grad_()  # 3 x 1025 = odd count
    with torch.no_grad():
        same = torch.fft.rfft(frames, dim=-1)
    loss = SpectralL1Fn.apply(frames, same, "backward")
    (g,) = torch.autograd.grad(loss, frames)
    assert float(loss) == 0.0 and torch.count_nonzero(g) == 0
    other = torch.randn(3, 1, 1025, dtype=torch.complex64, device=cuda_device)
    loss = SpectralL1Fn.apply(frames, other, "backward")
    ref = torch.nn.functional.l1_loss(torch.fft.rfft(frames.detach(), dim=-1), other)
    torch.testing.assert_close(loss, ref, rtol=1e-5, atol=0)
