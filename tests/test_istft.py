"""iSTFT of the model output: torch.fft.irfft per frame plus the overlap-add kernel pair
(pmb_istft_overlap_add_forward / _backward via ISTFTOverlapAddFn, as roformer._istft_overlap_add runs it) against
torch.istft, value and the gradient with respect to the spectrum, to fp32 summation-order differences (1e-5 of the
largest value)."""
from __future__ import annotations

import pytest
import torch

from pymsst_b200.roformer import _istft_overlap_add

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_fft,hop,win,frames,length", [
    (2048, 512, 2048, 258, 131584),   # config 3's STFT
    (2048, 512, 2048, 40, None),       # no target length: the centre-trimmed signal
    (1024, 300, 800, 31, 9000),        # hop not dividing n_fft, window shorter than n_fft
    (1024, 256, 1024, 31, 9000),       # a target length past the signal's end: zeros there
])
@pytest.mark.parametrize("normalized", [False, True])
def test_istft_matches_torch(cuda_device, n_fft, hop, win, frames, length, normalized):
    g = torch.Generator().manual_seed(n_fft + hop + frames)
    z = torch.randn(3, n_fft // 2 + 1, frames, 2, generator=g).to(cuda_device)
    w = torch.hann_window(win, device=cuda_device)
    za = torch.view_as_complex(z.clone()).requires_grad_()
    ours = _istft_overlap_add(za, n_fft, hop, w, normalized, length)
    gy = torch.randn(ours.shape, generator=g).to(cuda_device)
    (gz,) = torch.autograd.grad(ours, za, gy)
    zb = torch.view_as_complex(z.clone()).requires_grad_()
    ref = torch.istft(zb, n_fft=n_fft, hop_length=hop, win_length=win, window=w, center=True, normalized=normalized,
                      onesided=True, length=length)
    (gr,) = torch.autograd.grad(ref, zb, gy)
    assert ours.shape == ref.shape
    torch.testing.assert_close(ours, ref, rtol=1e-5, atol=1e-5 * float(ref.abs().max()))
    torch.testing.assert_close(torch.view_as_real(gz), torch.view_as_real(gr), rtol=1e-5,
                               atol=1e-5 * float(torch.view_as_real(gr).abs().max()))
