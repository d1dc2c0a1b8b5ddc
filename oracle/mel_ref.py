"""Mel-band tables and gather / scatter-add-average recombination (CPU).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The Mel-band RoFormer of pymss-core 0.1.4 (absent here; reached from
src/pymsst/training/fused_roformer.py:827-873 and exercised by
tests/test_training_smoke.py:40-65) builds its bands from
``librosa.filters.mel(sr, n_fft, n_mels)`` (Slaney mel scale, Slaney area
normalisation, float32 weights), marks bin f in band b where the weight is
> 0, forces the first bin into the first band and the last bin into the last
band, and interleaves stereo channels as index 2*f + s.  librosa (ISC) is not
installed; ``slaney_mel_filterbank`` restates its published algorithm with
plain Python loops in float64, casting to float32 where librosa's array is
float32.  It is cross-checked against torchaudio's independent
``melscale_fbanks`` in tests/test_mel_tables.py.
"""
from __future__ import annotations

import math

import numpy as np
import torch

_F_SP = 200.0 / 3.0  # Hz per mel below 1 kHz (Slaney)
_MIN_LOG_HZ = 1000.0
_MIN_LOG_MEL = _MIN_LOG_HZ / _F_SP
_LOGSTEP = math.log(6.4) / 27.0


def hz_to_mel(f: float) -> float:
    if f >= _MIN_LOG_HZ:
        return _MIN_LOG_MEL + math.log(f / _MIN_LOG_HZ) / _LOGSTEP
    return f / _F_SP


def mel_to_hz(m: float) -> float:
    if m >= _MIN_LOG_MEL:
        return _MIN_LOG_HZ * math.exp(_LOGSTEP * (m - _MIN_LOG_MEL))
    return _F_SP * m


def slaney_mel_filterbank(sample_rate: int, n_fft: int, n_mels: int) -> np.ndarray:
    """float32 [n_mels, n_fft//2 + 1] triangular filters, Slaney-normalised."""
    n_freqs = n_fft // 2 + 1
    fmax = float(sample_rate) / 2
    # numpy.fft.rfftfreq(n_fft, d=1/sr): k * (1 / (n_fft * (1/sr)))
    bin_hz = 1.0 / (n_fft * (1.0 / sample_rate))
    fft_freqs = [k * bin_hz for k in range(n_freqs)]
    # numpy.linspace(lo, hi, n_mels + 2): i * step + lo, last point exactly hi
    lo, hi = hz_to_mel(0.0), hz_to_mel(fmax)
    step = (hi - lo) / (n_mels + 1)
    mels = [i * step + lo for i in range(n_mels + 1)] + [hi]
    mel_pts = [mel_to_hz(m) for m in mels]
    weights = np.zeros((n_mels, n_freqs), dtype=np.float32)
    for i in range(n_mels):
        d_lo = mel_pts[i + 1] - mel_pts[i]
        d_hi = mel_pts[i + 2] - mel_pts[i + 1]
        enorm = 2.0 / (mel_pts[i + 2] - mel_pts[i])
        for k, f in enumerate(fft_freqs):
            rising = -(mel_pts[i] - f) / d_lo
            falling = (mel_pts[i + 2] - f) / d_hi
            w32 = np.float32(max(0.0, min(rising, falling)))
            weights[i, k] = np.float32(float(w32) * enorm)
    return weights


def mel_band_tables(sample_rate: int, n_fft: int, num_bands: int, stereo: bool):
    """(freq_indices int64 [J], num_freqs_per_band [nb], num_bands_per_freq [F], bands bool [nb, F])."""
    fb = torch.from_numpy(slaney_mel_filterbank(sample_rate, n_fft, num_bands))
    fb[0, 0] = 1.0
    fb[-1, -1] = 1.0
    bands = fb > 0
    assert bands.any(dim=0).all(), "every frequency must be covered by a band"
    n_freqs = bands.shape[1]
    indices = torch.arange(n_freqs).repeat(num_bands, 1)[bands]
    if stereo:
        indices = (indices[:, None] * 2 + torch.arange(2)).reshape(-1)
    return indices, bands.sum(1), bands.sum(0), bands


def gather(stft: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """stft [B,S,F,T,2] -> feats [B,T,J*2]; feature j reads pair index[j] = f*S + s."""
    b, s, f, t, _ = stft.shape
    pairs = stft.permute(0, 2, 1, 3, 4).reshape(b, f * s, t, 2)  # 'b s f t c -> b (f s) t c'
    x = pairs[:, index]  # [B, J, T, 2]
    return x.permute(0, 2, 1, 3).reshape(b, t, -1)


def recombine(mask: torch.Tensor, stft: torch.Tensor, index: torch.Tensor, multiply: bool = True) -> torch.Tensor:
    """mask [B,N,T,J*2] -> out [B,N,S,F,T,2]: scatter-add over pairs / per-pair band count, times stft."""
    b, s, f, t, _ = stft.shape
    n = mask.shape[1]
    m = mask.reshape(b, n, t, -1, 2).permute(0, 1, 3, 2, 4)  # [B,N,J,T,2]
    summed = torch.zeros(b, n, f * s, t, 2, dtype=mask.dtype, device=mask.device)
    summed.index_add_(2, index, m)
    count = torch.zeros(f * s, dtype=mask.dtype, device=mask.device).index_add_(
        0, index, torch.ones(index.numel(), dtype=mask.dtype, device=mask.device))
    avg = summed / count.clamp_min(1e-8)[None, None, :, None, None]
    avg = avg.reshape(b, n, f, s, t, 2).permute(0, 1, 3, 2, 4, 5)  # [B,N,S,F,T,2]
    if not multiply:
        return avg
    st = stft[:, None]
    re = st[..., 0] * avg[..., 0] - st[..., 1] * avg[..., 1]
    im = st[..., 0] * avg[..., 1] + st[..., 1] * avg[..., 0]
    return torch.stack((re, im), -1)
