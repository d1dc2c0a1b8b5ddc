"""Band layouts of BS-RoFormer and Mel-band RoFormer (host-side tables).

BS-RoFormer splits the 1025 STFT bins into 62 contiguous bands
(``DEFAULT_FREQS_PER_BANDS``).  Mel-band RoFormer builds ``num_bands``
overlapping bands from a Slaney mel filterbank: bin f belongs to band b where
the filter weight is > 0, with the first bin forced into the first band and the
last bin into the last band (pymss-core's MelBandRoformer, as exercised by the
reference's tests/test_training_smoke.py:40-65; the filterbank is
``librosa.filters.mel``'s published algorithm, computed here with numpy in the
same float64 / float32 steps).

Both layouts are described by one ``BandIndex``: ``index[j] = f*S + s`` is the
(frequency, channel) pair that feeds band feature j (stereo interleaved), and
the CSR inverse (``inv_ptr``, ``inv_idx``) lists, for every pair, the features
it feeds.  The CUDA gather / recombine kernels take these as int32 tables.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

DEFAULT_FREQS_PER_BANDS = (
    (2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8 + (128, 129)
)


def _hz_to_mel(f: np.ndarray) -> np.ndarray:
    f_sp = 200.0 / 3
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    f = np.asarray(f, dtype=np.float64)
    mel = f / f_sp
    high = f >= min_log_hz
    mel = np.where(high, min_log_mel + np.log(np.maximum(f, 1e-30) / min_log_hz) / logstep, mel)
    return mel


def _mel_to_hz(m: np.ndarray) -> np.ndarray:
    f_sp = 200.0 / 3
    min_log_hz = 1000.0
    min_log_mel = min_log_hz / f_sp
    logstep = np.log(6.4) / 27.0
    m = np.asarray(m, dtype=np.float64)
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), f_sp * m)


def mel_filterbank(sample_rate: int, n_fft: int, n_mels: int) -> np.ndarray:
    """Slaney-scale, Slaney-normalised triangular filters, float32 [n_mels, n_fft//2+1]."""
    n_freqs = n_fft // 2 + 1
    fft_freqs = np.arange(n_freqs) * (1.0 / (n_fft * (1.0 / sample_rate)))
    mels = np.linspace(_hz_to_mel(0.0), _hz_to_mel(float(sample_rate) / 2), n_mels + 2)
    pts = _mel_to_hz(mels)
    fdiff = np.diff(pts)
    ramps = pts[:, None] - fft_freqs[None, :]
    weights = np.zeros((n_mels, n_freqs), dtype=np.float32)
    for i in range(n_mels):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        weights[i] = np.maximum(0, np.minimum(lower, upper))
    enorm = 2.0 / (pts[2 : n_mels + 2] - pts[:n_mels])
    weights *= enorm[:, None]
    return weights


def mel_band_membership(sample_rate: int, n_fft: int, num_bands: int) -> np.ndarray:
    """bool [num_bands, n_fft//2+1]: bin f is in band b (edges forced)."""
    fb = mel_filterbank(sample_rate, n_fft, num_bands)
    fb[0, 0] = 1.0
    fb[-1, -1] = 1.0
    bands = fb > 0
    if not bands.any(axis=0).all():
        raise ValueError("every frequency must be covered by a mel band")
    return bands


@dataclass(frozen=True)
class BandIndex:
    """Feature <-> (frequency, channel) tables for one band layout."""

    index: np.ndarray  # int64 [J]  pair feeding feature j (f*S + s)
    freqs_per_band: tuple[int, ...]  # bins per band
    channels: int
    freqs: int

    @property
    def pairs(self) -> int:
        return int(self.index.shape[0])

    @property
    def dim_inputs(self) -> tuple[int, ...]:
        """Band-split input widths: 2 (re/im) * channels * bins, per band."""
        return tuple(2 * self.channels * n for n in self.freqs_per_band)

    @property
    def counts(self) -> np.ndarray:
        """Features per (f*S + s) pair: bands covering that bin."""
        return np.bincount(self.index, minlength=self.freqs * self.channels)

    def inverse(self) -> tuple[np.ndarray, np.ndarray]:
        """CSR inverse (inv_ptr [F*S+1], inv_idx [J]) of ``index`` (ascending j per pair)."""
        order = np.argsort(self.index, kind="stable")
        ptr = np.zeros(self.freqs * self.channels + 1, dtype=np.int64)
        np.cumsum(self.counts, out=ptr[1:])
        return ptr, order

    def is_identity(self) -> bool:
        return self.pairs == self.freqs * self.channels and bool(np.all(self.index == np.arange(self.pairs)))

    def device_tables(self, device: torch.device) -> dict[str, torch.Tensor]:
        ptr, inv = self.inverse()
        return {
            "index": torch.as_tensor(self.index, dtype=torch.int32, device=device),
            "inv_ptr": torch.as_tensor(ptr, dtype=torch.int32, device=device),
            "inv_idx": torch.as_tensor(inv, dtype=torch.int32, device=device),
        }


def split_band_index(freqs_per_band, channels: int) -> BandIndex:
    """BS-RoFormer: contiguous, non-overlapping bands (identity index)."""
    freqs = int(sum(freqs_per_band))
    return BandIndex(np.arange(freqs * channels, dtype=np.int64), tuple(int(n) for n in freqs_per_band), channels,
                     freqs)


def mel_band_index(sample_rate: int, n_fft: int, num_bands: int, channels: int) -> BandIndex:
    """Mel-band RoFormer: overlapping mel bands, stereo interleaved as 2*f + s."""
    bands = mel_band_membership(sample_rate, n_fft, num_bands)
    freqs = bands.shape[1]
    per_band = np.nonzero(bands)[1]  # row-major: band 0's bins ascending, then band 1 ...
    index = (per_band[:, None] * channels + np.arange(channels)[None, :]).reshape(-1)
    return BandIndex(index.astype(np.int64), tuple(int(n) for n in bands.sum(1)), channels, freqs)
