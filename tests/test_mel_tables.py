"""Band tables: the product's mel tables are bit-exact with the oracle's
restatement of librosa's Slaney filterbank, which agrees with torchaudio's
independent filterbank on every >0 decision except the forced last bin."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import torchaudio

from oracle import mel_ref
from pymsst_b200 import bands


@pytest.mark.parametrize("sr,n_fft,n_mels", [(44100, 2048, 60), (44100, 64, 8), (44100, 4096, 128), (48000, 2048, 64)])
def test_filterbank_matches_oracle_bitwise(sr, n_fft, n_mels):
    ours = bands.mel_filterbank(sr, n_fft, n_mels)
    ref = mel_ref.slaney_mel_filterbank(sr, n_fft, n_mels)
    assert ours.dtype == np.float32
    np.testing.assert_array_equal(ours > 0, ref > 0)
    np.testing.assert_allclose(ours, ref, rtol=1e-6, atol=1e-12)


@pytest.mark.parametrize("sr,n_fft,n_mels", [(44100, 2048, 60), (44100, 64, 8)])
def test_oracle_filterbank_pinned_to_torchaudio(sr, n_fft, n_mels):
    ref = mel_ref.slaney_mel_filterbank(sr, n_fft, n_mels)
    ta = torchaudio.functional.melscale_fbanks(n_fft // 2 + 1, 0.0, sr / 2, n_mels, sr, norm="slaney",
                                               mel_scale="slaney").T.numpy()
    np.testing.assert_allclose(ref, ta, atol=1e-6)
    mismatch = np.argwhere((ref > 0) != (ta > 0))
    # Only the last bin of the last band may differ (a ~1e-18 weight that
    # pymss-core forces to 1 anyway); the first bin is 0 in both and forced.
    assert all(tuple(m) == (n_mels - 1, n_fft // 2) for m in mismatch)


def test_mel_index_tables_bit_exact():
    ours = bands.mel_band_index(44100, 2048, 60, channels=2)
    idx, nfb, nbf, _ = mel_ref.mel_band_tables(44100, 2048, 60, stereo=True)
    np.testing.assert_array_equal(ours.index, idx.numpy())
    assert ours.freqs_per_band == tuple(nfb.tolist())
    np.testing.assert_array_equal(ours.counts.reshape(-1, 2)[:, 0], nbf.numpy())
    assert sum(ours.freqs_per_band) == 1979
    assert ours.pairs == 1979 * 2
    assert ours.counts.min() >= 1 and ours.counts.max() == 2


def test_reference_tiny_mel_config():
    """The reference's tiny test model: n_fft 64, 8 bands (tests/test_training_smoke.py:61-65)."""
    ours = bands.mel_band_index(44100, 64, 8, channels=2)
    assert ours.freqs_per_band == (2, 2, 2, 3, 5, 7, 12, 20)
    assert ours.dim_inputs == tuple(4 * n for n in ours.freqs_per_band)


def test_split_index_is_identity_and_bsr_widths():
    idx = bands.split_band_index(bands.DEFAULT_FREQS_PER_BANDS, channels=2)
    assert len(bands.DEFAULT_FREQS_PER_BANDS) == 62
    assert sum(bands.DEFAULT_FREQS_PER_BANDS) == 1025
    assert idx.is_identity()
    assert sum(idx.dim_inputs) == 4100
    ptr, inv = idx.inverse()
    np.testing.assert_array_equal(ptr, np.arange(2051))


def test_inverse_tables_round_trip():
    idx = bands.mel_band_index(44100, 2048, 60, channels=2)
    ptr, inv = idx.inverse()
    for pair in (0, 1, 500, 2049):
        js = inv[ptr[pair] : ptr[pair + 1]]
        assert np.all(idx.index[js] == pair)
        assert list(js) == sorted(js)


def test_oracle_gather_recombine_shapes():
    idx, *_ = mel_ref.mel_band_tables(44100, 64, 8, stereo=True)
    stft = torch.randn(2, 2, 33, 5, 2, dtype=torch.float64)
    x = mel_ref.gather(stft, idx)
    assert x.shape == (2, 5, idx.numel() * 2)
    out = mel_ref.recombine(torch.ones(2, 1, 5, idx.numel() * 2, dtype=torch.float64), stft, idx, multiply=False)
    # averaging constant masks of (1 + 1i) gives (1 + 1i) everywhere
    torch.testing.assert_close(out, torch.ones_like(out))
