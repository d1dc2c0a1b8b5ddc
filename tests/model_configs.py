"""Model configurations shared by the model tests (kwargs of the model constructors)."""
from __future__ import annotations

# The reference's tiny test model (tests/test_training_smoke.py:40-65).
TINY = dict(dim=8, depth=1, stereo=True, num_stems=1, time_transformer_depth=1, freq_transformer_depth=1,
            linear_transformer_depth=0, dim_head=8, heads=1, attn_dropout=0.0, ff_dropout=0.0, flash_attn=False,
            stft_n_fft=64, stft_hop_length=16, stft_win_length=64, stft_normalized=False, mask_estimator_depth=1,
            mlp_expansion_factor=2)
TINY_BSR = dict(TINY, freqs_per_bands=(8, 8, 8, 9))
TINY_MBR = dict(TINY, num_bands=8, sample_rate=44100)

# Benchmark configuration 0 (BS-RoFormer) / 1 (Mel-band RoFormer).
CONFIG0_BSR = dict(dim=192, depth=6, stereo=True, num_stems=1, time_transformer_depth=1, freq_transformer_depth=1,
                   dim_head=64, heads=8, mask_estimator_depth=2, mlp_expansion_factor=4)
CONFIG1_MBR = dict(dim=192, depth=6, stereo=True, num_stems=1, time_transformer_depth=1, freq_transformer_depth=1,
                   dim_head=64, heads=8, num_bands=60, sample_rate=44100, mask_estimator_depth=2,
                   mlp_expansion_factor=4)
