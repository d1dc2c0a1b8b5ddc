"""Seeded synthetic stereo training audio (stand-in for MUSDB18-HQ).

The benchmark configurations describe the generator: 44.1 kHz stereo, the
mixture is a sum of 16 sinusoids with log-uniform frequencies in
[40 Hz, 16 kHz] (random phase, random amplitude) plus pink noise scaled to
RMS 0.1; the target is one of the sinusoids scaled by a random gain in
[0.3, 0.7].  For multi-stem training each stem is an independent draw of
the generator and the mixture is the sum of the stems.  Everything derives
from a ``torch.Generator`` seed, so a (seed, index) pair fixes a batch.
"""
from __future__ import annotations

import math

import torch

SAMPLE_RATE = 44100


def pink_noise(n: int, channels: int, gen: torch.Generator, rms: float = 0.1) -> torch.Tensor:
    """[channels, n] noise with a 1/f power spectrum, scaled to the given RMS."""
    white = torch.randn(channels, n, generator=gen, dtype=torch.float64)
    spec = torch.fft.rfft(white, dim=-1)
    f = torch.arange(spec.shape[-1], dtype=torch.float64)
    f[0] = 1.0
    spec = spec / torch.sqrt(f)
    spec[..., 0] = 0.0
    pink = torch.fft.irfft(spec, n=n, dim=-1)
    pink = pink / pink.pow(2).mean(dim=-1, keepdim=True).sqrt().clamp_min(1e-12) * rms
    return pink


def one_example(length: int, gen: torch.Generator, channels: int = 2, n_sines: int = 16,
                sample_rate: int = SAMPLE_RATE) -> tuple[torch.Tensor, torch.Tensor]:
    """(mixture [channels, length], target [channels, length]) in float64."""
    lo, hi = math.log(40.0), math.log(16000.0)
    freqs = torch.exp(lo + (hi - lo) * torch.rand(n_sines, generator=gen, dtype=torch.float64))
    amps = 0.05 + 0.15 * torch.rand(n_sines, 1, generator=gen, dtype=torch.float64)
    phases = 2 * math.pi * torch.rand(channels, n_sines, 1, generator=gen, dtype=torch.float64)
    t = torch.arange(length, dtype=torch.float64) / sample_rate
    comps = amps * torch.sin(2 * math.pi * freqs[:, None] * t[None, :] + phases)  # [C, n_sines, L]
    which = int(torch.randint(n_sines, (1,), generator=gen))
    gain = 0.3 + 0.4 * float(torch.rand(1, generator=gen, dtype=torch.float64))
    mixture = comps.sum(dim=1) + pink_noise(length, channels, gen)
    target = gain * comps[:, which]
    return mixture, target


def make_batch(batch: int, length: int, seed: int, stems: int = 1, channels: int = 2,
               dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """(mixture [B, C, L], target [B, C, L] or [B, stems, C, L]) for one seed."""
    gen = torch.Generator().manual_seed(int(seed))
    mixes, targets = [], []
    for _ in range(batch):
        if stems == 1:
            mix, tgt = one_example(length, gen, channels)
        else:
            draws = [one_example(length, gen, channels) for _ in range(stems)]
            tgt = torch.stack([m for m, _ in draws])  # each stem is a full draw
            mix = tgt.sum(dim=0)
        mixes.append(mix)
        targets.append(tgt)
    return torch.stack(mixes).to(dtype), torch.stack(targets).to(dtype)
