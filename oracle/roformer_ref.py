"""Pure-PyTorch BS-RoFormer and Mel-band RoFormer (CPU oracle and CPU baseline).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

pymss-core 0.1.4 holds the reference's model code and is not available here,
so this restates the published architecture it implements (the
BS-RoFormer / Mel-band RoFormer of Music-Source-Separation-Training, which
pymss-core keeps checkpoint-compatible: the reference strict-loads its
pretrained checkpoints, tests/test_pretrained_compat.py:27-50).  What the
reference itself pins is followed exactly:

* constructor arguments (tests/test_training_smoke.py:40-65,
  src/pymsst/training/module.py:330-336);
* module / parameter names used by the reference's patches:
  ``band_split.to_features[b][0].gamma`` / ``[1].weight,bias``
  (fused_roformer.py:383-402), ``mask_estimators[k].to_freqs[b][0]`` the MLP
  (test_training_smoke.py:138), ``Attention.norm / to_qkv / to_gates /
  to_out`` (fused_roformer.py:776-818);
* fused-op formulas: RMSNorm = F.normalize(x) * sqrt(D) * gamma
  (fused_roformer.py:1265-1271), interleaved-pair rotary on q/k
  (fused_roformer.py:710-732), sigmoid head gate (.cu:1804-1805), GLU mask
  head (.cu:2303-2308);
* MelBandRoformer's legacy mask-estimator depth: ``mask_estimator_depth``
  hidden layers when ``mlp_hidden_layers`` is absent (module.py:330-336,
  test_training_smoke.py:131-152).

Forward with a target returns the training loss: L1 on the waveform plus the
multi-resolution STFT L1 loss (windows 4096..256, hop 147).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from . import mel_ref

DEFAULT_FREQS_PER_BANDS = (2,) * 24 + (4,) * 12 + (12,) * 8 + (24,) * 8 + (48,) * 8 + (128, 129)


class RMSNorm(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.scale = dim**0.5
        self.gamma = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return F.normalize(x, dim=-1) * self.scale * self.gamma


class RotaryEmbedding(nn.Module):
    """Interleaved-pair rotary embedding (rotary-embedding-torch defaults, theta 10000)."""

    def __init__(self, dim: int, theta: float = 10000.0):
        super().__init__()
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
        self.freqs = nn.Parameter(freqs, requires_grad=False)

    def rotate(self, t):  # t [..., n, d]
        n = t.shape[-2]
        ang = torch.arange(n, dtype=self.freqs.dtype, device=self.freqs.device)[:, None] * self.freqs[None, :]
        cos, sin = ang.cos().to(t.dtype), ang.sin().to(t.dtype)
        e, o = t[..., 0::2], t[..., 1::2]
        return torch.stack((e * cos - o * sin, o * cos + e * sin), dim=-1).flatten(-2)


class Attention(nn.Module):
    def __init__(self, dim, heads=8, dim_head=64, dropout=0.0, rotary_embed=None, flash=True):
        super().__init__()
        self.heads = heads
        self.dim_head = dim_head
        self.rotary_embed = rotary_embed
        self.dropout = dropout
        inner = heads * dim_head
        self.norm = RMSNorm(dim)
        self.to_qkv = nn.Linear(dim, inner * 3, bias=False)
        self.to_gates = nn.Linear(dim, heads)
        self.to_out = nn.Sequential(nn.Linear(inner, dim, bias=False), nn.Dropout(dropout))

    def forward(self, x):
        b, n, _ = x.shape
        x = self.norm(x)
        q, k, v = self.to_qkv(x).reshape(b, n, 3, self.heads, self.dim_head).permute(2, 0, 3, 1, 4)
        if self.rotary_embed is not None:
            q = self.rotary_embed.rotate(q)
            k = self.rotary_embed.rotate(k)
        out = F.scaled_dot_product_attention(q, k, v, dropout_p=self.dropout if self.training else 0.0)
        gates = self.to_gates(x).sigmoid()  # [b, n, h]
        out = out * gates.permute(0, 2, 1)[..., None]
        out = out.permute(0, 2, 1, 3).reshape(b, n, -1)
        return self.to_out(out)


class FeedForward(nn.Module):
    def __init__(self, dim, mult=4, dropout=0.0):
        super().__init__()
        inner = int(dim * mult)
        self.net = nn.Sequential(
            RMSNorm(dim), nn.Linear(dim, inner), nn.GELU(), nn.Dropout(dropout), nn.Linear(inner, dim), nn.Dropout(dropout)
        )

    def forward(self, x):
        return self.net(x)


class Transformer(nn.Module):
    def __init__(self, *, dim, depth, dim_head=64, heads=8, attn_dropout=0.0, ff_dropout=0.0, ff_mult=4,
                 norm_output=True, rotary_embed=None, flash_attn=True):
        super().__init__()
        self.layers = nn.ModuleList(
            [
                nn.ModuleList(
                    [
                        Attention(dim, heads, dim_head, attn_dropout, rotary_embed, flash_attn),
                        FeedForward(dim, ff_mult, ff_dropout),
                    ]
                )
                for _ in range(depth)
            ]
        )
        self.norm = RMSNorm(dim) if norm_output else nn.Identity()

    def forward(self, x):
        for attn, ff in self.layers:
            x = attn(x) + x
            x = ff(x) + x
        return self.norm(x)


class BandSplit(nn.Module):
    def __init__(self, dim, dim_inputs):
        super().__init__()
        self.dim_inputs = tuple(dim_inputs)
        self.to_features = nn.ModuleList([nn.Sequential(RMSNorm(d), nn.Linear(d, dim)) for d in dim_inputs])

    def forward(self, x):
        parts = x.split(self.dim_inputs, dim=-1)
        return torch.stack([net(p) for p, net in zip(parts, self.to_features)], dim=-2)


def mlp(dim_in, dim_out, dim_hidden, hidden_layers):
    dims = (dim_in, *((dim_hidden,) * hidden_layers), dim_out)
    layers = []
    for i, (a, b) in enumerate(zip(dims[:-1], dims[1:])):
        layers.append(nn.Linear(a, b))
        if i < len(dims) - 2:
            layers.append(nn.Tanh())
    return nn.Sequential(*layers)


class MaskEstimator(nn.Module):
    def __init__(self, dim, dim_inputs, hidden_layers, mlp_expansion_factor=4):
        super().__init__()
        self.dim_inputs = tuple(dim_inputs)
        hidden = dim * mlp_expansion_factor
        self.to_freqs = nn.ModuleList(
            [nn.Sequential(mlp(dim, d * 2, hidden, hidden_layers), nn.GLU(dim=-1)) for d in dim_inputs]
        )

    def forward(self, x):
        return torch.cat([net(band) for band, net in zip(x.unbind(dim=-2), self.to_freqs)], dim=-1)


class _RoformerBase(nn.Module):
    def _init_common(self, dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                     linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn, stft_n_fft,
                     stft_hop_length, stft_win_length, stft_normalized, multi_stft_resolution_loss_weight,
                     multi_stft_resolutions_window_sizes, multi_stft_hop_size, multi_stft_normalized,
                     skip_connection):
        if linear_transformer_depth:
            raise NotImplementedError("linear attention layers are not part of this restatement")
        self.stereo = stereo
        self.audio_channels = 2 if stereo else 1
        self.num_stems = num_stems
        self.skip_connection = skip_connection
        kwargs = dict(dim=dim, heads=heads, dim_head=dim_head, attn_dropout=attn_dropout, ff_dropout=ff_dropout,
                      flash_attn=flash_attn, norm_output=False)
        time_rot = RotaryEmbedding(dim_head)
        freq_rot = RotaryEmbedding(dim_head)
        self.layers = nn.ModuleList(
            [
                nn.ModuleList(
                    [
                        Transformer(depth=time_transformer_depth, rotary_embed=time_rot, **kwargs),
                        Transformer(depth=freq_transformer_depth, rotary_embed=freq_rot, **kwargs),
                    ]
                )
                for _ in range(depth)
            ]
        )
        self.final_norm = RMSNorm(dim)
        self.stft_kwargs = dict(n_fft=stft_n_fft, hop_length=stft_hop_length, win_length=stft_win_length,
                                normalized=stft_normalized)
        self.stft_win_length = stft_win_length
        self.multi_stft_resolution_loss_weight = multi_stft_resolution_loss_weight
        self.multi_stft_resolutions_window_sizes = tuple(multi_stft_resolutions_window_sizes)
        self.multi_stft_n_fft = stft_n_fft
        self.multi_stft_kwargs = dict(hop_length=multi_stft_hop_size, normalized=multi_stft_normalized)

    def _stft(self, raw_audio):
        b, s, length = raw_audio.shape
        window = torch.hann_window(self.stft_win_length, device=raw_audio.device)
        spec = torch.stft(raw_audio.reshape(b * s, length), **self.stft_kwargs, window=window, return_complex=True)
        spec = torch.view_as_real(spec)  # [b*s, f, t, 2]
        return spec.reshape(b, s, *spec.shape[1:]), window

    def _axial(self, x):
        store = []
        for i, (time_t, freq_t) in enumerate(self.layers):
            if self.skip_connection:
                for prev in store:
                    x = x + prev
            b, t, f, d = x.shape
            x = time_t(x.permute(0, 2, 1, 3).reshape(b * f, t, d)).reshape(b, f, t, d).permute(0, 2, 1, 3)
            x = freq_t(x.reshape(b * t, f, d)).reshape(b, t, f, d)
            if self.skip_connection:
                store.append(x)
        return self.final_norm(x)

    def _istft(self, spec, window, length):  # spec [b, n, s, f, t, 2]
        b, n, s, f, t, _ = spec.shape
        z = torch.view_as_complex(spec.reshape(b * n * s, f, t, 2).contiguous())
        audio = torch.istft(z, **self.stft_kwargs, window=window, return_complex=False, length=length)
        audio = audio.reshape(b, n, s, -1)
        return audio[:, 0] if n == 1 else audio

    def _loss(self, recon, target):
        if self.num_stems > 1:
            assert target.ndim == 4 and target.shape[1] == self.num_stems
        if target.ndim == 2:
            target = target[:, None]
        target = target[..., : recon.shape[-1]]
        loss = F.l1_loss(recon, target)
        res_loss = 0.0
        for win in self.multi_stft_resolutions_window_sizes:
            kw = dict(n_fft=max(win, self.multi_stft_n_fft), win_length=win, return_complex=True,
                      window=torch.hann_window(win, device=recon.device), **self.multi_stft_kwargs)
            ry = torch.stft(recon.reshape(-1, recon.shape[-1]), **kw)
            ty = torch.stft(target.reshape(-1, target.shape[-1]), **kw)
            res_loss = res_loss + F.l1_loss(ry, ty)
        return loss + res_loss * self.multi_stft_resolution_loss_weight


class BSRoformer(_RoformerBase):
    def __init__(self, dim, *, depth, stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2,
                 linear_transformer_depth=0, freqs_per_bands=DEFAULT_FREQS_PER_BANDS, dim_head=64, heads=8,
                 attn_dropout=0.0, ff_dropout=0.0, flash_attn=True, dim_freqs_in=1025, stft_n_fft=2048,
                 stft_hop_length=512, stft_win_length=2048, stft_normalized=False, stft_window_fn=None,
                 mask_estimator_depth=2, multi_stft_resolution_loss_weight=1.0,
                 multi_stft_resolutions_window_sizes=(4096, 2048, 1024, 512, 256), multi_stft_hop_size=147,
                 multi_stft_normalized=False, multi_stft_window_fn=None, mlp_expansion_factor=4,
                 use_torch_checkpoint=False, skip_connection=False, zero_dc=False):
        super().__init__()
        self.zero_dc = zero_dc
        self._init_common(dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                          linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn, stft_n_fft,
                          stft_hop_length, stft_win_length, stft_normalized, multi_stft_resolution_loss_weight,
                          multi_stft_resolutions_window_sizes, multi_stft_hop_size, multi_stft_normalized,
                          skip_connection)
        freqs = stft_n_fft // 2 + 1
        assert sum(freqs_per_bands) == freqs, f"bands must cover {freqs} bins"
        dim_inputs = tuple(2 * f * self.audio_channels for f in freqs_per_bands)
        self.band_split = BandSplit(dim, dim_inputs)
        self.mask_estimators = nn.ModuleList(
            [MaskEstimator(dim, dim_inputs, mask_estimator_depth - 1, mlp_expansion_factor) for _ in range(num_stems)]
        )

    def forward(self, raw_audio, target=None):
        if raw_audio.ndim == 2:
            raw_audio = raw_audio[:, None]
        b, s, length = raw_audio.shape
        spec, window = self._stft(raw_audio)  # [b, s, f, t, 2]
        _, _, f, t, _ = spec.shape
        x = spec.permute(0, 3, 2, 1, 4).reshape(b, t, f * s * 2)  # 'b s f t c -> b t (f s c)'
        x = self._axial(self.band_split(x))
        mask = torch.stack([est(x) for est in self.mask_estimators], dim=1)  # [b, n, t, (f s c)]
        mask = mask.reshape(b, -1, t, f, s, 2).permute(0, 1, 4, 3, 2, 5)  # [b, n, s, f, t, 2]
        sp = spec[:, None]
        re = sp[..., 0] * mask[..., 0] - sp[..., 1] * mask[..., 1]
        im = sp[..., 0] * mask[..., 1] + sp[..., 1] * mask[..., 0]
        out = torch.stack((re, im), -1)
        if self.zero_dc:
            out = torch.cat((torch.zeros_like(out[:, :, :, :1]), out[:, :, :, 1:]), dim=3)
        recon = self._istft(out, window, length)
        return recon if target is None else self._loss(recon, target)


class MelBandRoformer(_RoformerBase):
    def __init__(self, dim, *, depth, stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2,
                 linear_transformer_depth=0, num_bands=60, dim_head=64, heads=8, attn_dropout=0.0, ff_dropout=0.0,
                 flash_attn=True, dim_freqs_in=1025, sample_rate=44100, stft_n_fft=2048, stft_hop_length=512,
                 stft_win_length=2048, stft_normalized=False, stft_window_fn=None, mask_estimator_depth=1,
                 mlp_hidden_layers=None, multi_stft_resolution_loss_weight=1.0,
                 multi_stft_resolutions_window_sizes=(4096, 2048, 1024, 512, 256), multi_stft_hop_size=147,
                 multi_stft_normalized=False, multi_stft_window_fn=None, match_input_audio_length=False,
                 mlp_expansion_factor=4, use_torch_checkpoint=False, skip_connection=False, zero_dc=False):
        super().__init__()
        self.zero_dc = zero_dc
        self._init_common(dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                          linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn, stft_n_fft,
                          stft_hop_length, stft_win_length, stft_normalized, multi_stft_resolution_loss_weight,
                          multi_stft_resolutions_window_sizes, multi_stft_hop_size, multi_stft_normalized,
                          skip_connection)
        self.match_input_audio_length = match_input_audio_length
        index, per_band, _, _ = mel_ref.mel_band_tables(sample_rate, stft_n_fft, num_bands, stereo)
        self.register_buffer("freq_indices", index, persistent=False)
        dim_inputs = tuple(2 * int(n) * self.audio_channels for n in per_band.tolist())
        hidden_layers = mask_estimator_depth if mlp_hidden_layers is None else mlp_hidden_layers
        self.band_split = BandSplit(dim, dim_inputs)
        self.mask_estimators = nn.ModuleList(
            [MaskEstimator(dim, dim_inputs, hidden_layers, mlp_expansion_factor) for _ in range(num_stems)]
        )

    def forward(self, raw_audio, target=None):
        if raw_audio.ndim == 2:
            raw_audio = raw_audio[:, None]
        b, s, length = raw_audio.shape
        spec, window = self._stft(raw_audio)
        x = mel_ref.gather(spec, self.freq_indices)  # [b, t, J*2]
        x = self._axial(self.band_split(x))
        mask = torch.stack([est(x) for est in self.mask_estimators], dim=1)  # [b, n, t, J*2]
        out = mel_ref.recombine(mask, spec, self.freq_indices, multiply=True)
        if self.zero_dc:
            out = torch.cat((torch.zeros_like(out[:, :, :, :1]), out[:, :, :, 1:]), dim=3)
        recon = self._istft(out, window, length if self.match_input_audio_length else None)
        return recon if target is None else self._loss(recon, target)


def build(model_type: str, **kwargs) -> nn.Module:
    if model_type == "bs_roformer":
        return BSRoformer(**kwargs)
    if model_type == "mel_band_roformer":
        return MelBandRoformer(**kwargs)
    raise ValueError("model_type must be 'bs_roformer' or 'mel_band_roformer'")

