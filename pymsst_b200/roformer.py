"""BS-RoFormer and Mel-band RoFormer on the fused sm_100a training path.

Drop-in for pymss-core 0.1.4's ``BSRoformer`` / ``MelBandRoformer`` as the
reference uses them (src/pymsst/training/module.py:76, tests/
test_training_smoke.py:40-152): the same constructor keyword arguments, the
same ``forward(raw_audio [B, S, L], target=None)`` (separated stems, or the
training loss when a target is given) and the same parameter names /
state-dict layout (``band_split.to_features[b][0].gamma``,
``layers[i][0|1].layers[j][0].to_qkv.weight``,
``mask_estimators[k].to_freqs[b][0][l].weight`` ...), so checkpoints move
between the two.

The per-layer hot path runs through :mod:`pymsst_b200.fused`:

* STFT -> band features: :class:`~pymsst_b200.fused.BandGatherFn` (Mel-band
  overlapping gather; identity layout for BS-RoFormer);
* BandSplit: :class:`~pymsst_b200.fused.BandSplitFn` (per-band RMSNorm +
  ragged Linear);
* transformer RMSNorm: :class:`~pymsst_b200.fused.RMSNormFn`;
* QKV projection + rotary: :class:`~pymsst_b200.fused.QKVRotaryFn`; head gate:
  :class:`~pymsst_b200.fused.AttentionGateFn`;
* MaskEstimator MLP + GLU: :class:`~pymsst_b200.fused.MaskEstimatorFn`;
* mask recombination (scatter-add-average) and complex mask product:
  :class:`~pymsst_b200.fused.BandRecombineFn`.

* attention core softmax(q k^T / sqrt(dh)) v: :class:`~pymsst_b200.fused.AttentionFn`
  (tcgen05 kernels; 16-bit, head dim 64) on the band axis, cuDNN's
  ``F.scaled_dot_product_attention`` on the longer time axis; any backend can
  be forced with ``set_cuda_attention_backend``.  Where the own kernels run
  on sequences stored in row order (the band axis),
  :class:`~pymsst_b200.fused.QKVAttentionFn` takes projection, rotary and
  attention together, so the attention backward writes the projection
  gradient itself.

The feed-forward projections and the attention output projection are cuBLAS
GEMMs (the feed-forward GELU and bias gradients run on this package's kernels).
There is no CPU path: a forward on CPU tensors raises
``FusedKernelUnavailable``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from . import bands as band_tables
from .fused import (
    AttentionFn,
    AttentionGateFn,
    BandGatherFn,
    BandRecombineFn,
    BandSplitFn,
    FeedForwardFn,
    ISTFTOverlapAddFn,
    MaskEstimatorFn,
    MaskEstimatorTCFn,
    OutProjFn,
    QKVAttentionFn,
    QKVAttentionGateFn,
    QKVRotaryFn,
    RMSNormFn,
    RMSNormResidualFn,
    compute_dtype,
    rotary_tables,
    attention_supported,
    stft_l1_loss,
    tensor_core_ok,
)

DEFAULT_FREQS_PER_BANDS = band_tables.DEFAULT_FREQS_PER_BANDS


_ENVELOPES: dict = {}


def _overlap_add(frames, hop):
    """frames [B, n, T] -> [B, n + hop * (T - 1)]: frame t added at offset t * hop.  With n a multiple of hop
    the frames are cut into n / hop hop-long pieces and summed as shifted, zero-padded copies (a few
    contiguous passes whose backward is a slice); otherwise torch's fold."""
    b, n, t = frames.shape
    if n % hop == 0:
        r = n // hop
        pieces = frames.transpose(1, 2).reshape(b, t, r, hop)
        y = None
        for i in range(r):
            part = F.pad(pieces[:, :, i, :], (0, 0, i, r - 1 - i))
            y = part if y is None else y + part
        return y.reshape(b, (t + r - 1) * hop)
    total = n + hop * (t - 1)
    return F.fold(frames, output_size=(1, total), kernel_size=(1, n), stride=(1, hop)).reshape(b, total)


def _istft_overlap_add(z, n_fft, hop, window, normalized, length):
    """Inverse STFT (center=True, onesided) as torch.istft computes it -- inverse real FFT of each frame,
    window, overlap-add, division by the overlap-added squared window, centre trim -- without torch.istft's
    host-side check of the window envelope, so a captured CUDA graph can contain it.  z [B, F, T] complex."""
    frames = torch.fft.irfft(z, n=n_fft, dim=-2, norm="ortho" if normalized else "backward")  # [B, n_fft, T]
    win = window
    if win.shape[0] < n_fft:
        left = (n_fft - win.shape[0]) // 2
        win = F.pad(win, (left, n_fft - win.shape[0] - left))
    t = frames.shape[-1]
    total = n_fft + hop * (t - 1)
    if frames.is_cuda:
        # window, overlap-add, envelope division and trim in one kernel each way
        return ISTFTOverlapAddFn.apply(frames, win, hop, length if length is not None else total - n_fft)
    y = _overlap_add(frames * win[:, None], hop)
    key = (n_fft, hop, t, win.device, win.data_ptr(), win._version)
    env = _ENVELOPES.get(key)
    if env is None:  # kept for the process lifetime: a captured step graph reads it on every replay
        env = _overlap_add((win * win)[None, :, None].expand(1, n_fft, t).contiguous(), hop).reshape(total)
        _ENVELOPES[key] = env
    start = n_fft // 2
    end = start + length if length is not None else total - n_fft // 2
    y = y[:, start:end] / env[start:end]
    if length is not None and y.shape[-1] < length:
        y = F.pad(y, (0, length - y.shape[-1]))
    return y


class RMSNorm(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.scale = dim**0.5
        self.gamma = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return RMSNormFn.apply(x, self.gamma)

    def with_residual(self, x):
        """(norm(x), x) for a pre-norm residual block: use the second output for the residual branch, so the
        backward adds that branch's gradient of x in the norm's own pass."""
        return RMSNormResidualFn.apply(x, self.gamma)


class RotaryEmbedding(nn.Module):
    """Interleaved-pair rotary frequencies (theta 10000); fp32 angle tables are cached per length."""

    def __init__(self, dim: int, theta: float = 10000.0):
        super().__init__()
        freqs = 1.0 / (theta ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
        self.freqs = nn.Parameter(freqs, requires_grad=False)
        self._tables: dict = {}

    def tables(self, n: int, device: torch.device):
        key = (n, device.type, device.index, self.freqs.data_ptr(), self.freqs._version)
        hit = self._tables.get(key)
        if hit is None:
            cos, sin = rotary_tables(self.freqs, n, device)
            self._tables = {key: (cos, sin, cos.t().contiguous(), sin.t().contiguous())}
            hit = self._tables[key]
        return hit


# Library attention kernel per sequence length, used where the own kernels do
# not apply (fp32, dropout, head dim other than 64) or when a library backend
# is asked for: from fwd+bwd timings of [B, 8, N, 64] bf16 on B200, cuDNN's
# fused attention is the fastest library kernel for the long (time-axis)
# sequences, the memory-efficient kernel for the short band axis.
_SHORT_SEQ = 128

# Names accepted by Attention.set_cuda_attention_backend: the reference's
# cuda_attention_backend choices (src/pymsst/cli.py:61) plus "pmb", this
# package's tcgen05 attention kernels.  "auto" / "default" take, per shape,
# the path measured on B200 for the axial shapes (bf16, 8 heads of 64,
# fwd + bwd): the own kernels up to _SHORT_SEQ positions (band axis, level
# with the memory-efficient kernel and deterministic), cuDNN above (time
# axis, where it is still ahead of the own backward).
ATTENTION_BACKENDS = ("auto", "default", "pmb", "cudnn", "efficient", "math", "flash")


def _own_attention(n, backend):
    """Whether a sequence of n positions takes the own attention kernels (when they support the shape)."""
    return backend == "pmb" or (backend in ("auto", "default") and n <= _SHORT_SEQ)


def _attention(q, k, v, dropout_p, backend="auto"):
    if attention_supported(q, dropout_p) and _own_attention(q.shape[-2], backend):
        return AttentionFn.apply(q, k, v)
    if q.is_cuda:
        from torch.nn.attention import SDPBackend, sdpa_kernel

        forced = {"cudnn": SDPBackend.CUDNN_ATTENTION, "efficient": SDPBackend.EFFICIENT_ATTENTION,
                  "math": SDPBackend.MATH, "flash": SDPBackend.FLASH_ATTENTION}.get(backend)
        if forced is not None:
            with sdpa_kernel([forced]):
                return F.scaled_dot_product_attention(q, k, v, dropout_p=dropout_p)
        if q.dtype in (torch.bfloat16, torch.float16):
            first = SDPBackend.EFFICIENT_ATTENTION if q.shape[-2] <= _SHORT_SEQ else SDPBackend.CUDNN_ATTENTION
            order = [first] + [b for b in (SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                                           SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH) if b != first]
            with sdpa_kernel(order, set_priority=True):
                return F.scaled_dot_product_attention(q, k, v, dropout_p=dropout_p)
    return F.scaled_dot_product_attention(q, k, v, dropout_p=dropout_p)


class Attention(nn.Module):
    def __init__(self, dim, heads=8, dim_head=64, dropout=0.0, rotary_embed=None, flash=True):
        super().__init__()
        self.heads = heads
        self.dim_head = dim_head
        self.dropout = dropout
        self.rotary_embed = rotary_embed
        inner = heads * dim_head
        self.norm = RMSNorm(dim)
        self.to_qkv = nn.Linear(dim, inner * 3, bias=False)
        self.to_gates = nn.Linear(dim, heads)
        self.to_out = nn.Sequential(nn.Linear(inner, dim, bias=False), nn.Dropout(dropout))
        self.attention_backend = "auto"

    def set_cuda_attention_backend(self, backend: str) -> None:
        """Attention kernel choice, the hook the reference's training module calls on every module
        (src/pymsst/training/module.py:416-425); one of ATTENTION_BACKENDS."""
        name = str(backend).strip().lower()
        if name not in ATTENTION_BACKENDS:
            raise ValueError(f"unknown cuda attention backend {backend!r}; expected one of {ATTENTION_BACKENDS}")
        self.attention_backend = name

    def forward(self, x, seq_len=None, inner=1, residual=None):
        """x [b, n, d]; or any [..., d] whose rows are ordered (outer, position, inner) with sequences of
        ``seq_len`` positions (sequence = outer * inner + inner index).  With ``residual`` (same shape as x)
        the block returns residual + attention(x), the addition done by the output projection GEMM."""
        d = x.shape[-1]
        n = x.shape[-2] if seq_len is None else seq_len
        rows = x.numel() // d
        b = rows // n
        if residual is x:
            # the residual branch's gradient of x is added in the norm's backward pass
            xn, residual = self.norm.with_residual(x)
        else:
            xn = self.norm(x)
        cos = sin = cos_t = sin_t = None
        if self.rotary_embed is not None:
            cos, sin, cos_t, sin_t = self.rotary_embed.tables(n, x.device)
        dropout_p = self.dropout if self.training else 0.0
        own = (inner == 1 and xn.is_cuda and xn.dtype in (torch.bfloat16, torch.float16) and d % 8 == 0
               and self.dim_head == 64 and dropout_p == 0.0 and _own_attention(n, self.attention_backend))
        if own and n <= 64:
            # short sequences in row order (the band axis): projection, attention and head gate in one Function;
            # the attention backward writes the projection gradient and the gate logits' gradient
            gated = QKVAttentionGateFn.apply(xn.reshape(b, n, d), self.to_qkv.weight, cos, sin, cos_t, sin_t,
                                             self.heads, self.to_gates.weight, self.to_gates.bias)
        else:
            # the projection passes xn through to the head gate, so the gate's gradient of xn joins the
            # projection's input gradient in one GEMM
            if own:
                # sequences in row order on the own kernels: the attention backward writes the projection gradient
                attn, xg = QKVAttentionFn.apply(xn.reshape(b, n, d), self.to_qkv.weight, cos, sin, cos_t, sin_t,
                                                self.heads, True)
            else:
                q, k, v, xg = QKVRotaryFn.apply(xn.reshape(b, n, d), self.to_qkv.weight, cos, sin, cos_t, sin_t,
                                                self.heads, inner, True)
                attn = _attention(q, k, v, dropout_p, self.attention_backend)
            gated = AttentionGateFn.apply(attn, xg.reshape(rows, d), self.to_gates.weight, self.to_gates.bias,
                                          inner)
        drop = self.to_out[1]
        if residual is not None and (not self.training or drop.p == 0.0):
            # residual + gated W^T in one GEMM (C = residual, beta = 1)
            res = residual.reshape(rows, d).to(gated.dtype)
            return OutProjFn.apply(res, gated, self.to_out[0].weight).reshape(x.shape)
        out = drop(F.linear(gated, self.to_out[0].weight.to(gated.dtype))).reshape(x.shape)
        return out if residual is None else out + residual


class FeedForward(nn.Module):
    def __init__(self, dim, mult=4, dropout=0.0):
        super().__init__()
        inner = int(dim * mult)
        self.net = nn.Sequential(
            RMSNorm(dim), nn.Linear(dim, inner), nn.GELU(), nn.Dropout(dropout), nn.Linear(inner, dim), nn.Dropout(dropout)
        )

    def forward(self, x, add_residual=False):
        """ff(x), or ff(x) + x with ``add_residual`` (the residual branch's gradient of x then joins the norm's
        backward pass)."""
        if add_residual:
            h, res = self.net[0].with_residual(x)
            return self._ff(h) + res
        return self._ff(self.net[0](x))

    def _ff(self, h):
        dt = h.dtype
        lin1, lin2 = self.net[1], self.net[4]
        dropout_live = self.training and (self.net[3].p > 0 or self.net[5].p > 0)
        if h.dtype in (torch.bfloat16, torch.float16) and not dropout_live and h.shape[-1] % 8 == 0 and \
                lin1.out_features % 8 == 0:
            shape = h.shape
            out = FeedForwardFn.apply(h.reshape(-1, shape[-1]), lin1.weight, lin1.bias, lin2.weight, lin2.bias)
            return out.reshape(shape)
        h = F.linear(h, self.net[1].weight.to(dt), self.net[1].bias.to(dt))
        h = self.net[3](F.gelu(h))
        h = F.linear(h, self.net[4].weight.to(dt), self.net[4].bias.to(dt))
        return self.net[5](h)


class Transformer(nn.Module):
    def __init__(self, *, dim, depth, dim_head=64, heads=8, attn_dropout=0.0, ff_dropout=0.0, ff_mult=4,
                 norm_output=True, rotary_embed=None, flash_attn=True, linear_attn=False):
        super().__init__()
        if linear_attn:
            raise NotImplementedError("linear attention layers are not supported (linear_transformer_depth must be 0)")
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

    def forward(self, x, seq_len=None, inner=1):
        """x [b, n, d], or rows in (outer, position, inner) order (see Attention.forward)."""
        for attn, ff in self.layers:
            x = attn(x, seq_len, inner, residual=x)
            x = ff(x, add_residual=True)
        return self.norm(x)


class BandSplit(nn.Module):
    def __init__(self, dim, dim_inputs):
        super().__init__()
        self.dim = dim
        self.dim_inputs = tuple(int(d) for d in dim_inputs)
        self.to_features = nn.ModuleList([nn.Sequential(RMSNorm(d), nn.Linear(d, dim)) for d in self.dim_inputs])

    def parameters_by_role(self):
        gammas = [f[0].gamma for f in self.to_features]
        weights = [f[1].weight for f in self.to_features]
        biases = [f[1].bias for f in self.to_features]
        return gammas, weights, biases

    def forward(self, x):  # [..., total] -> [..., nb, dim]
        lead = x.shape[:-1]
        g, w, b = self.parameters_by_role()
        out = BandSplitFn.apply(x.reshape(-1, x.shape[-1]), self.dim_inputs, self.dim, *g, *w, *b)
        return out.reshape(*lead, len(self.dim_inputs), self.dim)


def MLP(dim_in, dim_out, dim_hidden, hidden_layers):
    """Linear (+Tanh) stack: ``hidden_layers`` hidden Linear+Tanh layers, then the output Linear."""
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
        self.dim_inputs = tuple(int(d) for d in dim_inputs)
        self.hidden_layers = int(hidden_layers)
        self.dim = dim
        hidden = dim * mlp_expansion_factor
        self.hidden = hidden
        self.to_freqs = nn.ModuleList(
            [nn.Sequential(MLP(dim, d * 2, hidden, self.hidden_layers), nn.GLU(dim=-1)) for d in self.dim_inputs]
        )

    def ordered_parameters(self):
        params = []
        for layer in range(self.hidden_layers + 1):
            linears = [net[0][2 * layer] for net in self.to_freqs]
            params.extend(lin.weight for lin in linears)
            params.extend(lin.bias for lin in linears)
        return params

    def forward(self, x):  # [..., nb, dim] -> [..., total]
        lead = x.shape[:-2]
        x2 = x.reshape(-1, *x.shape[-2:])
        if tensor_core_ok(x2, self.dim, self.hidden):
            out = MaskEstimatorTCFn.apply(x2, self.dim_inputs, self.hidden_layers, self.hidden,
                                          *self.ordered_parameters())
        else:
            out = MaskEstimatorFn.apply(x2, self.dim_inputs, self.hidden_layers, *self.ordered_parameters())
        return out.reshape(*lead, out.shape[-1])


class _Roformer(nn.Module):
    """Shared STFT -> bands -> axial transformer -> masks -> iSTFT pipeline."""

    def _build_common(self, dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                      linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn, stft_n_fft,
                      stft_hop_length, stft_win_length, stft_normalized, multi_stft_resolution_loss_weight,
                      multi_stft_resolutions_window_sizes, multi_stft_hop_size, multi_stft_normalized,
                      skip_connection, use_torch_checkpoint):
        if linear_transformer_depth:
            raise NotImplementedError("linear_transformer_depth > 0 is not supported")
        self.stereo = stereo
        self.audio_channels = 2 if stereo else 1
        self.num_stems = num_stems
        self.skip_connection = skip_connection
        self.use_torch_checkpoint = use_torch_checkpoint
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
        self._device_tables: dict = {}
        self._windows: dict = {}

    # ------------------------------------------------------------ helpers
    def _window(self, n: int, device: torch.device) -> torch.Tensor:
        key = (n, device.type, device.index)
        w = self._windows.get(key)
        if w is None:
            w = self._windows[key] = torch.hann_window(n, device=device)
        return w

    def _loss_window(self, win: int, n_fft: int, device: torch.device) -> torch.Tensor:
        """Hann window of `win` samples zero-padded to n_fft as torch.stft pads it (centred)."""
        key = ("loss", win, n_fft, device.type, device.index)
        w = self._windows.get(key)
        if w is None:
            base = self._window(win, device)
            left = (n_fft - win) // 2
            w = self._windows[key] = F.pad(base, (left, n_fft - win - left)).contiguous()
        return w

    def _tables(self, device: torch.device) -> dict:
        key = (device.type, device.index)
        t = self._device_tables.get(key)
        if t is None:
            t = self._device_tables[key] = self.band_index.device_tables(device)
        return t

    def _stft(self, raw_audio):
        b, s, length = raw_audio.shape
        window = self._window(self.stft_win_length, raw_audio.device)
        with torch.autocast("cuda", enabled=False):
            spec = torch.stft(raw_audio.float().reshape(b * s, length), **self.stft_kwargs, window=window,
                              return_complex=True)
        spec = torch.view_as_real(spec).contiguous()  # [b*s, f, t, 2]
        return spec.reshape(b, s, *spec.shape[1:]), window

    def _axial(self, x):
        store = []
        for time_t, freq_t in self.layers:
            if self.skip_connection:
                for prev in store:
                    x = x + prev
            b, t, f, d = x.shape
            # rows stay in (b, t, f) order for both axes: the time transformer's sequences are (b, f) pairs
            # over t (inner = f), the frequency transformer's are (b, t) pairs over f
            x = self._run_transformer(time_t, x, seq_len=t, inner=f)
            x = self._run_transformer(freq_t, x.reshape(b * t, f, d)).reshape(b, t, f, d)
            if self.skip_connection:
                store.append(x)
        return self.final_norm(x)

    def _run_transformer(self, transformer, x, **kwargs):
        """One axial transformer; with ``use_torch_checkpoint`` (training, gradients on) its activations are
        recomputed in the backward instead of kept (torch.utils.checkpoint, non-reentrant), as pymss-core
        does per transformer.  Dropout masks are replayed exactly only when dropout is live (the RNG state is
        then saved, which a captured CUDA graph does not allow)."""
        if not (self.use_torch_checkpoint and self.training and torch.is_grad_enabled()):
            return transformer(x, **kwargs)
        from torch.utils.checkpoint import checkpoint

        dropout_live = any(isinstance(m, nn.Dropout) and m.p > 0 for m in transformer.modules()) or any(
            getattr(m, "dropout", 0.0) > 0 for m in transformer.modules() if isinstance(m, Attention))
        return checkpoint(transformer, x, use_reentrant=False, preserve_rng_state=dropout_live, **kwargs)

    def _istft(self, spec, window, length):  # spec fp32 [b, n, s, f, t, 2]
        b, n, s, f, t, _ = spec.shape
        z = torch.view_as_complex(spec.reshape(b * n * s, f, t, 2))
        with torch.autocast("cuda", enabled=False):
            audio = _istft_overlap_add(z, self.stft_kwargs["n_fft"], self.stft_kwargs["hop_length"], window,
                                       self.stft_kwargs["normalized"], length)
        audio = audio.reshape(b, n, s, -1)
        return audio[:, 0] if n == 1 else audio

    def loss(self, recon, target):
        """L1 on the waveform + weighted multi-resolution STFT L1 (fp32)."""
        if self.num_stems > 1 and not (target.ndim == 4 and target.shape[1] == self.num_stems):
            raise ValueError("multi-stem training needs a [B, stems, S, L] target")
        if target.ndim == 2:
            target = target[:, None]
        target = target[..., : recon.shape[-1]].float()
        recon = recon.float()
        with torch.autocast("cuda", enabled=False):
            loss = F.l1_loss(recon, target)
            res = 0.0
            for win in self.multi_stft_resolutions_window_sizes:
                n_fft = max(win, self.multi_stft_n_fft)
                if recon.is_cuda:
                    # torch.stft's framing with an overlap-add backward of this package (same spectra, frames
                    # first); the L1 mean does not depend on the layout
                    window = self._loss_window(win, n_fft, recon.device)
                    hop, norm = self.multi_stft_kwargs["hop_length"], self.multi_stft_kwargs["normalized"]
                    res = res + stft_l1_loss(recon.reshape(-1, recon.shape[-1]), target.reshape(-1, target.shape[-1]),
                                             n_fft, hop, window, norm)
                else:
                    kw = dict(n_fft=n_fft, win_length=win, return_complex=True,
                              window=self._window(win, recon.device), **self.multi_stft_kwargs)
                    ry = torch.stft(recon.reshape(-1, recon.shape[-1]), **kw)
                    ty = torch.stft(target.reshape(-1, target.shape[-1]), **kw)
                    res = res + F.l1_loss(ry, ty)
        return loss + res * self.multi_stft_resolution_loss_weight

    def _separate(self, raw_audio, length):
        if raw_audio.ndim == 2:
            raw_audio = raw_audio[:, None]
        spec, window = self._stft(raw_audio)  # [b, s, f, t, 2]
        b, s, f, t, _ = spec.shape
        tables = self._tables(raw_audio.device)
        dtype = compute_dtype(raw_audio)
        x = BandGatherFn.apply(spec, tables, dtype)  # [b, t, J*2]
        x = self._axial(self.band_split(x))
        masks = torch.stack([est(x) for est in self.mask_estimators], dim=1)  # [b, n, t, J*2]
        out = BandRecombineFn.apply(masks, spec, tables)  # [b, n, s, f, t, 2]
        if self.zero_dc:  # drop the DC bin of the separated spectrum
            out = torch.cat((torch.zeros_like(out[:, :, :, :1]), out[:, :, :, 1:]), dim=3)
        return self._istft(out, window, length)

    def forward(self, raw_audio, target=None):
        recon = self._separate(raw_audio, self._istft_length(raw_audio))
        return recon if target is None else self.loss(recon, target)


class BSRoformer(_Roformer):
    def __init__(self, dim, *, depth, stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2,
                 linear_transformer_depth=0, freqs_per_bands=DEFAULT_FREQS_PER_BANDS, dim_head=64, heads=8,
                 attn_dropout=0.0, ff_dropout=0.0, flash_attn=True, dim_freqs_in=1025, stft_n_fft=2048,
                 stft_hop_length=512, stft_win_length=2048, stft_normalized=False, stft_window_fn=None,
                 mask_estimator_depth=2, multi_stft_resolution_loss_weight=1.0,
                 multi_stft_resolutions_window_sizes=(4096, 2048, 1024, 512, 256), multi_stft_hop_size=147,
                 multi_stft_normalized=False, multi_stft_window_fn=None, mlp_expansion_factor=4,
                 use_torch_checkpoint=False, skip_connection=False, zero_dc=False):
        super().__init__()
        self._build_common(dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                           linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn,
                           stft_n_fft, stft_hop_length, stft_win_length, stft_normalized,
                           multi_stft_resolution_loss_weight, multi_stft_resolutions_window_sizes,
                           multi_stft_hop_size, multi_stft_normalized, skip_connection, use_torch_checkpoint)
        self.zero_dc = zero_dc
        freqs = stft_n_fft // 2 + 1
        if sum(freqs_per_bands) != freqs:
            raise ValueError(f"the bands must cover {freqs} frequency bins, got {sum(freqs_per_bands)}")
        self.band_index = band_tables.split_band_index(freqs_per_bands, self.audio_channels)
        self.band_split = BandSplit(dim, self.band_index.dim_inputs)
        self.mask_estimators = nn.ModuleList(
            [MaskEstimator(dim, self.band_index.dim_inputs, mask_estimator_depth - 1, mlp_expansion_factor)
             for _ in range(num_stems)]
        )

    def _istft_length(self, raw_audio):
        return raw_audio.shape[-1]


class MelBandRoformer(_Roformer):
    def __init__(self, dim, *, depth, stereo=False, num_stems=1, time_transformer_depth=2, freq_transformer_depth=2,
                 linear_transformer_depth=0, num_bands=60, dim_head=64, heads=8, attn_dropout=0.0, ff_dropout=0.0,
                 flash_attn=True, dim_freqs_in=1025, sample_rate=44100, stft_n_fft=2048, stft_hop_length=512,
                 stft_win_length=2048, stft_normalized=False, stft_window_fn=None, mask_estimator_depth=1,
                 mlp_hidden_layers=None, multi_stft_resolution_loss_weight=1.0,
                 multi_stft_resolutions_window_sizes=(4096, 2048, 1024, 512, 256), multi_stft_hop_size=147,
                 multi_stft_normalized=False, multi_stft_window_fn=None, match_input_audio_length=False,
                 mlp_expansion_factor=4, use_torch_checkpoint=False, skip_connection=False, zero_dc=False):
        super().__init__()
        self._build_common(dim, depth, stereo, num_stems, time_transformer_depth, freq_transformer_depth,
                           linear_transformer_depth, dim_head, heads, attn_dropout, ff_dropout, flash_attn,
                           stft_n_fft, stft_hop_length, stft_win_length, stft_normalized,
                           multi_stft_resolution_loss_weight, multi_stft_resolutions_window_sizes,
                           multi_stft_hop_size, multi_stft_normalized, skip_connection, use_torch_checkpoint)
        self.zero_dc = zero_dc
        self.match_input_audio_length = match_input_audio_length
        self.band_index = band_tables.mel_band_index(sample_rate, stft_n_fft, num_bands, self.audio_channels)
        hidden_layers = mask_estimator_depth if mlp_hidden_layers is None else mlp_hidden_layers
        self.band_split = BandSplit(dim, self.band_index.dim_inputs)
        self.mask_estimators = nn.ModuleList(
            [MaskEstimator(dim, self.band_index.dim_inputs, hidden_layers, mlp_expansion_factor)
             for _ in range(num_stems)]
        )

    def _istft_length(self, raw_audio):
        return raw_audio.shape[-1] if self.match_input_audio_length else None
