"""The reference's own CUDA kernels, timed on this GPU as the per-kernel bar to beat.

The reference ships its fused training kernels as one pybind11 extension
(src/pymsst/training/cuda/fused_band_split.{cpp,cu}); ``oracle/build_ref.py``
compiles it from the reference sources into ``oracle/_ref/`` (test
infrastructure; skipped when that build is absent).  Each case calls one of the
reference's functions and the same-named function of this package's operator
API (``pymsst_b200.extension.ops``: same arguments, same results) on the same
inputs at the config-3 shapes (BS-RoFormer, 4 x 258 frames: 1032 band rows,
62 bands over 4100 features, 63984 transformer rows of 192, band-axis
sequences of 62 positions), fp16 (the reference's AMP type), and requires this
package to be faster.  The training path's tensor-core variants of BandSplit
and MaskEstimator are timed beside them for the record.  Only the reference's
"direct" MaskEstimator kernels run: its "grouped" variant passes host pointer
arrays to cublasGemmGroupedBatchedEx and faulted on this GPU
(fused_band_split.cu:2258-2279), so it is never called.

Run with ``-s`` to see the table (median of 10 calls after 3 warm-ups, CUDA
events around each call queued behind a GPU sleep so they bracket device
work, outputs allocated inside the call on both sides).
"""
from __future__ import annotations

import pytest
import torch

from pymsst_b200.bands import DEFAULT_FREQS_PER_BANDS
from pymsst_b200.extension import ops

pytestmark = pytest.mark.gpu


def _reference_module():
    from oracle.build_ref import OUT_DIR, MODULE, load

    path = OUT_DIR / f"{MODULE}.so"
    if not path.is_file():
        pytest.skip("the reference extension was not built (oracle/_ref missing)")
    return load(path)


def _time(fn, iters=10, warmup=3, graph=False):
    """Median device time of fn in microseconds.  Each timed call is queued behind a short GPU sleep, so the
    host has issued the whole call before the GPU reaches it and the events bracket device work (host-side
    waits inside the call, such as a synchronous pointer-table upload, still count).  graph=True times replays
    of fn captured into a CUDA graph (for the training-path autograd Functions)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        a.record()
        if g is not None:
            g.replay()
        else:
            fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2] * 1e3


def _cases(device):
    g = torch.Generator().manual_seed(0)
    dt = torch.float16

    def rn(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dt).to(device)

    rows, dim = 63984, 192
    x = rn(rows, dim)
    gamma = (torch.rand(dim, generator=g) + 0.5).to(dt).to(device)
    normed, inv = ops.rms_norm_forward(x, gamma)[1:]
    dy = rn(rows, dim)
    cases = [
        ("rms_norm_forward", (x, gamma)),
        ("rms_norm_backward", (dy, normed, inv, gamma)),
    ]
    t = rn(1032, 62, 8, 64)
    ang = torch.arange(62, dtype=torch.float32)[:, None] * (1.0 / 10000 ** (torch.arange(0, 64, 2) / 64))[None]
    cos, sin = (v.reshape(1, 62, 1, 32).to(dt).to(device) for v in (ang.cos(), ang.sin()))
    cases.append(("rotary_forward", (t, cos, sin)))
    widths = [4 * f for f in DEFAULT_FREQS_PER_BANDS]
    offsets = torch.tensor([0] + torch.tensor(widths).cumsum(0).tolist(), dtype=torch.int64, device=device)
    xb = rn(1032, sum(widths))
    gammas = [(torch.rand(w, generator=g) + 0.5).to(dt).to(device) for w in widths]
    weights = [rn(192, w, scale=w ** -0.5) for w in widths]
    biases = [rn(192, scale=0.1) for _ in widths]
    cases.append(("band_split_ragged_forward", (xb, gammas, weights, biases, widths, offsets)))
    _, bnormed, binv = ops.band_split_ragged_forward(xb, gammas, weights, biases, widths, offsets)
    bdy = rn(1032, 62, 192)
    cases.append(("band_split_ragged_backward", (bdy, bnormed, binv, gammas, weights, widths, offsets)))
    hx = rn(1032, 62, 768)
    mweights = [rn(2 * w, 768, scale=768 ** -0.5) for w in widths]
    mbias = rn(2 * sum(widths), scale=0.1)
    cases.append(("mask_estimator_final_direct_forward", (hx, mweights, mbias, widths, offsets)))
    _, pre, _ = ops.mask_estimator_final_direct_forward(hx, mweights, mbias, widths, offsets)
    mdy = rn(1032, sum(widths))
    cases.append(("mask_estimator_final_direct_backward", (mdy, hx, pre, mweights, widths, offsets)))
    return cases


def test_package_kernels_beat_the_reference_kernels(cuda_device):
    ref = _reference_module()
    rows = []
    for name, args in _cases(cuda_device):
        t_ref = _time(lambda: getattr(ref, name)(*args))
        t_ours = _time(lambda: getattr(ops, name)(*args))
        rows.append((name, t_ref, t_ours))
    print()
    print(f"{'reference function (config-3 shape, fp16)':44s} {'reference':>11s} {'pymsst_b200':>12s} {'speed-up':>9s}")
    for name, t_ref, t_ours in rows:
        print(f"{name:44s} {t_ref:9.1f} us {t_ours:9.1f} us {t_ref / t_ours:8.1f}x")
    slower = [(n, r, o) for n, r, o in rows if o >= r]
    assert not slower, slower


def test_training_path_kernels_timed_beside_the_reference(cuda_device):
    """The tensor-core BandSplit and MaskEstimator final layer of the training path (bf16, the bench's type) on
    the same shapes, for the table; they replace the reference's ragged BandSplit and final MaskEstimator."""
    _reference_module()
    from pymsst_b200.fused import BandSplitFn, MaskEstimatorTCFn

    g = torch.Generator().manual_seed(1)
    dt = torch.bfloat16
    widths = tuple(4 * f for f in DEFAULT_FREQS_PER_BANDS)
    ld = (sum(widths) + 7) // 8 * 8
    xb = torch.randn(1032, ld, generator=g).to(dt).to(cuda_device)[:, : sum(widths)]
    params = ([torch.rand(w, generator=g).add(0.5).to(cuda_device) for w in widths]
              + [(torch.randn(192, w, generator=g) * w ** -0.5).to(cuda_device) for w in widths]
              + [torch.zeros(192, device=cuda_device) for _ in widths])
    t_band = _time(lambda: BandSplitFn.apply(xb, widths, 192, *params), graph=True)
    hx = torch.randn(1032, 62, 192, generator=g).to(dt).to(cuda_device)
    mparams = []
    for layer, (cin, cout) in enumerate(((192, 768), (768, None))):
        outs = [768] * 62 if cout else [2 * w for w in widths]
        mparams += [(torch.randn(o, cin, generator=g) * cin ** -0.5).to(cuda_device) for o in outs]
        mparams += [torch.zeros(o, device=cuda_device) for o in outs]
    t_mask = _time(lambda: MaskEstimatorTCFn.apply(hx, widths, 1, 768, *mparams), graph=True)
    print(f"\ntraining path, bf16: BandSplit tcgen05 forward {t_band:.1f} us; "
          f"MaskEstimator tcgen05 forward (both layers) {t_mask:.1f} us")
    assert t_band > 0 and t_mask > 0
