"""Record golden vectors of the reference's own fused CUDA kernels.

Run on a GPU box (the reference extension is built by ``oracle/build_ref.py``
from the reference sources into ``oracle/_ref/``):

    python tests/golden/make_golden.py --out tests/golden/reference_kernels.pt

Every case calls one function of the reference extension module
(src/pymsst/training/cuda/fused_band_split.cpp:731-753) on small seeded
inputs and stores the inputs and outputs (CPU tensors).  The shapes include the
reference's own test shapes (ragged widths (3, 5, 2, 7) from
tests/test_training_smoke.py:512-571 and (3, 4, 2, 5, 6) from :574-615).
The committed file is read by ``tests/test_golden_reference.py`` to pin the
CPU oracle (``oracle/ops_ref.py``) and, on the GPU, this package's kernels.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))


def _g(seed):
    g = torch.Generator().manual_seed(seed)
    return g


def _randn(g, *shape, dtype=torch.float32):
    return torch.randn(*shape, generator=g).to(dtype)


def cases():
    """(name, function, args) with CPU tensors; args are moved to CUDA at call time."""
    out = []
    g = _g(1)
    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        x = _randn(g, 5, 7, 24, dtype=dt)
        gamma = (torch.rand(24, generator=g) + 0.5).to(dt)
        out.append((f"rms_norm_forward_{tag}", "rms_norm_forward", [x, gamma]))
        normed = _randn(g, 5, 7, 24, dtype=dt)
        inv = torch.rand(35, generator=g) + 0.1
        dy = _randn(g, 5, 7, 24, dtype=dt)
        out.append((f"rms_norm_backward_{tag}", "rms_norm_backward", [dy, normed, inv, gamma]))
    x = _randn(g, 6, 32, dtype=torch.float16)
    gamma32 = torch.rand(32, generator=g) + 0.5
    out.append(("rms_norm_forward_fp32_gamma", "rms_norm_forward_fp32_gamma", [x, gamma32]))
    out.append(("rms_norm_backward_fp32_gamma", "rms_norm_backward_fp32_gamma",
                [_randn(g, 6, 32, dtype=torch.float16), _randn(g, 6, 32, dtype=torch.float16),
                 torch.rand(6, generator=g) + 0.1, gamma32]))
    xb = _randn(g, 6, 32, dtype=torch.bfloat16)
    out.append(("rms_norm_forward_mixed", "rms_norm_forward_mixed", [xb, gamma32]))
    out.append(("rms_norm_backward_mixed", "rms_norm_backward_mixed",
                [_randn(g, 6, 32), _randn(g, 6, 32), torch.rand(6, generator=g) + 0.1, gamma32, xb]))

    t = _randn(g, 2, 5, 3, 8)
    ang = torch.arange(5)[:, None] * torch.rand(4, generator=g)
    cos, sin = ang.cos().reshape(1, 5, 1, 4), ang.sin().reshape(1, 5, 1, 4)
    out.append(("rotary_forward", "rotary_forward", [t, cos, sin]))
    out.append(("rotary_backward", "rotary_backward", [_randn(g, 2, 5, 3, 8), cos, sin]))

    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        x = _randn(g, 4, 3, 6, dtype=dt)
        gamma = (torch.rand(3, 6, generator=g) + 0.5).to(dt)
        w = (_randn(g, 3, 5, 6) * 0.3).to(dt)
        b = _randn(g, 3, 5, dtype=dt)
        out.append((f"band_split_forward_{tag}", "band_split_forward", [x, gamma, w, b]))
        normed = _randn(g, 4, 3, 6, dtype=dt)
        inv = torch.rand(4, 3, generator=g) + 0.1
        dy = _randn(g, 4, 3, 5, dtype=dt)
        for v in ("band_split_backward", "band_split_backward_v2", "band_split_backward_v3"):
            out.append((f"{v}_{tag}", v, [dy, normed, inv, gamma, w, True]))
    out.append(("band_split_forward_nobias", "band_split_forward", [_randn(g, 4, 3, 6), torch.rand(3, 6, generator=g) + 0.5,
                                                                      _randn(g, 3, 5, 6), None]))

    widths = [3, 5, 2, 7]
    offsets = torch.tensor([0, 3, 8, 10, 17])
    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        x = _randn(g, 5, 17, dtype=dt)
        gammas = [(torch.rand(w, generator=g) + 0.5).to(dt) for w in widths]
        weights = [(_randn(g, 4, w) * 0.4).to(dt) for w in widths]
        biases = [_randn(g, 4, dtype=dt) for _ in widths]
        out.append((f"band_split_ragged_forward_{tag}", "band_split_ragged_forward",
                    [x, gammas, weights, biases, widths, offsets]))
        dy = _randn(g, 5, 4, 4, dtype=dt)
        normed = _randn(g, 5, 17, dtype=dt)
        inv = torch.rand(5, 4, generator=g) + 0.1
        out.append((f"band_split_ragged_backward_{tag}", "band_split_ragged_backward",
                    [dy, normed, inv, gammas, weights, widths, offsets]))

    out.append(("grouped_linear_forward", "grouped_linear_forward",
                [_randn(g, 4, 3, 6), _randn(g, 3, 5, 6), _randn(g, 3, 5)]))

    attn = _randn(g, 6, 2, 4)
    xg = _randn(g, 6, 8)
    wg = _randn(g, 2, 8) * 0.5
    bg = _randn(g, 2)
    out.append(("attention_gate_forward", "attention_gate_forward", [attn, xg, wg, bg]))
    gate = torch.rand(6, 2, generator=g)
    out.append(("attention_gate_backward", "attention_gate_backward", [_randn(g, 6, 8), attn, xg, wg, gate]))

    mwidths = [3, 4, 2, 5, 6]
    moff = torch.tensor([0, 3, 7, 9, 14, 20])
    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        x = _randn(g, 4, 5, 16, dtype=dt)
        weights = [(_randn(g, 2 * w, 16) * 0.3).to(dt) for w in mwidths]
        bias = _randn(g, 40, dtype=dt)
        # Only the "direct" kernels: the reference's "grouped" variant hands host
        # std::vector pointer arrays to cublasGemmGroupedBatchedEx (which needs
        # device-resident pointer arrays) and raised an illegal memory access on
        # the B200 (fused_band_split.cu:2258-2279); it is not run again.
        out.append((f"mask_estimator_final_direct_forward_{tag}", "mask_estimator_final_direct_forward",
                    [x, weights, bias, mwidths, moff]))
        dy = _randn(g, 4, 20, dtype=dt)
        pre = _randn(g, 4, 40, dtype=dt)
        out.append((f"mask_estimator_final_direct_backward_{tag}", "mask_estimator_final_direct_backward",
                    [dy, x, pre, weights, mwidths, moff]))
    return out


def _to(obj, device):
    if isinstance(obj, torch.Tensor):
        return obj.to(device)
    if isinstance(obj, list):
        return [_to(o, device) for o in obj]
    return obj


def _cpu(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, (list, tuple)):
        return [_cpu(o) for o in obj]
    return obj


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--out", type=Path, default=REPO / "tests" / "golden" / "reference_kernels.pt")
    args = parser.parse_args()
    from oracle.build_ref import load

    ext = load()
    device = torch.device("cuda", 0)
    record = {"device": torch.cuda.get_device_name(0), "torch": str(torch.__version__), "cases": {}}
    for name, fn, fargs in cases():
        try:
            result = getattr(ext, fn)(*_to(fargs, device))
            torch.cuda.synchronize()
        except RuntimeError as exc:  # recorded, e.g. a cuBLAS path rejecting a shape
            record.setdefault("failed", {})[name] = str(exc)
            print(name, "FAILED", exc, flush=True)
            continue
        outputs = list(result) if isinstance(result, (list, tuple)) else [result]
        record["cases"][name] = {"fn": fn, "args": _cpu(fargs), "outputs": _cpu(outputs)}
        print(name, "ok", flush=True)
    args.out.parent.mkdir(parents=True, exist_ok=True)
    torch.save(record, args.out)
    print("wrote", args.out, args.out.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
