"""Pin the oracle, and the sm_100a kernels, to the reference's own CUDA kernels.

``tests/golden/reference_kernels.pt`` holds inputs and outputs of every
function of the reference's compiled extension (recorded on a B200 by
``tests/golden/make_golden.py``).  The CPU test checks the oracle restatement
(``oracle/ops_ref.py``) against them; the GPU test runs this package's
reference-compatible ops on the same inputs.

Tolerances: fp32 outputs 1e-5 relative / absolute (the reference is built
with --use_fast_math, so its sqrt/div/exp differ by a few ulp); fp16 / bf16
outputs 3e-3 (one or two half-precision ulps, sums scaled by their length).
"""
from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import ops_ref

GOLDEN_PATH = Path(__file__).resolve().parent / "golden" / "reference_kernels.pt"
GOLDEN = torch.load(GOLDEN_PATH, weights_only=True)
CASES = sorted(GOLDEN["cases"])


def _to(obj, device=None, dtype=None):
    if isinstance(obj, torch.Tensor):
        t = obj
        if dtype is not None and t.is_floating_point():
            t = t.to(dtype)
        return t.to(device) if device is not None else t
    if isinstance(obj, list):
        return [_to(o, device, dtype) for o in obj]
    return obj


def _flatten(outputs):
    flat = []
    for o in outputs:
        if isinstance(o, (list, tuple)):
            flat.extend(_flatten(o))
        else:
            flat.append(o)
    return flat


def _compare(actual, expected, name):
    actual, expected = _flatten(actual), _flatten(expected)
    assert len(actual) == len(expected), f"{name}: {len(actual)} outputs vs {len(expected)}"
    for k, (a, e) in enumerate(zip(actual, expected)):
        if e is None or (isinstance(e, torch.Tensor) and e.numel() == 0 and a is None):
            continue
        assert a is not None, f"{name}: output {k} missing"
        low = e.dtype in (torch.float16, torch.bfloat16)
        tol = 3e-3 if low else 1e-5
        scale = max(1.0, float(e.double().abs().max()))
        torch.testing.assert_close(
            a.detach().double().cpu(), e.double(), rtol=tol, atol=tol * scale, msg=lambda m: f"{name}[{k}]: {m}"
        )


def test_golden_file_covers_the_reference_surface():
    fns = {case["fn"] for case in GOLDEN["cases"].values()}
    expected = {
        "rms_norm_forward", "rms_norm_backward", "rms_norm_forward_fp32_gamma", "rms_norm_backward_fp32_gamma",
        "rms_norm_forward_mixed", "rms_norm_backward_mixed", "rotary_forward", "rotary_backward",
        "band_split_forward", "band_split_backward", "band_split_backward_v2", "band_split_backward_v3",
        "band_split_ragged_forward", "band_split_ragged_backward", "grouped_linear_forward",
        "attention_gate_forward", "attention_gate_backward", "mask_estimator_final_direct_forward",
    }
    assert expected <= fns


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_kernels(name):
    case = GOLDEN["cases"][name]
    fn = getattr(ops_ref, case["fn"])
    args = _to(case["args"], dtype=torch.float64)
    result = fn(*args)
    result = list(result) if isinstance(result, (list, tuple)) else [result]
    _compare(result, case["outputs"], name)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_kernels_match_reference_kernels(cuda_device, name):
    from pymsst_b200.extension import ops

    case = GOLDEN["cases"][name]
    fn = getattr(ops, case["fn"])
    result = fn(*_to(case["args"], device=cuda_device))
    result = list(result) if isinstance(result, (list, tuple)) else [result]
    if case["fn"] == "attention_gate_forward":
        result, expected = result[:2], case["outputs"][:2]
    else:
        expected = case["outputs"]
    _compare(result, expected, name)
