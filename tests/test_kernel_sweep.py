"""The config-2 kernel sweep's case list (``kernel_bench --sweep``): host logic only, checked without a GPU
against the shapes the benchmark configuration names."""
from __future__ import annotations

from pymsst_b200.kernel_bench import sweep_cases

L2_BYTES = 126 * 2 ** 20


def test_sweep_covers_config2_shapes():
    cases = sweep_cases()
    rms = [s for op, s in cases if op == "rms"]
    assert {(s["dtype"], s["dim"]) for s in rms} == {(d, k) for d in ("bf16", "fp32") for k in (192, 384)}
    assert max(s["rows"] for s in rms) == 8 * 62 * 1024  # B·F up to 8 x 62 bands, T up to 1024
    rot = [s for op, s in cases if op == "rotary"]
    assert {s["seq"] for s in rot} == {62, 1024} and all(s["heads"] == 8 and s["dim"] == 64 for s in rot)
    assert ("band", {"rows": 8 * 1024}) in cases
    assert ("mel", {"batch": 4, "frames": 1024}) in cases  # [8, 1025, 1024] complex stereo


def test_sweep_reaches_beyond_l2():
    """RMSNorm's and rotary's largest tensors exceed the L2; the mel case is the configuration's own
    [8, 1025, 1024] complex input (67 MB, half the L2), timed cold because the L2 is flushed between calls."""
    es = {"bf16": 2, "fp32": 4}
    cases = sweep_cases()
    assert max(s["rows"] * s["dim"] * es[s["dtype"]] for op, s in cases if op == "rms") > L2_BYTES
    assert max(s["batch"] * s["seq"] * s["heads"] * s["dim"] * es[s["dtype"]] for op, s in cases
               if op == "rotary") > L2_BYTES
    mel = next(s for op, s in cases if op == "mel")
    assert mel["batch"] * 2 * 1025 * mel["frames"] * 2 * 4 > L2_BYTES / 2
