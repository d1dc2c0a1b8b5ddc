"""Roofline work models (pymsst_b200/roofline.py) on the CPU: every entry point the bench times has one, and the
dominant entries' algorithmic bytes at the config-3 shapes are the figures the bench reports."""
from __future__ import annotations

import ast
from pathlib import Path

import pytest

from pymsst_b200 import roofline

REPO = Path(__file__).resolve().parents[1]


def _timed_entries() -> list[str]:
    tree = ast.parse((REPO / "bench.py").read_text())
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "TIMED_ENTRIES" for t in node.targets):
            return [ast.literal_eval(e) for e in node.value.elts]
    raise AssertionError("bench.py has no TIMED_ENTRIES list")


def test_every_timed_entry_has_a_work_model():
    src = (REPO / "pymsst_b200" / "roofline.py").read_text()
    missing = [name for name in _timed_entries() if f'"{name}"' not in src]
    assert not missing, f"entries timed by the bench without a work model: {missing}"


def _qkv_args(sequences, seq_len, inner):
    # pmb_qkv_linear_rotary_forward(x, w, cos_t, sin_t, batch, seq_len, dim, heads, dim_head, q, k, v, rotate,
    #                               dtype, seq_inner, stream)
    return (1, 1, 1, 1, sequences, seq_len, 192, 8, 64, 1, 1, 1, 1, 2, inner, None)


def test_qkv_projection_bytes_at_config3():
    """The bench line's algorithmic_bytes_per_call for the dominant entry is the mean of the time-axis call
    (248 sequences of 258 positions) and the band-axis call (1032 sequences of 62 positions)."""
    rows, dim, n = 63984, 192, 3 * 8 * 64
    base = (rows * dim + n * dim + rows * n) * 2
    t_bytes, t_flops = roofline.work("pmb_qkv_linear_rotary_forward", _qkv_args(248, 258, 62))
    b_bytes, b_flops = roofline.work("pmb_qkv_linear_rotary_forward", _qkv_args(1032, 62, 1))
    assert t_bytes == base + 2 * 258 * 32 * 4  # plus the two angle tables
    assert b_bytes == base + 2 * 62 * 32 * 4
    assert (t_bytes + b_bytes) / 2 == 221759488
    assert t_flops == b_flops == 2.0 * rows * n * dim


def test_gated_attention_backward_bytes_at_config3():
    seqs, n, h, dh = 1032, 62, 8, 64
    args = [1] * 25
    args[15], args[16], args[17], args[18], args[21] = seqs, n, h, dh, 2
    byt, flops = roofline.work("pmb_attention_backward_gated", tuple(args))
    plane = seqs * n * h * dh * 2
    # Q, K, V, gated output, its gradient read; dQ, dK, dV written; lse / logits / logit gradient rows
    assert byt == 8 * plane + 12 * seqs * h * n + 2 * seqs * n * h * 2
    assert flops == 10.0 * seqs * h * n * n * dh


def test_dense_gemm_bytes():
    # pmb_gemm_tc(a, lda, a_mn, b, ldb, b_mn, c, ldc, c_dtype, bias, bias_dtype, act, m, n, k, dtype, stream)
    byt, flops = roofline.work("pmb_gemm_tc", (1, 192, 0, 1, 192, 0, 1, 768, 2, 1, 0, 0, 63984, 768, 192, 2, None))
    assert byt == (63984 * 192 + 768 * 192) * 2 + 63984 * 768 * 2 + 768 * 4
    assert flops == 2.0 * 63984 * 768 * 192


@pytest.mark.parametrize("in_step", [True, False])
def test_roofline_picks_the_binding_roof(in_step):
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "source": "test"}
    args = [_qkv_args(1032, 62, 1)] * 4
    r = roofline.roofline("pmb_qkv_linear_rotary_forward", 4, 4 * 0.08, args, peaks, in_step=in_step)
    # 221.7 MB against 37.7 GFLOP: HBM binds (37 us at 6 TB/s against 24-27 us of tensor time)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert r["achieved"] == pytest.approx(221734400 / 80e-6 / 1e9, rel=1e-3)
    assert r["frac"] == pytest.approx(r["achieved"] / 6000.0, rel=1e-3)
