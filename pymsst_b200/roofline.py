"""Algorithmic work models of the C-ABI entry points, for roofline reporting.

For one call, ``work(name, args)`` returns the algorithmic HBM bytes (every
operand read once, every result written once) and floating-point operations
of the op, computed from the call's own arguments.  ``roofline`` turns the
measured average duration of those calls into the achieved rate against the
binding roof: HBM bandwidth or the dense bf16 tensor peak, whichever bounds
the op at its arithmetic intensity.
"""
from __future__ import annotations

import json
from pathlib import Path

ES = {0: 4, 1: 2, 2: 2}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks(path: str | Path | None = None) -> dict:
    candidates = [Path(path)] if path else []
    candidates.append(Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json")
    for c in candidates:
        if c.is_file():
            data = json.loads(c.read_text())
            return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                    "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                    "source": "measured"}
    return dict(FALLBACK_PEAKS)


def _widths(ptr, n):
    return [int(ptr[i]) for i in range(n)]


def work(name: str, a: tuple) -> tuple[float, float]:
    """(bytes, flops) of one call of entry point ``name`` with ctypes args ``a``."""
    if name == "pmb_rms_norm_forward":
        rows, dim, xd, gd, od = a[5], a[6], a[7], a[8], a[9]
        outs = 1 + (a[3] is not None)
        return rows * dim * (ES[xd] + outs * ES[od]) + 4 * rows + dim * ES[gd], 4.0 * rows * dim
    if name == "pmb_rms_norm_backward":
        rows, dim, gd, gmd, gxd = a[7], a[8], a[9], a[10], a[11]
        return rows * dim * (2 * ES[gd] + (ES[gxd] if a[5] is not None else 0)) + 4 * rows + 2 * dim * ES[gmd], \
            8.0 * rows * dim
    if name == "pmb_rms_norm_backward_add":  # dy, x and the residual gradient read, grad_x written
        rows, dim, gd, gmd, gxd = a[8], a[9], a[10], a[11], a[12]
        return rows * dim * (2 * ES[gd] + 2 * ES[gxd]) + 4 * rows + 2 * dim * ES[gmd], 9.0 * rows * dim
    if name in ("pmb_qkv_rotary_split", "pmb_qkv_rotary_merge"):
        b, n, h, dh = (a[3], a[4], a[5], a[6]) if name.endswith("split") else (a[5], a[6], a[7], a[8])
        dt = a[11]
        return 2.0 * b * n * 3 * h * dh * ES[dt] + 2 * n * dh // 2 * 4, 6.0 * b * n * 2 * h * dh
    if name == "pmb_attention_gate_forward":
        rows, h, dh, dim, dt, pt = a[8], a[9], a[10], a[11], a[14], a[15]
        return rows * (2 * h * dh + dim + h) * ES[dt] + h * (dim + 1) * ES[pt], 2.0 * rows * h * (dim + dh)
    if name == "pmb_attention_gate_backward":
        rows, h, dh, dim, dt, pt = a[9], a[10], a[11], a[12], a[17], a[18]
        return rows * (3 * h * dh + 2 * dim + h) * ES[dt] + 8 * rows * h + 2 * h * (dim + 1) * ES[pt], \
            4.0 * rows * h * (dim + dh)
    if name == "pmb_band_gather_forward":
        b, s, f, t, j, xd = a[2], a[3], a[4], a[5], a[6], a[9]
        return b * t * j * 2 * (4 + ES[xd]) + 4 * j, 0.0
    if name == "pmb_band_recombine_forward":
        b, n, s, f, t, j, mult, md = a[4], a[5], a[6], a[7], a[8], a[9], a[10], a[12]
        return b * n * t * j * 2 * ES[md] + (b * s * f * t * 8 if mult else 0) + b * n * s * f * t * 8, \
            8.0 * b * n * s * f * t
    if name == "pmb_band_recombine_backward":
        b, n, s, f, t, j, mult, md = a[4], a[5], a[6], a[7], a[8], a[9], a[10], a[12]
        return b * n * s * f * t * 8 + (b * s * f * t * 8 if mult else 0) + b * n * t * j * 2 * ES[md], \
            8.0 * b * n * t * j
    if name == "pmb_band_split_forward":
        rows, nb, o, dt, pt = a[1], a[5], a[10], a[14], a[15]
        total = sum(_widths(a[6], nb))
        normed = a[12] is not None
        byt = rows * total * ES[dt] * (1 + normed) + rows * nb * (o * ES[dt] + 4) + (total * (o + 1) + nb * o) * ES[pt]
        return byt, 2.0 * rows * total * o
    if name == "pmb_band_split_backward":
        rows, nb, o, dt, pt = a[3], a[4], a[8], a[13], a[14]
        total = sum(_widths(a[5], nb))
        gx = a[9] is not None
        byt = rows * nb * o * ES[dt] + rows * total * ES[dt] * (1 + gx) + 4 * rows * nb + 2 * (total * (o + 1) + nb * o) * ES[pt]
        return byt, 2.0 * rows * total * o * (2 if gx else 1)
    if name == "pmb_grouped_linear_forward":
        rows, g, i, o, dt, pt = a[1], a[2], a[3], a[4], a[12], a[13]
        return rows * g * (i + o) * ES[dt] + g * o * (i + 1) * ES[pt], 2.0 * rows * g * i * o
    if name == "pmb_grouped_linear_backward":
        rows, g, i, o, dt, pt = a[3], a[4], a[5], a[6], a[13], a[14]
        gx = a[8] is not None
        return rows * g * (2 * o + i * (1 + gx)) * ES[dt] + 2 * g * o * (i + 1) * ES[pt], \
            2.0 * rows * g * i * o * (2 if gx else 1)
    if name == "pmb_mask_estimator_final_forward":
        rows, nb, h, dt, pt = a[1], a[2], a[3], a[9], a[10]
        total = sum(_widths(a[4], nb))
        return rows * (nb * h + 3 * total) * ES[dt] + 2 * total * (h + 1) * ES[pt], 4.0 * rows * h * total
    if name == "pmb_mask_estimator_final_backward":
        rows, nb, h, dt, pt = a[3], a[4], a[5], a[11], a[12]
        total = sum(_widths(a[6], nb))
        return rows * (2 * nb * h + 3 * total) * ES[dt] + 2 * 2 * total * (h + 1) * ES[pt], 8.0 * rows * h * total
    if name == "pmb_gemm_tc":  # A [m, k] and B [n, k] read, C [m, n] written, the bias slice read
        m, n, k, cd, bd, dt = a[12], a[13], a[14], a[8], a[10], a[15]
        return (m * k + n * k) * ES[dt] + m * n * ES[cd] + (n * ES[bd] if a[9] else 0), 2.0 * m * n * k
    if name == "pmb_qkv_linear_rotary_forward":
        rows, dim, n, dt = a[4] * a[5], a[6], 3 * a[7] * a[8], a[13]
        return (rows * dim + n * dim + rows * n) * ES[dt] + 2 * a[5] * a[8] // 2 * 4, 2.0 * rows * n * dim
    if name == "pmb_band_split_tc_forward":
        # x read once, out and inv written once, parameters read once
        rows, nb, o, dt, pt = a[1], a[3], a[8], a[12], a[13]
        total = sum(_widths(a[4], nb))
        byt = rows * total * ES[dt] + rows * nb * (o * ES[dt] + 4) + (total * (o + 1) + nb * o) * ES[pt]
        return byt, 2.0 * rows * total * o
    if name == "pmb_band_split_tc_backward":
        # dY, x and inv read once; W read; grad W, gamma, bias written
        rows, nb, o, dt, pt = a[4], a[5], a[9], a[13], a[14]
        total = sum(_widths(a[6], nb))
        byt = rows * nb * (o * ES[dt] + 4) + rows * total * ES[dt] + (2 * total * o + 2 * total + 2 * nb * o) * ES[pt]
        return byt, 2.0 * rows * total * o
    if name in ("pmb_mask_estimator_tc_forward", "pmb_mask_estimator_tc_backward"):
        fwd = name.endswith("forward")
        rows, nb, dim, hid, layers = a[1 if fwd else 5], a[2 if fwd else 6], a[3 if fwd else 7], \
            a[4 if fwd else 8], a[5 if fwd else 9]
        widths = _widths(a[6 if fwd else 10], nb)
        dt, pt = (a[13], a[14]) if fwd else (a[14], a[15])
        total = sum(widths)
        hin = hid if layers > 0 else dim
        flops = 2.0 * rows * (nb * dim * hid * (layers > 0) + max(layers - 1, 0) * nb * hid * hid + 2 * total * hin)
        params = nb * dim * hid * (layers > 0) + max(layers - 1, 0) * nb * hid * hid + 2 * total * hin
        acts = rows * (nb * dim + layers * nb * hid + 2 * total + total)
        if fwd:
            return acts * ES[dt] + params * (ES[pt] + ES[dt]), flops
        return (acts + rows * total) * ES[dt] + 2 * params * ES[pt], 2 * flops
    if name == "pmb_attention_forward":
        seqs, n, h, dh, dt = a[5], a[6], a[7], a[8], a[11]
        plane = seqs * n * h * dh * ES[dt]
        return 4.0 * plane + 4.0 * seqs * h * n, 4.0 * seqs * h * n * n * dh
    if name == "pmb_attention_backward":
        seqs, n, h, dh, dt = a[9], a[10], a[11], a[12], a[15]
        plane = seqs * n * h * dh * ES[dt]
        # q, k, v, o, dO read; dQ, dK, dV written; lse read, D written and read back
        return 8.0 * plane + 12.0 * seqs * h * n, 10.0 * seqs * h * n * n * dh
    if name == "pmb_attention_backward_rotary":  # the same, plus the two fp32 angle tables
        seqs, n, h, dh, dt = a[11], a[12], a[13], a[14], a[17]
        plane = seqs * n * h * dh * ES[dt]
        return 8.0 * plane + 12.0 * seqs * h * n + 2 * 4.0 * n * dh // 2, 10.0 * seqs * h * n * n * dh
    if name in ("pmb_stft_frames_forward", "pmb_stft_frames_backward"):
        b, length, n_fft, frames = a[3], a[4], a[5], a[7]
        return 4.0 * (b * length + b * frames * n_fft + n_fft), 1.0 * b * frames * n_fft
    if name == "pmb_istft_overlap_add_forward":  # frames read once, the signal written
        b, n, t, length = a[4], a[5], a[6], a[8]
        return 4.0 * b * (n * t + length), 3.0 * b * n * t
    if name == "pmb_istft_overlap_add_backward":  # the signal's gradient read, the frames' written
        b, n, t, length = a[3], a[4], a[5], a[7]
        return 4.0 * b * (n * t + length), 2.0 * b * n * t
    if name == "pmb_spectral_l1_forward":  # two complex64 spectra read
        return 16.0 * a[2], 4.0 * a[2]
    if name == "pmb_spectral_l1_backward":  # two read, the gradient written
        return 24.0 * a[2], 8.0 * a[2]
    if name == "pmb_attention_forward_gated":  # the attention forward plus the [rows, heads] logits
        seqs, n, h, dh, dt = a[6], a[7], a[8], a[9], a[12]
        plane = seqs * n * h * dh * ES[dt]
        return 4.0 * plane + 4.0 * seqs * h * n + seqs * n * h * ES[dt], 4.0 * seqs * h * n * n * dh
    if name == "pmb_attention_backward_gated":  # the backward plus logits read and their gradient written
        seqs, n, h, dh, dt = a[15], a[16], a[17], a[18], a[21]
        plane = seqs * n * h * dh * ES[dt]
        return 8.0 * plane + 12.0 * seqs * h * n + 2.0 * seqs * n * h * ES[dt], 10.0 * seqs * h * n * n * dh
    if name == "pmb_gelu_forward":
        return 2.0 * a[2] * ES[a[3]], 0.0
    if name == "pmb_gelu_backward":
        return 3.0 * a[3] * a[4] * ES[a[7]], 0.0
    if name == "pmb_column_sum":
        return 1.0 * a[1] * a[2] * ES[a[5]], 0.0
    return 0.0, 0.0


# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of each entry's main kernel, from one
# `ncu --set full --clock-control none` capture of that kernel on the config-3 shapes
# (`python -m pymsst_b200.kernel_bench <op> --iters 2 --warmup 1`; the attention entries on the band-axis
# shape the step runs them on).  Writes that still sit in the 126 MB L2 when a kernel ends are not counted,
# so traffic can read below the algorithmic bytes; well above them would mean re-reads.
MEASURED_TRAFFIC = {
    "config3": {
        "pmb_qkv_linear_rotary_forward": 168.3e6,
        "pmb_attention_forward": 235.2e6,
        "pmb_attention_backward": 483.7e6,
        "pmb_attention_gate_forward": 118.5e6,
        "pmb_attention_gate_backward": 216.1e6,
        "pmb_rms_norm_forward": 26.1e6,
        "pmb_rms_norm_backward": 50.4e6,
        "pmb_gelu_forward": 152.6e6,
    },
}


def roofline(name: str, calls: int, total_ms: float, args_list: list, peaks: dict, traffic=None,
             in_step: bool = True) -> dict:
    """Achieved rate of the timed calls against the roof that binds this op.

    ``in_step``: the calls were timed inside a long training step, so the tensor roof is the sustained bf16
    figure (the GPU settles at a lower clock under its power cap); otherwise the burst figure of a kernel
    timed alone.  HBM has one measured figure for both."""
    tflops = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) if in_step else peaks["bf16_tflops"]
    byt = sum(work(name, a)[0] for a in args_list)
    flops = sum(work(name, a)[1] for a in args_list)
    secs = total_ms / 1e3
    t_hbm = byt / (peaks["hbm_gbs"] * 1e9)
    t_tc = flops / (tflops * 1e12)
    per_launch_ms = total_ms / max(calls, 1)
    if t_tc > t_hbm:
        achieved = flops / secs / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": tflops, "unit": "TFLOP/s",
                "frac": round(achieved / tflops, 4), "traffic": traffic, "kernel": name,
                "peak_kind": "sustained" if in_step else "burst",
                "calls": calls, "ms_per_call": round(per_launch_ms, 4), "peak_source": peaks["source"],
                "algorithmic_flops_per_call": flops / max(calls, 1)}
    achieved = byt / secs / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic, "kernel": name, "calls": calls,
            "ms_per_call": round(per_launch_ms, 4), "peak_source": peaks["source"],
            "algorithmic_bytes_per_call": byt / max(calls, 1)}

