"""Per-kernel timings of the C-ABI entry points at the config-3 shapes.

``python -m pymsst_b200.kernel_bench [op ...] [--iters N] [--json PATH]``;
``--sweep`` runs the config-2 kernel sweep instead (isolated kernels up to
tensors well beyond L2, bf16 and fp32: ``sweep_cases``).

Each op is one entry-point call on synthetic device tensors with the shapes a
config-3 training step uses (BS-RoFormer dim 192, 8 heads of 64, batch 4 x
258 frames x 62 bands = 63984 transformer rows).  Calls are timed with CUDA
events on the launching stream after 3 warm-up calls, with a 256 MB buffer
written between timed calls so every call starts with a cold L2.  The line
printed per op gives the median time, the algorithmic bytes (each operand
read once, each result written once) and the achieved fraction of the
measured HBM bandwidth, or TFLOP/s for the GEMMs.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _native as nat
from .roofline import load_peaks

ROWS, DIM, HEADS, DHEAD = 63984, 192, 8, 64
SEQ_BATCH, SEQ = 248, 258


class _Bench:
    def __init__(self, device: torch.device, iters: int, warmup: int = 3, graphs: bool = True):
        self.device = device
        self.graphs = graphs
        self.iters = iters
        self.warmup = warmup
        self.flush = torch.empty(64 * 1024 * 1024, device=device)
        # every op runs on this side stream (made current by main), the stream its graphs are captured on
        self.stream = torch.cuda.Stream(device)
        self.results: dict[str, dict] = {}
        self.peaks = load_peaks()

    def time(self, name: str, fn, bytes_: float = 0.0, flops: float = 0.0) -> dict:
        """Median device time of ``fn``: captured once into a CUDA graph after the warm-up calls and replayed
        (so host launch work between an op's kernels is not timed), 256 MB written between replays so L2
        starts cold; ops that cannot be captured are timed as eager calls."""
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize(self.device)
        graph = None
        if self.graphs:
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=self.stream):
                    fn()
            except Exception:  # not capturable: time eager calls instead
                graph = None
                torch.cuda.synchronize(self.device)
        times = []
        for _ in range(self.iters):
            self.flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(self.stream)
            if graph is not None:
                graph.replay()
            else:
                fn()
            b.record(self.stream)
            torch.cuda.synchronize(self.device)
            times.append(a.elapsed_time(b))
        times.sort()
        us = times[len(times) // 2] * 1e3
        rec = {"us": round(us, 2), "bytes": bytes_, "flops": flops}
        if flops > 0 and flops / (self.peaks["bf16_tflops"] * 1e12) > bytes_ / (self.peaks["hbm_gbs"] * 1e9):
            rec["tflops"] = round(flops / us / 1e6, 1)
            rec["frac"] = round(rec["tflops"] / self.peaks["bf16_tflops"], 3)
            what = f"{rec['tflops']:8.1f} TFLOP/s"
        else:
            rec["gbs"] = round(bytes_ / us / 1e3, 1)
            rec["frac"] = round(rec["gbs"] / self.peaks["hbm_gbs"], 3)
            what = f"{rec['gbs']:8.1f} GB/s"
        self.results[name] = rec
        print(f"{name:34s} {us:9.1f} us {bytes_ / 1e6:9.1f} MB {what}  frac {rec['frac']:.3f}", flush=True)
        return rec


def _gemm(a, lda, a_mn, b, ldb, b_mn, c, m, n, k, bias=None, act=0):
    nat.call("pmb_gemm_tc", a.data_ptr(), lda, a_mn, b.data_ptr(), ldb, b_mn, c.data_ptr(), c.stride(0),
             nat.dtype_code(c.dtype), nat.ptr(bias), nat.dtype_code(bias.dtype) if bias is not None else 0, act,
             m, n, k, nat.dtype_code(a.dtype), nat.stream_handle(a.device))


def op_gate(bench: _Bench):
    dev, bf, f32 = bench.device, torch.bfloat16, torch.float32
    x = torch.randn(ROWS, DIM, device=dev, dtype=bf)
    # [b, h, n, dh] view of a [b, n, h, dh] plane, the layout the attention kernels write
    attn = torch.randn(SEQ_BATCH, SEQ, HEADS, DHEAD, device=dev, dtype=bf).transpose(1, 2)
    w = torch.randn(HEADS, DIM, device=dev, dtype=f32) * 0.1
    b = torch.randn(HEADS, device=dev, dtype=f32)
    out = torch.empty(ROWS, HEADS * DHEAD, device=dev, dtype=bf)
    gate = torch.empty(ROWS, HEADS, device=dev, dtype=bf)
    st = nat.stream_handle(dev)
    strides = (attn.stride(0), attn.stride(2), attn.stride(1))

    def fwd():
        nat.call("pmb_attention_gate_forward", attn.data_ptr(), SEQ, *strides, x.data_ptr(), w.data_ptr(),
                 b.data_ptr(), ROWS, HEADS, DHEAD, DIM, out.data_ptr(), gate.data_ptr(), nat.dtype_code(bf),
                 nat.dtype_code(f32), 1, st)

    e = 2
    bench.time("attention_gate_forward", fwd, ROWS * (DIM + 2 * HEADS * DHEAD + HEADS) * e)
    dy = torch.randn(ROWS, HEADS * DHEAD, device=dev, dtype=bf)
    ga, gx = torch.empty_like(attn), torch.empty_like(x)
    gw, gb = torch.empty_like(w), torch.empty_like(b)
    wsb = nat.library().pmb_attention_gate_backward_workspace_size(ROWS, HEADS, DIM)
    ws = nat.workspace(wsb, dev)

    def bwd():
        nat.call("pmb_attention_gate_backward", dy.data_ptr(), attn.data_ptr(), SEQ, *strides, x.data_ptr(),
                 w.data_ptr(), gate.data_ptr(), ROWS, HEADS, DHEAD, DIM, ga.data_ptr(), gx.data_ptr(), gw.data_ptr(),
                 gb.data_ptr(), nat.dtype_code(bf), nat.dtype_code(f32), ws.data_ptr(), wsb, 1, st)

    bench.time("attention_gate_backward", bwd, ROWS * (3 * HEADS * DHEAD + 2 * DIM + HEADS) * e)


def op_rms(bench: _Bench):
    dev, bf = bench.device, torch.bfloat16
    x = torch.randn(ROWS, DIM, device=dev, dtype=bf)
    g = torch.ones(DIM, device=dev, dtype=bf)
    out, normed = torch.empty_like(x), torch.empty_like(x)
    inv = torch.empty(ROWS, device=dev)
    st = nat.stream_handle(dev)
    bench.time("rms_norm_forward", lambda: nat.call(
        "pmb_rms_norm_forward", x.data_ptr(), g.data_ptr(), out.data_ptr(), normed.data_ptr(), inv.data_ptr(), ROWS,
        DIM, 2, 2, 2, st), ROWS * DIM * 2 * 3 + ROWS * 4)
    dy = torch.randn_like(x)
    gx, gg = torch.empty_like(x), torch.empty_like(g)
    wsb = nat.library().pmb_rms_norm_backward_workspace_size(ROWS, DIM)
    ws = nat.workspace(wsb, dev)
    bench.time("rms_norm_backward", lambda: nat.call(
        "pmb_rms_norm_backward", dy.data_ptr(), x.data_ptr(), 1, inv.data_ptr(), g.data_ptr(), gx.data_ptr(),
        gg.data_ptr(), ROWS, DIM, 2, 2, 2, 2, ws.data_ptr(), wsb, st), ROWS * DIM * 2 * 3 + ROWS * 4)
    res = torch.randn_like(x)
    bench.time("rms_norm_backward_add (+ residual gradient)", lambda: nat.call(
        "pmb_rms_norm_backward_add", dy.data_ptr(), x.data_ptr(), 1, inv.data_ptr(), g.data_ptr(), res.data_ptr(),
        gx.data_ptr(), gg.data_ptr(), ROWS, DIM, 2, 2, 2, 2, ws.data_ptr(), wsb, st), ROWS * DIM * 2 * 4 + ROWS * 4)
    bench.time("torch add (the residual sum it replaces)", lambda: torch.add(gx, res, out=out), ROWS * DIM * 2 * 3)


def op_qkv(bench: _Bench):
    dev, bf = bench.device, torch.bfloat16
    n3 = 3 * HEADS * DHEAD
    x = torch.randn(ROWS, DIM, device=dev, dtype=bf)
    w = torch.randn(n3, DIM, device=dev, dtype=bf) * 0.05
    qkv = torch.empty(ROWS, n3, device=dev, dtype=bf)
    flops = 2.0 * ROWS * n3 * DIM
    bench.time("gemm_tc qkv (x W^T)", lambda: _gemm(x, DIM, 0, w, DIM, 0, qkv, ROWS, n3, DIM),
               (ROWS * DIM + n3 * DIM + ROWS * n3) * 2, flops)
    bench.time("torch qkv (x W^T)", lambda: torch.matmul(x, w.t(), out=qkv), (ROWS * DIM + n3 * DIM + ROWS * n3) * 2,
               flops)
    dx = torch.empty(ROWS, DIM, device=dev, dtype=bf)
    bench.time("gemm_tc dx (dqkv W)", lambda: _gemm(qkv, n3, 0, w, DIM, 1, dx, ROWS, DIM, n3),
               (ROWS * DIM + n3 * DIM + ROWS * n3) * 2, flops)
    bench.time("torch dx (dqkv W)", lambda: torch.matmul(qkv, w, out=dx), (ROWS * DIM + n3 * DIM + ROWS * n3) * 2,
               flops)
    cos = torch.randn(SEQ, DHEAD // 2, device=dev)
    sin = torch.randn(SEQ, DHEAD // 2, device=dev)
    q = torch.empty(SEQ_BATCH, HEADS, SEQ, DHEAD, device=dev, dtype=bf)
    k, v = torch.empty_like(q), torch.empty_like(q)
    st = nat.stream_handle(dev)
    bench.time("qkv_rotary_split", lambda: nat.call(
        "pmb_qkv_rotary_split", qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), SEQ_BATCH, SEQ, HEADS, DHEAD,
        q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 2, 1, st), ROWS * n3 * 2 * 2)
    bench.time("qkv_rotary_merge", lambda: nat.call(
        "pmb_qkv_rotary_merge", q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), SEQ_BATCH,
        SEQ, HEADS, DHEAD, qkv.data_ptr(), 1, 2, q.stride(0), q.stride(1), q.stride(2), 1, st), ROWS * n3 * 2 * 2)
    cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
    pq, pk, pv = (torch.empty(ROWS, HEADS * DHEAD, device=dev, dtype=bf) for _ in range(3))
    bench.time("qkv_linear_rotary_forward", lambda: nat.call(
        "pmb_qkv_linear_rotary_forward", x.data_ptr(), w.data_ptr(), cos_t.data_ptr(), sin_t.data_ptr(), SEQ_BATCH,
        SEQ, DIM, HEADS, DHEAD, pq.data_ptr(), pk.data_ptr(), pv.data_ptr(), 1, 2, 1, st),
        (ROWS * DIM + n3 * DIM + ROWS * n3) * 2, flops)
    gw = torch.empty(n3, DIM, device=dev)
    wsb = nat.library().pmb_gemm_tc_wgrad_workspace_size(n3, DIM, ROWS)
    ws = nat.workspace(wsb, dev)
    bench.time("gemm_tc_wgrad (dqkv^T x)", lambda: nat.call(
        "pmb_gemm_tc_wgrad", qkv.data_ptr(), n3, x.data_ptr(), DIM, n3, DIM, ROWS, gw.data_ptr(), DIM, 0, 2,
        ws.data_ptr(), wsb, st), (ROWS * n3 + ROWS * DIM) * 2 + n3 * DIM * 4, flops)
    bench.time("torch wgrad (dqkv^T x)", lambda: torch.matmul(qkv.t(), x),
               (ROWS * n3 + ROWS * DIM) * 2 + n3 * DIM * 2, flops)


def op_ff(bench: _Bench):
    dev, bf = bench.device, torch.bfloat16
    hid = 4 * DIM
    x = torch.randn(ROWS, DIM, device=dev, dtype=bf)
    w1 = torch.randn(hid, DIM, device=dev, dtype=bf) * 0.05
    b1 = torch.randn(hid, device=dev, dtype=bf)
    h = torch.empty(ROWS, hid, device=dev, dtype=bf)
    flops = 2.0 * ROWS * hid * DIM
    byt = (ROWS * DIM + hid * DIM + ROWS * hid) * 2
    bench.time("gemm_tc ff1 (+bias)", lambda: _gemm(x, DIM, 0, w1, DIM, 0, h, ROWS, hid, DIM, bias=b1), byt, flops)
    bench.time("torch ff1 (+bias)", lambda: torch.nn.functional.linear(x, w1, b1), byt, flops)
    w1f, b1f = w1.float(), b1.float()
    w2 = torch.randn(DIM, hid, device=dev, dtype=bf) * 0.05
    w2f, b2f = w2.float(), torch.randn(DIM, device=dev)
    pre, act = torch.empty(ROWS, hid, device=dev, dtype=bf), torch.empty(ROWS, hid, device=dev, dtype=bf)
    out = torch.empty(ROWS, DIM, device=dev, dtype=bf)
    st = nat.stream_handle(dev)
    fwd_bytes = (ROWS * DIM * 2 + ROWS * hid * 2) * 2
    bench.time("feed_forward_forward", lambda: nat.call(
        "pmb_feed_forward_forward", x.data_ptr(), w1.data_ptr(), b1f.data_ptr(), w2.data_ptr(), b2f.data_ptr(), ROWS,
        DIM, hid, pre.data_ptr(), act.data_ptr(), out.data_ptr(), 2, 0, st), fwd_bytes, 2 * flops)
    gy = torch.randn(ROWS, DIM, device=dev, dtype=bf)
    gx = torch.empty_like(x)
    gw1, gb1, gw2, gb2 = torch.empty_like(w1f), torch.empty_like(b1f), torch.empty_like(w2f), torch.empty_like(b2f)
    wsb = nat.library().pmb_feed_forward_backward_workspace_size(ROWS, DIM, hid, 2)
    ws = nat.workspace(wsb, dev)
    gwsb = nat.library().pmb_rows_pass_workspace_size(ROWS, hid)
    gws = nat.workspace(gwsb, dev)
    gpre = torch.empty_like(pre)
    bench.time("gelu_forward", lambda: nat.call("pmb_gelu_forward", pre.data_ptr(), act.data_ptr(), pre.numel(), 2, st),
               2 * ROWS * hid * 2)
    bench.time("gelu_backward (+bias grad)", lambda: nat.call(
        "pmb_gelu_backward", act.data_ptr(), pre.data_ptr(), gpre.data_ptr(), ROWS, hid, gb1.data_ptr(), 0, 2,
        gws.data_ptr(), gwsb, st), 3 * ROWS * hid * 2)
    bench.time("column_sum [rows, dim]", lambda: nat.call(
        "pmb_column_sum", gy.data_ptr(), ROWS, DIM, gb2.data_ptr(), 0, 2, gws.data_ptr(), gwsb, st), ROWS * DIM * 2)
    bwd_bytes = (3 * ROWS * DIM + 4 * ROWS * hid) * 2
    bench.time("feed_forward_backward", lambda: nat.call(
        "pmb_feed_forward_backward", gy.data_ptr(), x.data_ptr(), pre.data_ptr(), act.data_ptr(), w1.data_ptr(),
        w2.data_ptr(), ROWS, DIM, hid, gx.data_ptr(), gw1.data_ptr(), gb1.data_ptr(), gw2.data_ptr(), gb2.data_ptr(),
        2, 0, ws.data_ptr(), wsb, st), bwd_bytes, 4 * flops)
    lin1 = torch.nn.Linear(DIM, hid, device=dev)
    lin2 = torch.nn.Linear(hid, DIM, device=dev)
    xr = x.detach().requires_grad_()

    def torch_ff():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = lin2(torch.nn.functional.gelu(lin1(xr)))
        _grads(y, [xr, *lin1.parameters(), *lin2.parameters()], gy)

    bench.time("torch feed-forward fwd+bwd", torch_ff, fwd_bytes + bwd_bytes, 6 * flops)


def _grads(y, inputs, gy):
    """The backward of y for the given inputs without accumulating into their .grad (no accumulation kernels
    are timed with the op)."""
    return torch.autograd.grad(y, inputs, gy)


def op_sdpa(bench: _Bench):
    """Attention core (library kernels) fwd+bwd per backend, q/k/v as [B, H, N, Dh] views of [B, N, H, Dh]."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    dev, bf = bench.device, torch.bfloat16
    for nb, n in ((SEQ_BATCH, SEQ), (ROWS // 62, 62)):
        qkv = [torch.randn(nb, n, HEADS, DHEAD, device=dev, dtype=bf).transpose(1, 2).requires_grad_()
               for _ in range(3)]
        gy = torch.randn(nb, HEADS, n, DHEAD, device=dev, dtype=bf)
        flops = 4.0 * nb * HEADS * n * n * DHEAD * 3.5
        for backend in (SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION):
            def run():
                with sdpa_kernel(backend):
                    y = torch.nn.functional.scaled_dot_product_attention(*qkv)
                _grads(y, qkv, gy)
            try:
                bench.time(f"sdpa {backend.name} n={n}", run, 0.0, flops)
            except RuntimeError as e:
                print(f"sdpa {backend.name} n={n}: unavailable ({str(e).splitlines()[0][:80]})")


def op_attn(bench: _Bench):
    """Own attention kernels (fwd, fwd+bwd) on the two axial shapes, q/k/v as views of a packed projection."""
    from .fused import AttentionFn

    dev, bf = bench.device, torch.bfloat16
    for nb, n in ((SEQ_BATCH, SEQ), (ROWS // 62, 62)):
        packed = torch.randn(nb, n, 3, HEADS, DHEAD, device=dev, dtype=bf)
        qkv = [packed[:, :, i].transpose(1, 2).requires_grad_() for i in range(3)]
        gy = torch.randn(nb, n, HEADS, DHEAD, device=dev, dtype=bf).transpose(1, 2)
        fl_f = 4.0 * nb * HEADS * n * n * DHEAD
        by = 4 * nb * n * HEADS * DHEAD * 2

        def fwd():
            with torch.no_grad():
                AttentionFn.apply(*qkv)

        def run():
            _grads(AttentionFn.apply(*qkv), qkv, gy)

        bench.time(f"attention fwd n={n}", fwd, by, fl_f)
        bench.time(f"attention fwd+bwd n={n}", run, by * 3, fl_f * 3.5)
    _op_qkv_attention(bench)


def _op_qkv_attention(bench: _Bench):
    """Projection + rotary + attention on the band axis (62 positions), fwd+bwd: QKVAttentionFn (the attention
    backward writes the projection gradient, rotated back) against QKVRotaryFn + AttentionFn (merge pass)."""
    from .fused import AttentionFn, QKVAttentionFn, QKVRotaryFn, rotary_tables

    dev, bf = bench.device, torch.bfloat16
    nb, n = ROWS // 62, 62
    x = torch.randn(nb, n, DIM, device=dev, dtype=bf).requires_grad_()
    w = (torch.randn(3 * HEADS * DHEAD, DIM, device=dev) / DIM ** 0.5).requires_grad_()
    freqs = 1.0 / (10000 ** (torch.arange(0, DHEAD, 2, device=dev).float() / DHEAD))
    cos, sin = rotary_tables(freqs, n, dev)
    cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
    gy = torch.randn(nb, HEADS, n, DHEAD, device=dev, dtype=bf)
    by = ROWS * (DIM + 3 * HEADS * DHEAD) * 2 * 3

    def fused():
        _grads(QKVAttentionFn.apply(x, w, cos, sin, cos_t, sin_t, HEADS), [x, w], gy)

    def split():
        q, k, v = QKVRotaryFn.apply(x, w, cos, sin, cos_t, sin_t, HEADS)
        _grads(AttentionFn.apply(q, k, v), [x, w], gy)

    bench.time(f"qkv+attention fwd+bwd n={n} (QKVAttentionFn)", fused, by)
    bench.time(f"qkv+attention fwd+bwd n={n} (QKVRotaryFn + AttentionFn)", split, by)

    from .fused import AttentionGateFn, QKVAttentionGateFn

    wg = (torch.randn(HEADS, DIM, device=dev) / DIM ** 0.5).requires_grad_()
    bg = torch.zeros(HEADS, device=dev).requires_grad_()
    gg = torch.randn(ROWS, HEADS * DHEAD, device=dev, dtype=bf)
    byg = by + ROWS * HEADS * DHEAD * 2 * 3

    def gated():
        _grads(QKVAttentionGateFn.apply(x, w, cos, sin, cos_t, sin_t, HEADS, wg, bg), [x, w, wg, bg], gg)

    def gate_apart():
        o = QKVAttentionFn.apply(x, w, cos, sin, cos_t, sin_t, HEADS)
        _grads(AttentionGateFn.apply(o, x.reshape(ROWS, DIM), wg, bg, 1), [x, w, wg, bg], gg)

    bench.time(f"qkv+attention+gate fwd+bwd n={n} (QKVAttentionGateFn)", gated, byg)
    bench.time(f"qkv+attention+gate fwd+bwd n={n} (QKVAttentionFn + AttentionGateFn)", gate_apart, byg)


def op_attn_gated(bench: _Bench):
    """The band-axis attention of the training step alone: projection, rotary, attention and head gate forward and
    backward through QKVAttentionGateFn (62 positions); its first backward launch is the gated one-pass kernel."""
    from .fused import QKVAttentionGateFn, rotary_tables

    dev, bf = bench.device, torch.bfloat16
    nb, n = ROWS // 62, 62
    x = torch.randn(nb, n, DIM, device=dev, dtype=bf).requires_grad_()
    w = (torch.randn(3 * HEADS * DHEAD, DIM, device=dev) / DIM ** 0.5).requires_grad_()
    wg = (torch.randn(HEADS, DIM, device=dev) / DIM ** 0.5).requires_grad_()
    bg = torch.zeros(HEADS, device=dev).requires_grad_()
    freqs = 1.0 / (10000 ** (torch.arange(0, DHEAD, 2, device=dev).float() / DHEAD))
    cos, sin = rotary_tables(freqs, n, dev)
    cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
    gg = torch.randn(ROWS, HEADS * DHEAD, device=dev, dtype=bf)
    byg = ROWS * (DIM + 3 * HEADS * DHEAD) * 2 * 3 + ROWS * HEADS * DHEAD * 2 * 3
    bench.time(f"qkv+attention+gate fwd+bwd n={n} (QKVAttentionGateFn)", lambda: _grads(
        QKVAttentionGateFn.apply(x, w, cos, sin, cos_t, sin_t, HEADS, wg, bg), [x, w, wg, bg], gg), byg)


def op_band(bench: _Bench):
    """BandSplit (config-3 bands: 62 bands over 1025 stereo complex bins, 1032 rows, D = 192)."""
    _op_band_rows(bench, 1032)


def _op_band_rows(bench: _Bench, rows: int):
    import ctypes

    from .bands import DEFAULT_FREQS_PER_BANDS

    dev, bf = bench.device, torch.bfloat16
    widths = [4 * f for f in DEFAULT_FREQS_PER_BANDS]
    nb, total, D = len(widths), sum(widths), DIM
    sfx = "" if rows == 1032 else f" [{rows} rows]"
    ld = (total + 7) // 8 * 8  # the band gather's 16-byte rows
    xbuf = torch.randn(rows, ld, device=dev, dtype=bf)
    x = xbuf[:, :total]
    gam = [torch.ones(w, device=dev) for w in widths]
    wts = [torch.randn(D, w, device=dev) / w ** 0.5 for w in widths]
    bss = [torch.zeros(D, device=dev) for _ in widths]
    warr = nat.i64_array(widths)
    sizes = (ctypes.c_int64 * 4)()
    nat.call("pmb_band_split_tc_sizes", rows, nb, warr, D, 2, sizes)
    packed = nat.workspace(sizes[0], dev)
    inv = torch.empty(rows, nb, device=dev)
    out = torch.empty(rows, nb, D, device=dev, dtype=bf)
    st = nat.stream_handle(dev)
    pg, pw, pb = nat.ptr_array(gam), nat.ptr_array(wts), nat.ptr_array(bss)
    flops = 2.0 * rows * total * D
    # algorithmic bytes: x read once, out and inv written once, fp32 W / gamma / bias read once
    byt = rows * total * 2 + rows * nb * (D * 2 + 4) + (total * (D + 1) + nb * D) * 4
    bench.time("band_split_tc_forward" + sfx, lambda: nat.call(
        "pmb_band_split_tc_forward", x.data_ptr(), rows, ld, nb, warr, pg, pw, pb, D, packed.data_ptr(),
        inv.data_ptr(), out.data_ptr(), 2, 0, st), byt, flops)
    xc = x.contiguous()
    normed = torch.empty_like(xc)
    sbyt = rows * total * 2 * 2 + rows * nb * (D * 2 + 4) + (total * (D + 1) + nb * D) * 4
    bench.time("band_split_forward (SIMT)" + sfx, lambda: nat.call(
        "pmb_band_split_forward", xc.data_ptr(), rows, total, -1, 1, nb, warr, pg, pw, pb, D, out.data_ptr(),
        normed.data_ptr(), inv.data_ptr(), 2, 0, st), sbyt, flops)
    gy = torch.randn(rows, nb, D, device=dev, dtype=bf)
    gg = [torch.empty_like(g) for g in gam]
    gw = [torch.empty_like(w) for w in wts]
    gb = [torch.empty_like(b) for b in bss]
    ws = nat.workspace(sizes[1], dev)
    # dY, x and inv read once; W read, grad W / gamma / bias written (fp32)
    bbyt = rows * nb * (D * 2 + 4) + rows * total * 2 + (total * D * 2 + 2 * total + 2 * nb * D) * 4
    bench.time("band_split_tc_backward" + sfx, lambda: nat.call(
        "pmb_band_split_tc_backward", gy.data_ptr(), x.data_ptr(), ld, inv.data_ptr(), rows, nb, warr, pg, pw, D,
        nat.ptr_array(gg), nat.ptr_array(gw), nat.ptr_array(gb), 2, 0, ws.data_ptr(), sizes[1], st), bbyt, flops)
    swsb = nat.library().pmb_band_split_backward_workspace_size(rows, nb, warr, D, 0)
    sws = nat.workspace(swsb, dev)
    bench.time("band_split_backward (SIMT)" + sfx, lambda: nat.call(
        "pmb_band_split_backward", gy.data_ptr(), normed.data_ptr(), inv.data_ptr(), rows, nb, warr, pg, pw, D, None,
        nat.ptr_array(gg), nat.ptr_array(gw), nat.ptr_array(gb), 2, 0, sws.data_ptr(), swsb, st), bbyt, flops)


def op_mel(bench: _Bench):
    """Mel-band gather / scatter-add-average recombine (60 overlapping mel bands, stereo, batch 4 x 258 frames)."""
    _op_mel_shape(bench, 4, 258)


def _op_mel_shape(bench: _Bench, b: int, t: int):
    from . import bands
    from . import extension as ext

    dev = bench.device
    index = bands.mel_band_index(44100, 2048, 60, channels=2)
    tables = index.device_tables(dev)
    f = 1025
    sfx = "" if (b, t) == (4, 258) else f" [{b}x2, {f}, {t}]"
    j = int(tables["index"].numel())
    stft = torch.randn(b, 2, f, t, 2, device=dev)
    x = ext.band_gather(stft, tables, torch.bfloat16)
    bench.time("band_gather_forward" + sfx, lambda: ext.band_gather(stft, tables, torch.bfloat16),
               b * t * j * 2 * (4 + 2) + 4 * j)
    gx = torch.randn_like(x)
    bench.time("band_gather_backward" + sfx, lambda: ext.band_gather_backward(gx, tables, 2, f),
               b * t * j * 2 * 2 + b * 2 * f * t * 2 * 4)
    mask = torch.randn(b, 1, t, j * 2, device=dev, dtype=torch.bfloat16)
    out = ext.band_recombine(mask, stft, tables, 2, f)
    bench.time("band_recombine_forward" + sfx, lambda: ext.band_recombine(mask, stft, tables, 2, f),
               b * t * j * 2 * 2 + 2 * b * 2 * f * t * 8)
    go = torch.randn_like(out)
    bench.time("band_recombine_backward" + sfx,
               lambda: ext.band_recombine_backward(go, stft, tables, torch.bfloat16),
               2 * b * 2 * f * t * 8 + b * t * j * 2 * 2)


def op_mask(bench: _Bench):
    """MaskEstimator on the tensor cores (config 3: 62 bands, dim 192, hidden 768, one hidden layer, 1032 rows)."""
    from .bands import DEFAULT_FREQS_PER_BANDS
    from .fused import MaskEstimatorTCFn

    dev = bench.device
    widths = [2 * 2 * f for f in DEFAULT_FREQS_PER_BANDS]
    nb, rows, hid = len(widths), 1032, 4 * DIM
    params = []
    for w_in, w_out in ((DIM, hid), (hid, None)):
        outs = [hid] * nb if w_out is not None else [2 * w for w in widths]
        params += [torch.randn(o, w_in, device=dev) / w_in ** 0.5 for o in outs]
        params += [torch.zeros(o, device=dev) for o in outs]
    params = [p.requires_grad_() for p in params]
    x = torch.randn(rows, nb, DIM, device=dev, dtype=torch.bfloat16)
    flops = 2.0 * rows * (nb * DIM * hid + hid * 2 * sum(widths))
    byt = rows * (nb * DIM + nb * hid + 3 * sum(widths)) * 2

    def fwd():
        with torch.no_grad():
            MaskEstimatorTCFn.apply(x, widths, 1, hid, *params)

    bench.time("mask_estimator_tc_forward", fwd, byt, flops)
    xr = x.detach().requires_grad_()
    gy = torch.randn(rows, sum(widths), device=dev, dtype=torch.bfloat16)

    def fwd_bwd():
        _grads(MaskEstimatorTCFn.apply(xr, widths, 1, hid, *params), [xr, *params], gy)

    bench.time("mask_estimator_tc fwd+bwd", fwd_bwd, 3 * byt, 3 * flops)


def op_stft(bench: _Bench):
    """Loss and output transforms of config 3: one resolution of the multi-resolution STFT loss (8 signals of
    131584 samples, n_fft 2048, hop 147: spectral L1 forward and backward) and the iSTFT overlap-add of the model
    output (8 signals, n_fft 2048, hop 512, 258 frames)."""
    dev = bench.device
    st = nat.stream_handle(dev)
    nsig, length, n_fft = 8, 131584, 2048
    frames = 1 + length // 147
    count = nsig * frames * (n_fft // 2 + 1)
    yr = torch.randn(count * 2, device=dev)
    yt = torch.randn(count * 2, device=dev)
    gy = torch.empty_like(yr)
    loss = torch.empty((), device=dev)
    one = torch.ones(1, device=dev)
    wsb = int(nat.library().pmb_spectral_l1_workspace_size(count))
    ws = nat.workspace(wsb, dev)
    bench.time("spectral_l1_forward [8, 896, 1025]", lambda: nat.call(
        "pmb_spectral_l1_forward", yr.data_ptr(), yt.data_ptr(), count, loss.data_ptr(), ws.data_ptr(), wsb, st),
        16.0 * count)
    bench.time("spectral_l1_backward [8, 896, 1025]", lambda: nat.call(
        "pmb_spectral_l1_backward", yr.data_ptr(), yt.data_ptr(), count, n_fft // 2 + 1, n_fft, one.data_ptr(),
        gy.data_ptr(), st), 24.0 * count)
    hop, t = 512, 258
    fr = torch.randn(nsig, n_fft, t, device=dev)
    win = torch.hann_window(n_fft, device=dev)
    y = torch.empty(nsig, length, device=dev)
    gfr = torch.empty_like(fr)
    strides = nat.i64_array(list(fr.stride()))
    byt = 4.0 * nsig * (n_fft * t + length)
    bench.time("istft_overlap_add_forward [8, 2048, 258]", lambda: nat.call(
        "pmb_istft_overlap_add_forward", fr.data_ptr(), strides, win.data_ptr(), y.data_ptr(), nsig, n_fft, t, hop,
        length, st), byt)
    bench.time("istft_overlap_add_backward [8, 2048, 258]", lambda: nat.call(
        "pmb_istft_overlap_add_backward", y.data_ptr(), win.data_ptr(), gfr.data_ptr(), nsig, n_fft, t, hop, length,
        st), byt)


def op_band_sweep(bench: _Bench):
    """BandSplit at the config-2 sweep size (8192 rows), for profiling it alone."""
    _op_band_rows(bench, 8 * 1024)


OPS = {"gate": op_gate, "band": op_band, "band8192": op_band_sweep, "mel": op_mel, "mask": op_mask, "rms": op_rms,
       "qkv": op_qkv, "ff": op_ff, "sdpa": op_sdpa, "attn": op_attn, "attn_gated": op_attn_gated, "stft": op_stft}
# ops that only isolate one case of another op (for profiler captures); run when named
NAMED_ONLY = {"attn_gated"}


# ---------------------------------------------------------------------------
# Config-2 sweep: the hot kernels in isolation, up to tensors well beyond the 126 MB
# L2 (which is flushed between timed calls in any case), random normal inputs (seed 0), bf16 and fp32 where the
# kernel takes both.
def sweep_cases() -> list[tuple[str, dict]]:
    """(op, shape) cases of the sweep, in run order; pure host logic (tests check it without a GPU)."""
    cases = []
    for dtype in ("bf16", "fp32"):
        for dim in (192, 384):
            for bf, t in ((62, 1024), (496, 1024)):  # B·F rows of T frames: one and eight batch items of 62 bands
                cases.append(("rms", {"dtype": dtype, "rows": bf * t, "dim": dim}))
    for dtype in ("bf16", "fp32"):
        for n, b in ((62, 2048), (1024, 128)):  # [B, N, 8, 64]: 2048 x 62 and 128 x 1024 positions
            cases.append(("rotary", {"dtype": dtype, "batch": b, "seq": n, "heads": 8, "dim": 64}))
    cases.append(("band", {"rows": 8 * 1024}))  # ragged BandSplit, 62 bands -> 192, M = 8 x 1024 rows
    cases.append(("mel", {"batch": 4, "frames": 1024}))  # [8 = 4 x stereo, 1025, 1024] complex
    return cases


_TORCH_DT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def _sweep_rms(bench: _Bench, dtype: str, rows: int, dim: int):
    dev, dt = bench.device, _TORCH_DT[dtype]
    code, es = nat.dtype_code(dt), torch.tensor([], dtype=dt).element_size()
    x = torch.randn(rows, dim, device=dev, dtype=dt)
    g = torch.ones(dim, device=dev, dtype=dt)
    out, normed = torch.empty_like(x), torch.empty_like(x)
    inv = torch.empty(rows, device=dev)
    st = nat.stream_handle(dev)
    tag = f"{dtype} [{rows}, {dim}]"
    bench.time(f"rms fwd {tag}", lambda: nat.call(
        "pmb_rms_norm_forward", x.data_ptr(), g.data_ptr(), out.data_ptr(), normed.data_ptr(), inv.data_ptr(), rows,
        dim, code, code, code, st), rows * dim * es * 3 + rows * 4)
    dy = torch.randn_like(x)
    gx, gg = torch.empty_like(x), torch.empty_like(g)
    wsb = nat.library().pmb_rms_norm_backward_workspace_size(rows, dim)
    ws = nat.workspace(wsb, dev)
    bench.time(f"rms bwd {tag}", lambda: nat.call(
        "pmb_rms_norm_backward", dy.data_ptr(), x.data_ptr(), 1, inv.data_ptr(), g.data_ptr(), gx.data_ptr(),
        gg.data_ptr(), rows, dim, code, code, code, code, ws.data_ptr(), wsb, st), rows * dim * es * 3 + rows * 4)


def _sweep_rotary(bench: _Bench, dtype: str, batch: int, seq: int, heads: int, dim: int):
    dev, dt = bench.device, _TORCH_DT[dtype]
    code, es = nat.dtype_code(dt), torch.tensor([], dtype=dt).element_size()
    t = torch.randn(batch, seq, heads, dim, device=dev, dtype=dt)
    cos = torch.randn(seq, dim // 2, device=dev, dtype=dt)
    sin = torch.randn(seq, dim // 2, device=dev, dtype=dt)
    out = torch.empty_like(t)
    st = nat.stream_handle(dev)
    byt = 2 * t.numel() * es + 2 * seq * (dim // 2) * es
    tag = f"{dtype} [{batch}, {seq}, {heads}, {dim}]"
    bench.time(f"rotary fwd {tag}", lambda: nat.call(
        "pmb_rotary_forward", t.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(), batch, seq, heads, dim,
        code, st), byt)
    bench.time(f"rotary bwd {tag}", lambda: nat.call(
        "pmb_rotary_backward", out.data_ptr(), cos.data_ptr(), sin.data_ptr(), t.data_ptr(), batch, seq, heads, dim,
        code, st), byt)


def run_sweep(bench: _Bench) -> None:
    torch.manual_seed(0)
    for op, shape in sweep_cases():
        if op == "rms":
            _sweep_rms(bench, **shape)
        elif op == "rotary":
            _sweep_rotary(bench, **shape)
        elif op == "band":
            _op_band_rows(bench, shape["rows"])
        elif op == "mel":
            _op_mel_shape(bench, shape["batch"], shape["frames"])


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("ops", nargs="*", help=f"ops to run (default all): {', '.join(OPS)}")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3, help="untimed calls per op before timing (0 with --iters 1 "
                   "launches each kernel once, for profiler captures)")
    p.add_argument("--json", default=None)
    p.add_argument("--eager", action="store_true",
                   help="time eager calls instead of CUDA-graph replays (host launch time then counts)")
    p.add_argument("--sweep", action="store_true",
                   help="run the config-2 kernel sweep (RMSNorm, rotary, BandSplit, mel at sizes beyond L2) "
                        "instead of the config-3 ops")
    args = p.parse_args(argv)
    device = torch.device("cuda", torch.cuda.current_device())
    bench = _Bench(device, max(args.iters, 1), args.warmup, graphs=not args.eager and args.warmup > 0)
    with torch.cuda.stream(bench.stream):
        if args.sweep:
            run_sweep(bench)
        for name in ([] if args.sweep else args.ops or [k for k in OPS if k not in NAMED_ONLY]):
            if name not in OPS:
                raise SystemExit(f"unknown op {name!r}; choose from {', '.join(OPS)}")
            OPS[name](bench)
    torch.cuda.synchronize(device)
    timeout = nat.library().pmb_umma_timeout(1)
    if timeout:
        raise RuntimeError(f"tcgen05 wait timed out (site {timeout:#x})")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(bench.results, f, indent=1)


if __name__ == "__main__":
    main()
