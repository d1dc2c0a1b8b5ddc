"""Autograd Functions of the fused training path (the product's hot path).

Each Function calls the sm_100a C-ABI library through :mod:`pymsst_b200._native`;
there is no CPU or torch fallback (CPU tensors raise
:class:`~pymsst_b200._native.FusedKernelUnavailable`).  They play the role of
the reference's autograd wrappers (src/pymsst/training/fused_roformer.py:
888-1262) for this package's own model modules.

Precision: activations are in the *compute dtype* (fp32, or the autocast
dtype bf16 / fp16 under ``torch.autocast``); parameters stay fp32 masters and
are read directly by the kernels (no per-step cast copies); parameter
gradients are produced in fp32.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _native as nat
from . import extension as ext


def compute_dtype(t: torch.Tensor) -> torch.dtype:
    if t.device.type == "cuda" and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return t.dtype if t.is_floating_point() else torch.float32


def _rows(x: torch.Tensor) -> int:
    return x.numel() // x.shape[-1] if x.shape[-1] else 0


# ------------------------------------------------------------------ RMSNorm
class RMSNormFn(torch.autograd.Function):
    """y = F.normalize(x) * sqrt(D) * gamma; saves x and the fp32 inverse norms."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, gamma: torch.Tensor):
        device = nat.require_cuda(x, gamma, name="RMSNorm")
        x = x.contiguous()
        dim = x.shape[-1]
        rows = _rows(x)
        out = torch.empty_like(x)
        inv = torch.empty(rows, dtype=torch.float32, device=device)
        nat.call(
            "pmb_rms_norm_forward", x.data_ptr(), gamma.data_ptr(), out.data_ptr(), None, inv.data_ptr(), rows, dim,
            nat.dtype_code(x.dtype), nat.dtype_code(gamma.dtype), nat.dtype_code(x.dtype), nat.stream_handle(device),
        )
        ctx.save_for_backward(x, inv, gamma)
        return out

    @staticmethod
    def backward(ctx, grad):
        x, inv, gamma = ctx.saved_tensors
        gx, gg = ext.rms_norm_backward_into(
            grad.to(x.dtype).contiguous(), x, inv, gamma, saved_is_input=True,
            grad_x_dtype=x.dtype if ctx.needs_input_grad[0] else None, grad_gamma_dtype=gamma.dtype,
            name="RMSNorm.backward",
        )
        return gx, gg


class RMSNormResidualFn(torch.autograd.Function):
    """RMSNormFn for a pre-norm residual block: returns (y, x), the second output being x itself for the block's
    residual branch.  The backward then receives both gradients of x and writes grad_x = RMSNorm'(grad_y) +
    grad_residual in the norm's own pass (pmb_rms_norm_backward_add), instead of the norm's pass followed by
    autograd's elementwise sum of the two gradients."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, gamma: torch.Tensor):
        device = nat.require_cuda(x, gamma, name="RMSNormResidual")
        xc = x.contiguous()
        dim = xc.shape[-1]
        rows = _rows(xc)
        out = torch.empty_like(xc)
        inv = torch.empty(rows, dtype=torch.float32, device=device)
        nat.call(
            "pmb_rms_norm_forward", xc.data_ptr(), gamma.data_ptr(), out.data_ptr(), None, inv.data_ptr(), rows, dim,
            nat.dtype_code(xc.dtype), nat.dtype_code(gamma.dtype), nat.dtype_code(xc.dtype), nat.stream_handle(device),
        )
        ctx.save_for_backward(xc, inv, gamma)
        return out, x

    @staticmethod
    def backward(ctx, grad, grad_res):
        x, inv, gamma = ctx.saved_tensors
        need_x = ctx.needs_input_grad[0]
        if grad is None:  # only the residual branch was used
            return grad_res, None
        gx, gg = ext.rms_norm_backward_into(
            grad.to(x.dtype).contiguous(), x, inv, gamma, saved_is_input=True,
            grad_x_dtype=x.dtype if need_x else None, grad_gamma_dtype=gamma.dtype,
            grad_residual=grad_res.reshape(x.shape) if need_x and grad_res is not None else None,
            name="RMSNormResidual.backward",
        )
        return gx, gg


# ---------------------------------------------------------------- BandSplit
class BandSplitFn(torch.autograd.Function):
    """feats [rows, total] -> [rows, nb, O]; per band RMSNorm + Linear (ragged).

    16-bit activations whose input needs no gradient (the STFT features of
    training) take the tcgen05 path (pmb_band_split_tc_forward / _backward:
    the GEMM reads the features in place -- rows 16-byte aligned, as the band
    gather writes them; anything else is first copied into such rows -- and
    applies the per-(row, band) norm scale in its epilogue; the backward
    reads the features and the saved inverse norms); otherwise the exact SIMT
    kernels (pmb_band_split_forward / _backward)."""

    @staticmethod
    def forward(ctx, x, widths, out_features, *params):
        nb = len(widths)
        gammas, weights, biases = params[:nb], params[nb : 2 * nb], params[2 * nb :]
        device = nat.require_cuda(x, name="BandSplit")
        rows, total = x.shape
        inv = torch.empty(rows, nb, dtype=torch.float32, device=device)
        pdt = weights[0].dtype
        ctx.widths = widths
        ctx.out_features = out_features
        ctx.tc = (x.dtype in (torch.bfloat16, torch.float16) and not ctx.needs_input_grad[0]
                  and out_features % 64 == 0)
        if ctx.tc:
            warr = nat.i64_array(widths)
            sizes = (ctypes.c_int64 * 4)()
            nat.call("pmb_band_split_tc_sizes", rows, nb, warr, out_features, nat.dtype_code(x.dtype), sizes)
            align = int(sizes[2])
            if not (x.stride(-1) == 1 and x.stride(0) % align == 0 and x.stride(0) >= total
                    and x.data_ptr() % 16 == 0):
                ld = (total + align - 1) // align * align
                buf = torch.empty(rows, ld, dtype=x.dtype, device=device)
                buf[:, :total].copy_(x)
                x = buf[:, :total]
            out = torch.empty(rows, nb, out_features, dtype=x.dtype, device=device)
            packed = nat.workspace(sizes[0], device)
            nat.call(
                "pmb_band_split_tc_forward", x.data_ptr(), rows, x.stride(0), nb, warr, nat.ptr_array(gammas),
                nat.ptr_array(weights), nat.ptr_array(biases), out_features, packed.data_ptr(), inv.data_ptr(),
                out.data_ptr(), nat.dtype_code(x.dtype), nat.dtype_code(pdt), nat.stream_handle(device),
            )
            ctx.ws_bytes = int(sizes[1])
            ctx.save_for_backward(x, inv, *gammas, *weights)
            return out
        x = x.contiguous()
        out = torch.empty(rows, nb, out_features, dtype=x.dtype, device=device)
        normed = torch.empty_like(x)
        ext.band_split_forward_into(x, rows, (total, -1, 1), widths, gammas, weights, biases, out_features, out,
                                    normed, inv, param_dtype=pdt)
        ctx.save_for_backward(normed, inv, *gammas, *weights)
        return out

    @staticmethod
    def backward(ctx, grad):
        nb = len(ctx.widths)
        if ctx.tc:
            x, inv, *rest = ctx.saved_tensors
            gammas, weights = rest[:nb], rest[nb:]
            device = x.device
            grad = grad.to(x.dtype).contiguous()
            rows = grad.shape[0]
            g_gammas = [torch.empty_like(g) for g in gammas]
            g_weights = [torch.empty_like(w) for w in weights]
            g_biases = [torch.empty(ctx.out_features, dtype=weights[0].dtype, device=device) for _ in weights]
            ws = nat.workspace(ctx.ws_bytes, device)
            nat.call(
                "pmb_band_split_tc_backward", grad.data_ptr(), x.data_ptr(), x.stride(0), inv.data_ptr(), rows, nb,
                nat.i64_array(ctx.widths), nat.ptr_array(gammas), nat.ptr_array(weights), ctx.out_features,
                nat.ptr_array(g_gammas), nat.ptr_array(g_weights), nat.ptr_array(g_biases),
                nat.dtype_code(grad.dtype), nat.dtype_code(weights[0].dtype), ws.data_ptr(), ctx.ws_bytes,
                nat.stream_handle(device),
            )
            return (None, None, None, *g_gammas, *g_weights, *g_biases)
        normed, inv, *rest = ctx.saved_tensors
        gammas, weights = rest[:nb], rest[nb:]
        grad = grad.to(normed.dtype).contiguous()
        grad_x = torch.empty_like(normed) if ctx.needs_input_grad[0] else None
        g_gammas = [torch.empty_like(g) for g in gammas]
        g_weights = [torch.empty_like(w) for w in weights]
        g_biases = [torch.empty(ctx.out_features, dtype=weights[0].dtype, device=grad.device) for _ in weights]
        ext.band_split_backward_into(grad, normed, inv, ctx.widths, gammas, weights, ctx.out_features, grad_x,
                                     g_gammas, g_weights, g_biases, param_dtype=weights[0].dtype)
        return (grad_x, None, None, *g_gammas, *g_weights, *g_biases)


# ----------------------------------------------------------- MaskEstimator
class MaskEstimatorFn(torch.autograd.Function):
    """x [rows, nb, D] -> mask [rows, total]: per band (Linear+Tanh)^L, Linear, GLU.

    params: for each hidden layer, nb weights then nb biases; then the nb
    final weights and nb final biases.
    """

    @staticmethod
    def forward(ctx, x, widths, hidden_layers, *params):
        nb = len(widths)
        nat.require_cuda(x, name="MaskEstimator")
        x = x.contiguous()
        rows = x.shape[0]
        pdtype = params[0].dtype
        acts = [x]
        h = x
        for layer in range(hidden_layers):
            ws = params[2 * nb * layer : 2 * nb * layer + nb]
            bs = params[2 * nb * layer + nb : 2 * nb * (layer + 1)]
            h = ext.grouped_linear_forward_lists(h, ws, bs, ws[0].shape[0], pdtype, activation=1)
            acts.append(h)
        fw = params[2 * nb * hidden_layers : 2 * nb * hidden_layers + nb]
        fb = params[2 * nb * hidden_layers + nb :]
        total = sum(widths)
        out = torch.empty(rows, total, dtype=x.dtype, device=x.device)
        pre = torch.empty(rows, 2 * total, dtype=x.dtype, device=x.device)
        ext.mask_estimator_final_forward_into(h, fw, fb, widths, out, pre, pdtype)
        ctx.widths = widths
        ctx.hidden_layers = hidden_layers
        ctx.save_for_backward(pre, *acts, *params)
        return out

    @staticmethod
    def backward(ctx, grad):
        nb = len(ctx.widths)
        L = ctx.hidden_layers
        pre, *rest = ctx.saved_tensors
        acts, params = rest[: L + 1], rest[L + 1 :]
        pdtype = params[0].dtype
        grad = grad.to(pre.dtype).contiguous()
        fw = params[2 * nb * L : 2 * nb * L + nb]
        h = acts[-1]
        grad_h = torch.empty_like(h)
        g_fw = [torch.empty_like(w) for w in fw]
        g_fb = [torch.empty(w.shape[0], dtype=pdtype, device=grad.device) for w in fw]
        ext.mask_estimator_final_backward_into(grad, h, pre, fw, ctx.widths, grad_h, g_fb, g_fw, pdtype)
        layer_grads = []
        for layer in reversed(range(L)):
            ws = params[2 * nb * layer : 2 * nb * layer + nb]
            x_in, y = acts[layer], acts[layer + 1]
            need_x = layer > 0 or ctx.needs_input_grad[0]
            gx = torch.empty_like(x_in) if need_x else None
            g_w = [torch.empty_like(w) for w in ws]
            g_b = [torch.empty(w.shape[0], dtype=pdtype, device=grad.device) for w in ws]
            ext.grouped_linear_backward_lists(grad_h, x_in, y, ws, ws[0].shape[0], pdtype, gx, g_w, g_b, activation=1)
            layer_grads.append((g_w, g_b))
            grad_h = gx
        flat = []
        for g_w, g_b in reversed(layer_grads):
            flat.extend(g_w)
            flat.extend(g_b)
        flat.extend(g_fw)
        flat.extend(g_fb)
        return (grad_h if ctx.needs_input_grad[0] else None, None, None, *flat)


class MaskEstimatorTCFn(torch.autograd.Function):
    """Tensor-core (tcgen05) MaskEstimator for 16-bit activations; same contract as MaskEstimatorFn."""

    @staticmethod
    def forward(ctx, x, widths, hidden_layers, hidden, *params):
        import ctypes

        nb = len(widths)
        device = nat.require_cuda(x, name="MaskEstimatorTC")
        x = x.contiguous()
        rows, _, dim = x.shape
        warr = nat.i64_array(widths)
        sizes = (ctypes.c_int64 * 5)()
        nat.call("pmb_mask_estimator_tc_sizes", rows, nb, dim, hidden, hidden_layers, warr, sizes)
        packed = torch.empty(max(sizes[0], 1), dtype=torch.uint8, device=device)
        acts = torch.empty(max(sizes[1], 1), dtype=torch.uint8, device=device)
        pre = torch.empty(max(sizes[2], 1), dtype=torch.uint8, device=device)
        total = sum(widths)
        out = torch.empty(rows, total, dtype=x.dtype, device=device)
        layers = hidden_layers + 1
        weights = [params[2 * nb * l + b] for l in range(layers) for b in range(nb)]
        biases = [params[2 * nb * l + nb + b] for l in range(layers) for b in range(nb)]
        nat.call(
            "pmb_mask_estimator_tc_forward", x.data_ptr(), rows, nb, dim, hidden, hidden_layers, warr,
            nat.ptr_array(weights), nat.ptr_array(biases), packed.data_ptr(), acts.data_ptr(), pre.data_ptr(),
            out.data_ptr(), nat.dtype_code(x.dtype), nat.dtype_code(params[0].dtype), nat.stream_handle(device),
        )
        ctx.meta = (widths, hidden_layers, hidden, int(sizes[3]))
        ctx.save_for_backward(x, packed, acts, pre, *params)
        return out

    @staticmethod
    def backward(ctx, grad):
        widths, hidden_layers, hidden, ws_bytes = ctx.meta
        x, packed, acts, pre, *params = ctx.saved_tensors
        nb = len(widths)
        rows, _, dim = x.shape
        device = x.device
        grad = grad.to(x.dtype).contiguous()
        grads = [torch.empty_like(p) for p in params]
        layers = hidden_layers + 1
        gw = [grads[2 * nb * l + b] for l in range(layers) for b in range(nb)]
        gb = [grads[2 * nb * l + nb + b] for l in range(layers) for b in range(nb)]
        grad_x = torch.empty_like(x) if ctx.needs_input_grad[0] else None
        ws = nat.workspace(ws_bytes, device)
        nat.call(
            "pmb_mask_estimator_tc_backward", grad.data_ptr(), x.data_ptr(), acts.data_ptr(), pre.data_ptr(),
            packed.data_ptr(), rows, nb, dim, hidden, hidden_layers, nat.i64_array(widths), nat.ptr_array(gw),
            nat.ptr_array(gb), nat.ptr(grad_x), nat.dtype_code(x.dtype), nat.dtype_code(params[0].dtype),
            ws.data_ptr(), ws_bytes, nat.stream_handle(device),
        )
        return (grad_x, None, None, None, *grads)


def tensor_core_ok(x: torch.Tensor, *dims: int) -> bool:
    """16-bit activations and 64-aligned feature widths take the tcgen05 path."""
    return x.dtype in (torch.bfloat16, torch.float16) and all(d % 64 == 0 for d in dims)


# ------------------------------------------------------- attention pieces
def lowp_weight(p: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Parameter ``p`` in the activation type ``dtype``: inside the trainer's own forward / backward, its
    low-precision mirror of the parameters (the same values p.to(dtype) gives, made for all parameters by one
    copy kernel at the start of that step instead of one cast kernel per weight); anywhere else p.to(dtype).
    The trainer opens that scope only right after refreshing the mirror, so a mirror older than the
    parameters is never handed out (a captured optimizer update does not move version counters, so those
    cannot tell)."""
    half = getattr(p, "_pmb_half", None)
    live = getattr(p, "_pmb_half_live", None)
    if half is not None and live is not None and live[0] and half.dtype == dtype:
        return half
    return p.to(dtype)


class OutProjFn(torch.autograd.Function):
    """residual + gated W^T in one GEMM (torch.addmm with the residual as C), W in the activation type; the
    gradients are those autograd gives through W.to(dtype), with the same products: grad_gated = g W,
    grad_W = (gated^T g)^T cast to W's type, grad_residual = g."""

    @staticmethod
    def forward(ctx, res, gated, w):
        wl = lowp_weight(w, gated.dtype)
        ctx.w_dtype = w.dtype
        ctx.save_for_backward(gated, wl)
        return torch.addmm(res, gated, wl.t())

    @staticmethod
    def backward(ctx, g):
        gated, wl = ctx.saved_tensors
        g_gated = g.mm(wl) if ctx.needs_input_grad[1] else None
        # the product autograd forms for addmm's second operand (gated^T g), transposed back: same rounding
        g_w = gated.t().mm(g).t().to(ctx.w_dtype) if ctx.needs_input_grad[2] else None
        return g, g_gated, g_w


def _weight_grad(a: torch.Tensor, b: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """a @ b as the gradient of a parameter of type ``dtype``: for fp32 parameters and 16-bit operands one GEMM
    with an fp32 result (cuBLAS accumulates in fp32 either way), instead of a 16-bit product and a cast kernel."""
    if dtype == torch.float32 and a.dtype in (torch.bfloat16, torch.float16) and a.is_cuda:
        return torch.mm(a, b, out_dtype=torch.float32)
    return torch.matmul(a, b).to(dtype)


def _input_grad(gqkv, w, gx_pass, shape):
    """gqkv W, plus the gradient that reached the input through its pass-through output (the head gate's input
    gradient) as the GEMM's C operand: one GEMM instead of a GEMM and an elementwise sum."""
    if gx_pass is None:
        return torch.matmul(gqkv, w).reshape(shape)
    c = gx_pass.reshape(gqkv.shape[0], w.shape[1]).to(gqkv.dtype)
    return torch.addmm(c, gqkv, w).reshape(shape)


class QKVRotaryFn(torch.autograd.Function):
    """xn [b, n, D] -> q, k, v [b, h, n, dh]: projection, split, rotary on q/k.

    ``inner`` > 1: the b*n rows of xn are ordered (outer, position, inner)
    rather than (sequence, position) -- sequence = outer * inner + inner
    index -- so an axial transformer passes its activations without a
    permuted copy; q, k, v are always in sequence order.

    16-bit activations with D % 8 == 0 and dh % 32 == 0: one tensor-core GEMM
    with the rotation in its epilogue writes q, k, v as [b, n, h, dh] planes
    (pmb_qkv_linear_rotary_forward); the returned [b, h, n, dh] tensors are
    views of them, which the attention kernel reads in place.  cos_t / sin_t
    are the transposed angle tables ([dh/2, n]) that epilogue reads.
    Otherwise (fp32, other shapes): a torch projection plus the split kernel.
    The backward merges the three gradients, in whatever layout the attention
    backward produced them, with the inverse rotation (pmb_qkv_rotary_merge)
    and runs the two projection-gradient GEMMs.  With ``pass_x`` xn is also
    returned, for another consumer of the same input (the head gate): the
    gradient coming back through it is the C operand of the input-gradient
    GEMM, so the two gradients of xn are not summed by a separate pass."""

    @staticmethod
    def forward(ctx, xn, weight, cos, sin, cos_t, sin_t, heads, inner=1, pass_x=False):
        device = nat.require_cuda(xn, weight, name="QKVRotary")
        b, n, d = xn.shape
        dh = weight.shape[0] // (3 * heads)
        w = lowp_weight(weight, xn.dtype).contiguous()
        x2 = xn.reshape(b * n, d).contiguous()
        rotate = int(cos is not None)
        if rotate and (tuple(cos.shape) != (n, dh // 2) or tuple(sin.shape) != (n, dh // 2)):
            raise ValueError(f"QKVRotary: angle tables must be [{n}, {dh // 2}] (rotation of the whole head), "
                             f"got {tuple(cos.shape)} and {tuple(sin.shape)}")
        if xn.dtype in (torch.bfloat16, torch.float16) and d % 8 == 0 and dh % 32 == 0:
            if rotate and cos_t is None:
                cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
            planes = [torch.empty(b, n, heads, dh, dtype=xn.dtype, device=device) for _ in range(3)]
            nat.call(
                "pmb_qkv_linear_rotary_forward", x2.data_ptr(), w.data_ptr(), nat.ptr(cos_t), nat.ptr(sin_t), b, n,
                d, heads, dh, planes[0].data_ptr(), planes[1].data_ptr(), planes[2].data_ptr(), rotate,
                nat.dtype_code(xn.dtype), inner, nat.stream_handle(device),
            )
            q, k, v = (p.transpose(1, 2) for p in planes)
        else:
            qkv = torch.matmul(x2, w.t())
            q = torch.empty(b, heads, n, dh, dtype=xn.dtype, device=device)
            k = torch.empty_like(q)
            v = torch.empty_like(q)
            nat.call(
                "pmb_qkv_rotary_split", qkv.data_ptr(), nat.ptr(cos), nat.ptr(sin), b, n, heads, dh, q.data_ptr(),
                k.data_ptr(), v.data_ptr(), rotate, nat.dtype_code(xn.dtype), inner, nat.stream_handle(device),
            )
        ctx.heads = heads
        ctx.inner = inner
        ctx.weight_dtype = weight.dtype
        ctx.save_for_backward(x2, w, cos, sin)
        return (q, k, v, xn) if pass_x else (q, k, v)

    @staticmethod
    def backward(ctx, gq, gk, gv, gx_pass=None):
        x2, w, cos, sin = ctx.saved_tensors
        heads = ctx.heads
        device = x2.device
        ref = next(g for g in (gq, gk, gv) if g is not None)
        b, _, n, dh = ref.shape
        grads = [torch.zeros_like(ref) if g is None else g.to(x2.dtype) for g in (gq, gk, gv)]
        strides = grads[0].stride()
        if strides[-1] != 1 or any(g.stride() != strides for g in grads[1:]):
            grads = [g.contiguous() for g in grads]
            strides = grads[0].stride()
        gqkv = torch.empty(b * n, 3 * heads * dh, dtype=x2.dtype, device=device)
        nat.call(
            "pmb_qkv_rotary_merge", grads[0].data_ptr(), grads[1].data_ptr(), grads[2].data_ptr(), nat.ptr(cos),
            nat.ptr(sin), b, n, heads, dh, gqkv.data_ptr(), int(cos is not None), nat.dtype_code(x2.dtype),
            strides[0], strides[1], strides[2], ctx.inner, nat.stream_handle(device),
        )
        gx = _input_grad(gqkv, w, gx_pass, (b, n, -1)) if ctx.needs_input_grad[0] else None
        gw = _weight_grad(gqkv.t(), x2, ctx.weight_dtype) if ctx.needs_input_grad[1] else None
        return gx, gw, None, None, None, None, None, None, None


class FeedForwardFn(torch.autograd.Function):
    """xn [rows, D] -> gelu(xn W1^T + b1) W2^T + b2 (16-bit activations).

    The two Linear layers and their weight / input gradients are plain
    library GEMMs (cuBLAS through torch, bias in the GEMM epilogue, operands
    cast to the activation dtype as autocast does); GELU, its derivative and
    both bias gradients are this package's kernels: the GELU derivative and
    the first bias gradient come out of one pass over the hidden activations
    (pmb_gelu_backward), the second bias gradient from pmb_column_sum.  (The
    fused block pmb_feed_forward_forward -- bias and GELU in the tcgen05 GEMM
    epilogue -- measured 118.7 us per call at config-3 shapes against 112 us
    for cuBLAS + the GELU pass, so the step keeps the latter.)"""

    @staticmethod
    def forward(ctx, xn, w1, b1, w2, b2):
        device = nat.require_cuda(xn, w1, b1, w2, b2, name="FeedForward")
        dt = xn.dtype
        xn = xn.contiguous()
        w1c, w2c = lowp_weight(w1, dt), lowp_weight(w2, dt)
        pre = F.linear(xn, w1c, lowp_weight(b1, dt))
        act = torch.empty_like(pre)
        nat.call("pmb_gelu_forward", pre.data_ptr(), act.data_ptr(), pre.numel(), nat.dtype_code(dt),
                 nat.stream_handle(device))
        out = F.linear(act, w2c, lowp_weight(b2, dt))
        ctx.param_dtypes = (w1.dtype, b1.dtype, w2.dtype, b2.dtype)
        ctx.save_for_backward(xn, pre, act, w1c, w2c)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        xn, pre, act, w1c, w2c = ctx.saved_tensors
        rows, dim = xn.shape
        hidden = pre.shape[1]
        device = xn.device
        dt = xn.dtype
        st = nat.stream_handle(device)
        g = grad_out.to(dt).contiguous()
        dts = ctx.param_dtypes
        gb2 = torch.empty(dim, dtype=dts[3], device=device)
        wsb = nat.library().pmb_rows_pass_workspace_size(rows, max(dim, hidden))
        ws = nat.workspace(wsb, device)
        nat.call("pmb_column_sum", g.data_ptr(), rows, dim, gb2.data_ptr(), nat.dtype_code(dts[3]),
                 nat.dtype_code(dt), ws.data_ptr(), wsb, st)
        gw2 = _weight_grad(g.t(), act, dts[2])
        da = torch.matmul(g, w2c)
        dpre = torch.empty_like(pre)
        gb1 = torch.empty(hidden, dtype=dts[1], device=device)
        nat.call("pmb_gelu_backward", da.data_ptr(), pre.data_ptr(), dpre.data_ptr(), rows, hidden, gb1.data_ptr(),
                 nat.dtype_code(dts[1]), nat.dtype_code(dt), ws.data_ptr(), wsb, st)
        gw1 = _weight_grad(dpre.t(), xn, dts[0])
        gx = torch.matmul(dpre, w1c) if ctx.needs_input_grad[0] else None
        return gx, gw1, gb1, gw2, gb2


class AttentionGateFn(torch.autograd.Function):
    """attn [b, h, n, dh] (any strides, dh contiguous), xn [b*n, D] -> gated [b*n, h*dh]; the rows of xn and of
    the result follow the ``inner`` row order of QKVRotaryFn."""

    @staticmethod
    def forward(ctx, attn, xn, weight, bias, inner=1):
        device = nat.require_cuda(attn, xn, weight, bias, name="AttentionGate")
        if attn.stride(-1) != 1:
            attn = attn.contiguous()
        b, h, n, dh = attn.shape
        ctx.x_dtype = xn.dtype
        xn = xn.to(attn.dtype).contiguous()  # the kernel reads attn and xn in one activation type
        rows, dim = xn.shape
        out = torch.empty(rows, h * dh, dtype=attn.dtype, device=device)
        gate = torch.empty(rows, h, dtype=attn.dtype, device=device)
        nat.call(
            "pmb_attention_gate_forward", attn.data_ptr(), n, attn.stride(0), attn.stride(2), attn.stride(1),
            xn.data_ptr(), weight.data_ptr(), bias.data_ptr(), rows, h, dh, dim, out.data_ptr(), gate.data_ptr(),
            nat.dtype_code(attn.dtype), nat.dtype_code(weight.dtype), inner, nat.stream_handle(device),
        )
        ctx.inner = inner
        ctx.save_for_backward(attn, xn, weight, gate)
        return out

    @staticmethod
    def backward(ctx, grad):
        attn, xn, weight, gate = ctx.saved_tensors
        device = attn.device
        b, h, n, dh = attn.shape
        rows, dim = xn.shape
        grad = grad.to(attn.dtype).contiguous()
        grad_attn = torch.empty_strided(attn.shape, attn.stride(), dtype=attn.dtype, device=device)
        grad_x = torch.empty_like(xn)
        gw = torch.empty_like(weight)
        gb = torch.empty(h, dtype=weight.dtype, device=device)
        lib = nat.library()
        ws_bytes = int(lib.pmb_attention_gate_backward_workspace_size(rows, h, dim))
        ws = nat.workspace(ws_bytes, device)
        nat.call(
            "pmb_attention_gate_backward", grad.data_ptr(), attn.data_ptr(), n, attn.stride(0), attn.stride(2),
            attn.stride(1), xn.data_ptr(), weight.data_ptr(), gate.data_ptr(), rows, h, dh, dim,
            grad_attn.data_ptr(), grad_x.data_ptr(), gw.data_ptr(), gb.data_ptr(), nat.dtype_code(attn.dtype),
            nat.dtype_code(weight.dtype), ws.data_ptr(), ws_bytes, ctx.inner, nat.stream_handle(device),
        )
        return grad_attn, grad_x.to(ctx.x_dtype), gw, gb, None


def _attn_plane(t: torch.Tensor) -> torch.Tensor:
    """[b, h, n, dh] view whose strides the attention kernels accept: head dim contiguous, 16-byte rows, and the
    non-overlapping order of a [b, n, h, dh] plane (head >= dh, position >= h heads, sequence >= n positions;
    size-1 dimensions are free); anything else is copied into such a plane."""
    b, h, n, dh = t.shape
    sb, sh, sn, sd = t.stride()
    sh = dh if h == 1 else sh
    sn = h * sh if n == 1 else sn
    sb = n * sn if b == 1 else sb
    ok = (sd == 1 and t.data_ptr() % 16 == 0 and not any(s % 8 for s in t.stride()[:3])
          and sh >= dh and sn >= h * sh and sb >= n * sn)
    if not ok:
        t = t.transpose(1, 2).contiguous().transpose(1, 2)
    return t


def _attn_strides(*planes: torch.Tensor) -> list[int]:
    """(sequence, position, head) element strides of [b, h, n, dh] views, plane by plane."""
    out: list[int] = []
    for t in planes:
        out += [t.stride(0), t.stride(2), t.stride(1)]
    return out


def _bnhd_empty(b, h, n, dh, dtype, device) -> torch.Tensor:
    return torch.empty(b, n, h, dh, dtype=dtype, device=device).transpose(1, 2)


def attention_supported(q: torch.Tensor, dropout_p: float = 0.0) -> bool:
    """Shapes and types the attention kernels take: CUDA, bf16/fp16, head dim 64, no dropout."""
    return (q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and q.dim() == 4 and q.shape[-1] == 64
            and dropout_p == 0.0)


class AttentionFn(torch.autograd.Function):
    """softmax(q k^T / sqrt(dh)) v for q, k, v [b, h, n, 64] (any strides with the head dim contiguous, such as
    views of [b, n, h, 64] planes) -> o [b, h, n, 64], a view of a [b, n, h, 64] plane.  Drop-in for
    F.scaled_dot_product_attention(q, k, v) without mask or dropout; deterministic backward."""

    @staticmethod
    def forward(ctx, q, k, v):
        device = nat.require_cuda(q, k, v, name="Attention")
        q, k, v = _attn_plane(q), _attn_plane(k), _attn_plane(v)
        b, h, n, dh = q.shape
        o = _bnhd_empty(b, h, n, dh, q.dtype, device)
        lse = torch.empty(b * h, (n + 3) // 4 * 4, dtype=torch.float32, device=device)  # rows padded to 16 bytes
        nat.call(
            "pmb_attention_forward", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, n, h,
            dh, nat.i64_array(_attn_strides(q, k, v, o)), dh ** -0.5, nat.dtype_code(q.dtype),
            nat.stream_handle(device),
        )
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, grad):
        q, k, v, o, lse = ctx.saved_tensors
        device = q.device
        b, h, n, dh = q.shape
        grad = _attn_plane(grad.to(q.dtype))
        dq, dk, dv = (_bnhd_empty(b, h, n, dh, q.dtype, device) for _ in range(3))
        ws_bytes = int(nat.library().pmb_attention_backward_workspace_size(b, n, h))
        ws = nat.workspace(ws_bytes, device)
        nat.call(
            "pmb_attention_backward", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), grad.data_ptr(),
            lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), b, n, h, dh,
            nat.i64_array(_attn_strides(q, k, v, o, grad, dq, dk, dv)), dh ** -0.5, nat.dtype_code(q.dtype),
            ws.data_ptr(), ws_bytes, nat.stream_handle(device),
        )
        return dq, dk, dv


class QKVAttentionFn(torch.autograd.Function):
    """Attention input projection with rotary (QKVRotaryFn's tensor-core path) followed by the own attention
    kernels (AttentionFn): xn [b, n, D] (rows in sequence order, as on an axial transformer's band axis) ->
    o [b, h, n, 64], a view of a [b, n, h, 64] plane.  The forward is those two ops.  The backward writes dQ and
    dK rotated back to the projection's space, and dV, straight into the [b * n, 3 * h * 64] projection gradient
    (pmb_attention_backward_rotary given strided views of it), so QKVRotaryFn.backward's merge pass and its
    round trip of that gradient go; the two projection-gradient GEMMs follow as there (``pass_x`` as there).
    Reference semantics:
    qkv_to_bnhd + rotary + scaled-dot-product attention of the patched Attention.forward
    (src/pymsst/training/fused_roformer.py:793-818)."""

    @staticmethod
    def forward(ctx, xn, weight, cos, sin, cos_t, sin_t, heads, pass_x=False):
        device = nat.require_cuda(xn, weight, name="QKVAttention")
        b, n, d = xn.shape
        dh = weight.shape[0] // (3 * heads)
        if not (xn.dtype in (torch.bfloat16, torch.float16) and d % 8 == 0 and dh == 64):
            raise ValueError("QKVAttention: 16-bit activations, D % 8 == 0 and 64-element heads only")
        w = lowp_weight(weight, xn.dtype).contiguous()
        x2 = xn.reshape(b * n, d).contiguous()
        rotate = int(cos is not None)
        if rotate:
            if tuple(cos.shape) != (n, dh // 2) or tuple(sin.shape) != (n, dh // 2):
                raise ValueError(f"QKVAttention: angle tables must be [{n}, {dh // 2}], got {tuple(cos.shape)} "
                                 f"and {tuple(sin.shape)}")
            cos, sin = cos.float().contiguous(), sin.float().contiguous()
            if cos_t is None:
                cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
        planes = [torch.empty(b, n, heads, dh, dtype=xn.dtype, device=device) for _ in range(3)]
        stream = nat.stream_handle(device)
        nat.call(
            "pmb_qkv_linear_rotary_forward", x2.data_ptr(), w.data_ptr(), nat.ptr(cos_t), nat.ptr(sin_t), b, n, d,
            heads, dh, planes[0].data_ptr(), planes[1].data_ptr(), planes[2].data_ptr(), rotate,
            nat.dtype_code(xn.dtype), 1, stream,
        )
        q, k, v = (pl.transpose(1, 2) for pl in planes)
        o = _bnhd_empty(b, heads, n, dh, xn.dtype, device)
        lse = torch.empty(b * heads, (n + 3) // 4 * 4, dtype=torch.float32, device=device)
        nat.call(
            "pmb_attention_forward", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), b, n,
            heads, dh, nat.i64_array(_attn_strides(q, k, v, o)), dh ** -0.5, nat.dtype_code(xn.dtype), stream,
        )
        ctx.weight_dtype = weight.dtype
        ctx.save_for_backward(x2, w, cos, sin, q, k, v, o, lse)
        return (o, xn) if pass_x else o

    @staticmethod
    def backward(ctx, grad, gx_pass=None):
        x2, w, cos, sin, q, k, v, o, lse = ctx.saved_tensors
        device = q.device
        b, h, n, dh = q.shape
        grad = _attn_plane(grad.to(q.dtype))
        gqkv = torch.empty(b * n, 3 * h * dh, dtype=q.dtype, device=device)
        parts = gqkv.view(b, n, 3, h, dh)
        dq, dk, dv = (parts[:, :, i].transpose(1, 2) for i in range(3))
        ws_bytes = int(nat.library().pmb_attention_backward_workspace_size(b, n, h))
        ws = nat.workspace(ws_bytes, device)
        strides = nat.i64_array(_attn_strides(q, k, v, o, grad, dq, dk, dv))
        head = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), grad.data_ptr(), lse.data_ptr())
        tail = (b, n, h, dh, strides, dh ** -0.5, nat.dtype_code(q.dtype), ws.data_ptr(), ws_bytes,
                nat.stream_handle(device))
        if cos is not None:
            nat.call("pmb_attention_backward_rotary", *head, cos.data_ptr(), sin.data_ptr(), dq.data_ptr(),
                     dk.data_ptr(), dv.data_ptr(), *tail)
        else:
            nat.call("pmb_attention_backward", *head, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), *tail)
        gx = _input_grad(gqkv, w, gx_pass, (b, n, -1)) if ctx.needs_input_grad[0] else None
        gw = _weight_grad(gqkv.t(), x2, ctx.weight_dtype) if ctx.needs_input_grad[1] else None
        return gx, gw, None, None, None, None, None, None


class QKVAttentionGateFn(torch.autograd.Function):
    """QKVAttentionFn with the head gate folded into the attention kernels, for sequences of up to 64 positions
    in row order (the band axis): xn [b, n, D] -> gated [b * n, h * 64] = attention * sigmoid(xn W_g^T + b_g)
    per head, the AttentionGateFn output.

    Forward: the gate logits come from one small GEMM in the activation type (as autocast computes the gate
    Linear), and the attention kernel writes the gated output in place of o (pmb_attention_forward_gated).
    Backward: pmb_attention_backward_gated writes dQ / dK rotated back, dV and the logits' gradient
    rowsum(dGated * gated) (1 - gate) into one [b * n, 3 h 64 + h] buffer E, so the input gradient
    E [W_qkv; W_g] and the weight gradients E^T xn are one GEMM each and the gate has no pass of its own.
    Reference semantics: the patched Attention.forward, src/pymsst/training/fused_roformer.py:793-818."""

    @staticmethod
    def forward(ctx, xn, weight, cos, sin, cos_t, sin_t, heads, w_gate, b_gate):
        device = nat.require_cuda(xn, weight, w_gate, b_gate, name="QKVAttentionGate")
        b, n, d = xn.shape
        dh = weight.shape[0] // (3 * heads)
        if not (xn.dtype in (torch.bfloat16, torch.float16) and d % 8 == 0 and dh == 64 and n <= 64):
            raise ValueError("QKVAttentionGate: 16-bit activations, D % 8 == 0, 64-element heads and at most 64 "
                             "positions only")
        dt = xn.dtype
        w = lowp_weight(weight, dt).contiguous()
        wg = lowp_weight(w_gate, dt).contiguous()
        bg = lowp_weight(b_gate, dt)
        x2 = xn.reshape(b * n, d).contiguous()
        rotate = int(cos is not None)
        if rotate:
            if tuple(cos.shape) != (n, dh // 2) or tuple(sin.shape) != (n, dh // 2):
                raise ValueError(f"QKVAttentionGate: angle tables must be [{n}, {dh // 2}], got {tuple(cos.shape)} "
                                 f"and {tuple(sin.shape)}")
            cos, sin = cos.float().contiguous(), sin.float().contiguous()
            if cos_t is None:
                cos_t, sin_t = cos.t().contiguous(), sin.t().contiguous()
        planes = [torch.empty(b, n, heads, dh, dtype=dt, device=device) for _ in range(3)]
        stream = nat.stream_handle(device)
        nat.call(
            "pmb_qkv_linear_rotary_forward", x2.data_ptr(), w.data_ptr(), nat.ptr(cos_t), nat.ptr(sin_t), b, n, d,
            heads, dh, planes[0].data_ptr(), planes[1].data_ptr(), planes[2].data_ptr(), rotate, nat.dtype_code(dt),
            1, stream,
        )
        q, k, v = (pl.transpose(1, 2) for pl in planes)
        logits = torch.addmm(bg, x2, wg.t())  # [b * n, heads]
        gated = torch.empty(b * n, heads * dh, dtype=dt, device=device)
        gp = gated.view(b, n, heads, dh).transpose(1, 2)
        lse = torch.empty(b * heads, (n + 3) // 4 * 4, dtype=torch.float32, device=device)
        nat.call(
            "pmb_attention_forward_gated", q.data_ptr(), k.data_ptr(), v.data_ptr(), logits.data_ptr(),
            gated.data_ptr(), lse.data_ptr(), b, n, heads, dh, nat.i64_array(_attn_strides(q, k, v, gp)), dh ** -0.5,
            nat.dtype_code(dt), stream,
        )
        ctx.dtypes = (weight.dtype, w_gate.dtype, b_gate.dtype)
        ctx.save_for_backward(x2, w, wg, cos, sin, q, k, v, gated, lse, logits)
        return gated

    @staticmethod
    def backward(ctx, grad):
        x2, w, wg, cos, sin, q, k, v, gated, lse, logits = ctx.saved_tensors
        device = q.device
        b, h, n, dh = q.shape
        rows, inner = b * n, h * dh
        g2 = grad.to(q.dtype).contiguous()
        width = 3 * inner + h
        # rows padded to 8 elements: the kernels take plane strides that are multiples of 8
        ext = torch.empty(rows, (width + 7) // 8 * 8, dtype=q.dtype, device=device)[:, :width]
        dq, dk, dv = (ext[:, i * inner:(i + 1) * inner].view(b, n, h, dh).transpose(1, 2) for i in range(3))
        gp = gated.view(b, n, h, dh).transpose(1, 2)
        dgp = g2.view(b, n, h, dh).transpose(1, 2)
        ws_bytes = int(nat.library().pmb_attention_backward_workspace_size(b, n, h))
        ws = nat.workspace(ws_bytes, device)
        # per (sequence pair, head, 32-row group) sums of the logit gradient: the gate bias gradient's partials
        bpart = torch.empty(int(nat.library().pmb_attention_gate_bias_partials(b, h)), dtype=torch.float32,
                            device=device)
        nat.call(
            "pmb_attention_backward_gated", q.data_ptr(), k.data_ptr(), v.data_ptr(), gated.data_ptr(),
            g2.data_ptr(), lse.data_ptr(), logits.data_ptr(), nat.ptr(cos), nat.ptr(sin), dq.data_ptr(),
            dk.data_ptr(), dv.data_ptr(), ext[:, 3 * inner:].data_ptr(), ext.stride(0), bpart.data_ptr(), b, n, h, dh,
            nat.i64_array(_attn_strides(q, k, v, gp, dgp, dq, dk, dv)), dh ** -0.5, nat.dtype_code(q.dtype),
            ws.data_ptr(), ws_bytes, nat.stream_handle(device),
        )
        gx = gw = gwg = gbg = None
        if ctx.needs_input_grad[0]:
            gx = torch.matmul(ext, torch.cat([w, wg], 0)).reshape(b, n, -1)
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[7]:
            gw_ext = _weight_grad(ext.t(), x2, ctx.dtypes[0])
            gw = gw_ext[:3 * inner]
            gwg = gw_ext[3 * inner:].to(ctx.dtypes[1])
        if ctx.needs_input_grad[8]:
            gbg = bpart.view(-1, h, 4).sum((0, 2)).to(ctx.dtypes[2])
        return gx, gw, None, None, None, None, None, gwg, gbg


class STFTFramesFn(torch.autograd.Function):
    """x [B, L] fp32 -> windowed frames [B, T, n_fft] of the centred, reflect-padded signal, as torch.stft frames
    it (window: n_fft values, zero-padded as torch.stft pads a shorter window).  Forward: one kernel writes the
    frames (pmb_stft_frames_forward).  Backward: one deterministic overlap-add per sample with the reflection
    folded in (pmb_stft_frames_backward) instead of torch's atomic index_add and reflection-pad backward."""

    @staticmethod
    def forward(ctx, x, window, n_fft, hop):
        device = nat.require_cuda(x, window, name="STFTFrames")
        x = x.float().contiguous()
        b, length = x.shape
        t = 1 + (length + 2 * (n_fft // 2) - n_fft) // hop
        frames = torch.empty(b, t, n_fft, dtype=torch.float32, device=device)
        nat.call("pmb_stft_frames_forward", x.data_ptr(), window.data_ptr(), frames.data_ptr(), b, length, n_fft, hop,
                 t, nat.stream_handle(device))
        ctx.save_for_backward(window)
        ctx.meta = (x.shape[-1], n_fft, hop, device)
        return frames

    @staticmethod
    def backward(ctx, grad):
        (window,) = ctx.saved_tensors
        length, n_fft, hop, device = ctx.meta
        g = grad.float().contiguous()
        b, t, _ = g.shape
        gx = torch.empty(b, length, dtype=torch.float32, device=device)
        nat.call("pmb_stft_frames_backward", g.data_ptr(), window.data_ptr(), gx.data_ptr(), b, length, n_fft, hop, t,
                 nat.stream_handle(device))
        return gx, None, None, None


_INVERSE_NORM = {"backward": "forward", "ortho": "ortho", "forward": "backward"}
_HALF_BINS: dict = {}


class RealFFTFn(torch.autograd.Function):
    """torch.fft.rfft over the last dimension, with a shorter backward.

    For y_k = sum_n x_n e^(-2 pi i k n / N) over the onesided bins k = 0..N/2 and torch's gradient convention
    (g = dL/dRe y + i dL/dIm y), dL/dx_n = Re sum_k g_k e^(+2 pi i k n / N).  An inverse real FFT counts every
    bin strictly between 0 and N/2 twice, so that sum is irfft(h) with those bins of g halved and the
    normalisation swapped.  torch's own backward instead zero-pads g to all N bins, runs a complex FFT and
    returns the strided real part (copied again by the framing backward): one multiply and a half-size
    c2r transform replace a memset, a copy, a full c2c transform and the real-part copy."""

    @staticmethod
    def forward(ctx, x, norm):
        ctx.n = x.shape[-1]
        ctx.norm = norm
        return torch.fft.rfft(x, dim=-1, norm=norm)

    @staticmethod
    def backward(ctx, g):
        n = ctx.n
        key = (n, g.device)
        w = _HALF_BINS.get(key)
        if w is None:
            w = torch.ones(n // 2 + 1, device=g.device)
            w[1 : (n - 1) // 2 + 1] = 0.5
            _HALF_BINS[key] = w
        return torch.fft.irfft(g * w, n=n, dim=-1, norm=_INVERSE_NORM[ctx.norm]), None


class ISTFTOverlapAddFn(torch.autograd.Function):
    """The overlap-add of torch.istft (center=True) after the per-frame inverse real FFT: frames fp32
    [B, n_fft, T] (any strides, e.g. torch.fft.irfft along dim -2 of a [B, F, T] spectrum) -> y [B, length] =
    the window-weighted overlap-add divided by the overlap-added squared window, centre-trimmed, zero past the
    signal's end.  One kernel each way (pmb_istft_overlap_add_forward / _backward)."""

    @staticmethod
    def forward(ctx, frames, window, hop, length):
        device = nat.require_cuda(frames, window, name="ISTFTOverlapAdd")
        frames = frames.float()
        window = window.float().contiguous()
        b, n, t = frames.shape
        y = torch.empty(b, length, dtype=torch.float32, device=device)
        nat.call("pmb_istft_overlap_add_forward", frames.data_ptr(), nat.i64_array(list(frames.stride())),
                 window.data_ptr(), y.data_ptr(), b, n, t, hop, length, nat.stream_handle(device))
        ctx.save_for_backward(window)
        ctx.meta = (b, n, t, hop, length)
        return y

    @staticmethod
    def backward(ctx, g):
        (window,) = ctx.saved_tensors
        b, n, t, hop, length = ctx.meta
        g = g.float().contiguous()
        gf = torch.empty(b, n, t, dtype=torch.float32, device=g.device)
        nat.call("pmb_istft_overlap_add_backward", g.data_ptr(), window.data_ptr(), gf.data_ptr(), b, n, t, hop,
                 length, nat.stream_handle(g.device))
        return gf, None, None, None


class SpectralL1Fn(torch.autograd.Function):
    """mean |rfft(frames) - target_spec| (F.l1_loss of two onesided spectra) with the rfft inside.  Forward:
    torch.fft.rfft, then one pass for the mean (pmb_spectral_l1_forward, deterministic).  Backward: one pass
    writes (Y - T) / |Y - T| times the upstream gradient / count and the inverse real FFT's bin weights
    (pmb_spectral_l1_backward), then the inverse real FFT: the elementwise difference, abs, mean, their
    backward and RealFFTFn's bin weighting in two passes over the spectrum."""

    @staticmethod
    def forward(ctx, frames, target_spec, norm):
        device = nat.require_cuda(frames, target_spec, name="SpectralL1")
        y = torch.fft.rfft(frames, dim=-1, norm=norm)
        t = target_spec.contiguous()
        if t.shape != y.shape or t.dtype != y.dtype:
            raise ValueError(f"SpectralL1: target spectrum {tuple(t.shape)} {t.dtype} must match {tuple(y.shape)} "
                             f"{y.dtype}")
        count = y.numel()
        wsb = int(nat.library().pmb_spectral_l1_workspace_size(count))
        ws = nat.workspace(wsb, device)
        loss = torch.empty((), dtype=torch.float32, device=device)
        nat.call("pmb_spectral_l1_forward", torch.view_as_real(y).data_ptr(), torch.view_as_real(t).data_ptr(), count,
                 loss.data_ptr(), ws.data_ptr(), wsb, nat.stream_handle(device))
        ctx.n = frames.shape[-1]
        ctx.norm = norm
        ctx.save_for_backward(y, t)
        return loss

    @staticmethod
    def backward(ctx, g):
        y, t = ctx.saved_tensors
        gl = g.float().reshape(1).contiguous()
        gy = torch.empty_like(y)
        nat.call("pmb_spectral_l1_backward", torch.view_as_real(y).data_ptr(), torch.view_as_real(t).data_ptr(),
                 y.numel(), y.shape[-1], ctx.n, gl.data_ptr(), torch.view_as_real(gy).data_ptr(),
                 nat.stream_handle(y.device))
        return torch.fft.irfft(gy, n=ctx.n, dim=-1, norm=_INVERSE_NORM[ctx.norm]), None, None


def stft_l1_loss(recon: torch.Tensor, target: torch.Tensor, n_fft: int, hop: int, window: torch.Tensor,
                 normalized: bool) -> torch.Tensor:
    """F.l1_loss(stft(recon), stft(target)) for fp32 CUDA signals [B, L] (torch.stft's spectra, frames first):
    the framing kernels, the rfft, and SpectralL1Fn's one-pass mean and gradient.  The target's spectrum carries no
    gradient (a training target); with a target that needs one, the two spectra go through F.l1_loss."""
    norm = "ortho" if normalized else "backward"
    if target.requires_grad:
        return F.l1_loss(stft_loss_spectrum(recon, n_fft, hop, window, normalized),
                         stft_loss_spectrum(target, n_fft, hop, window, normalized))
    with torch.no_grad():
        ty = stft_loss_spectrum(target, n_fft, hop, window, normalized)
    return SpectralL1Fn.apply(STFTFramesFn.apply(recon, window, n_fft, hop), ty, norm)


def stft_loss_spectrum(x: torch.Tensor, n_fft: int, hop: int, window: torch.Tensor, normalized: bool) -> torch.Tensor:
    """torch.stft(x, n_fft, hop, window=window, center=True, pad_mode="reflect", onesided, return_complex) for
    fp32 CUDA x [B, L], as [B, T, F] (frames first); window already zero-padded to n_fft."""
    frames = STFTFramesFn.apply(x, window, n_fft, hop)
    return RealFFTFn.apply(frames, "ortho" if normalized else "backward")


# -------------------------------------------------------- band index ops
class BandGatherFn(torch.autograd.Function):
    """stft fp32 [B,S,F,T,2] -> band features [B,T,J*2] in out_dtype."""

    @staticmethod
    def forward(ctx, stft, tables, out_dtype):
        ctx.tables = tables
        ctx.shape = stft.shape
        return ext.band_gather(stft, tables, out_dtype)

    @staticmethod
    def backward(ctx, grad):
        _, s, f, _, _ = ctx.shape
        return ext.band_gather_backward(grad, ctx.tables, s, f), None, None


class BandRecombineFn(torch.autograd.Function):
    """masks [B,N,T,J*2] x stft [B,S,F,T,2] -> masked STFT fp32 [B,N,S,F,T,2] (overlaps averaged)."""

    @staticmethod
    def forward(ctx, mask, stft, tables):
        ctx.tables = tables
        ctx.mask_dtype = mask.dtype
        ctx.save_for_backward(stft)
        _, s, f, _, _ = stft.shape
        return ext.band_recombine(mask, stft, tables, s, f, multiply=True)

    @staticmethod
    def backward(ctx, grad):
        (stft,) = ctx.saved_tensors
        gm = ext.band_recombine_backward(grad, stft, ctx.tables, ctx.mask_dtype, multiply=True)
        return gm, None, None


def rotary_tables(freqs: torch.Tensor, n: int, device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin [n, dh/2] for positions 0..n-1 (exact fp32 positions); .t().contiguous() of them are the
    transposed tables the fused projection epilogue reads."""
    pos = torch.arange(n, device=device, dtype=torch.float32)
    ang = pos[:, None] * freqs.detach().to(device=device, dtype=torch.float32)[None, :]
    return ang.cos().contiguous(), ang.sin().contiguous()

