"""Reference-compatible operator set backed by the sm_100a C-ABI library.

:data:`ops` exposes the same functions, argument meanings, return tuples and
argument checks as the reference's pybind11 extension module
(src/pymsst/training/cuda/fused_band_split.cpp:731-753, loaded by
src/pymsst/training/fused_extension.py:15-57).  An object with this surface is
what the reference's plugin boundary ``apply_roformer_fused_training_backend(
model, "cuda_ext", extension=...)`` (src/pymsst/training/fused_roformer.py:56-136)
accepts, so the reference's own autograd wrappers can run on these kernels.

Argument validation raises ``RuntimeError`` with the reference's messages
(``TORCH_CHECK`` surfaces as ``RuntimeError`` in Python).  Outputs are
allocated with torch on the input's device; the library itself never
allocates.  There is no CPU path: CPU tensors are rejected.
"""
from __future__ import annotations

from types import SimpleNamespace

import torch

from . import _native as nat


def _check(cond: bool, message: str) -> None:
    if not cond:
        raise RuntimeError(message)


def _contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


# ----------------------------------------------------------------- RMSNorm
def _rms_forward(x: torch.Tensor, gamma: torch.Tensor, out_dtype: torch.dtype, name: str):
    device = nat.require_cuda(x, gamma, name=name)
    x = _contig(x)
    gamma = _contig(gamma)
    dim = x.shape[-1]
    rows = x.numel() // dim if dim else 0
    out = torch.empty(x.shape, dtype=out_dtype, device=device)
    normed = torch.empty(x.shape, dtype=out_dtype, device=device)
    inv_norm = torch.empty(rows, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_rms_norm_forward",
            x.data_ptr(), gamma.data_ptr(), out.data_ptr(), normed.data_ptr(), inv_norm.data_ptr(),
            rows, dim, nat.dtype_code(x.dtype), nat.dtype_code(gamma.dtype), nat.dtype_code(out_dtype),
            nat.stream_handle(device),
        )
    return out, normed, inv_norm


def rms_norm_backward_into(
    grad_out: torch.Tensor,
    saved: torch.Tensor,
    inv_norm: torch.Tensor,
    gamma: torch.Tensor,
    *,
    saved_is_input: bool,
    grad_x_dtype: torch.dtype | None,
    grad_gamma_dtype: torch.dtype,
    grad_residual: torch.Tensor | None = None,
    name: str = "rms_norm_backward",
):
    """Shared RMSNorm backward; ``grad_x_dtype=None`` skips grad_x.  ``grad_residual`` (same shape as x, in
    ``grad_x_dtype``) is added to grad_x in the same pass (pmb_rms_norm_backward_add)."""
    device = nat.require_cuda(grad_out, saved, inv_norm, gamma, name=name)
    grad_out = _contig(grad_out)
    saved = _contig(saved)
    dim = grad_out.shape[-1]
    rows = grad_out.numel() // dim if dim else 0
    grad_x = None if grad_x_dtype is None else torch.empty(grad_out.shape, dtype=grad_x_dtype, device=device)
    grad_gamma = torch.empty(dim, dtype=grad_gamma_dtype, device=device)
    lib = nat.library()
    ws_bytes = int(lib.pmb_rms_norm_backward_workspace_size(rows, dim))
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    head = (grad_out.data_ptr(), saved.data_ptr(), int(saved_is_input), inv_norm.data_ptr(), _contig(gamma).data_ptr())
    tail = (nat.ptr(grad_x), grad_gamma.data_ptr(), rows, dim, nat.dtype_code(grad_out.dtype),
            nat.dtype_code(gamma.dtype), nat.dtype_code(grad_x_dtype or grad_out.dtype),
            nat.dtype_code(grad_gamma_dtype), workspace.data_ptr(), ws_bytes, nat.stream_handle(device))
    with torch.cuda.device(device):
        if grad_residual is None:
            nat.call("pmb_rms_norm_backward", *head, *tail)
        else:
            _check(grad_x is not None, f"{name}: grad_residual needs grad_x")
            grad_residual = _contig(grad_residual.to(grad_x_dtype))
            _check(grad_residual.numel() == grad_out.numel(), f"{name}: grad_residual must match x")
            nat.call("pmb_rms_norm_backward_add", *head, grad_residual.data_ptr(), *tail)
    return grad_x, grad_gamma


def _check_rms_forward_args(x, gamma):
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(gamma.is_cuda, "gamma must be a CUDA tensor")
    _check(x.dim() >= 2, "x must have at least 2 dimensions")
    _check(gamma.dim() == 1, "gamma must have shape [D]")
    _check(gamma.size(0) == x.size(-1), "gamma dimension must match x last dimension")


def _check_rms_backward_args(grad_out, normed, inv_norm, gamma):
    _check(grad_out.is_cuda, "grad_out must be a CUDA tensor")
    _check(normed.is_cuda, "normed must be a CUDA tensor")
    _check(inv_norm.is_cuda, "inv_norm must be a CUDA tensor")
    _check(gamma.is_cuda, "gamma must be a CUDA tensor")
    _check(grad_out.dim() >= 2, "grad_out must have at least 2 dimensions")
    _check(normed.shape == grad_out.shape, "normed shape must match grad_out")
    _check(gamma.dim() == 1, "gamma must have shape [D]")
    _check(gamma.size(0) == grad_out.size(-1), "gamma dimension must match grad_out last dimension")
    _check(inv_norm.dim() == 1, "inv_norm must have shape [M]")
    _check(inv_norm.size(0) * gamma.size(0) == grad_out.numel(), "inv_norm length must match flattened rows")
    _check(inv_norm.dtype == torch.float32, "inv_norm must be float32")


def rms_norm_forward(x: torch.Tensor, gamma: torch.Tensor):
    """``(out, normed, inv_norm)``; reference .cpp:434-444."""
    _check_rms_forward_args(x, gamma)
    _check(gamma.dtype == x.dtype, "gamma dtype must match x")
    return _rms_forward(x, gamma, x.dtype, "rms_norm_forward")


def rms_norm_backward(grad_out, normed, inv_norm, gamma):
    """``(grad_x, grad_gamma)``; reference .cpp:446-458."""
    _check_rms_backward_args(grad_out, normed, inv_norm, gamma)
    _check(normed.dtype == grad_out.dtype, "normed dtype must match grad_out")
    _check(gamma.dtype == grad_out.dtype, "gamma dtype must match grad_out")
    return rms_norm_backward_into(
        grad_out, normed, inv_norm, gamma, saved_is_input=False, grad_x_dtype=grad_out.dtype,
        grad_gamma_dtype=grad_out.dtype,
    )


def rms_norm_forward_fp32_gamma(x, gamma):
    """Half activations, fp32 gamma; reference .cpp:469-479."""
    _check_rms_forward_args(x, gamma)
    _check(gamma.dtype == torch.float32, "gamma must be float32")
    return _rms_forward(x, gamma, x.dtype, "rms_norm_forward_fp32_gamma")


def rms_norm_backward_fp32_gamma(grad_out, normed, inv_norm, gamma):
    """fp32 grad_gamma; reference .cpp:481-498."""
    _check_rms_backward_args(grad_out, normed, inv_norm, gamma)
    _check(normed.dtype == grad_out.dtype, "normed dtype must match grad_out")
    _check(gamma.dtype == torch.float32, "gamma must be float32")
    return rms_norm_backward_into(
        grad_out, normed, inv_norm, gamma, saved_is_input=False, grad_x_dtype=grad_out.dtype,
        grad_gamma_dtype=torch.float32,
    )


def rms_norm_forward_mixed(x, gamma):
    """fp32 out/normed from half x; reference .cpp:500-510."""
    _check_rms_forward_args(x, gamma)
    _check(gamma.dtype == torch.float32, "gamma must be float32")
    return _rms_forward(x, gamma, torch.float32, "rms_norm_forward_mixed")


def rms_norm_backward_mixed(grad_out, normed, inv_norm, gamma, x_meta):
    """grad_x in x_meta's dtype; reference .cpp:512-537."""
    _check_rms_backward_args(grad_out, normed, inv_norm, gamma)
    _check(x_meta.is_cuda, "x_meta must be a CUDA tensor")
    _check(grad_out.dtype == torch.float32, "grad_out must be float32")
    _check(normed.dtype == torch.float32, "normed must be float32")
    _check(gamma.dtype == torch.float32, "gamma must be float32")
    return rms_norm_backward_into(
        grad_out, normed, inv_norm, gamma, saved_is_input=False, grad_x_dtype=x_meta.dtype,
        grad_gamma_dtype=torch.float32,
    )


# ------------------------------------------------------------------ rotary
def _check_rotary_args(t, cos, sin, tname):
    _check(t.is_cuda, f"{tname} must be a CUDA tensor")
    _check(cos.is_cuda, "cos must be a CUDA tensor")
    _check(sin.is_cuda, "sin must be a CUDA tensor")
    _check(t.dim() == 4, f"{tname} must have shape [B, N, H, D]")
    _check(cos.dim() == 4, "cos must have shape [1, N, 1, D/2]")
    _check(sin.dim() == 4, "sin must have shape [1, N, 1, D/2]")
    _check(t.size(3) % 2 == 0, f"{tname} last dimension must be even")
    _check(cos.size(0) == 1 and cos.size(2) == 1, "cos must broadcast over batch and heads")
    _check(sin.size(0) == 1 and sin.size(2) == 1, "sin must broadcast over batch and heads")
    _check(cos.size(1) == t.size(1), f"cos sequence dimension must match {tname}")
    _check(sin.size(1) == t.size(1), f"sin sequence dimension must match {tname}")
    _check(cos.size(3) == t.size(3) // 2, f"cos rotary dimension must match {tname}")
    _check(sin.size(3) == t.size(3) // 2, f"sin rotary dimension must match {tname}")
    _check(cos.dtype == t.dtype, f"cos dtype must match {tname}")
    _check(sin.dtype == t.dtype, f"sin dtype must match {tname}")


def _rotary(entry: str, t, cos, sin):
    device = nat.require_cuda(t, cos, sin, name=entry)
    t = _contig(t)
    cos = _contig(cos)
    sin = _contig(sin)
    out = torch.empty_like(t)
    b, n, h, d = t.shape
    with torch.cuda.device(device):
        nat.call(
            entry, t.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(), b, n, h, d,
            nat.dtype_code(t.dtype), nat.stream_handle(device),
        )
    return out


def rotary_forward(t, cos, sin):
    """Reference .cpp:390-410."""
    _check_rotary_args(t, cos, sin, "t")
    return _rotary("pmb_rotary_forward", t, cos, sin)


def rotary_backward(grad_out, cos, sin):
    """Reference .cpp:412-430."""
    _check_rotary_args(grad_out, cos, sin, "grad_out")
    return _rotary("pmb_rotary_backward", grad_out, cos, sin)


# --------------------------------------------------------------- BandSplit
def _elsize(t: torch.Tensor) -> int:
    return t.element_size()


def _rows_ptrs(base: torch.Tensor, count: int, step_elems: int) -> list[int]:
    return [base.data_ptr() + g * step_elems * _elsize(base) for g in range(count)]


def band_split_forward_into(x, rows, strides, widths, gammas, weights, biases, out_features, out, normed, inv_norm,
                            param_dtype=None, name="band_split_forward"):
    """Low-level call: per-band pointer lists, caller-allocated outputs."""
    device = x.device
    with torch.cuda.device(device):
        nat.call(
            "pmb_band_split_forward", x.data_ptr(), rows, strides[0], strides[1], strides[2], len(widths),
            nat.i64_array(widths), nat.ptr_array(gammas), nat.ptr_array(weights),
            None if biases is None else nat.ptr_array(biases), out_features, out.data_ptr(),
            nat.ptr(normed), inv_norm.data_ptr(), nat.dtype_code(x.dtype), nat.dtype_code(param_dtype or x.dtype),
            nat.stream_handle(device),
        )


def band_split_backward_into(grad_out, normed, inv_norm, widths, gammas, weights, out_features, grad_x,
                             grad_gammas, grad_weights, grad_biases, param_dtype=None, name="band_split_backward"):
    device = grad_out.device
    rows = grad_out.shape[0]
    lib = nat.library()
    warr = nat.i64_array(widths)
    ws_bytes = int(lib.pmb_band_split_backward_workspace_size(rows, len(widths), warr, out_features,
                                                              int(grad_x is not None)))
    ws = nat.workspace(ws_bytes, device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_band_split_backward", grad_out.data_ptr(), normed.data_ptr(), inv_norm.data_ptr(), rows,
            len(widths), warr, nat.ptr_array(gammas), nat.ptr_array(weights), out_features, nat.ptr(grad_x),
            nat.ptr_array(grad_gammas), nat.ptr_array(grad_weights),
            None if grad_biases is None else nat.ptr_array(grad_biases), nat.dtype_code(grad_out.dtype),
            nat.dtype_code(param_dtype or grad_out.dtype), ws.data_ptr(), ws_bytes, nat.stream_handle(device),
        )


def band_split_forward(x, gamma, weight, bias=None):
    """Grouped BandSplit forward; reference .cpp:141-170 -> (out, normed, inv_norm)."""
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(gamma.is_cuda, "gamma must be a CUDA tensor")
    _check(weight.is_cuda, "weight must be a CUDA tensor")
    if bias is not None:
        _check(bias.is_cuda, "bias must be a CUDA tensor")
    _check(x.dim() == 3, "x must have shape [M, G, I]")
    _check(gamma.dim() == 2, "gamma must have shape [G, I]")
    _check(weight.dim() == 3, "weight must have shape [G, O, I]")
    _check(gamma.size(0) == x.size(1), "gamma group dimension must match x")
    _check(gamma.size(1) == x.size(2), "gamma input dimension must match x")
    _check(weight.size(0) == x.size(1), "weight group dimension must match x")
    _check(weight.size(2) == x.size(2), "weight input dimension must match x")
    if bias is not None:
        _check(bias.dim() == 2, "bias must have shape [G, O]")
        _check(bias.size(0) == x.size(1), "bias group dimension must match x")
        _check(bias.size(1) == weight.size(1), "bias output dimension must match weight")
        _check(bias.dtype == x.dtype, "bias dtype must match x")
    _check(gamma.dtype == x.dtype, "gamma dtype must match x")
    _check(weight.dtype == x.dtype, "weight dtype must match x")
    nat.require_cuda(x, gamma, weight, bias, name="band_split_forward")
    m, g, i = x.shape
    o = weight.shape[1]
    gamma, weight = _contig(gamma), _contig(weight)
    bias = None if bias is None else _contig(bias)
    out = torch.empty(m, g, o, dtype=x.dtype, device=x.device)
    normed = torch.empty(m, g, i, dtype=x.dtype, device=x.device)
    inv = torch.empty(m, g, dtype=torch.float32, device=x.device)
    band_split_forward_into(
        x, m, (x.stride(0), x.stride(1), x.stride(2)), [i] * g, _rows_ptrs(gamma, g, i), _rows_ptrs(weight, g, o * i),
        None if bias is None else _rows_ptrs(bias, g, o), o, out, normed, inv,
    )
    return out, normed, inv


def _band_split_backward_grouped(grad_out, normed, inv_norm, gamma, weight, has_bias):
    _check(grad_out.is_cuda, "grad_out must be a CUDA tensor")
    _check(normed.is_cuda, "normed must be a CUDA tensor")
    _check(inv_norm.is_cuda, "inv_norm must be a CUDA tensor")
    _check(gamma.is_cuda, "gamma must be a CUDA tensor")
    _check(weight.is_cuda, "weight must be a CUDA tensor")
    _check(grad_out.dim() == 3, "grad_out must have shape [M, G, O]")
    _check(normed.dim() == 3, "normed must have shape [M, G, I]")
    _check(inv_norm.dim() == 2, "inv_norm must have shape [M, G]")
    _check(gamma.dim() == 2, "gamma must have shape [G, I]")
    _check(weight.dim() == 3, "weight must have shape [G, O, I]")
    _check(normed.size(0) == grad_out.size(0), "normed M must match grad_out")
    _check(normed.size(1) == grad_out.size(1), "normed G must match grad_out")
    _check(inv_norm.size(0) == grad_out.size(0), "inv_norm M must match grad_out")
    _check(inv_norm.size(1) == grad_out.size(1), "inv_norm G must match grad_out")
    _check(gamma.size(0) == grad_out.size(1), "gamma G must match grad_out")
    _check(gamma.size(1) == normed.size(2), "gamma I must match normed")
    _check(weight.size(0) == grad_out.size(1), "weight G must match grad_out")
    _check(weight.size(1) == grad_out.size(2), "weight O must match grad_out")
    _check(weight.size(2) == normed.size(2), "weight I must match normed")
    _check(normed.dtype == grad_out.dtype, "normed dtype must match grad_out")
    _check(gamma.dtype == grad_out.dtype, "gamma dtype must match grad_out")
    _check(weight.dtype == grad_out.dtype, "weight dtype must match grad_out")
    _check(inv_norm.dtype == torch.float32, "inv_norm must be float32")
    nat.require_cuda(grad_out, normed, inv_norm, gamma, weight, name="band_split_backward")
    m, g, o = grad_out.shape
    i = normed.shape[2]
    grad_out, normed, inv_norm = _contig(grad_out), _contig(normed), _contig(inv_norm)
    gamma, weight = _contig(gamma), _contig(weight)
    grad_x = torch.empty_like(normed)
    grad_gamma = torch.empty_like(gamma)
    grad_weight = torch.empty_like(weight)
    grad_bias = torch.empty(g, o, dtype=grad_out.dtype, device=grad_out.device) if has_bias else None
    band_split_backward_into(
        grad_out, normed, inv_norm, [i] * g, _rows_ptrs(gamma, g, i), _rows_ptrs(weight, g, o * i), o, grad_x,
        _rows_ptrs(grad_gamma, g, i), _rows_ptrs(grad_weight, g, o * i),
        None if grad_bias is None else _rows_ptrs(grad_bias, g, o),
    )
    return grad_x, grad_gamma, grad_weight, grad_bias


def band_split_backward(grad_out, normed, inv_norm, gamma, weight, has_bias):
    """Reference .cpp:172-203 -> (grad_x, grad_gamma, grad_weight, grad_bias|None)."""
    return _band_split_backward_grouped(grad_out, normed, inv_norm, gamma, weight, has_bias)


def band_split_backward_v2(grad_out, normed, inv_norm, gamma, weight, has_bias):
    """Reference .cpp:205-236 (same values as v1)."""
    return _band_split_backward_grouped(grad_out, normed, inv_norm, gamma, weight, has_bias)


def band_split_backward_v3(grad_out, normed, inv_norm, gamma, weight, has_bias):
    """Reference .cpp:238-269 (same values as v1)."""
    return _band_split_backward_grouped(grad_out, normed, inv_norm, gamma, weight, has_bias)


def _check_offsets(dim_offsets, dim_inputs, count):
    _check(dim_offsets.dim() == 1, "dim_offsets must be 1D")
    _check(dim_offsets.dtype == torch.int64, "dim_offsets must be int64")
    _check(dim_offsets.size(0) == count + 1, "dim_offsets length must be band count + 1")


def band_split_ragged_forward(x, gammas, weights, biases, dim_inputs, dim_offsets):
    """Reference .cpp:271-314 -> (out [M,nb,O], normed [M,total], inv_norm [M,nb])."""
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(dim_offsets.is_cuda, "dim_offsets must be a CUDA tensor")
    _check(x.dim() == 2, "x must have shape [M, total]")
    _check(len(gammas) == len(weights), "gammas length must match weights length")
    _check(len(biases) == len(weights), "biases length must match weights length")
    _check(len(dim_inputs) == len(weights), "dim_inputs length must match weights length")
    _check(len(weights) > 0, "weights must not be empty")
    _check_offsets(dim_offsets, dim_inputs, len(weights))
    o = weights[0].size(0)
    for gamma, weight, bias, w in zip(gammas, weights, biases, dim_inputs):
        _check(gamma.dim() == 1, "gamma must have shape [I]")
        _check(weight.dim() == 2, "weight must have shape [O, I]")
        _check(bias.dim() == 1, "bias must have shape [O]")
        _check(gamma.size(0) == w, "gamma dimension must match dim_inputs")
        _check(weight.size(0) == o, "all weights must share output dimension")
        _check(weight.size(1) == w, "weight input dimension must match dim_inputs")
        _check(bias.size(0) == o, "bias output dimension must match weight")
        _check(gamma.dtype == x.dtype, "gamma dtype must match x")
        _check(weight.dtype == x.dtype, "weight dtype must match x")
        _check(bias.dtype == x.dtype, "bias dtype must match x")
    _check(x.size(1) == sum(int(w) for w in dim_inputs), "x total dimension must match dim_inputs")
    nat.require_cuda(x, *gammas, *weights, *biases, name="band_split_ragged_forward")
    x = _contig(x)
    gammas = [_contig(t) for t in gammas]
    weights = [_contig(t) for t in weights]
    biases = [_contig(t) for t in biases]
    m, total = x.shape
    nb = len(weights)
    out = torch.empty(m, nb, o, dtype=x.dtype, device=x.device)
    normed = torch.empty(m, total, dtype=x.dtype, device=x.device)
    inv = torch.empty(m, nb, dtype=torch.float32, device=x.device)
    band_split_forward_into(x, m, (total, -1, 1), dim_inputs, gammas, weights, biases, o, out, normed, inv)
    return out, normed, inv


def band_split_ragged_backward(grad_out, normed, inv_norm, gammas, weights, dim_inputs, dim_offsets):
    """Reference .cpp:316-356 -> [grad_x, *grad_gammas, *grad_weights, *grad_biases]."""
    _check(grad_out.is_cuda, "grad_out must be a CUDA tensor")
    _check(grad_out.dim() == 3, "grad_out must have shape [M, B, O]")
    _check(normed.dim() == 2, "normed must have shape [M, total]")
    _check(inv_norm.dim() == 2, "inv_norm must have shape [M, B]")
    _check(len(gammas) == len(weights), "gammas length must match weights length")
    _check(len(dim_inputs) == len(weights), "dim_inputs length must match weights length")
    _check(len(weights) > 0, "weights must not be empty")
    _check_offsets(dim_offsets, dim_inputs, len(weights))
    _check(normed.size(0) == grad_out.size(0), "normed M must match grad_out")
    _check(inv_norm.size(0) == grad_out.size(0), "inv_norm M must match grad_out")
    _check(inv_norm.size(1) == grad_out.size(1), "inv_norm band count must match grad_out")
    _check(len(weights) == grad_out.size(1), "weights length must match grad_out band count")
    _check(normed.dtype == grad_out.dtype, "normed dtype must match grad_out")
    _check(inv_norm.dtype == torch.float32, "inv_norm must be float32")
    _check(normed.size(1) == sum(int(w) for w in dim_inputs), "normed total dimension must match dim_inputs")
    nat.require_cuda(grad_out, normed, inv_norm, *gammas, *weights, name="band_split_ragged_backward")
    o = grad_out.size(2)
    grad_out, normed, inv_norm = _contig(grad_out), _contig(normed), _contig(inv_norm)
    gammas = [_contig(t) for t in gammas]
    weights = [_contig(t) for t in weights]
    grad_x = torch.empty_like(normed)
    grad_gammas = [torch.empty_like(t) for t in gammas]
    grad_weights = [torch.empty_like(t) for t in weights]
    grad_biases = [torch.empty(o, dtype=grad_out.dtype, device=grad_out.device) for _ in weights]
    band_split_backward_into(grad_out, normed, inv_norm, dim_inputs, gammas, weights, o, grad_x, grad_gammas,
                             grad_weights, grad_biases)
    return [grad_x, *grad_gammas, *grad_weights, *grad_biases]


# ---------------------------------------------------------- grouped linear
def grouped_linear_forward(x, weight, bias=None, activation: int = 0):
    """Reference .cpp:358-388 (x [M,G,I] any strides) -> out [M,G,O]."""
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(weight.is_cuda, "weight must be a CUDA tensor")
    _check(x.dim() == 3, "x must have shape [M, G, I]")
    _check(weight.dim() == 3, "weight must have shape [G, O, I]")
    _check(weight.size(0) == x.size(1), "weight group dimension must match x")
    _check(weight.size(2) == x.size(2), "weight input dimension must match x")
    if bias is not None:
        _check(bias.dim() == 2, "bias must have shape [G, O]")
        _check(bias.size(0) == x.size(1), "bias group dimension must match x")
        _check(bias.size(1) == weight.size(1), "bias output dimension must match weight")
        _check(bias.dtype == x.dtype, "bias dtype must match x")
    _check(weight.dtype == x.dtype, "weight dtype must match x")
    nat.require_cuda(x, weight, bias, name="grouped_linear_forward")
    g = x.shape[1]
    o, i = weight.shape[1], weight.shape[2]
    weight = _contig(weight)
    bias = None if bias is None else _contig(bias)
    return grouped_linear_forward_lists(
        x, _rows_ptrs(weight, g, o * i), None if bias is None else _rows_ptrs(bias, g, o), o, weight.dtype, activation
    )


def grouped_linear_forward_lists(x, weights, biases, out_features, param_dtype, activation: int = 0,
                                 out: torch.Tensor | None = None):
    """x [M,G,I] (any strides), per-group weight / bias pointers or tensors -> out [M,G,O]."""
    device = x.device
    m, g, i = x.shape
    if out is None:
        out = torch.empty(m, g, out_features, dtype=x.dtype, device=device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_grouped_linear_forward", x.data_ptr(), m, g, i, out_features, x.stride(0), x.stride(1),
            x.stride(2), nat.ptr_array(weights), None if biases is None else nat.ptr_array(biases), out.data_ptr(),
            activation, nat.dtype_code(x.dtype), nat.dtype_code(param_dtype), nat.stream_handle(device),
        )
    return out


def grouped_linear_backward(grad_out, x, out, weight, activation: int = 0, need_grad_x: bool = True,
                            has_bias: bool = True):
    """Backward of :func:`grouped_linear_forward` -> (grad_x|None, grad_weight, grad_bias|None)."""
    device = nat.require_cuda(grad_out, x, out, weight, name="grouped_linear_backward")
    weight = _contig(weight)
    g, o, i = weight.shape
    grad_x = torch.empty_like(x) if need_grad_x else None
    grad_weight = torch.empty_like(weight)
    grad_bias = torch.empty(g, o, dtype=weight.dtype, device=device) if has_bias else None
    grouped_linear_backward_lists(
        grad_out, x, out, _rows_ptrs(weight, g, o * i), o, weight.dtype, grad_x, _rows_ptrs(grad_weight, g, o * i),
        None if grad_bias is None else _rows_ptrs(grad_bias, g, o), activation,
    )
    return grad_x, grad_weight, grad_bias


def grouped_linear_backward_lists(grad_out, x, out, weights, out_features, param_dtype, grad_x, grad_weights,
                                  grad_biases, activation: int = 0):
    """Backward with per-group pointer lists; x/grad_out/out must be contiguous [M,G,*]."""
    device = grad_out.device
    grad_out, x = _contig(grad_out), _contig(x)
    out = None if out is None else _contig(out)
    m, g, i = x.shape
    lib = nat.library()
    ws_bytes = int(lib.pmb_grouped_linear_backward_workspace_size(m, g, out_features))
    ws = nat.workspace(ws_bytes, device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_grouped_linear_backward", grad_out.data_ptr(), x.data_ptr(), nat.ptr(out), m, g, i, out_features,
            nat.ptr_array(weights), nat.ptr(grad_x), nat.ptr_array(grad_weights),
            None if grad_biases is None else nat.ptr_array(grad_biases), activation, nat.dtype_code(x.dtype),
            nat.dtype_code(param_dtype), ws.data_ptr(), ws_bytes, nat.stream_handle(device),
        )


# ----------------------------------------------------------- attention gate
def attention_gate_forward(attn, x, weight, bias):
    """Reference .cpp:539-561 -> (out [M,H*DH], gate [M,H], attn, x)."""
    _check(attn.is_cuda, "attn must be a CUDA tensor")
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(weight.is_cuda, "weight must be a CUDA tensor")
    _check(bias.is_cuda, "bias must be a CUDA tensor")
    _check(attn.dim() == 3, "attn must have shape [M, H, DH]")
    _check(x.dim() == 2, "x must have shape [M, D]")
    _check(weight.dim() == 2, "weight must have shape [H, D]")
    _check(bias.dim() == 1, "bias must have shape [H]")
    _check(attn.size(0) == x.size(0), "attn and x row counts must match")
    _check(attn.size(1) == weight.size(0), "attn heads must match weight")
    _check(weight.size(1) == x.size(1), "weight input dimension must match x")
    _check(bias.size(0) == weight.size(0), "bias heads must match weight")
    _check(x.dtype == attn.dtype, "x dtype must match attn")
    _check(weight.dtype == attn.dtype, "weight dtype must match attn")
    _check(bias.dtype == attn.dtype, "bias dtype must match attn")
    device = nat.require_cuda(attn, x, weight, bias, name="attention_gate_forward")
    attn, x, weight, bias = _contig(attn), _contig(x), _contig(weight), _contig(bias)
    rows, heads, dh = attn.shape
    out = torch.empty(rows, heads * dh, dtype=attn.dtype, device=device)
    gate = torch.empty(rows, heads, dtype=attn.dtype, device=device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_attention_gate_forward", attn.data_ptr(), 1, heads * dh, 0, dh, x.data_ptr(), weight.data_ptr(),
            bias.data_ptr(), rows, heads, dh, x.shape[1], out.data_ptr(), gate.data_ptr(),
            nat.dtype_code(attn.dtype), nat.dtype_code(weight.dtype), 1, nat.stream_handle(device),
        )
    return out, gate, attn, x


def attention_gate_backward(grad_out, attn, x, weight, gate):
    """Reference .cpp:563-591 -> (grad_attn, grad_x, grad_weight, grad_bias)."""
    _check(grad_out.dim() == 2, "grad_out must have shape [M, H*DH]")
    _check(attn.dim() == 3, "attn must have shape [M, H, DH]")
    _check(x.dim() == 2, "x must have shape [M, D]")
    _check(weight.dim() == 2, "weight must have shape [H, D]")
    _check(gate.dim() == 2, "gate must have shape [M, H]")
    _check(grad_out.size(0) == attn.size(0), "grad_out rows must match attn")
    _check(grad_out.size(1) == attn.size(1) * attn.size(2), "grad_out columns must match flattened attn")
    _check(attn.size(0) == x.size(0), "attn and x row counts must match")
    _check(attn.size(1) == weight.size(0), "attn heads must match weight")
    _check(weight.size(1) == x.size(1), "weight input dimension must match x")
    _check(gate.size(0) == attn.size(0), "gate rows must match attn")
    _check(gate.size(1) == attn.size(1), "gate heads must match attn")
    for t, n in ((attn, "attn"), (x, "x"), (weight, "weight"), (gate, "gate")):
        _check(t.dtype == grad_out.dtype, f"{n} dtype must match grad_out")
    device = nat.require_cuda(grad_out, attn, x, weight, gate, name="attention_gate_backward")
    grad_out, attn, x, weight, gate = map(_contig, (grad_out, attn, x, weight, gate))
    rows, heads, dh = attn.shape
    dim = x.shape[1]
    grad_attn = torch.empty_like(attn)
    grad_x = torch.empty_like(x)
    grad_weight = torch.empty_like(weight)
    grad_bias = torch.empty(heads, dtype=grad_out.dtype, device=device)
    lib = nat.library()
    ws_bytes = int(lib.pmb_attention_gate_backward_workspace_size(rows, heads, dim))
    ws = nat.workspace(ws_bytes, device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_attention_gate_backward", grad_out.data_ptr(), attn.data_ptr(), 1, heads * dh, 0, dh,
            x.data_ptr(), weight.data_ptr(), gate.data_ptr(), rows, heads, dh, dim, grad_attn.data_ptr(),
            grad_x.data_ptr(), grad_weight.data_ptr(), grad_bias.data_ptr(), nat.dtype_code(grad_out.dtype),
            nat.dtype_code(weight.dtype), ws.data_ptr(), ws_bytes, 1, nat.stream_handle(device),
        )
    return grad_attn, grad_x, grad_weight, grad_bias


# ------------------------------------------------- MaskEstimator final + GLU
def _check_mask_forward(x, weights, bias, dim_inputs, dim_offsets):
    _check(x.is_cuda, "x must be a CUDA tensor")
    _check(bias.is_cuda, "bias must be a CUDA tensor")
    _check(dim_offsets.is_cuda, "dim_offsets must be a CUDA tensor")
    _check(x.dim() == 3, "x must have shape [M, G, H]")
    _check(bias.dim() == 1, "bias must have shape [2 * total]")
    _check(len(weights) == x.size(1), "weights length must match band count")
    _check(len(dim_inputs) == len(weights), "dim_inputs length must match weights length")
    _check_offsets(dim_offsets, dim_inputs, len(weights))
    _check(bias.size(0) == 2 * sum(int(w) for w in dim_inputs), "bias dimension must match dim_inputs")
    _check(bias.dtype == x.dtype, "bias dtype must match x")
    for weight, w in zip(weights, dim_inputs):
        _check(weight.dim() == 2, "weight must have shape [2 * O, H]")
        _check(weight.size(1) == x.size(2), "weight hidden dimension must match x")
        _check(weight.size(0) == int(w) * 2, "weight output dimension must match dim_inputs")
        _check(weight.dtype == x.dtype, "weight dtype must match x")


def _flat_band_ptrs(flat: torch.Tensor, dim_inputs, factor: int = 2) -> list[int]:
    """Per-band pointers into a flat [factor*total] vector."""
    ptrs, off = [], 0
    for w in dim_inputs:
        ptrs.append(flat.data_ptr() + factor * off * flat.element_size())
        off += int(w)
    return ptrs


def mask_estimator_final_forward_into(x, weights, biases, dim_inputs, out, pre, param_dtype):
    """Per-band weights / biases (tensors or pointers) -> out [M,total], pre [M,2*total]."""
    device = x.device
    rows, nb, hidden = x.shape
    with torch.cuda.device(device):
        nat.call(
            "pmb_mask_estimator_final_forward", x.data_ptr(), rows, nb, hidden, nat.i64_array(dim_inputs),
            nat.ptr_array(weights), nat.ptr_array(biases), out.data_ptr(), pre.data_ptr(), nat.dtype_code(x.dtype),
            nat.dtype_code(param_dtype), nat.stream_handle(device),
        )


def mask_estimator_final_backward_into(grad_out, x, pre, weights, dim_inputs, grad_x, grad_biases, grad_weights,
                                       param_dtype):
    device = grad_out.device
    rows, nb, hidden = x.shape
    warr = nat.i64_array(dim_inputs)
    lib = nat.library()
    ws_bytes = int(lib.pmb_mask_estimator_final_backward_workspace_size(rows, nb, warr))
    ws = nat.workspace(ws_bytes, device)
    with torch.cuda.device(device):
        nat.call(
            "pmb_mask_estimator_final_backward", grad_out.data_ptr(), x.data_ptr(), pre.data_ptr(), rows, nb,
            hidden, warr, nat.ptr_array(weights), grad_x.data_ptr(), nat.ptr_array(grad_biases),
            nat.ptr_array(grad_weights), nat.dtype_code(grad_out.dtype), nat.dtype_code(param_dtype), ws.data_ptr(),
            ws_bytes, nat.stream_handle(device),
        )


def mask_estimator_final_forward(x, weights, bias, dim_inputs, dim_offsets):
    """Reference .cpp:560-589 ("grouped") -> (out [M,total], pre [M,2*total], x)."""
    _check_mask_forward(x, weights, bias, dim_inputs, dim_offsets)
    nat.require_cuda(x, bias, *weights, name="mask_estimator_final_forward")
    x, bias = _contig(x), _contig(bias)
    weights = [_contig(w) for w in weights]
    total = sum(int(w) for w in dim_inputs)
    out = torch.empty(x.shape[0], total, dtype=x.dtype, device=x.device)
    pre = torch.empty(x.shape[0], 2 * total, dtype=x.dtype, device=x.device)
    mask_estimator_final_forward_into(x, weights, _flat_band_ptrs(bias, dim_inputs), dim_inputs, out, pre, bias.dtype)
    return out, pre, x


def mask_estimator_final_backward(grad_out, x, pre, weights, dim_inputs, dim_offsets):
    """Reference .cpp:591-625 -> [grad_x, grad_bias, *grad_weights]."""
    _check(grad_out.dim() == 2, "grad_out must have shape [M, total]")
    _check(x.dim() == 3, "x must have shape [M, G, H]")
    _check(pre.dim() == 2, "pre must have shape [M, 2 * total]")
    _check(grad_out.size(0) == x.size(0), "grad_out M must match x")
    _check(pre.size(0) == x.size(0), "pre M must match x")
    _check(pre.size(1) == grad_out.size(1) * 2, "pre total dimension must be twice grad_out")
    _check_offsets(dim_offsets, dim_inputs, x.size(1))
    _check(len(weights) == x.size(1), "weights length must match band count")
    _check(grad_out.dtype == x.dtype, "grad_out dtype must match x")
    _check(pre.dtype == x.dtype, "pre dtype must match x")
    nat.require_cuda(grad_out, x, pre, *weights, name="mask_estimator_final_backward")
    grad_out, x, pre = _contig(grad_out), _contig(x), _contig(pre)
    weights = [_contig(w) for w in weights]
    grad_x = torch.empty_like(x)
    grad_bias = torch.empty(pre.shape[1], dtype=grad_out.dtype, device=grad_out.device)
    grad_weights = [torch.empty_like(w) for w in weights]
    mask_estimator_final_backward_into(grad_out, x, pre, weights, dim_inputs, grad_x,
                                       _flat_band_ptrs(grad_bias, dim_inputs), grad_weights, grad_bias.dtype)
    return [grad_x, grad_bias, *grad_weights]


def mask_estimator_final_direct_forward(x, weights, bias, dim_inputs, dim_offsets):
    """Reference .cpp:660-693 ("direct"); same kernels as the grouped form."""
    return mask_estimator_final_forward(x, weights, bias, dim_inputs, dim_offsets)


def mask_estimator_final_direct_backward(grad_out, x, pre, weights, dim_inputs, dim_offsets):
    """Reference .cpp:695-729 ("direct"); same kernels as the grouped form."""
    return mask_estimator_final_backward(grad_out, x, pre, weights, dim_inputs, dim_offsets)


# ------------------------------------------------------- band index kernels
def band_gather(stft: torch.Tensor, tables: dict, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """stft fp32 [B,S,F,T,2] -> band features [B,T,J*2] (``tables`` from BandIndex.device_tables).

    The result is a view whose rows (one per frame) start 16 bytes apart: the
    storage is [B, T, ld] with ld = J*2 rounded up to 8 elements, so the
    tensor-core BandSplit reads it in place with TMA."""
    device = nat.require_cuda(stft, name="band_gather")
    _check(stft.dtype == torch.float32 and stft.dim() == 5 and stft.shape[-1] == 2, "stft must be fp32 [B,S,F,T,2]")
    stft = _contig(stft)
    b, s, f, t, _ = stft.shape
    j = tables["index"].numel()
    ld = (2 * j + 7) // 8 * 8
    x = torch.empty(b, t, ld, dtype=out_dtype, device=device)
    with torch.cuda.device(device):
        nat.call("pmb_band_gather_forward", stft.data_ptr(), tables["index"].data_ptr(), b, s, f, t, j, x.data_ptr(),
                 ld, nat.dtype_code(out_dtype), nat.stream_handle(device))
    return x[..., : 2 * j]


def band_gather_backward(grad_x: torch.Tensor, tables: dict, channels: int, freqs: int) -> torch.Tensor:
    device = nat.require_cuda(grad_x, name="band_gather_backward")
    grad_x = _contig(grad_x)
    b, t, j2 = grad_x.shape
    grad = torch.empty(b, channels, freqs, t, 2, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        nat.call("pmb_band_gather_backward", grad_x.data_ptr(), tables["inv_ptr"].data_ptr(),
                 tables["inv_idx"].data_ptr(), b, channels, freqs, t, j2 // 2, grad.data_ptr(),
                 nat.dtype_code(grad_x.dtype), nat.stream_handle(device))
    return grad


def band_recombine(mask: torch.Tensor, stft: torch.Tensor | None, tables: dict, channels: int, freqs: int,
                   multiply: bool = True) -> torch.Tensor:
    """mask [B,N,T,J*2] (+ stft [B,S,F,T,2]) -> masked STFT fp32 [B,N,S,F,T,2]."""
    device = nat.require_cuda(mask, stft, name="band_recombine")
    mask = _contig(mask)
    b, n, t, j2 = mask.shape
    if multiply:
        _check(stft is not None and stft.dtype == torch.float32, "stft must be fp32 [B,S,F,T,2]")
        stft = _contig(stft)
    out = torch.empty(b, n, channels, freqs, t, 2, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        nat.call("pmb_band_recombine_forward", mask.data_ptr(), nat.ptr(stft if multiply else None),
                 tables["inv_ptr"].data_ptr(), tables["inv_idx"].data_ptr(), b, n, channels, freqs, t, j2 // 2,
                 int(multiply), out.data_ptr(), nat.dtype_code(mask.dtype), nat.stream_handle(device))
    return out


def band_recombine_backward(grad_out: torch.Tensor, stft: torch.Tensor | None, tables: dict,
                            mask_dtype: torch.dtype = torch.float32, multiply: bool = True) -> torch.Tensor:
    device = nat.require_cuda(grad_out, stft, name="band_recombine_backward")
    grad_out = _contig(grad_out).float()
    b, n, s, f, t, _ = grad_out.shape
    j = tables["index"].numel()
    grad_mask = torch.empty(b, n, t, j * 2, dtype=mask_dtype, device=device)
    with torch.cuda.device(device):
        nat.call("pmb_band_recombine_backward", grad_out.data_ptr(), nat.ptr(_contig(stft) if multiply else None),
                 tables["index"].data_ptr(), tables["inv_ptr"].data_ptr(), b, n, s, f, t, j, int(multiply),
                 grad_mask.data_ptr(), nat.dtype_code(mask_dtype), nat.stream_handle(device))
    return grad_mask


#: The reference-compatible operator namespace (``extension=ops``).
ops = SimpleNamespace(
    rms_norm_forward=rms_norm_forward,
    rms_norm_backward=rms_norm_backward,
    rms_norm_forward_fp32_gamma=rms_norm_forward_fp32_gamma,
    rms_norm_backward_fp32_gamma=rms_norm_backward_fp32_gamma,
    rms_norm_forward_mixed=rms_norm_forward_mixed,
    rms_norm_backward_mixed=rms_norm_backward_mixed,
    rotary_forward=rotary_forward,
    rotary_backward=rotary_backward,
    band_split_forward=band_split_forward,
    band_split_backward=band_split_backward,
    band_split_backward_v2=band_split_backward_v2,
    band_split_backward_v3=band_split_backward_v3,
    band_split_ragged_forward=band_split_ragged_forward,
    band_split_ragged_backward=band_split_ragged_backward,
    grouped_linear_forward=grouped_linear_forward,
    attention_gate_forward=attention_gate_forward,
    attention_gate_backward=attention_gate_backward,
    mask_estimator_final_forward=mask_estimator_final_forward,
    mask_estimator_final_backward=mask_estimator_final_backward,
    mask_estimator_final_direct_forward=mask_estimator_final_direct_forward,
    mask_estimator_final_direct_backward=mask_estimator_final_direct_backward,
)


def load_fused_band_split_extension() -> SimpleNamespace:
    """Drop-in for the reference loader (fused_extension.py:15-20)."""
    if not torch.cuda.is_available():
        raise nat.FusedKernelUnavailable("CUDA is not available")
    nat.library()
    return ops


__all__ = [
    "ops", "load_fused_band_split_extension", "rms_norm_backward_into", "band_split_forward_into",
    "band_split_backward_into", "grouped_linear_backward", "grouped_linear_forward_lists",
    "grouped_linear_backward_lists", "mask_estimator_final_forward_into",
    "mask_estimator_final_backward_into", "band_gather", "band_gather_backward", "band_recombine",
    "band_recombine_backward",
] + [
    name for name in vars(ops)
]
