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
    name: str = "rms_norm_backward",
):
    """Shared RMSNorm backward; ``grad_x_dtype=None`` skips grad_x."""
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
    with torch.cuda.device(device):
        nat.call(
            "pmb_rms_norm_backward",
            grad_out.data_ptr(), saved.data_ptr(), int(saved_is_input), inv_norm.data_ptr(), _contig(gamma).data_ptr(),
            nat.ptr(grad_x), grad_gamma.data_ptr(), rows, dim, nat.dtype_code(grad_out.dtype),
            nat.dtype_code(gamma.dtype), nat.dtype_code(grad_x_dtype or grad_out.dtype),
            nat.dtype_code(grad_gamma_dtype), workspace.data_ptr(), ws_bytes, nat.stream_handle(device),
        )
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
)


def load_fused_band_split_extension() -> SimpleNamespace:
    """Drop-in for the reference loader (fused_extension.py:15-20)."""
    if not torch.cuda.is_available():
        raise nat.FusedKernelUnavailable("CUDA is not available")
    nat.library()
    return ops


__all__ = ["ops", "load_fused_band_split_extension", "rms_norm_backward_into"] + [
    name for name in vars(ops)
]
