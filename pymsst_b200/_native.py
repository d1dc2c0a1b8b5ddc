"""ctypes binding of the C-ABI library ``_lib/libpymsst_b200.so``.

The library is the product: every fused op in this package calls it, and there
is no fallback.  If the library is missing the import of an op raises
:class:`FusedKernelUnavailable`, mirroring the reference's loader error
(src/pymsst/training/fused_extension.py:11-19), but it is never swallowed.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libpymsst_b200.so"

F32, F16, BF16 = 0, 1, 2
_DTYPE_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_f32 = ctypes.c_float
_pp = ctypes.POINTER(ctypes.c_void_p)
_pi64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes).  Kept in the order of include/pymsst_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "pmb_version": (ctypes.c_char_p, []),
    "pmb_last_error": (ctypes.c_char_p, []),
    "pmb_launch_count": (ctypes.c_uint64, []),
    "pmb_umma_timeout": (ctypes.c_uint, [_i]),
    "pmb_gemm_tc": (_i, [_p, _i64, _i, _p, _i64, _i, _p, _i64, _i, _p, _i, _i, _i64, _i64, _i64, _i, _p]),
    "pmb_gemm_tc_wgrad_workspace_size": (_i64, [_i64, _i64, _i64]),
    "pmb_gemm_tc_wgrad": (_i, [_p, _i64, _p, _i64, _i64, _i64, _i64, _p, _i64, _i, _i, _p, _i64, _p]),
    "pmb_qkv_linear_rotary_forward": (
        _i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i, _i, _i64, _p]),
    "pmb_feed_forward_forward": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i, _i, _p]),
    "pmb_feed_forward_backward_workspace_size": (_i64, [_i64, _i64, _i64, _i]),
    "pmb_feed_forward_backward": (
        _i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i, _i, _p, _i64, _p]),
    "pmb_gelu_forward": (_i, [_p, _p, _i64, _i, _p]),
    "pmb_rows_pass_workspace_size": (_i64, [_i64, _i64]),
    "pmb_gelu_backward": (_i, [_p, _p, _p, _i64, _i64, _p, _i, _i, _p, _i64, _p]),
    "pmb_column_sum": (_i, [_p, _i64, _i64, _p, _i, _i, _p, _i64, _p]),
    "pmb_band_split_tc_sizes": (_i, [_i64, _i, _p, _i64, _i, _p]),
    "pmb_band_split_tc_forward": (
        _i, [_p, _i64, _i64, _i, _p, _p, _p, _p, _i64, _p, _p, _p, _i, _i, _p]),
    "pmb_band_split_tc_backward": (
        _i, [_p, _p, _i64, _p, _i64, _i, _p, _p, _p, _i64, _p, _p, _p, _i, _i, _p, _i64, _p]),
    "pmb_rms_norm_forward": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i, _i, _i, _p]),
    "pmb_rms_norm_backward_workspace_size": (_i64, [_i64, _i64]),
    "pmb_rms_norm_backward": (_i, [_p, _p, _i, _p, _p, _p, _p, _i64, _i64, _i, _i, _i, _i, _p, _i64, _p]),
    "pmb_rms_norm_backward_add": (
        _i, [_p, _p, _i, _p, _p, _p, _p, _p, _i64, _i64, _i, _i, _i, _i, _p, _i64, _p]),
    "pmb_rms_norm_backward_noalloc": (_i, [_p, _p, _i, _p, _p, _p, _p, _i64, _i64, _i, _i, _i, _i, _p]),
    "pmb_rotary_forward": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "pmb_rotary_backward": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i, _p]),
    "pmb_band_split_forward": (
        _i, [_p, _i64, _i64, _i64, _i64, _i, _pi64, _pp, _pp, _pp, _i64, _p, _p, _p, _i, _i, _p]),
    "pmb_band_split_backward_workspace_size": (_i64, [_i64, _i, _pi64, _i64, _i]),
    "pmb_band_split_backward": (
        _i, [_p, _p, _p, _i64, _i, _pi64, _pp, _pp, _i64, _p, _pp, _pp, _pp, _i, _i, _p, _i64, _p]),
    "pmb_grouped_linear_forward": (
        _i, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _pp, _pp, _p, _i, _i, _i, _p]),
    "pmb_grouped_linear_backward_workspace_size": (_i64, [_i64, _i64, _i64]),
    "pmb_grouped_linear_backward": (
        _i, [_p, _p, _p, _i64, _i64, _i64, _i64, _pp, _p, _pp, _pp, _i, _i, _i, _p, _i64, _p]),
    "pmb_mask_estimator_final_forward": (_i, [_p, _i64, _i, _i64, _pi64, _pp, _pp, _p, _p, _i, _i, _p]),
    "pmb_mask_estimator_final_backward_workspace_size": (_i64, [_i64, _i, _pi64]),
    "pmb_mask_estimator_final_backward": (
        _i, [_p, _p, _p, _i64, _i, _i64, _pi64, _pp, _p, _pp, _pp, _i, _i, _p, _i64, _p]),
    "pmb_attention_gate_forward": (
        _i, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i, _i, _i64, _p]),
    "pmb_attention_gate_backward_workspace_size": (_i64, [_i64, _i64, _i64]),
    "pmb_attention_gate_backward": (
        _i, [_p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _i, _i, _p, _i64,
             _i64, _p]),
    "pmb_band_gather_forward": (_i, [_p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i64, _i, _p]),
    "pmb_band_gather_backward": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i, _p]),
    "pmb_band_recombine_forward": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i, _p, _i, _p]),
    "pmb_band_recombine_backward": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i, _p, _i, _p]),
    "pmb_mask_estimator_tc_sizes": (_i, [_i64, _i, _i64, _i64, _i, _pi64, _pi64]),
    "pmb_mask_estimator_tc_forward": (
        _i, [_p, _i64, _i, _i64, _i64, _i, _pi64, _pp, _pp, _p, _p, _p, _p, _i, _i, _p]),
    "pmb_mask_estimator_tc_backward": (
        _i, [_p, _p, _p, _p, _p, _i64, _i, _i64, _i64, _i, _pi64, _pp, _pp, _p, _i, _i, _p, _i64, _p]),
    "pmb_qkv_rotary_split": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _p, _i, _i, _i64, _p]),
    "pmb_qkv_rotary_merge": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i, _i, _i64, _i64, _i64, _i64, _p]),
    "pmb_attention_row_pitch": (_i64, [_i64]),
    "pmb_attention_forward": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _pi64, _f32, _i, _p]),
    "pmb_attention_backward_workspace_size": (_i64, [_i64, _i64, _i64]),
    "pmb_attention_backward": (
        _i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _pi64, _f32, _i, _p, _i64, _p]),
    "pmb_attention_forward_gated": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _pi64, _f32, _i, _p]),
    "pmb_attention_gate_bias_partials": (_i64, [_i64, _i64]),
    "pmb_attention_backward_gated": (
        _i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _pi64, _f32, _i,
             _p, _i64, _p]),
    "pmb_attention_backward_rotary": (
        _i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _pi64, _f32, _i, _p, _i64, _p]),
    "pmb_istft_overlap_add_forward": (_i, [_p, _pi64, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "pmb_istft_overlap_add_backward": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "pmb_spectral_l1_workspace_size": (_i64, [_i64]),
    "pmb_spectral_l1_forward": (_i, [_p, _p, _i64, _p, _p, _i64, _p]),
    "pmb_spectral_l1_backward": (_i, [_p, _p, _i64, _i64, _i64, _p, _p, _p]),
    "pmb_stft_frames_forward": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "pmb_stft_frames_backward": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
}


class FusedKernelUnavailable(RuntimeError):
    """The sm_100a kernel library cannot be used (not built, or no CUDA device)."""


class KernelError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and return the C-ABI library with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.is_file():
            raise FusedKernelUnavailable(
                f"{target} is missing; build it with `python -m pymsst_b200.build`"
            )
        lib = ctypes.CDLL(str(target))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if path is None:
            _lib = lib
        return lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from exc


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(status: int, name: str) -> None:
    if status != 0:
        message = library().pmb_last_error().decode("utf-8", "replace")
        raise KernelError(f"{name} failed with status {status}: {message}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# Entry points whose calls are bracketed by CUDA events (see ``time_entries``).
_TIMED: dict[str, list] = {}
_TIMED_EXTERNAL = [False]


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    rec = _TIMED.get(name) if _TIMED else None
    if rec is None:
        check(getattr(library(), name)(*args), name)
        return
    start = torch.cuda.Event(enable_timing=True, external=_TIMED_EXTERNAL[0])
    end = torch.cuda.Event(enable_timing=True, external=_TIMED_EXTERNAL[0])
    start.record()
    check(getattr(library(), name)(*args), name)
    end.record()
    rec.append((start, end, args))


class time_entries:
    """Context manager: record CUDA events around every call of the given entry
    points (on the current stream, where the library launches).  ``result()``
    returns {name: (calls, total_ms, [args of each call])} after a synchronize.

    ``external=True`` makes the events graph nodes when the calls are captured
    into a CUDA graph: every replay of that graph records them again, so
    ``result()`` after a replay gives each entry's device time inside the
    replayed step (no host launch time in it)."""

    def __init__(self, names, external: bool = False):
        self.names = list(names)
        self.external = bool(external)

    def __enter__(self):
        for n in self.names:
            _TIMED[n] = []
        _TIMED_EXTERNAL[0] = self.external
        return self

    def __exit__(self, *exc):
        self.records = {n: _TIMED.pop(n) for n in self.names}
        _TIMED_EXTERNAL[0] = False
        return False

    def result(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for n, recs in self.records.items():
            total = sum(s.elapsed_time(e) for s, e, _ in recs)
            out[n] = (len(recs), total, [a for _, _, a in recs])
        return out


def i64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * len(values))(*values)


def ptr_array(values) -> ctypes.Array:
    """Host array of device pointers (ints or tensors; None becomes NULL)."""
    out = []
    for v in values:
        if v is None:
            out.append(None)
        elif isinstance(v, torch.Tensor):
            out.append(v.data_ptr())
        else:
            out.append(int(v))
    return (ctypes.c_void_p * len(out))(*out)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def require_cuda(*tensors: torch.Tensor | None, name: str) -> torch.device:
    """Fail loudly unless every tensor is on one CUDA device."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise FusedKernelUnavailable(
                f"{name}: tensors must be CUDA tensors (got {t.device}); this package has no CPU path"
            )
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"{name}: tensors are on different devices ({device} and {t.device})")
    if device is None:
        raise ValueError(f"{name}: no tensor arguments")
    return device
