"""The C-ABI library loads on the CPU host and exports what the header declares."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from pymsst_b200 import _native as nat

HEADER = Path(__file__).resolve().parents[1] / "include" / "pymsst_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^PMB_API\s+[\w\s\*]+?\b(pmb_\w+)\s*\(", text, flags=re.M)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "pmb_rms_norm_forward" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = nat.library()
    missing = [name for name in declared_symbols() if not hasattr(lib, name)]
    assert not missing, f"library does not export {missing}"


def test_binding_table_matches_header():
    assert set(nat.SIGNATURES) == set(declared_symbols())


def test_version_and_empty_error():
    lib = nat.library()
    assert lib.pmb_version().decode() == "0.1.0"
    assert isinstance(lib.pmb_last_error(), bytes)


def test_argument_validation_reports_errors_without_a_gpu():
    lib = nat.library()
    status = lib.pmb_rms_norm_forward(None, None, None, None, None, 4, 0, 0, 0, 0, None)
    assert status == -1
    assert b"bad shape" in lib.pmb_last_error()
    status = lib.pmb_rotary_forward(None, None, None, None, 1, 2, 3, 5, 0, None)
    assert status == -1
    assert b"must be even" in lib.pmb_last_error()
    status = lib.pmb_rms_norm_forward(None, None, None, None, None, 4, 8, 7, 0, 0, None)
    assert status in (-1, -2)


def test_workspace_sizes_are_positive():
    lib = nat.library()
    assert lib.pmb_rms_norm_backward_workspace_size(1000, 192) > 0
    assert lib.pmb_rms_norm_backward_workspace_size(0, 192) == 0


def test_product_ops_reject_cpu_tensors():
    import torch

    from pymsst_b200.extension import ops

    x = torch.randn(4, 8)
    g = torch.ones(8)
    with pytest.raises((RuntimeError, nat.FusedKernelUnavailable)):
        ops.rms_norm_forward(x, g)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(nat.FusedKernelUnavailable):
        nat.library(tmp_path / "missing.so")
