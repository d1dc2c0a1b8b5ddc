"""The normal-CDF coefficient table of the 16-bit GELU kernels (csrc/gelu.cuh) against its generator
(pymsst_b200.gelu_fit), and the generator's own fp32 emulation over every finite bf16 / fp16 input."""
from __future__ import annotations

import pathlib
import re

import numpy as np
import pytest

scipy = pytest.importorskip("scipy")

from pymsst_b200 import gelu_fit  # noqa: E402


def test_gelu_fit_reproduces_the_kernel_table():
    src = (pathlib.Path(gelu_fit.__file__).parent / "csrc" / "gelu.cuh").read_text()
    table = re.search(r"kPhiH\[10\] = \{([^}]*)\}", src).group(1)
    in_kernel = np.array([float(v.strip().rstrip("f")) for v in table.split(",")], dtype=np.float32)
    np.testing.assert_allclose(in_kernel, gelu_fit.fit(), rtol=1e-6, atol=0)


def test_gelu_fit_emulation_matches_exact_gelu():
    """bf16: every finite input rounds to the exact GELU; fp16: all but a few dozen."""
    result = gelu_fit.check(gelu_fit.fit())
    assert result["bf16"][0] == 0
    assert result["fp16"][0] <= 64
