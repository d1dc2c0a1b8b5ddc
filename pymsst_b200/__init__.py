"""pymsst_b200 — B200-native (sm_100a) kernels for the BS-RoFormer /
Mel-band RoFormer training hot path, behind the reference's plugin API.

Public entry points:

* :mod:`pymsst_b200.extension` — ``ops``, the reference-compatible fused
  operator set (same 21 functions as the reference's CUDA extension), and
  ``load_fused_band_split_extension()``.
* :mod:`pymsst_b200.build` — compiles the C-ABI library in-tree.
"""
from __future__ import annotations

__version__ = "0.1.0"
