"""mosyne_bposit -- W8A8 bposit pipeline on NVIDIA B200 (sm_100a).

Drop-in for the reference package's public API
(packages/mosyne_bposit/src/mosyne_bposit/__init__.py:11-30)::

    from mosyne_bposit import linear_w8a8
    y = linear_w8a8(x, w)

Build the shared library once with ``mosyne-bposit_b200/build.py`` (or
``mosyne_bposit.build_library()``); it compiles the tcgen05 INT8 GEMM, the
quantisers, the quire256 exact-sum kernels and the bposit16 ALU for sm_100a.
"""
from __future__ import annotations

from ._api import (
    linear_w8a8,
    linear_w8a8_dev,
    linear_w8a8_dev_bf16,
    linear_w8a8_dev_bf16_io,
    linear_w8a8_dev_fp16,
    linear_w8a8_dev_fp16_io,
    quantize_weight_per_channel_dev,
    shutdown,
    library_path,
)
from .build_so import build as build_library

__version__ = "0.1.0"

__all__ = [
    "linear_w8a8",
    "linear_w8a8_dev",
    "linear_w8a8_dev_bf16",
    "linear_w8a8_dev_bf16_io",
    "linear_w8a8_dev_fp16",
    "linear_w8a8_dev_fp16_io",
    "quantize_weight_per_channel_dev",
    "shutdown",
    "library_path",
    "build_library",
    "__version__",
]
