"""Shared test set-up.

* ``gpu`` marks tests that need a CUDA device (run on a B200 with
  ``pytest -m gpu``); everything else runs on the CPU.
* The repository root (for ``oracle``), ``mosyne-bposit_b200`` (for the
  ``mosyne_bposit`` package) and ``tests/golden`` (for ``configs``, the
  seeded inputs of the benchmark configurations) are put on ``sys.path``.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "mosyne-bposit_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG_DIR), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name: str):
    return json.loads((GOLDEN / name).read_text())


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA library on a GPU: loaded and initialised.  A GPU test fails
    (not skips) when the library is missing, so a silent fallback cannot
    pass."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from mosyne_bposit import _api
    lib = _api.load_library(init=True)
    return lib
