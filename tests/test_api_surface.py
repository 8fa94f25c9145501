"""CPU-side checks of the public surface: package import, validation before
the library loads (reference tests/test_api_validation.py), and that the
built C-ABI library loads and exports every symbol include/*.h declares."""
from __future__ import annotations

import ctypes
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_package_imports_and_version():
    import mosyne_bposit
    assert isinstance(mosyne_bposit.__version__, str) and mosyne_bposit.__version__
    assert {"linear_w8a8", "shutdown", "library_path", "build_library"} <= set(mosyne_bposit.__all__)


def test_library_path_resolves_next_to_module():
    import mosyne_bposit
    from mosyne_bposit import _api
    p = mosyne_bposit.library_path()
    assert isinstance(p, Path)
    assert p.name == "libmosyne_bposit.so"
    assert p.parent == Path(_api.__file__).resolve().parent


def test_linear_w8a8_rejects_non_2d_inputs():
    from mosyne_bposit import linear_w8a8
    with pytest.raises(ValueError, match="must be 2-D"):
        linear_w8a8(np.zeros(8, np.float32), np.zeros((8, 8), np.float32))
    with pytest.raises(ValueError, match="must be 2-D"):
        linear_w8a8(np.zeros((8, 8), np.float32), np.zeros((8, 8, 8), np.float32))


def test_linear_w8a8_rejects_shape_mismatch():
    from mosyne_bposit import linear_w8a8
    with pytest.raises(ValueError, match="shape mismatch"):
        linear_w8a8(np.zeros((4, 8), np.float32), np.zeros((16, 4), np.float32))


def test_shutdown_is_safe_when_library_not_loaded():
    from mosyne_bposit import _api, shutdown
    saved = _api._lib
    _api._lib = None
    try:
        shutdown()
    finally:
        _api._lib = saved


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from mosyne_bposit import _api
    monkeypatch.setattr(_api, "_lib", None)
    monkeypatch.setenv("MOSYNE_BPOSIT_SO", str(tmp_path / "nope.so"))
    with pytest.raises(RuntimeError, match="not found"):
        _api.load_library()


def _header_symbols():
    txt = (ROOT / "include" / "mosyne_bposit.h").read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b((?:mosyne_bposit|shannon_entropy_bposit16)\w*)\s*\(", txt)))


@pytest.fixture(scope="module")
def built_lib():
    from mosyne_bposit import _api
    so = _api.library_path()
    if not so.exists():
        subprocess.run([sys.executable, str(ROOT / "mosyne-bposit_b200" / "build.py")], check=True)
    return so


def test_library_exports_every_declared_symbol(built_lib):
    syms = _header_symbols()
    assert "mosyne_bposit_init" in syms and "mosyne_bposit_gemm_i8" in syms
    assert len(syms) >= 30
    lib = ctypes.CDLL(str(built_lib))
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    nm = subprocess.run(["nm", "-D", "--defined-only", str(built_lib)], capture_output=True, text=True)
    exported = set(re.findall(r"\b((?:mosyne_bposit|shannon_entropy_bposit16)\w*)\b", nm.stdout))
    assert set(syms) <= exported


def test_python_binding_declares_every_symbol(built_lib):
    from mosyne_bposit import _api
    assert set(_header_symbols()) == set(_api._SIGS)
    _api._lib = None
    lib = _api.load_library(init=False)      # no GPU needed to load and bind
    assert lib.mosyne_bposit_version().decode().endswith("sm_100a tcgen05")


def test_reference_abi_symbols_present(built_lib):
    ref9 = ["mosyne_bposit_init", "mosyne_bposit_shutdown",
            "mosyne_bposit_quantize_weight_per_channel", "mosyne_bposit_linear_w8a8",
            "mosyne_bposit_linear_w8a8_bf16", "mosyne_bposit_linear_w8a8_bf16_io",
            "mosyne_bposit_linear_w8a8_fp16", "mosyne_bposit_linear_w8a8_fp16_io",
            "mosyne_bposit_linear_w8a8_host",
            # kernels/shannon_entropy_bposit16.cu:124 (the entropy library's export)
            "shannon_entropy_bposit16_cuda"]
    lib = ctypes.CDLL(str(built_lib))
    for s in ref9:
        assert hasattr(lib, s), s
