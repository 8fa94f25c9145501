"""The library's bposit encoders/decoders (csrc/bposit.cuh, the same source
the CUDA kernels compile) built for the host with g++ and checked against
the oracle -- encoder logic verified without a GPU."""
from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import bposit_oracle as O

HERE = Path(__file__).resolve().parent
CSRC = HERE.parent / "mosyne-bposit_b200" / "csrc"


@pytest.fixture(scope="module")
def hlib(tmp_path_factory):
    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("host") / "libhost_encoders.so"
    subprocess.run([gxx, "-O2", "-std=c++17", "-fopenmp", "-shared", "-fPIC", "-I", str(CSRC),
                    str(HERE / "host_encoders.cpp"), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    return lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_int64_encoders(hlib):
    rng = np.random.default_rng(11)
    I = np.concatenate([rng.integers(-(2 ** 62), 2 ** 62, 20000), rng.integers(-5000, 5000, 5000),
                        np.array([0, 1, -1, 2 ** 63 - 1, -(2 ** 63) + 1])]).astype(np.int64)
    sh = rng.integers(-40, 120, I.size).astype(np.int32)
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(I.size, dtype=np.uint32)
            hlib.h_from_int64(_p(I), _p(sh), ctypes.c_size_t(I.size), nb, rtne, _p(out))
            mode = "rtne" if rtne else "truncate"
            exp = np.array([O.encode_int(int(a), int(s), nb, mode) for a, s in zip(I, sh)], dtype=np.uint32)
            assert np.array_equal(out, exp), (nb, mode)


def test_int32_fast_path(hlib):
    rng = np.random.default_rng(12)
    I = np.concatenate([rng.integers(-(2 ** 31), 2 ** 31, 50000), np.arange(-70000, 70000),
                        np.array([-(2 ** 31), 2 ** 31 - 1])]).astype(np.int32)
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(I.size, dtype=np.uint32)
            hlib.h_from_int32(_p(I), ctypes.c_size_t(I.size), nb, rtne, _p(out))
            exp = O.encode_int_array(I.astype(np.int64), 0, nb, "rtne" if rtne else "truncate")
            assert np.array_equal(out, exp.astype(np.uint32)), (nb, rtne)


@pytest.mark.parametrize("shift", list(range(32)))
def test_int32_table_path(hlib, shift):
    """The epilogue's table-driven encoder equals the oracle on every scale
    (each power of two and its neighbours) and on random values, for the
    plain integer (shift 0) and for I / 2^shift (negative scales)."""
    rng = np.random.default_rng(15)
    edges = []
    for b in range(31):
        for d in (-2, -1, 0, 1, 2):
            v = (1 << b) + d
            if 0 < v < 2 ** 31:
                edges += [v, -v]
    I = np.concatenate([rng.integers(-(2 ** 31), 2 ** 31, 40000), np.array(edges),
                        np.array([0, -(2 ** 31), 2 ** 31 - 1])]).astype(np.int32)
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(I.size, dtype=np.uint32)
            hlib.h_from_int32_tab(_p(I), ctypes.c_size_t(I.size), nb, rtne, _p(out), shift)
            exp = O.encode_int_array(I.astype(np.int64), shift, nb, "rtne" if rtne else "truncate")
            assert np.array_equal(out, exp.astype(np.uint32)), (nb, rtne, shift)


def test_quire_encoders(hlib, golden):
    qs = [int(c["q"]) for c in golden("pyref_samples.json")["quire"]]
    rng = np.random.default_rng(13)
    for _ in range(3000):
        bits = int(rng.integers(0, 250))
        v = int.from_bytes(rng.bytes(32), "little") & ((1 << bits) - 1)
        qs.append(v if rng.integers(0, 2) else -v)
    qs += [_q for _q in (0, 1, -1, (1 << 255) - 1, -(1 << 255) + 1, 1 << 200, -(1 << 200))]
    qs += [s * ((1 << b) + d) for b in range(0, 255, 7) for d in (-1, 0, 1) for s in (1, -1)
           if 0 < (1 << b) + d < (1 << 255)]
    w = np.array([O.quire_to_words(q) for q in qs], dtype=np.uint64)
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(len(qs), dtype=np.uint32)
            hlib.h_from_quire(_p(w), ctypes.c_size_t(len(qs)), nb, rtne, _p(out))
            mode = "rtne" if rtne else "truncate"
            exp = np.array([O.quire_to_bposit(q, nb, mode) for q in qs], dtype=np.uint32)
            assert np.array_equal(out, exp), (nb, mode)
            sel = np.empty(len(qs), dtype=np.uint32)      # the element-wise kernels' form
            hlib.h_from_quire_sel(_p(w), ctypes.c_size_t(len(qs)), nb, rtne, _p(sel))
            assert np.array_equal(sel, exp), (nb, mode)


def test_bp16_decode_all_codes(hlib):
    p = np.arange(65536, dtype=np.uint16)
    w = np.empty((65536, 4), dtype=np.uint64)
    hlib.h_bp16_to_quire(_p(p), ctypes.c_size_t(65536), _p(w))
    for i in range(65536):
        assert O.words_to_quire(w[i]) == O.bposit16_to_quire(i), i


def test_double_encoder(hlib):
    rng = np.random.default_rng(14)
    x = np.concatenate([rng.standard_normal(20000) * 10.0 ** rng.integers(-20, 20, 20000),
                        np.array([0.0, -0.0, 5e-324, 1e300, -1e-300, 2.0 ** -48, 2.0 ** 48])])
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(x.size, dtype=np.uint32)
            hlib.h_from_double(_p(x), ctypes.c_size_t(x.size), nb, rtne, _p(out))
            exp = O.float_to_bposit_array(x, nb, "rtne" if rtne else "truncate").astype(np.uint32)
            assert np.array_equal(out, exp), (nb, rtne)


def test_float_encoder(hlib):
    """The single-precision encoder (32-bit arithmetic) equals the oracle's
    exact encoding of the same values: normals over the whole exponent range
    (saturating beyond +-2^48), subnormals, zeros, inf/nan, and the
    neighbours of every power of two in range."""
    rng = np.random.default_rng(16)
    bits = rng.integers(0, 2 ** 32, 60000, dtype=np.uint64).astype(np.uint32)
    edges = []
    for e in range(-60, 61):
        f = np.float32(2.0 ** e)
        edges += [f, np.nextafter(f, np.float32(0)), np.nextafter(f, np.float32(np.inf))]
    x = np.concatenate([bits.view(np.float32), np.array(edges, dtype=np.float32),
                        -np.array(edges, dtype=np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4e38],
                                 dtype=np.float32)])
    finite = np.isfinite(x)
    for nb in (16, 32):
        for rtne in (0, 1):
            out = np.empty(x.size, dtype=np.uint32)
            hlib.h_from_float(_p(x), ctypes.c_size_t(x.size), nb, rtne, _p(out))
            exp = O.float_to_bposit_array(x[finite].astype(np.float64), nb,
                                          "rtne" if rtne else "truncate").astype(np.uint32)
            assert np.array_equal(out[finite], exp), (nb, rtne)
            assert np.all(out[~finite] == (1 << (nb - 1))), (nb, rtne)   # NaR
            tab = np.empty(x.size, dtype=np.uint32)
            hlib.h_from_float_tab(_p(x), ctypes.c_size_t(x.size), nb, rtne, _p(tab))
            assert np.array_equal(tab, out), (nb, rtne)   # table form == direct form


def test_sum16_int64_path(hlib):
    """The ALU's int64 bposit16 sum equals the quire path (itself pinned to
    the oracle) for every code against 300 partners -- special codes, the
    extremes of the regime range, random codes -- and against the codes next
    to -a and a."""
    rng = np.random.default_rng(17)
    special = [0, 0x8000, 0x0001, 0xFFFF, 0x7FFF, 0x8001, 0x4000, 0xC000, 0x0002, 0x7FFE,
               0x0100, 0xFF00, 0x3FFF, 0x4001]
    bs = np.array(special + list(rng.integers(0, 65536, 300 - len(special))), dtype=np.uint16)
    hlib.h_sum16_check.restype = ctypes.c_size_t
    assert hlib.h_sum16_check(_p(bs), ctypes.c_size_t(bs.size)) == 0


def test_alu_32bit_forms(hlib):
    """The ALU's floating-point adder (TwoSum of the exact values) and 32-bit
    exact multiplier against the int64 forms: every code against 300 codes
    and against the codes next to its negation and itself (the GPU test
    covers all 2^32 pairs)."""
    rng = np.random.default_rng(41)
    special = [0, 0x8000, 0x0001, 0xFFFF, 0x7FFF, 0x8001, 0x4000, 0xC000, 0x0002, 0x7FFE,
               0x0100, 0xFF00, 0x3FFF, 0x4001, 0x0003, 0x0010, 0xFFF0]
    bs = np.array(special + list(rng.integers(0, 65536, 300 - len(special))), dtype=np.uint16)
    hlib.h_alu32_check.restype = ctypes.c_size_t
    assert hlib.h_alu32_check(_p(bs), ctypes.c_size_t(bs.size)) == 0


def test_headline_sum(hlib, golden):
    _, _, codes = O.det_headline_inputs()
    w = np.empty(4, dtype=np.uint64)
    hlib.h_quire_sum(_p(codes), ctypes.c_size_t(codes.size), _p(w))
    assert [f"{int(x):016x}" for x in w] == golden("headline.json")["quire_words"]


def test_bposit8_to_int8_table(hlib, golden):
    """The library's bposit8 decode (built on the host, uploaded with each
    launch) equals the reference's table for all 256 codes."""
    out = np.zeros(256, dtype=np.int8)
    hlib.h_bp8_to_i8(_p(out))
    assert out.tolist() == golden("bposit8.json")["to_int8"]


def test_sum16_f32_every_pair(hlib):
    """The ALU's floating-point bposit16 sum equals the int64 sum on all 2^32
    pairs of codes (the int64 sum is pinned to the quire path above)."""
    hlib.h_sum16_f32_exhaustive.restype = ctypes.c_size_t
    assert hlib.h_sum16_f32_exhaustive() == 0


def test_float_table_encoder_every_pattern(hlib):
    """The kernels' table encoder (one 256-entry lookup by the float's biased
    exponent, then shifts and the RTNE increment) equals the direct float
    encoder on every one of the 2^32 float bit patterns, for bposit16 and
    bposit32, truncate and RTNE (the direct encoder is pinned to the oracle in
    test_float_encoder)."""
    hlib.h_from_float_tab_exhaustive.restype = ctypes.c_size_t
    assert hlib.h_from_float_tab_exhaustive() == 0


def test_sum_regime_bins_every_code(hlib):
    """The exact sum's branch-free decode (regime bin and signed within-regime
    integer, folded as v * 2^(8k + 85) into the quire) equals quire_from_bp16 on
    every code, and the fold's right shift for the lowest regimes drops no bit."""
    hlib.h_sum_bin16_check.restype = ctypes.c_size_t
    assert hlib.h_sum_bin16_check() == 0


def test_quire_halves_every_code(hlib):
    """The element-wise bposit16 -> quire kernel's per-lane half (32-bit words,
    two's complement carried across the halves) equals quire_from_bp16 on
    every code."""
    hlib.h_quire_half_check.restype = ctypes.c_size_t
    assert hlib.h_quire_half_check() == 0

