"""Pin the CPU oracle to the reference: its known-answer tables, its Python
arithmetic (sampled into tests/golden by make_golden.py), its published
determinism headline and its published W8A8 probe hashes.  CPU only."""
from __future__ import annotations

import hashlib
import math
import random
import struct
from fractions import Fraction
from pathlib import Path

import numpy as np
import pytest

from oracle import bposit_oracle as O


def _q(words):
    return O.words_to_quire([int(w, 16) for w in words])


def test_kat_quire_to_bp16(golden):
    cases = golden("kat_quire_to_bp16.json")
    assert len(cases) == 25
    for c in cases:
        assert O.quire_to_bposit(_q(c["w"]), 16) == c["expected"], c["note"]


def test_kat_quire_to_bp32(golden):
    cases = golden("kat_quire_to_bp32.json")
    assert len(cases) == 20
    for c in cases:
        assert O.quire_to_bposit(_q(c["w"]), 32) == c["expected"], c["note"]


def test_kat_int32_to_bp32(golden):
    for c in golden("kat_int32_to_bp32.json"):
        assert O.encode_int(c["input"], c["scale_shift"], 32) == c["expected"], c
        got = O.int_to_bposit32_array(np.array([c["input"]]), c["scale_shift"])[0]
        assert int(got) == c["expected"], c


def test_kat_add_mul(golden):
    for c in golden("kat_add.json"):
        assert O.add16(c["a"], c["b"]) == c["expected"], c["note"]
    for c in golden("kat_mul.json"):
        assert O.mul16(c["a"], c["b"]) == c["expected"], c["note"]


def test_kat_unary(golden):
    k = golden("kat_unary.json")
    fns = {"sqrt": O.sqrt16, "recip": O.recip16, "exp2": O.exp2_16}
    for op, cases in k.items():
        assert cases, op
        for c in cases:
            assert fns[op](c["in"]) == c["expected"], (op, c["note"])


def test_pyref_samples_quire(golden):
    s = golden("pyref_samples.json")
    for c in s["quire"]:
        q = int(c["q"])
        assert O.quire_to_bposit(q, 16) == c["bp16"]
        assert O.quire_to_bposit(q, 32) == c["bp32"]
        assert O.quire_to_bposit(q, 16, "rtne") == c["bp16_rtne"]


def test_pyref_samples_int_and_float(golden):
    s = golden("pyref_samples.json")
    I = np.array([c["I"] for c in s["int"]], dtype=np.int64)
    for sh in {c["shift"] for c in s["int"]}:
        sel = [i for i, c in enumerate(s["int"]) if c["shift"] == sh]
        got32 = O.encode_int_array(I[sel], sh, 32)
        got16 = O.encode_int_array(I[sel], sh, 16)
        for j, i in enumerate(sel):
            assert int(got32[j]) == s["int"][i]["bp32"]
            assert int(got16[j]) == s["int"][i]["bp16"]
    xs = np.array([float.fromhex(c["x"]) for c in s["float"]])
    r16 = O.float_to_bposit_array(xs, 16, "rtne")
    t16 = O.float_to_bposit_array(xs, 16)
    t32 = O.float_to_bposit_array(xs, 32)
    for i, c in enumerate(s["float"]):
        assert int(r16[i]) == c["bp16_rtne"]
        assert int(t16[i]) == c["bp16"]
        assert int(t32[i]) == c["bp32"]


def test_vector_encoder_matches_scalar():
    rng = np.random.default_rng(7)
    I = np.concatenate([rng.integers(-(2 ** 62), 2 ** 62, 3000), rng.integers(-300, 300, 1000),
                        np.array([0, 1, -1, 2 ** 62, -(2 ** 62)])]).astype(np.int64)
    for nb in (16, 32):
        for mode in O.MODES:
            for sh in (0, 7, 96, -20):
                got = O.encode_int_array(I, sh, nb, mode)
                for j in range(0, len(I), 13):
                    assert int(got[j]) == O.encode_int(int(I[j]), sh, nb, mode)


def test_decode_vector_all_codes():
    mant, sh = O.bposit16_decode_array(np.arange(65536, dtype=np.uint16))
    for p in range(0, 65536, 7):
        assert (int(mant[p]) << int(sh[p])) == O.bposit16_to_quire(p)


def test_lut_hashes_oracle(golden):
    g = golden("lut_sha256.json")
    tabs = O.build_tables()
    for name in ("log2", "exp2", "sqrt", "recip", "term", "square"):
        h = hashlib.sha256(struct.pack("<65536H", *tabs[name])).hexdigest()
        assert h == g[name], name
    words = []
    for i in range(65536):
        words.extend(O.quire_to_words(O.bposit16_to_quire(i)))
    assert hashlib.sha256(struct.pack("<262144Q", *words)).hexdigest() == g["to_quire"]


def test_shannon_entropy_goldens(golden):
    """The oracle's entropy (term table + exact sum + truncating bposit32)
    equals the reference's integer pipeline on every golden case."""
    for case in golden("kat_entropy.json"):
        codes = (np.arange(65536, dtype=np.uint16) if case["codes"] == "range(65536)"
                 else np.asarray(case["codes"], dtype=np.uint16))
        q = O.shannon_entropy_quire(codes)
        assert [f"{x:016x}" for x in O.quire_to_words(q)] == case["quire_words"], case["name"]
        assert O.shannon_entropy_bposit(codes) == case["bp32"], case["name"]


def test_build_time_tables_match_oracle(golden):
    """The tables the library is built from (mosyne_bposit._tables) are the
    reference's, term table included."""
    from mosyne_bposit import _tables
    g = golden("lut_sha256.json")
    tabs = _tables.build_all()
    for name in _tables.TABLE_ORDER:
        assert hashlib.sha256(struct.pack("<65536H", *tabs[name])).hexdigest() == g[name], name
    assert np.array_equal(np.asarray(tabs["term"], dtype=np.uint16), O.term_table())


def test_determinism_headline(golden):
    h = golden("headline.json")
    _, _, codes = O.det_headline_inputs()
    q = O.quire_sum_bposit16(codes)
    w = O.quire_to_words(q)
    assert f"{w[1]:016x}" == h["published_quire_w1"]
    assert [f"{x:016x}" for x in w] == h["quire_words"]
    assert O.quire_to_bposit(q, 16) == h["published_bp16"] == 0x7627
    assert O.quire_to_bposit(q, 32) == h["pyref_bp32"]
    # the committed codes bench.py runs on every GPU are the same bits
    fixture = np.load(Path(__file__).resolve().parent / "golden" / "headline_codes.npy")
    assert fixture.dtype == np.uint16 and np.array_equal(fixture, codes)


def test_probe_hashes(golden):
    torch = pytest.importorskip("torch")
    g = golden("probe_hashes.json")
    for key, (M, K, N) in g["shapes"].items():
        gen = torch.Generator(device="cpu").manual_seed(g["seed"])
        x = torch.randn(M, K, generator=gen, dtype=torch.float32) * 0.3
        w = torch.randn(N, K, generator=gen, dtype=torch.float32) * (1.0 / K ** 0.5)
        y = O.linear_w8a8(x.numpy(), w.numpy().T)[0]
        assert hashlib.sha256(np.ascontiguousarray(y).tobytes()).hexdigest() == g["hashes"][key]


# --- RTNE properties (kernels/test_encode_rtne.py restated on the oracle) ---

def _relerr(v: float, mode: str) -> float:
    p = O.encode_fraction(Fraction(v), 16, mode)
    d = float(O.decode(p, 16))
    return abs(d - v) / abs(v)


def test_rtne_properties():
    for v in [1.0, 2.0, 4.0, 0.5, 0.25, 0.125, -1.0, -8.0]:
        assert O.encode_fraction(Fraction(v), 16, "truncate") == O.encode_fraction(Fraction(v), 16, "rtne")
    rng = random.Random(0xB0517)
    vals = [rng.uniform(-1e3, 1e3) for _ in range(2000)] + [rng.uniform(-1e-3, 1e-3) for _ in range(2000)]
    better = 0
    for v in vals:
        if v == 0:
            continue
        et, er = _relerr(v, "truncate"), _relerr(v, "rtne")
        assert er <= et + 1e-15
        better += er + 1e-15 < et
    assert better > 0
    assert O.encode_fraction(Fraction(2) ** 60, 16, "rtne") == 0x7FFF
    with pytest.raises(ValueError, match="unknown rounding mode"):
        O.encode_int(1, 0, 16, "banker")


def test_rtne_bp32_against_rational_rounding():
    """bposit32 RTNE is unpinned by the reference; pin it to exact rational
    round-half-even of the kept fraction instead."""
    rng = random.Random(3)
    for _ in range(3000):
        I = rng.randint(1, 2 ** 40)
        sh = rng.randint(0, 60)
        code = O.encode_int(I, sh, 32, "rtne")
        lo = O.encode_int(I, sh, 32, "truncate")
        v = Fraction(I, 1 << sh)
        if lo == 0x7FFFFFFF:
            continue
        a, b = O.decode(lo, 32), O.decode(lo + 1, 32)
        assert a <= v < b
        if v - a < b - v:
            assert code == lo
        elif v - a > b - v:
            assert code == lo + 1
        else:
            assert code == (lo if lo % 2 == 0 else lo + 1)


def test_exact_sum_inputs_are_rtne():
    v, codes = O.exact_sum_inputs(500, seed=1)
    for x, c in zip(v[:200], codes[:200]):
        assert int(c) == O.encode_fraction(Fraction(float(x)), 16, "rtne")
    assert math.isfinite(float(np.abs(v).max()))


def test_bposit8_tables(golden):
    """bposit8 -> quire words (build_bposit_luts.py:302-311 via pyref) and the
    int8 decode table derived from them (test_mera_isometry_imma.cu:166-197)."""
    g = golden("bposit8.json")
    for i in range(256):
        w = O.quire_to_words(O.bposit8_to_quire(i))
        assert [f"{x:016x}" for x in w] == g["to_quire_words"][i], i
        assert O.bposit8_to_int8(i) == g["to_int8"][i], i
    assert O.bposit8_to_int8(0x40) == 64                  # 1.0 -> 2^6


def test_c5_golden_hashes_reproduce_on_256_rows(golden):
    """The committed C5 output hashes come from configs.c5_inputs and the
    oracle: the first 256 rows (all 28,672 columns, K = 8192) reproduce."""
    import hashlib

    import configs
    want = golden("c5_hashes.json")["rows"]["256"]
    x, w = configs.c5_inputs(256)
    wq, ws = O.quant_per_channel(w.T)
    xq, xs = O.quant_per_token(x)
    acc = O.gemm_exact(xq, wq)                                   # [256, N]
    at = np.ascontiguousarray(acc.T)
    bp = np.concatenate([O.encode_int_array(c, 0, 32) for c in np.array_split(at.reshape(-1), 64)])
    y = np.ascontiguousarray(O.dequant(acc, xs, ws).T)
    assert hashlib.sha256(bp.tobytes()).hexdigest() == want["bp32"]
    assert hashlib.sha256(y.tobytes()).hexdigest() == want["y_f32"]
