"""Regenerate the golden fixtures in this directory from the reference.

Run from the repository root, giving the reference checkout as the first
argument (else ``$MOSYNE_REFERENCE_ROOT``, else a directory named
``reference`` beside this repository)::

    python tests/golden/make_golden.py [/path/to/reference [fixture.json ...]]

It reads the reference's known-answer tables as text, calls the
reference's own Python arithmetic (kernels/bposit16_reference.py) on seeded
random samples and on every bposit16 code, and writes small JSON fixtures.
The tests only read the JSON; nothing at test time touches the reference.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import random
import re
import struct
import sys
import time
from fractions import Fraction
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = Path(sys.argv[1] if len(sys.argv) > 1 else
           os.environ.get("MOSYNE_REFERENCE_ROOT", str(HERE.parents[2] / "reference")))
KERN = REF / "kernels"
sys.path.insert(0, str(KERN))
import bposit16_reference as R  # noqa: E402

sys.path.insert(0, str(HERE.parent.parent))
from oracle import bposit_oracle as O  # noqa: E402  (only for the headline inputs)


def _write(name: str, obj) -> None:
    (HERE / name).write_text(json.dumps(obj, indent=1) + "\n")
    print("wrote", name)


def _src(rel: str) -> str:
    return (REF / rel).read_text()


def kat_quire_to_bp16():
    """kernels/test_cases_quire_inline.h:8-32."""
    txt = _src("kernels/test_cases_quire_inline.h")
    pat = re.compile(r"\{\s*\{\s*0x([0-9a-f]+)ULL,\s*0x([0-9a-f]+)ULL,\s*0x([0-9a-f]+)ULL,\s*0x([0-9a-f]+)ULL\s*\},\s*0x([0-9a-f]+),\s*\"([^\"]*)\"")
    out = [{"w": [m.group(i) for i in range(1, 5)], "expected": int(m.group(5), 16), "note": m.group(6)}
           for m in pat.finditer(txt)]
    assert len(out) == 25, len(out)
    return out


def kat_quire_to_bp32():
    """kernels/gen_test_cases_quire_to_bp32.py:39-60 with pyref expectations."""
    spec = importlib.util.spec_from_file_location("genbp32", KERN / "gen_test_cases_quire_to_bp32.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = []
    for note, val in mod.CASES:
        w = mod.value_to_quire_words(val)
        out.append({"w": [f"{x:016x}" for x in w], "expected": R.encode_bposit32(val) & 0xFFFFFFFF, "note": note})
    return out


def kat_int32_to_bp32():
    """kernels/test_int32_to_bposit32.cu:141-154."""
    txt = _src("kernels/test_int32_to_bposit32.cu")
    pat = re.compile(r"\{\s*(-?\d+),\s*(\d+),\s*0x([0-9a-f]+),\s*\"")
    out = [{"input": int(m.group(1)), "scale_shift": int(m.group(2)), "expected": int(m.group(3), 16)}
           for m in pat.finditer(txt)]
    assert len(out) == 11, len(out)
    return out


def kat_binary(rel: str, n: int):
    """kernels/test_cases_{add,mul}_inline.h."""
    pat = re.compile(r"\{\s*0x([0-9a-f]+),\s*0x([0-9a-f]+),\s*0x([0-9a-f]+),\s*\"([^\"]*)\"")
    out = [{"a": int(m.group(1), 16), "b": int(m.group(2), 16), "expected": int(m.group(3), 16), "note": m.group(4)}
           for m in pat.finditer(_src(rel))]
    assert len(out) == n, (rel, len(out))
    return out


def kat_unary(rel: str):
    """Inline Tcase tables of kernels/test_{sqrt,recip,exp2}.cu."""
    pat = re.compile(r"\{\s*0x([0-9a-f]+),\s*0x([0-9a-f]+),\s*\"([^\"]*)\"")
    return [{"in": int(m.group(1), 16), "expected": int(m.group(2), 16), "note": m.group(3)}
            for m in pat.finditer(_src(rel))]


def pyref_samples():
    rng = random.Random(0xB0517)
    quires = []
    for _ in range(1500):
        mag = rng.randint(0, 200)
        quires.append(rng.getrandbits(mag) * rng.choice([-1, 1]))
    quires += [0, 1, -1, 1 << 96, -(1 << 96), (1 << 145), -(1 << 145), (1 << 48) - 1]
    q16 = [{"q": str(q), "bp16": R.quire256_to_bposit16(q), "bp32": R.quire256_to_bposit32(q),
            "bp16_rtne": (R.encode_bposit16(Fraction(q, 1 << 96), mode="rtne") if q else 0)} for q in quires]
    ints = []
    for _ in range(1500):
        I = rng.randint(-(2 ** 31) + 1, 2 ** 31 - 1)
        sh = rng.choice([0, 0, 0, 12, 24])
        ints.append({"I": I, "shift": sh, "bp32": R.encode_bposit32(Fraction(I, 1 << sh)),
                     "bp16": R.encode_bposit16(Fraction(I, 1 << sh))})
    floats = []
    for _ in range(1000):
        x = rng.choice([rng.uniform(-1e3, 1e3), rng.uniform(-1e-3, 1e-3), 2.0 ** rng.uniform(-50, 50)])
        floats.append({"x": x.hex(), "bp16_rtne": R.encode_bposit16(Fraction(x), mode="rtne"),
                       "bp16": R.encode_bposit16(Fraction(x)), "bp32": R.encode_bposit32(Fraction(x))})
    return {"quire": q16, "int": ints, "float": floats}


def lut_hashes():
    """SHA-256 of the ALU tables exactly as kernels/build_bposit_luts.py:34-286
    bakes them (little-endian uint16 / 4 x uint64 per entry)."""
    t0 = time.time()
    log2 = [R.bposit16_log2(i) for i in range(65536)]
    tabs = {
        "log2": log2,
        "exp2": [R.bposit16_exp2(i) for i in range(65536)],
        "sqrt": [R.bposit16_sqrt(i) for i in range(65536)],
        "recip": [R.bposit16_reciprocal(i) for i in range(65536)],
        "term": [R.NAR if log2[i] == R.NAR else R.bposit16_mul(i, log2[i]) for i in range(65536)],
        "square": [R.bposit16_mul(i, i) for i in range(65536)],
    }
    out = {k: hashlib.sha256(struct.pack("<65536H", *v)).hexdigest() for k, v in tabs.items()}
    words = []
    for i in range(65536):
        q = R.bposit16_to_quire(i) & ((1 << 256) - 1)
        words.extend((q >> (64 * w)) & 0xFFFFFFFFFFFFFFFF for w in range(4))
    out["to_quire"] = hashlib.sha256(struct.pack("<262144Q", *words)).hexdigest()
    out["samples"] = {k: {str(i): v[i] for i in range(0, 65536, 997)} for k, v in tabs.items()}
    print("tables in", round(time.time() - t0, 1), "s")
    return out


def headline():
    """docs/research/repro_bench_cross_gpu_2026-05-09.md:14 (published values)
    plus the full quire of the det:181-189 inputs summed with pyref."""
    txt = _src("docs/research/repro_bench_cross_gpu_2026-05-09.md")
    m = re.search(r"quire_hi=0x([0-9a-f]{16})`<br>`bp16=0x([0-9a-f]{4})", txt)
    _, _, codes = O.det_headline_inputs()
    q = sum(R.bposit16_to_quire(int(c)) for c in codes)
    return {"published_quire_w1": m.group(1), "published_bp16": int(m.group(2), 16),
            "quire_words": [f"{x:016x}" for x in O.quire_to_words(q)],
            "pyref_bp16": R.quire256_to_bposit16(q), "pyref_bp32": R.quire256_to_bposit32(q),
            "n": len(codes), "seed": 0x5EED1234}


def bposit8():
    """bposit8 -> quire table words exactly as kernels/build_bposit_luts.py:302-311
    bakes them, and the int8 decode table the reference derives from those
    words (kernels/test_mera_isometry_imma.cu:166-197, restated here: signed
    w[1], bit 63 forced on for a negative quire, arithmetic shift by 26,
    clamp to int8)."""
    words, to_i8 = [], []
    for i in range(256):
        q = R.bposit8_to_quire(i)
        if q < 0:
            q += 1 << 256
        w = [(q >> (64 * k)) & 0xFFFFFFFFFFFFFFFF for k in range(4)]
        words.append([f"{x:016x}" for x in w])
        hi = w[1] - (1 << 64) if w[1] >> 63 else w[1]
        if (w[3] >> 63) and hi >= 0:
            hi -= 1 << 63
        to_i8.append(max(-128, min(127, hi >> 26)))
    return {"to_quire_words": words, "to_int8": to_i8}


def probe():
    """packages/mosyne_bposit/src/mosyne_bposit/cross_gpu_probe.py:52-57 and
    examples/canonical_probe_references/probe_{3090,5090}_*.json."""
    d = REF / "packages/mosyne_bposit/examples/canonical_probe_references"
    refs = {p.name: json.loads(p.read_text())["hashes"] for p in sorted(d.glob("probe_*.json"))}
    hashes = list(refs.values())
    assert all(h == hashes[0] for h in hashes)
    return {"seed": 1234, "shapes": {"small": [64, 2048, 2048], "llama_ffn": [128, 4096, 11008],
                                     "square": [256, 4096, 4096]},
            "hashes": hashes[0], "sources": sorted(refs)}


def entropy():
    """Shannon entropy of bposit16 probabilities through the reference's own
    integer pipeline (kernels/bposit16_reference.py:813-824; the test case of
    pyref:850-853 first): bposit32 result and the quire it encodes, for
    uniform and seeded random distributions, mixed codes (zero, NaR,
    negatives, saturating values) and every bposit16 code."""
    def case(name, codes):
        codes = [int(c) & 0xFFFF for c in codes]
        q = sum(-R.bposit16_to_quire(R.bposit16_mul(p, R.bposit16_log2(p))) for p in codes)
        bp32 = R.shannon_entropy_bposit16(codes)
        assert bp32 == R.quire256_to_bposit32(q)
        return {"name": name, "codes": codes, "bp32": bp32,
                "quire_words": [f"{x:016x}" for x in O.quire_to_words(q)]}
    rng = random.Random(20261202)
    out = [case("uniform4 (pyref:850-853)", [R.encode_bposit16(Fraction(1, 4))] * 4)]
    for n in (2, 3, 5, 10, 64, 1000):
        out.append(case(f"uniform{n}", [R.encode_bposit16(Fraction(1, n))] * n))
    for n in (16, 256, 1024):
        w = [rng.random() for _ in range(n)]
        t = sum(w)
        out.append(case(f"random{n}", [R.encode_bposit16(Fraction(x / t)) for x in w]))
    out.append(case("mixed512", [rng.randrange(65536) for _ in range(508)] + [0, 0x8000, 0x7FFF, 0x8001]))
    allc = case("all_codes", range(65536))
    allc["codes"] = "range(65536)"
    out.append(allc)
    return out


FIXTURES = {
    "kat_quire_to_bp16.json": kat_quire_to_bp16,
    "kat_quire_to_bp32.json": kat_quire_to_bp32,
    "kat_int32_to_bp32.json": kat_int32_to_bp32,
    "kat_add.json": lambda: kat_binary("kernels/test_cases_add_inline.h", 21),
    "kat_mul.json": lambda: kat_binary("kernels/test_cases_mul_inline.h", 24),
    "kat_unary.json": lambda: {op: kat_unary(f"kernels/test_{op}.cu") for op in ("sqrt", "recip", "exp2")},
    "probe_hashes.json": probe,
    "headline.json": headline,
    "pyref_samples.json": pyref_samples,
    "lut_sha256.json": lut_hashes,
    "bposit8.json": bposit8,
    "kat_entropy.json": entropy,
}


def main():
    """All fixtures, or only those named after the reference path."""
    only = sys.argv[2:]
    for name, make in FIXTURES.items():
        if not only or name in only:
            _write(name, make())


if __name__ == "__main__":
    main()
