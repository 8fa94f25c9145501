"""Build-time generator of the bposit16 ALU tables (log2, exp2, sqrt, recip,
term).

The tables follow the reference's definitions exactly
(kernels/build_bposit_luts.py:34-259 over kernels/bposit16_reference.py):

* ``log2[p]``  = bposit16(log2(value(p))) via the float ``math.log2``; NaR for
  zero, NaR and negative codes (bposit16_reference.py:519-531)
* ``sqrt[p]``  = bposit16(math.sqrt(value(p))); 0 -> 0, NaR/negative -> NaR
  (bposit16_reference.py:545-559)
* ``exp2[p]``  = bposit16(2.0 ** value(p)), input clamped to +-48; 0 -> one
  (bposit16_reference.py:562-584)
* ``recip[p]`` = bposit16(1 / value(p)) computed exactly; 0/NaR -> NaR
  (bposit16_reference.py:587-599)
* ``term[p]``  = bposit16(p * log2(p)): NaR where ``log2[p]`` is NaR, else the
  truncated exact product of ``p`` and ``log2[p]`` (kernels/build_bposit_luts.py:
  102-110 with bposit16_reference.py:507-516) -- the Shannon-entropy term

Float results enter the encoder the way the reference's boundary conversion
does: ``Fraction(x).limit_denominator(10**12)`` and then the truncating
encode (bposit16_reference.py:490-494).  That narrowing decides a handful
of codes (values within ~1e-12 of a bposit16 boundary), so it is kept.

The tables are computed once by the build and compiled into the library;
nothing here runs on the hot path.
"""
from __future__ import annotations

import math
from fractions import Fraction

NAR = 0x8000
ONE = 0x4000
TABLE_ORDER = ("log2", "exp2", "sqrt", "recip", "term")   # device table index order


def value16(p: int):
    """Exact value of bposit16 code ``p`` (``None`` for NaR)."""
    p &= 0xFFFF
    if p == 0:
        return Fraction(0)
    if p == NAR:
        return None
    neg = p >> 15
    mag = ((-p) & 0x7FFF) if neg else (p & 0x7FFF)
    lead = mag >> 14
    run = 1
    while run < 15 and ((mag >> (14 - run)) & 1) == lead:
        run += 1
    if run == 15:
        k, e, fbits, fw = (14 if lead else -15), 0, 0, 0
    else:
        k = run - 1 if lead else -run
        left = 14 - run                       # bits after the terminator
        ew = min(3, left)
        e = ((mag >> (left - ew)) & ((1 << ew) - 1)) << (3 - ew) if ew else 0
        fw = left - ew
        fbits = mag & ((1 << fw) - 1)
    exp = 8 * k + e - fw
    num = (1 << fw) | fbits
    v = Fraction(num << exp) if exp >= 0 else Fraction(num, 1 << -exp)
    return -v if neg else v


def encode16(v: Fraction) -> int:
    """Truncating bposit16 encode of an exact rational."""
    if v == 0:
        return 0
    neg = v < 0
    if neg:
        v = -v
    n, d = v.numerator, v.denominator
    t = n.bit_length() - d.bit_length()       # floor(log2 v) or one more
    if (n << max(0, -t)) < (d << max(0, t)):
        t -= 1
    if t > 48:
        field = 0x7FFF
    elif t < -48:
        field = 0x0001
    else:
        k, e = t >> 3, t & 7
        if k >= 0:
            rlen, regime = k + 2, ((1 << (k + 1)) - 1) << (14 - k)
        else:
            rlen, regime = 1 - k, 1 << (15 - (1 - k))
        fw = 15 - rlen - 3
        sh = fw - t
        scaled = (n << sh) // d if sh >= 0 else n // (d << -sh)
        field = regime | (e << fw) | (scaled - (1 << fw))
    return (0x8000 | ((-field) & 0x7FFF)) if neg else field


def encode16_float(x: float) -> int:
    if x == 0:
        return 0
    return encode16(Fraction(x).limit_denominator(10 ** 12))


def _log2(p):
    v = value16(p)
    if v is None or v <= 0:
        return NAR
    return encode16_float(math.log2(float(v)))


def _exp2(p):
    v = value16(p)
    if v is None:
        return NAR
    if v == 0:
        return ONE
    if v >= 49:
        return encode16_float(2.0 ** 48)
    if v <= -49:
        return encode16_float(2.0 ** -48)
    return encode16_float(2.0 ** float(v))


def _sqrt(p):
    v = value16(p)
    if v is None or v < 0:
        return NAR
    if v == 0:
        return 0
    return encode16_float(math.sqrt(float(v)))


def _recip(p):
    v = value16(p)
    if v is None or v == 0:
        return NAR
    return encode16(1 / v)


def _mul_exact(a: int, b: int) -> int:
    """Truncated exact product; zero is checked before NaR
    (bposit16_reference.py:507-516)."""
    va, vb = value16(a), value16(b)
    if va == 0 or vb == 0:
        return 0
    if va is None or vb is None:
        return NAR
    return encode16(va * vb)


def _term_table(log2: list) -> list:
    return [NAR if lg == NAR else _mul_exact(p, lg) for p, lg in enumerate(log2)]


_FUNCS = {"log2": _log2, "exp2": _exp2, "sqrt": _sqrt, "recip": _recip}


def build_table(name: str) -> list:
    if name == "term":
        return _term_table(build_table("log2"))
    f = _FUNCS[name]
    return [f(p) for p in range(65536)]


def build_all() -> dict:
    out = {name: build_table(name) for name in TABLE_ORDER if name != "term"}
    out["term"] = _term_table(out["log2"])
    return {name: out[name] for name in TABLE_ORDER}


def write_c_include(path, tables: dict | None = None) -> None:
    """Write ``kBposit16Tables[len(TABLE_ORDER)][65536]`` as a C include file."""
    tables = tables or build_all()
    lines = ["// generated by mosyne_bposit._tables -- do not edit",
             f"static const uint16_t kBposit16Tables[{len(TABLE_ORDER)}][65536] = {{"]
    for name in TABLE_ORDER:
        t = tables[name]
        lines.append("  { // " + name)
        for i in range(0, 65536, 16):
            lines.append("    " + ",".join(f"0x{v:04x}" for v in t[i:i + 16]) + ",")
        lines.append("  },")
    lines.append("};")
    with open(path, "w") as fh:
        fh.write("\n".join(lines) + "\n")
