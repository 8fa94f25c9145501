"""Bit-exact CPU restatement of the reference's bposit / W8A8 arithmetic.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed CPU
baseline.  The shipped library never imports this module.

Citations are ``file:line`` inside the reference project:

* ``pyref``   = kernels/bposit16_reference.py
* ``enc.cuh`` = kernels/bposit16_encode.cuh
* ``pkglib``  = packages/mosyne_bposit/src/mosyne_bposit/_cuda/libmosyne_bposit.cu
* ``det``     = kernels/test_determinism_headline.cu
* ``i2b``     = kernels/test_int32_to_bposit32.cu

Two layers live here:

1. scalar exact functions on Python ints / ``Fraction`` (the "port" of
   pyref, used on small cases and golden vectors);
2. vectorised numpy functions for full-size arrays (quantisers, exact GEMM,
   dequant, integer -> bposit encoders, exact bposit16 sums), cross-checked
   against layer 1 in tests/test_oracle_pins.py.
"""
from __future__ import annotations

import math
from fractions import Fraction

import numpy as np

QUIRE_FRAC_BITS = 96          # pyref:537
ES = 3                        # pyref:24 (bposit16), pyref:33 (bposit32)
ES8 = 2                       # pyref:151
SCALE_LIMIT = 48              # pyref:412-415 (bp16), pyref:103-106 (bp32)
NAR16 = 0x8000                # pyref:25
NAR32 = 0x80000000            # pyref:34
ONE16 = 0x4000                # pyref:27
MODES = ("truncate", "rtne")

# ---------------------------------------------------------------------------
# Layer 1: scalar exact arithmetic
# ---------------------------------------------------------------------------


def _check_mode(mode: str) -> None:
    if mode not in MODES:
        raise ValueError(f"unknown rounding mode: {mode!r}")   # pyref:392-393


def encode_int(I: int, shift: int, nbits: int, mode: str = "truncate") -> int:
    """bposit<nbits> code of the exact rational ``I / 2**shift``.

    Restates ``_encode_unsigned`` (pyref:378-482; bposit16 truncate and
    RTNE), ``_encode_unsigned_32`` (pyref:93-131; bposit32 truncate), the
    sign handling of ``encode_bposit16`` (pyref:485-503) and
    ``encode_bposit32`` (pyref:134-146), and ``int_to_bposit32`` (i2b:94-112)
    when ``nbits == 32`` and ``shift`` is the fixed-point shift.  The quire
    encoders are ``I = q, shift = 96`` (enc.cuh:113-418).

    ``nbits == 32, mode == "rtne"`` applies the bposit16 RTNE rule
    (enc.cuh:299-311) at the 31-bit field; the reference has no bposit32
    RTNE encoder, so that combination is unpinned.
    """
    _check_mode(mode)
    if I == 0:
        return 0
    n1 = nbits - 1
    fmask = (1 << n1) - 1
    sign = I < 0
    a = -I if sign else I
    msb = a.bit_length() - 1
    scale = msb - shift                      # floor(log2 |value|)
    if scale > SCALE_LIMIT:
        field = fmask                        # +maxpos (pyref:412-413)
    elif scale < -SCALE_LIMIT:
        field = 1                            # +minpos (pyref:414-415)
    else:
        k = scale >> 3                       # regime, useed = 256 (pyref:418)
        e = scale & 7                        # 3 exponent bits (pyref:419)
        if k >= 0:                           # k+1 ones then a 0 (pyref:426-428)
            rlen = k + 2
            regime = ((1 << (k + 1)) - 1) << (n1 - (k + 1))
        else:                                # -k zeros then a 1 (pyref:429-431)
            rlen = 1 - k
            regime = 1 << (n1 - rlen)
        fw = n1 - rlen - 3                   # fraction bits left in the field
        frac = a - (1 << msb)
        drop = msb - fw
        if drop > 0:
            f = frac >> drop
            rem = frac & ((1 << drop) - 1)
            rbit = (rem >> (drop - 1)) & 1
            sticky = (rem & ((1 << (drop - 1)) - 1)) != 0
        else:
            f = frac << (-drop)
            rbit, sticky = 0, False
        field = regime | (e << fw) | f
        if mode == "rtne" and rbit and (sticky or (f & 1)) and field < fmask:
            field += 1                       # pyref:477-480 (saturating)
    if sign:
        field = (-field) & fmask             # pyref:501-502
    return (int(sign) << n1) | field


def encode_fraction(value, nbits: int = 16, mode: str = "truncate") -> int:
    """Exact encode of a rational (``Fraction`` or ``int``); pyref:485-503
    with a non-float argument, pyref:134-146 for nbits=32."""
    _check_mode(mode)
    v = Fraction(value)
    if v == 0:
        return 0
    sign = v < 0
    a = -v if sign else v
    p, q = a.numerator, a.denominator
    t = p.bit_length() - q.bit_length()
    if t >= 0:
        if p < (q << t):
            t -= 1
    elif (p << -t) < q:
        t -= 1
    # a in [2^t, 2^(t+1)).  Take W+1 significant bits and a sticky sentinel.
    W = nbits + 8
    num = p << max(0, W - t)
    den = q << max(0, t - W)
    I = num // den
    sticky = 1 if num - I * den else 0
    I2 = (I << 1) | sticky
    return encode_int(-I2 if sign else I2, W - t + 1, nbits, mode)


_LIMIT_DEN = {8: 10 ** 8, 16: 10 ** 12, 32: 10 ** 16}   # pyref:257, :494, :137


def encode_float_pyref(x: float, nbits: int = 16, mode: str = "truncate") -> int:
    """The reference's float boundary conversion: ``Fraction(x)`` narrowed by
    ``limit_denominator`` before the exact encode (pyref:490-494 for
    bposit16, pyref:135-137 for bposit32)."""
    if x == 0:
        return 0
    v = Fraction(x).limit_denominator(_LIMIT_DEN[nbits])
    if v == 0:
        return 0
    return encode_fraction(v, nbits, mode)


def decode(p: int, nbits: int = 16, es: int = ES):
    """Exact value of a bposit code as a ``Fraction`` (``None`` for NaR).

    Restates decode_bposit16 + decoded_to_fraction (pyref:302-374),
    decode_bposit32 + decoded_to_fraction_32 (pyref:39-90) and the bposit8
    pair (pyref:158-209)."""
    mask = (1 << nbits) - 1
    p &= mask
    if p == 0:
        return Fraction(0)
    if p == 1 << (nbits - 1):
        return None
    n1 = nbits - 1
    sign = p >> n1
    rest = p & ((1 << n1) - 1)
    if sign:
        rest = (-rest) & ((1 << n1) - 1)
    lead = (rest >> (n1 - 1)) & 1
    rs = 0
    while rs < n1 and ((rest >> (n1 - 1 - rs)) & 1) == lead:
        rs += 1
    if rs == n1:
        k = (n1 - 1) if lead else -n1
        e, fw, fb = 0, 0, 0
    else:
        k = (rs - 1) if lead else -rs
        remaining = n1 - (rs + 1)
        rest2 = rest & ((1 << remaining) - 1)
        ew = min(es, remaining)
        e = (((rest2 >> (remaining - ew)) & ((1 << ew) - 1)) << (es - ew)) if ew > 0 else 0
        remaining -= ew
        fw = remaining
        fb = rest2 & ((1 << fw) - 1) if fw > 0 else 0
    useed = Fraction(1 << (1 << es))
    val = useed ** k * Fraction(1 << e) * Fraction((1 << fw) + fb, 1 << fw)
    return -val if sign else val


def bposit16_to_quire(p: int) -> int:
    """pyref:602-609: exact fixed point x 2^96, truncated toward zero
    (only codes below 2^-96 lose bits)."""
    v = decode(p, 16)
    if v is None or v == 0:
        return 0
    return int(v * (1 << QUIRE_FRAC_BITS))


def bposit8_to_quire(p: int) -> int:
    """pyref:281-287."""
    v = decode(p, 8, ES8)
    if v is None or v == 0:
        return 0
    return int(v * (1 << QUIRE_FRAC_BITS))


def bposit8_to_int8(p: int) -> int:
    """bposit8 -> int8 fixed point, 6 fraction bits, as the reference builds
    its decode table (kernels/test_mera_isometry_imma.cu:166-197) from the
    bposit8 quire table words (kernels/build_bposit_luts.py:302-311): the
    signed high word w[1] (bit 63 forced on when the quire is negative)
    shifted right by 26 (floor), clamped to [-128, 127]."""
    w = quire_to_words(bposit8_to_quire(p))
    hi = w[1] - (1 << 64) if w[1] >> 63 else w[1]
    if (w[3] >> 63) and hi >= 0:
        hi -= 1 << 63
    v = hi >> (QUIRE_FRAC_BITS - 6 - 64)
    return max(-128, min(127, v))


def bposit8_to_int8_array(codes) -> np.ndarray:
    """Vectorised bposit8_to_int8 over a uint8 array."""
    tab = np.array([bposit8_to_int8(i) for i in range(256)], dtype=np.int8)
    return tab[np.asarray(codes, dtype=np.uint8)]


def quire_to_bposit(q: int, nbits: int = 16, mode: str = "truncate") -> int:
    """quire256 (signed int, 96 fraction bits) -> bposit.  pyref:616-631
    (bp16), pyref:775-794 (bp32), enc.cuh:113-204 / 221-321 / 333-418."""
    return encode_int(q, QUIRE_FRAC_BITS, nbits, mode)


def quire_to_words(q: int) -> tuple:
    """256-bit two's complement, four little-endian u64 words (enc.cuh:30)."""
    q &= (1 << 256) - 1
    return tuple((q >> (64 * i)) & 0xFFFFFFFFFFFFFFFF for i in range(4))


def words_to_quire(w) -> int:
    q = 0
    for i in range(4):
        q |= (int(w[i]) & 0xFFFFFFFFFFFFFFFF) << (64 * i)
    if q >> 255:
        q -= 1 << 256
    return q


# ----- bposit16 ALU (pyref port) -------------------------------------------


def neg16(x: int) -> int:
    """enc.cuh:437-443."""
    if x in (0, NAR16):
        return x
    return (-x) & 0xFFFF


def neg16_ones_complement(x: int) -> int:
    """enc.cuh:461-467."""
    if x in (0, NAR16):
        return x
    return (~x) & 0xFFFF


def log2_16(p: int) -> int:
    """pyref:519-531."""
    v = decode(p, 16)
    if v is None or v <= 0:
        return NAR16
    return encode_float_pyref(math.log2(float(v)), 16)


def sqrt16(p: int) -> int:
    """pyref:545-559."""
    v = decode(p, 16)
    if v is None:
        return NAR16
    if v == 0:
        return 0
    if v < 0:
        return NAR16
    return encode_float_pyref(math.sqrt(float(v)), 16)


def exp2_16(p: int) -> int:
    """pyref:562-584."""
    v = decode(p, 16)
    if v is None:
        return NAR16
    if v == 0:
        return ONE16
    if v >= 49:
        return encode_float_pyref(2.0 ** 48, 16)
    if v <= -49:
        return encode_float_pyref(2.0 ** -48, 16)
    return encode_float_pyref(2.0 ** float(v), 16)


def recip16(p: int) -> int:
    """pyref:587-599."""
    v = decode(p, 16)
    if v is None or v == 0:
        return NAR16
    return encode_fraction(Fraction(1) / v, 16)


def mul16_exact(a: int, b: int) -> int:
    """pyref:507-516 (zero is checked before NaR, as there)."""
    va, vb = decode(a, 16), decode(b, 16)
    if va == 0 or vb == 0:
        return 0
    if va is None or vb is None:
        return NAR16
    return encode_fraction(va * vb, 16)


def add16(a: int, b: int) -> int:
    """pyref:758-772 / enc.cuh:472-483."""
    if a == NAR16 or b == NAR16:
        return NAR16
    if a == 0:
        return b
    if b == 0:
        return a
    return quire_to_bposit(bposit16_to_quire(a) + bposit16_to_quire(b), 16)


def mul16(a: int, b: int, log2_tab=None, exp2_tab=None) -> int:
    """pyref:634-677 / enc.cuh:491-537 (log2 + quire add + exp2)."""
    if a == NAR16 or b == NAR16:
        return NAR16
    if a == 0 or b == 0:
        return 0
    if a == ONE16:
        return b
    if b == ONE16:
        return a
    rs = ((a >> 15) ^ (b >> 15)) & 1

    def absb(x):
        return x if not (x >> 15) else ((-x) & 0x7FFF)

    lg = log2_tab.__getitem__ if log2_tab is not None else log2_16
    ex = exp2_tab.__getitem__ if exp2_tab is not None else exp2_16
    la, lb = lg(absb(a)), lg(absb(b))
    log_sum = quire_to_bposit(bposit16_to_quire(la) + bposit16_to_quire(lb), 16)
    mag = ex(log_sum)
    if mag == NAR16 or mag == 0:
        return mag
    return ((-mag) & 0xFFFF) if rs else mag


def build_tables() -> dict:
    """The 65,536-entry bposit16 ALU tables (kernels/build_bposit_luts.py:34-286)."""
    log2 = [log2_16(i) for i in range(65536)]
    return {
        "log2": log2,
        "exp2": [exp2_16(i) for i in range(65536)],
        "sqrt": [sqrt16(i) for i in range(65536)],
        "recip": [recip16(i) for i in range(65536)],
        "term": [NAR16 if log2[i] == NAR16 else mul16_exact(i, log2[i]) for i in range(65536)],
        "square": [mul16_exact(i, i) for i in range(65536)],
    }


# ---------------------------------------------------------------------------
# Layer 2: vectorised numpy
# ---------------------------------------------------------------------------

_F127 = np.float32(127.0)
_EPS = np.float32(1e-8)


def quant_scale(amax: np.ndarray) -> np.ndarray:
    """``127.f / max`` in fp32, 1.0 when max <= 1e-8 (pkglib:170, :234)."""
    amax = np.asarray(amax, dtype=np.float32)
    with np.errstate(divide="ignore"):
        s = _F127 / np.where(amax > _EPS, amax, np.float32(1.0))
    return np.where(amax > _EPS, s, np.float32(1.0)).astype(np.float32)


def quantize(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """``rint(clamp(x*s, +-127))`` in fp32 (pkglib:178-180, :240-242)."""
    v = (np.asarray(x, dtype=np.float32) * np.asarray(scale, dtype=np.float32)).astype(np.float32)
    v = np.minimum(_F127, np.maximum(-_F127, v))
    return np.rint(v).astype(np.int8)


def quant_per_token(x: np.ndarray):
    """Row-wise (token) scales over a logical [M,K] array; pkglib:206-244."""
    x = np.asarray(x, dtype=np.float32)
    s = quant_scale(np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], np.float32))
    return quantize(x, s[:, None]), s


def quant_per_channel(w: np.ndarray):
    """Column-wise (output channel) scales over a logical [K,N] array;
    pkglib:162-181."""
    w = np.asarray(w, dtype=np.float32)
    s = quant_scale(np.abs(w).max(axis=0) if w.shape[0] else np.zeros(w.shape[1], np.float32))
    return quantize(w, s[None, :]), s


def quant_per_tensor(t: np.ndarray):
    """One scale for the whole tensor, with the per-token convention
    (inverse scale 127/max, multiply, clamp, rint); the reference has no
    data-dependent per-tensor kernel (closest: test_ffn_layer_perch.cu:84-92)."""
    t = np.asarray(t, dtype=np.float32)
    s = quant_scale(np.float32(np.abs(t).max()) if t.size else np.float32(0))
    return quantize(t, s), np.float32(s)


def gemm_exact(a_i8: np.ndarray, b_i8: np.ndarray) -> np.ndarray:
    """Exact ``C = A @ B`` as int64 (the value cuBLASLt's COMPUTE_32I IMMA
    returns, pkglib:274-319).  float64 BLAS is exact while every partial sum
    stays below 2^53, which 127*127*K guarantees for K < 5.5e11."""
    K = a_i8.shape[1]
    assert 127 * 127 * max(K, 1) < 2 ** 53
    c = np.asarray(a_i8, dtype=np.float64) @ np.asarray(b_i8, dtype=np.float64)
    return c.astype(np.int64)


def dequant(acc: np.ndarray, xs: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """``(float)y_i32 / (x_scale[i] * w_scale[j])`` in fp32 (pkglib:252-262)."""
    xs = np.asarray(xs, dtype=np.float32)
    ws = np.asarray(ws, dtype=np.float32)
    den = (xs.reshape(-1, 1) * ws.reshape(1, -1)).astype(np.float32)
    return (np.asarray(acc).astype(np.float32) / den).astype(np.float32)


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """``silu(g) * u`` with ``silu(v) = v / (1 + exp(-v))`` in fp32
    (kernels/test_ffn_layer_real_qwen.cu:101-108).  The reference evaluates
    CUDA's ``expf``; numpy's float32 ``exp`` may differ from it in the last
    place, so this stage is compared within a tolerance."""
    g = np.asarray(g, dtype=np.float32)
    with np.errstate(over="ignore"):
        e = np.exp(-g).astype(np.float32)
    return ((g / (np.float32(1) + e)).astype(np.float32) * np.asarray(u, np.float32)).astype(np.float32)


def ffn_swiglu_w8a8(x: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray):
    """The W8A8 SwiGLU FFN of kernels/test_ffn_layer_real_qwen.cu:300-334 on
    row-major x [M, D] and nn.Linear weights (gate/up [F, D], down [D, F]).
    Returns (y, act, xq, xs) with every stage in fp32 as the reference does."""
    xq, xs = quant_per_token(x)
    gq, gs = quant_per_channel(np.asarray(w_gate, np.float32).T)
    uq, us = quant_per_channel(np.asarray(w_up, np.float32).T)
    dq, ds = quant_per_channel(np.asarray(w_down, np.float32).T)
    g = dequant(gemm_exact(xq, gq), xs, gs)
    u = dequant(gemm_exact(xq, uq), xs, us)
    act = swiglu(g, u)
    hq, hs = quant_per_token(act)
    y = dequant(gemm_exact(hq, dq), hs, ds)
    return y, act, xq, xs


def f32_to_bf16_bits(y: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit pattern (``__float2bfloat16``)."""
    u = np.ascontiguousarray(y, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def linear_w8a8(x: np.ndarray, w: np.ndarray):
    """The reference's W8A8 linear (pkglib:183-193 + 322-348) on logical
    row-major x [M,K] and w [K,N]: per-channel weight quant, per-token
    activation quant, exact INT32 GEMM, fp32 dequant.  Returns
    ``(y_f32, acc_int64, xq, xs, wq, ws)``."""
    wq, ws = quant_per_channel(w)
    xq, xs = quant_per_token(x)
    acc = gemm_exact(xq, wq)
    return dequant(acc, xs, ws), acc, xq, xs, wq, ws


def _bit_length_u64(a: np.ndarray) -> np.ndarray:
    """Exact floor(log2(a)) + 1 for uint64 a > 0 (0 for a == 0)."""
    a = np.asarray(a, dtype=np.uint64)
    f = np.floor(np.log2(np.maximum(a, 1).astype(np.float64))).astype(np.int64)
    f = np.clip(f, 0, 63)
    one = np.uint64(1)
    too_big = (one << f.astype(np.uint64)) > a
    f = np.where(too_big, f - 1, f)
    f1 = np.clip(f + 1, 0, 63)
    too_small = ((one << f1.astype(np.uint64)) <= a) & (f + 1 <= 63)
    f = np.where(too_small, f + 1, f)
    return np.where(a == 0, 0, f + 1)


def encode_int_array(I: np.ndarray, shift, nbits: int, mode: str = "truncate") -> np.ndarray:
    """Vectorised :func:`encode_int` for int64 ``I`` (|I| < 2^63) and an int
    or int-array ``shift``.  Returns uint16 (nbits=16) or uint32 codes."""
    _check_mode(mode)
    I = np.asarray(I, dtype=np.int64)
    shift = np.asarray(shift, dtype=np.int64)
    n1 = nbits - 1
    fmask = np.int64((1 << n1) - 1)
    sign = I < 0
    a = np.abs(I).astype(np.uint64)
    zero = a == 0
    msb = _bit_length_u64(a) - 1
    msb = np.where(zero, 0, msb)
    scale = msb - shift
    k = scale >> 3
    e = scale & 7
    kc = np.clip(k, -6, 6)
    rlen = np.where(kc >= 0, kc + 2, 1 - kc)
    ones = (np.int64(1) << (kc + 1).clip(0, 62)) - 1
    regime = np.where(kc >= 0, ones << (n1 - (kc + 1)).clip(0, 62), np.int64(1) << (n1 - rlen).clip(0, 62))
    fw = n1 - rlen - 3
    frac = (a - (np.uint64(1) << msb.astype(np.uint64))).astype(np.uint64)
    drop = msb - fw
    dpos = np.clip(drop, 0, 63).astype(np.uint64)
    dneg = np.clip(-drop, 0, 63).astype(np.uint64)
    f_drop = (frac >> dpos).astype(np.int64)
    rem = frac & ((np.uint64(1) << dpos) - np.uint64(1))
    rsh = np.clip(drop - 1, 0, 63).astype(np.uint64)
    rbit = np.where(drop > 0, (rem >> rsh) & np.uint64(1), np.uint64(0)).astype(np.int64)
    sticky = np.where(drop > 1, (rem & ((np.uint64(1) << rsh) - np.uint64(1))) != 0, False)
    f = np.where(drop > 0, f_drop, (frac << dneg).astype(np.int64))
    field = regime | (e << fw.clip(0, 62)) | f
    if mode == "rtne":
        up = (rbit == 1) & (sticky | ((f & 1) == 1)) & (field < fmask)
        field = np.where(up, field + 1, field)
    field = np.where(scale > SCALE_LIMIT, fmask, field)
    field = np.where(scale < -SCALE_LIMIT, np.int64(1), field)
    field = np.where(sign, (-field) & fmask, field)
    out = (sign.astype(np.int64) << n1) | field
    out = np.where(zero, 0, out)
    return out.astype(np.uint16 if nbits == 16 else np.uint32)


def int_to_bposit32_array(I: np.ndarray, scale_shift: int = 0, mode: str = "truncate") -> np.ndarray:
    """i2b:94-112 over an int array (value = I / 2^scale_shift)."""
    return encode_int_array(I, scale_shift, 32, mode)


def float_to_bposit_array(x: np.ndarray, nbits: int = 16, mode: str = "truncate") -> np.ndarray:
    """Exact rounding of binary floating-point values (the exact rational
    each fp64/fp32 number denotes, i.e. ``encode_bposit16(Fraction(v))``)."""
    x = np.asarray(x, dtype=np.float64)
    m, e = np.frexp(x)                              # x = m * 2^e, |m| in [0.5, 1)
    I = np.round(m * 2.0 ** 53).astype(np.int64)    # exact: 53-bit significand
    return encode_int_array(I, 53 - e.astype(np.int64), nbits, mode)


def bposit16_decode_array(p: np.ndarray):
    """Vectorised bposit16 -> (signed mantissa int64, power-of-two shift)
    such that the quire value is ``trunc(mant * 2**shift)`` with
    ``shift`` relative to the quire's 2^-96 unit (pyref:602-609)."""
    p = np.asarray(p, dtype=np.uint16).astype(np.int64)
    sign = (p >> 15) & 1
    rest = p & 0x7FFF
    rest = np.where(sign == 1, (-rest) & 0x7FFF, rest)
    lead = (rest >> 14) & 1
    x = np.where(lead == 1, (~rest) & 0x7FFF, rest)      # leading run -> zeros
    blen = _bit_length_u64(x.astype(np.uint64))           # 0..15
    rs = 15 - blen                                        # run length
    full = rs >= 15
    k = np.where(lead == 1, rs - 1, -rs)
    k = np.where(full, np.where(lead == 1, 14, -15), k)
    remaining = np.clip(15 - (rs + 1), 0, 15)
    rest2 = rest & ((np.int64(1) << remaining) - 1)
    ew = np.minimum(3, remaining)
    e = np.where(ew > 0, ((rest2 >> (remaining - ew)) & ((np.int64(1) << ew) - 1)) << (3 - ew), 0)
    fw = remaining - ew
    fb = rest2 & ((np.int64(1) << fw) - 1)
    e = np.where(full, 0, e)
    fw = np.where(full, 0, fw)
    fb = np.where(full, 0, fb)
    mant = (np.int64(1) << fw) + fb
    shift = 8 * k + e - fw + QUIRE_FRAC_BITS
    special = (p == 0) | (p == NAR16)
    mant = np.where(special, 0, mant)
    # values below the quire's LSB truncate toward zero
    neg_sh = np.clip(-shift, 0, 62)
    mant = np.where(shift < 0, mant >> neg_sh, mant)
    shift = np.where(shift < 0, 0, shift)
    mant = np.where(sign == 1, -mant, mant)
    return mant, shift


def quire_sum_bposit16(p: np.ndarray) -> int:
    """Exact sum of bposit16 codes as a quire integer (det:65-91, the order
    independent integer reduction), computed by binning equal shifts."""
    mant, shift = bposit16_decode_array(p)
    total = 0
    for s in np.unique(shift):
        sel = shift == s
        total += int(mant[sel].sum(dtype=np.int64)) << int(s)
    return total


_TERM_TABLE = None


def term_table() -> np.ndarray:
    """bposit16(p * log2(p)) for every code p (kernels/build_bposit_luts.py:
    102-110): NaR where log2 is NaR, else the truncated exact product."""
    global _TERM_TABLE
    if _TERM_TABLE is None:
        t = [NAR16 if (lg := log2_16(i)) == NAR16 else mul16_exact(i, lg) for i in range(65536)]
        _TERM_TABLE = np.asarray(t, dtype=np.uint16)
    return _TERM_TABLE


def shannon_entropy_quire(p: np.ndarray) -> int:
    """H = -sum quire(term(p_i)) as a quire integer (pyref:813-824; the kernel
    kernels/shannon_entropy_bposit16.cu:63-119 negates the sum once, which is
    the same two's-complement value)."""
    codes = term_table()[np.asarray(p, dtype=np.uint16)]
    return -quire_sum_bposit16(codes)


def shannon_entropy_bposit(p: np.ndarray, nbits: int = 32, mode: str = "truncate") -> int:
    """bposit encoding of :func:`shannon_entropy_quire` (the reference returns
    ``quire256_to_bposit32``, truncating: pyref:824, shannon:112-118)."""
    return quire_to_bposit(shannon_entropy_quire(p), nbits, mode)


# ----- determinism headline inputs (det:110-189) ----------------------------


def det_encode_bposit16_host(v: float) -> int:
    """det:110-148: the headline's float64 truncating encoder (not pyref)."""
    if v == 0.0:
        return 0
    sign = 1 if v < 0 else 0
    a = -v if sign else v
    e2 = math.floor(math.log2(a))
    if e2 > 48:
        return 0x8001 if sign else 0x7FFF
    if e2 < -48:
        return 0xFFFF if sign else 0x0001
    if e2 >= 0:
        k, ef = e2 // 8, e2 % 8
    else:
        ae = -e2
        ak, aem = ae // 8, ae % 8
        k, ef = (-ak, 0) if aem == 0 else (-ak - 1, 8 - aem)
    frac = a / math.pow(2.0, float(e2)) - 1.0
    mag = 0
    if k >= 0:
        ones = min(k + 1, 14)
        mag |= ((1 << ones) - 1) << (15 - ones)
        top = 14 - (ones + 1)
    else:
        zeros = min(-k, 14)
        mag |= 1 << (14 - zeros)
        top = 14 - zeros - 1
    eb = 3 if top + 1 >= 3 else (top + 1 if top + 1 > 0 else 0)
    if eb > 0:
        mag |= (ef >> (3 - eb)) << (top - eb + 1)
    fb = top - eb + 1 if top - eb + 1 > 0 else 0
    if fb > 0:
        ff = int(frac * float(1 << fb))
        if ff >= (1 << fb):
            ff = (1 << fb) - 1
        mag |= ff
    if sign:
        mag = (-mag) & 0x7FFF
    return (sign << 15) | mag


def det_headline_inputs(n: int = 65536, seed: int = 0x5EED1234):
    """det:181-189: LCG log-uniform values on [1e-3, 1e3] and their bposit16
    codes.  Returns (float64 values, float32 values, uint16 codes)."""
    vals = np.empty(n, dtype=np.float64)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u = float(s >> 1) / float(0x7FFFFFFF)
        vals[i] = math.pow(10.0, -3.0 + 6.0 * u)
    codes = np.array([det_encode_bposit16_host(float(v)) for v in vals], dtype=np.uint16)
    return vals, vals.astype(np.float32), codes


def exact_sum_inputs(n: int, seed: int = 0):
    """The exact-reduction workload: magnitudes 2^U, U ~ Uniform[-24, 24],
    random signs, rounded RTNE to bposit16 from the exact float64 value.
    Returns (float64 values, uint16 codes)."""
    rng = np.random.default_rng(seed)
    u = rng.uniform(-24.0, 24.0, n)
    sg = rng.integers(0, 2, n)
    v = np.where(sg == 1, -1.0, 1.0) * np.exp2(u)
    return v, float_to_bposit_array(v, 16, "rtne")
