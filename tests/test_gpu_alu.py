"""GPU parity: the bposit16 ALU (tables, unary and binary ops) vs the
reference's known answers, table hashes and the oracle."""
from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _t(codes):
    return torch.from_numpy(np.asarray(codes, dtype=np.uint16).view(np.int16).copy()).cuda()


def _u(t):
    return t.cpu().numpy().view(np.uint16)


def test_device_tables_match_reference_hashes(cuda_lib, golden):
    from mosyne_bposit import _api
    g = golden("lut_sha256.json")
    for name in ("log2", "exp2", "sqrt", "recip"):
        tab = _api.bposit16_table(name)
        assert hashlib.sha256(struct.pack("<65536H", *tab.tolist())).hexdigest() == g[name], name


def test_unary_ops_all_codes(cuda_lib):
    from mosyne_bposit import _api, ops
    codes = np.arange(65536, dtype=np.uint16)
    big = np.tile(codes, 64)                        # large enough for the staged-table kernel
    for name in ("log2", "exp2", "sqrt", "recip"):
        tab = _api.bposit16_table(name)
        assert np.array_equal(_u(ops.bposit16_op(name, _t(codes))), tab), name
        assert np.array_equal(_u(ops.bposit16_op(name, _t(big))), tab[big]), name
    neg = _u(ops.bposit16_op("neg", _t(codes)))
    assert [int(v) for v in neg[::97]] == [O.neg16(int(p)) for p in codes[::97]]
    n1 = _u(ops.bposit16_op("neg_ones_complement", _t(codes)))
    assert [int(v) for v in n1[::97]] == [O.neg16_ones_complement(int(p)) for p in codes[::97]]


def test_unary_kats(cuda_lib, golden):
    from mosyne_bposit import ops
    for op, cases in golden("kat_unary.json").items():
        got = _u(ops.bposit16_op(op, _t([c["in"] for c in cases])))
        assert [int(v) for v in got] == [c["expected"] for c in cases], op


def test_add_mul_kats(cuda_lib, golden):
    from mosyne_bposit import ops
    for name, op in (("kat_add.json", "add"), ("kat_mul.json", "mul")):
        cases = golden(name)
        got = _u(ops.bposit16_op(op, _t([c["a"] for c in cases]), _t([c["b"] for c in cases])))
        assert [int(v) for v in got] == [c["expected"] for c in cases], op


def test_binary_ops_random(cuda_lib):
    from mosyne_bposit import _api, ops
    rng = np.random.default_rng(31)
    a = rng.integers(0, 65536, 30000).astype(np.uint16)
    b = rng.integers(0, 65536, 30000).astype(np.uint16)
    a[:8] = [0, 0x8000, 0x4000, 0, 0x7FFF, 0x0001, 0xFFFF, 0x8001]
    b[:8] = [0x8000, 0, 0x1234, 0, 0x7FFF, 0x0001, 0x8001, 0xFFFF]
    # cancellation: b next to -a (every third pair is checked below)
    d = rng.integers(-2, 3, 9000)
    b[8:9008] = ((65536 - a[8:9008].astype(np.int64) + d) & 0xFFFF).astype(np.uint16)
    add = _u(ops.bposit16_op("add", _t(a), _t(b)))
    mex = _u(ops.bposit16_op("mul_exact", _t(a), _t(b)))
    mul = _u(ops.bposit16_op("mul", _t(a), _t(b)))
    lg, ex = _api.bposit16_table("log2").tolist(), _api.bposit16_table("exp2").tolist()
    for i in range(0, 30000, 3):
        x, y = int(a[i]), int(b[i])
        assert int(add[i]) == O.add16(x, y), (hex(x), hex(y))
        assert int(mex[i]) == O.mul16_exact(x, y), (hex(x), hex(y))
        assert int(mul[i]) == O.mul16(x, y, lg, ex), (hex(x), hex(y))


@pytest.mark.parametrize("op", ["add", "mul_exact", "quire_sum", "mul"])
def test_alu_32bit_forms_equal_int64_forms_on_every_pair(cuda_lib, op):
    """The adder, the exact multiplier, the quire sum and the log/exp
    multiplier run in 32-bit arithmetic; on all 2^32 pairs of codes they give
    the codes of the int64 forms they replaced (which the oracle pins)."""
    from mosyne_bposit import _api
    bad, first = _api.debug_alu_check(op)
    assert bad == 0, (op, bad, None if first is None else (hex(first >> 16), hex(first & 0xFFFF)))


def test_alu_add_staged_and_unstaged(cuda_lib):
    """The adder reads its decode table from shared memory on large launches
    and through L2 on small ones: both against the oracle."""
    from mosyne_bposit import ops
    rng = np.random.default_rng(31)
    for n in (1000, 148 * 16384 + 77):
        a = rng.integers(0, 65536, n).astype(np.uint16)
        b = rng.integers(0, 65536, n).astype(np.uint16)
        a[:8] = [0, 0x8000, 0x7FFF, 0x8001, 1, 0xFFFF, 0x4000, 0xC000]
        b[:8] = [0x4000, 5, 0x8001, 0x7FFF, 0xFFFF, 1, 0xC000, 0x4000]
        out = _u(ops.bposit16_op("add", _t(a), _t(b)))
        k = min(n, 4000)
        want = np.array([O.add16(int(x), int(y)) for x, y in zip(a[:k], b[:k])], dtype=np.uint16)
        assert np.array_equal(out[:k], want), n
        tail = slice(n - 2000, n)
        want_t = np.array([O.add16(int(x), int(y)) for x, y in zip(a[tail], b[tail])],
                          dtype=np.uint16)
        assert np.array_equal(out[tail], want_t), n


def test_dequant_division_equals_ieee(cuda_lib):
    """The GEMM epilogues divide (float)acc by x_scale * w_scale without a
    slow path when both scales are in [2^-45, 2^46): that division equals
    the IEEE one (__fdiv_rn) on 2^32 pseudo-random pairs spanning every
    exponent of that range, with all-ones and zero significands forced; and
    silu's g / (1 + expf(-g)) where its guard lets the fast divide run; and
    its reciprocal step is the correctly rounded reciprocal for every normal
    divisor in [2^-110, 2^111), the premise of the correction theorem."""
    from mosyne_bposit import _api
    for op in ("div_reciprocal", "dequant_div", "silu_div"):
        bad, first = _api.debug_alu_check(op)
        assert bad == 0, (op, bad, first)

