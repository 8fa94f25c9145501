"""GPU parity: element-wise bposit conversions vs the oracle (bit-exact)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _words_tensor(qs):
    w = np.array([O.quire_to_words(q) for q in qs], dtype=np.uint64).view(np.int64)
    return torch.from_numpy(w.copy()).cuda()


def _u(t, bits):
    a = t.cpu().numpy()
    return a.view(np.uint16 if bits == 16 else np.uint32)


def _quires(golden):
    qs = [int(c["q"]) for c in golden("pyref_samples.json")["quire"]]
    for name in ("kat_quire_to_bp16.json", "kat_quire_to_bp32.json"):
        qs += [O.words_to_quire([int(w, 16) for w in c["w"]]) for c in golden(name)]
    rng = np.random.default_rng(21)
    for _ in range(20000):
        bits = int(rng.integers(0, 252))
        v = int.from_bytes(rng.bytes(32), "little") & ((1 << bits) - 1)
        qs.append(-v if rng.integers(0, 2) else v)
    return qs


def test_quire_to_bposit_kats(cuda_lib, golden):
    from mosyne_bposit import ops
    for name, nb in (("kat_quire_to_bp16.json", 16), ("kat_quire_to_bp32.json", 32)):
        cases = golden(name)
        q = _words_tensor([O.words_to_quire([int(w, 16) for w in c["w"]]) for c in cases])
        got = _u(ops.quire_to_bposit(q, nb), nb)
        assert [int(g) for g in got] == [c["expected"] for c in cases], name


def test_quire_to_bposit_random(cuda_lib, golden):
    from mosyne_bposit import ops
    qs = _quires(golden)
    qt = _words_tensor(qs)
    for nb in (16, 32):
        for mode in O.MODES:
            got = _u(ops.quire_to_bposit(qt, nb, rtne=(mode == "rtne")), nb)
            exp = np.array([O.quire_to_bposit(q, nb, mode) for q in qs])
            bad = np.nonzero(got.astype(np.int64) != exp)[0]
            assert bad.size == 0, (nb, mode, [hex(qs[i]) for i in bad[:4]])


def test_bp16_to_quire_all_codes(cuda_lib):
    from mosyne_bposit import ops
    codes = torch.arange(65536, dtype=torch.int32).to(torch.int16).cuda()
    w = ops.bp16_to_quire(codes).cpu().numpy().view(np.uint64)
    for p in range(65536):
        assert O.words_to_quire(w[p]) == O.bposit16_to_quire(p), p


def test_int32_to_bp32(cuda_lib, golden):
    from mosyne_bposit import ops
    for c in golden("kat_int32_to_bp32.json"):
        x = torch.tensor([c["input"]], dtype=torch.int32).cuda()
        assert int(_u(ops.int32_to_bp32(x, c["scale_shift"]), 32)[0]) == c["expected"]
    rng = np.random.default_rng(22)
    I = np.concatenate([rng.integers(-(2 ** 31), 2 ** 31, 200000),
                        np.array([0, 1, -1, 2 ** 31 - 1, -(2 ** 31)])]).astype(np.int32)
    xt = torch.from_numpy(I).cuda()
    for sh in (0, 12, 24, 31, 60):
        for mode in O.MODES:
            got = _u(ops.int32_to_bp32(xt, sh, rtne=(mode == "rtne")), 32)
            exp = O.encode_int_array(I.astype(np.int64), sh, 32, mode)
            assert np.array_equal(got, exp), (sh, mode)


def test_float_to_bposit(cuda_lib, golden):
    from mosyne_bposit import ops
    rng = np.random.default_rng(23)
    x = np.concatenate([rng.standard_normal(100000) * 10.0 ** rng.integers(-18, 18, 100000),
                        np.array([0.0, 2.0 ** 48, 2.0 ** 49, 2.0 ** -48, -2.0 ** -49, 1.0, -1.0]),
                        np.array([float.fromhex(c["x"]) for c in golden("pyref_samples.json")["float"]])])
    for dt in (np.float64, np.float32):
        xv = x.astype(dt)
        xt = torch.from_numpy(xv).cuda()
        for nb in (16, 32):
            for mode in O.MODES:
                got = _u(ops.float_to_bposit(xt, nb, rtne=(mode == "rtne")), nb)
                exp = O.float_to_bposit_array(xv.astype(np.float64), nb, mode)
                assert np.array_equal(got, exp), (dt, nb, mode)


@pytest.mark.parametrize("M,N", [(256, 48), (130, 7)])
def test_epilogue_i32(cuda_lib, M, N):
    """The standalone epilogue over a column-major INT32 accumulator (the
    K-split's exact sum): M % 4 == 0 takes the 16-byte vector kernel, other
    M the per-element one; bposit32/16 in both roundings, fp32 and bf16
    dequant, per-row and scalar scales."""
    from mosyne_bposit import ops
    rng = np.random.default_rng(24)
    acc = rng.integers(-(2 ** 31), 2 ** 31, (M, N)).astype(np.int32)
    acc[0, :4] = [0, 1, -1, -(2 ** 31)]
    acc[1, :3] = [2 ** 31 - 1, 1 << 24, -(1 << 24) - 1]
    xs = (rng.random(M) + 0.5).astype(np.float32)
    ws = (rng.random(N) + 0.5).astype(np.float32)
    a_t, xs_t, ws_t = torch.from_numpy(acc).cuda(), torch.from_numpy(xs).cuda(), torch.from_numpy(ws).cuda()
    y_ref = O.dequant(acc.astype(np.int64), xs, ws)
    for mode in O.MODES:
        r = ops.epilogue_i32(a_t, bp32=True, bp16=True, y_dtype=torch.float32, x_scale=xs_t,
                             w_scale=ws_t, rtne32=(mode == "rtne"), rtne16=(mode == "rtne"))
        assert np.array_equal(_u(r["bp32"], 32), O.encode_int_array(acc.astype(np.int64), 0, 32, mode))
        assert np.array_equal(_u(r["bp16"], 16), O.encode_int_array(acc.astype(np.int64), 0, 16, mode))
        assert np.array_equal(r["y"].cpu().numpy().view(np.uint32), y_ref.view(np.uint32))
    rb = ops.epilogue_i32(a_t, bp32=False, y_dtype=torch.bfloat16, x_scale=xs_t[:1], w_scale=ws_t)
    y1 = O.dequant(acc.astype(np.int64), np.full(M, xs[0], np.float32), ws)
    assert torch.equal(rb["y"].cpu(), torch.from_numpy(y1).to(torch.bfloat16))


def test_empty_inputs(cuda_lib):
    from mosyne_bposit import ops
    z = torch.empty((0,), dtype=torch.int32, device="cuda")
    assert ops.int32_to_bp32(z).numel() == 0
    assert ops.bp16_to_quire(torch.empty((0,), dtype=torch.int16, device="cuda")).shape == (0, 4)


def test_bposit8_to_int8(cuda_lib, golden):
    """bposit8 -> int8 decode: every code against the reference's table, and
    a large ragged buffer through the vector path (same alignment phase on
    both sides) and the byte path (different phases)."""
    from mosyne_bposit import _api, ops
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).cuda()
    want = np.array(golden("bposit8.json")["to_int8"], dtype=np.int8)
    assert np.array_equal(ops.bposit8_to_int8(codes).cpu().numpy(), want)
    g = torch.Generator(device="cpu").manual_seed(8)
    n = (1 << 24) + 37
    big = torch.randint(0, 256, (n + 64,), generator=g, dtype=torch.int32).to(torch.uint8)
    ref = O.bposit8_to_int8_array(big.numpy())
    src = big.cuda()
    out = torch.full((n + 64,), 99, dtype=torch.int8, device="cuda")
    for si, oi in ((0, 0), (5, 5), (3, 7), (1, 0)):
        out.fill_(99)
        _api.bposit8_to_int8_dev(src[si:].data_ptr(), n, out[oi:].data_ptr())
        got = out.cpu().numpy()
        assert np.array_equal(got[oi:oi + n], ref[si:si + n]), (si, oi)
        assert (got[:oi] == 99).all() and (got[oi + n:] == 99).all(), (si, oi)
    assert _api.last_error() == 0
