"""GPU parity: exact quire256 sums (the determinism workload) vs the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _sum(codes_np, **kw):
    from mosyne_bposit import ops
    x = torch.from_numpy(codes_np.view(np.int16).copy()).cuda()
    q, b16, b32 = ops.quire_sum_bp16(x, **kw)
    torch.cuda.synchronize()
    w = q.cpu().numpy().view(np.uint64)
    return O.words_to_quire(w), int(b16.cpu().numpy().view(np.uint16)[0]), \
        int(b32.cpu().numpy().view(np.uint32)[0])


def test_determinism_headline(cuda_lib, golden):
    """kernels/test_determinism_headline.cu: 65,536 log-uniform values, five
    runs, one bit pattern: quire w[1] = 0x0049ec1830468000, bposit16 0x7627."""
    h = golden("headline.json")
    _, vals_f, codes = O.det_headline_inputs()
    seen = set()
    for run in range(5):
        q, b16, b32 = _sum(codes)
        seen.add((q, b16, b32))
    assert len(seen) == 1
    q, b16, b32 = seen.pop()
    assert [f"{x:016x}" for x in O.quire_to_words(q)] == h["quire_words"]
    assert b16 == h["published_bp16"] == 0x7627
    assert b32 == h["pyref_bp32"]
    # the IEEE control arm runs and lands near the exact value
    from mosyne_bposit import ops
    xf = torch.from_numpy(vals_f).cuda()
    s = float(ops.fp32_atomic_sum(xf).item())
    assert abs(s - float(np.sum(vals_f.astype(np.float64)))) / abs(s) < 1e-4


def test_determinism_headline_every_gpu(cuda_lib, golden):
    """The headline's cross-GPU claim: five runs on EVERY visible GPU of the
    box give one bit pattern (demo.sh:66-78 loops the headline binary over
    the GPUs; det:233-252 is the five-run loop)."""
    from mosyne_bposit import ops
    h = golden("headline.json")
    _, _, codes = O.det_headline_inputs()
    seen = {}
    for d in range(torch.cuda.device_count()):
        with torch.cuda.device(d):
            x = torch.from_numpy(codes.view(np.int16).copy()).to(f"cuda:{d}")
            for run in range(5):
                q, b16, b32 = ops.quire_sum_bp16(x)
                seen[(d, run)] = (bytes(q.cpu().numpy().tobytes()),
                                  int(b16.cpu().numpy().view(np.uint16)[0]),
                                  int(b32.cpu().numpy().view(np.uint32)[0]))
    assert len(seen) == 5 * torch.cuda.device_count()
    patterns = set(seen.values())
    assert len(patterns) == 1
    qb, b16, b32 = patterns.pop()
    w = np.frombuffer(qb, dtype=np.uint64)
    assert [f"{int(x):016x}" for x in w] == h["quire_words"]
    assert b16 == h["published_bp16"] and b32 == h["pyref_bp32"]


@pytest.mark.parametrize("n", [1, 2, 7, 8, 9, 1000, 65536, 1_000_003])
def test_exact_sum_sizes(cuda_lib, n):
    _, codes = O.exact_sum_inputs(n, seed=n)
    q, b16, b32 = _sum(codes)
    ref = O.quire_sum_bposit16(codes)
    assert q == ref
    assert b16 == O.quire_to_bposit(ref, 16)
    assert b32 == O.quire_to_bposit(ref, 32)
    _, b16r, b32r = _sum(codes, rtne16=True, rtne32=True)
    assert b16r == O.quire_to_bposit(ref, 16, "rtne")
    assert b32r == O.quire_to_bposit(ref, 32, "rtne")


def test_exact_sum_2_24_grid_independent(cuda_lib):
    """2^24 values; the quire is identical for any grid size (integer
    addition is associative)."""
    _, codes = O.exact_sum_inputs(1 << 24, seed=0)
    ref = O.quire_sum_bposit16(codes)
    results = {_sum(codes, max_blocks=mb) for mb in (0, 1, 3, 37, 148, 592)}
    assert len(results) == 1
    q, b16, b32 = results.pop()
    assert q == ref
    assert b16 == O.quire_to_bposit(ref, 16)


def test_exact_sum_every_code(cuda_lib):
    """All 65,536 codes (NaR and zero contribute nothing), including the
    extreme regimes whose quire images reach 2^208 and underflow 2^-96."""
    codes = np.arange(65536, dtype=np.uint16)
    q, _, _ = _sum(codes)
    assert q == sum(O.bposit16_to_quire(p) for p in range(65536))
    hi = np.array([0x7FFF] * 1000 + [0x7FFE] * 77, dtype=np.uint16)
    q, b16, _ = _sum(hi)
    assert q == O.quire_sum_bposit16(hi)
    assert b16 == 0x7FFF


def test_exact_sum_decode_every_code(cuda_lib):
    """The device decode each code takes in the exact sum (its regime and the
    signed integer within the regime, formed through one fused multiply-add)
    equals the code's quire image for all 65,536 codes; a sum over every code
    cannot show this, as each code cancels against its negation."""
    from mosyne_bposit import _api
    bad, first = _api.debug_alu_check("sum_decode")
    assert bad == 0, (bad, first)
    pos = np.arange(1, 0x8000, dtype=np.uint16)
    q, _, _ = _sum(pos)
    assert q == sum(O.bposit16_to_quire(p) for p in range(1, 0x8000))
    q, _, _ = _sum((0x10000 - pos.astype(np.uint32)).astype(np.uint16)[::3])
    assert q == -sum(O.bposit16_to_quire(p) for p in range(1, 0x8000, 3))


def test_exact_sum_large_inputs(cuda_lib):
    """Millions of codes: every code (zero, NaR, both extremes of the regime
    range) many times over, a sign-cancelling mix, an unaligned start with an
    odd length, and the whole input in a single block."""
    rng = np.random.default_rng(41)
    allc = np.tile(np.arange(65536, dtype=np.uint16), 33)
    rng.shuffle(allc)
    q, b16, b32 = _sum(allc)
    ref = O.quire_sum_bposit16(allc)
    assert q == ref and b16 == O.quire_to_bposit(ref, 16) and b32 == O.quire_to_bposit(ref, 32)
    pos = rng.integers(1, 0x8000, 1 << 20).astype(np.uint16)
    mixed = np.concatenate([pos, ((65536 - pos.astype(np.int64)) & 0xFFFF).astype(np.uint16),
                            np.array([0x4000, 0x0001, 0x7FFF], dtype=np.uint16)])
    rng.shuffle(mixed)
    q, _, _ = _sum(mixed)
    assert q == O.quire_sum_bposit16(mixed)
    from mosyne_bposit import ops
    _, codes = O.exact_sum_inputs((1 << 21) + 13, seed=9)
    x = torch.from_numpy(codes.view(np.int16).copy()).cuda()
    qd, _, _ = ops.quire_sum_bp16(x[3:])                # 6-byte offset: no 16-byte vectors
    assert O.words_to_quire(qd.cpu().numpy().view(np.uint64)) == O.quire_sum_bposit16(codes[3:])
    q1, _, _ = _sum(codes, max_blocks=1)
    assert q1 == O.quire_sum_bposit16(codes)


def test_unaligned_and_empty(cuda_lib):
    from mosyne_bposit import ops
    _, codes = O.exact_sum_inputs(5001, seed=5)
    x = torch.from_numpy(codes.view(np.int16).copy()).cuda()
    q, b16, _ = ops.quire_sum_bp16(x[1:])          # 2-byte aligned start
    assert O.words_to_quire(q.cpu().numpy().view(np.uint64)) == O.quire_sum_bposit16(codes[1:])
    q, b16, b32 = ops.quire_sum_bp16(x[:0])
    assert int(q.abs().sum()) == 0 and int(b16) == 0 and int(b32) == 0
