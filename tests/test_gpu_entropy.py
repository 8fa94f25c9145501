"""GPU parity: Shannon entropy of bposit16 probabilities (term table + exact
quire256 sum) vs the oracle and the reference's own golden vectors
(kernels/shannon_entropy_bposit16.cu, bposit16_reference.py:813-824)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _codes(case):
    if case["codes"] == "range(65536)":
        return np.arange(65536, dtype=np.uint16)
    return np.asarray(case["codes"], dtype=np.uint16)


def _entropy(codes_np, **kw):
    from mosyne_bposit import ops
    x = torch.from_numpy(codes_np.view(np.int16).copy()).cuda()
    q, b32, b16 = ops.shannon_entropy_bp16(x, **kw)
    torch.cuda.synchronize()
    return (O.words_to_quire(q.cpu().numpy().view(np.uint64)),
            int(b32.cpu().numpy().view(np.uint32)[0]), int(b16.cpu().numpy().view(np.uint16)[0]))


def test_device_term_table(cuda_lib, golden):
    """The device copy of bposit16(p * log2(p)) is the reference's table
    (SHA-256 of kernels/build_bposit_luts.py's term LUT)."""
    import hashlib
    out = np.zeros(65536, dtype=np.uint16)
    assert cuda_lib.mosyne_bposit16_table_host(4, out.ctypes.data_as(ctypes.c_void_p)) == 0
    assert hashlib.sha256(out.astype("<u2").tobytes()).hexdigest() == golden("lut_sha256.json")["term"]


def test_entropy_reference_goldens(cuda_lib, golden):
    """Every case the reference's integer pipeline produced (uniform and
    random distributions, mixed and saturating codes, all 65,536 codes):
    the same quire and the same bposit32."""
    for case in golden("kat_entropy.json"):
        codes = _codes(case)
        q, b32, b16 = _entropy(codes)
        assert [f"{x:016x}" for x in O.quire_to_words(q)] == case["quire_words"], case["name"]
        assert b32 == case["bp32"], case["name"]
        assert b16 == O.quire_to_bposit(q, 16), case["name"]


def test_reference_entry_point(cuda_lib, golden):
    """shannon_entropy_bposit16_cuda (kernels/shannon_entropy_bposit16.cu:124-146):
    same symbol, arguments and return codes; the result is in place on return."""
    lib = cuda_lib
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for case in golden("kat_entropy.json"):
        codes = _codes(case)
        x = torch.from_numpy(codes.view(np.int16).copy()).cuda()
        torch.cuda.synchronize()
        assert lib.shannon_entropy_bposit16_cuda(x.data_ptr(), x.numel(), out.data_ptr()) == 0
        assert int(out.cpu().numpy().view(np.uint32)[0]) == case["bp32"], case["name"]
    assert lib.shannon_entropy_bposit16_cuda(out.data_ptr(), 0, out.data_ptr()) == -1


@pytest.mark.parametrize("n", [1, 7, 8, 9, 4096, 65537, 1_000_003])
def test_entropy_sizes_and_modes(cuda_lib, n):
    """Normalised random distributions of many sizes (ragged tails), every
    output and both rounding modes."""
    rng = np.random.default_rng(n)
    w = rng.random(n)
    codes = O.float_to_bposit_array(w / w.sum(), 16, "truncate")
    ref = O.shannon_entropy_quire(codes)
    q, b32, b16 = _entropy(codes)
    assert q == ref
    assert b32 == O.quire_to_bposit(ref, 32) and b16 == O.quire_to_bposit(ref, 16)
    _, b32r, b16r = _entropy(codes, rtne32=True, rtne16=True)
    assert b32r == O.quire_to_bposit(ref, 32, "rtne") and b16r == O.quire_to_bposit(ref, 16, "rtne")


def test_entropy_large_grid_independent(cuda_lib):
    """2^22 mixed codes (zero, NaR, negatives, saturating terms): the quire
    is the same for any grid, and unaligned starts take the scalar path."""
    from mosyne_bposit import ops
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 65536, (1 << 22) + 5).astype(np.uint16)
    ref = O.shannon_entropy_quire(codes)
    results = {_entropy(codes, max_blocks=mb) for mb in (0, 1, 5, 148)}
    assert len(results) == 1
    assert results.pop()[0] == ref
    x = torch.from_numpy(codes.view(np.int16).copy()).cuda()
    q, _, _ = ops.shannon_entropy_bp16(x[3:])
    assert O.words_to_quire(q.cpu().numpy().view(np.uint64)) == O.shannon_entropy_quire(codes[3:])


def test_entropy_empty(cuda_lib):
    from mosyne_bposit import ops
    x = torch.zeros(4, dtype=torch.int16, device="cuda")
    q, b32, b16 = ops.shannon_entropy_bp16(x[:0])
    assert int(q.abs().sum()) == 0 and int(b32) == 0 and int(b16) == 0
