"""GPU parity of the INT64 accumulator kernels (the exact K-split sums beyond
the INT32 range): widening / accumulating INT32 partials and the epilogue
over an INT64 accumulator, bit for bit against the oracle, including values
far outside INT32 and the saturating bposit range."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_widen_and_accumulate(cuda_lib):
    from mosyne_bposit import ops
    g = torch.Generator(device="cpu").manual_seed(11)
    for n in (1, 3, 4, 1001, 1 << 20):
        a = torch.randint(-(1 << 31), 1 << 31, (n,), generator=g, dtype=torch.int64).to(torch.int32)
        b = torch.randint(-(1 << 31), 1 << 31, (n,), generator=g, dtype=torch.int64).to(torch.int32)
        d = ops.widen_i32(a.cuda())
        ops.widen_i32(b.cuda(), d, accumulate=True)
        ops.widen_i32(b.cuda(), d, accumulate=True)
        want = a.numpy().astype(np.int64) + 2 * b.numpy().astype(np.int64)
        assert np.array_equal(d.cpu().numpy(), want), n
    # an unaligned view takes the scalar path
    base = torch.arange(17, dtype=torch.int32).cuda()
    assert np.array_equal(ops.widen_i32(base[1:].contiguous()).cpu().numpy(), np.arange(1, 17))


@pytest.mark.parametrize("M,N", [(5, 3), (1024, 33), (3000, 7)])
def test_epilogue_i64_matches_oracle(cuda_lib, M, N):
    from mosyne_bposit import _api, ops
    rng = np.random.default_rng(M + N)
    mag = rng.integers(0, 62, (M, N))
    acc = (rng.integers(0, 1 << 62, (M, N), dtype=np.int64) >> (62 - mag).astype(np.int64))
    acc *= np.where(rng.random((M, N)) < 0.5, -1, 1).astype(np.int64)
    acc[0, 0] = 0
    acc[-1, -1] = (1 << 62) + 12345                      # saturates the bposit scale
    xs = (rng.random(M) + 0.5).astype(np.float32)
    ws = (rng.random(N) + 0.5).astype(np.float32)
    a = torch.from_numpy(np.ascontiguousarray(acc.T)).cuda().t()    # column-major [M, N]
    for rtne in (False, True):
        r = ops.epilogue_i64(a, bp32=True, bp16=True, y_dtype=torch.float32,
                             x_scale=torch.from_numpy(xs).cuda(), w_scale=torch.from_numpy(ws).cuda(),
                             rtne32=rtne, rtne16=rtne)
        mode = "rtne" if rtne else "truncate"
        assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32),
                              O.encode_int_array(acc, 0, 32, mode))
        assert np.array_equal(r["bp16"].cpu().numpy().view(np.uint16),
                              O.encode_int_array(acc, 0, 16, mode))
        assert np.array_equal(r["y"].cpu().numpy().view(np.uint32),
                              O.dequant(acc, xs, ws).view(np.uint32))
    r = ops.epilogue_i64(a, bp32=True, scale_shift=12)
    assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(acc, 12, 32))
    assert _api.last_error() == 0


def test_long_k_partials_in_int64_match_exact_sum(cuda_lib):
    """K = 140,000 all-127 codes: the INT32 accumulator would wrap; INT32
    partial GEMMs over K pieces, widened and summed in INT64, give the exact
    dot products (the single-GPU form of the wide K-split)."""
    from mosyne_bposit import ops
    from mosyne_bposit.dist import MAX_EXACT_K
    M, N, K = 64, 48, 140_000
    A = torch.full((M, K), 127, dtype=torch.int8)
    A[::3] = -127
    B = torch.full((N, K), 127, dtype=torch.int8)
    B[::5] = -127                                    # |sums| = 127^2 * K > 2^31
    Ad, Bd = A.cuda(), B.cuda()
    acc64 = torch.empty((N, M), dtype=torch.int64, device="cuda")
    tmp = torch.empty((N, M), dtype=torch.int32, device="cuda")
    for j, k0 in enumerate(range(0, K, MAX_EXACT_K)):
        k1 = min(K, k0 + MAX_EXACT_K)
        ops.gemm_i8(Ad[:, k0:k1].contiguous(), Bd[:, k0:k1].contiguous(), bp32=False, i32=True,
                    out={"i32": tmp.t()})
        ops.widen_i32(tmp, acc64, accumulate=j > 0)
    want = O.gemm_exact(A.numpy(), B.numpy().T)
    assert np.abs(want).max() > 2 ** 31              # beyond INT32
    assert np.array_equal(acc64.t().cpu().numpy(), want)
    r = ops.epilogue_i64(acc64.t(), bp32=True)
    assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(want, 0, 32))
