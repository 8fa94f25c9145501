"""GPU parity: the fused tcgen05 INT8 GEMM vs the oracle.

INT32 accumulators, bposit32/bposit16 codes (truncate and RTNE) and the
dequantised fp32/bf16/fp16 outputs are compared bit for bit.  Ragged shapes
cover partial tiles in M, N and K; K not a multiple of 16 takes the CUDA-core
path.  The full-size check compares the 4096^3 INT32 result with cuBLAS's
exact integer GEMM and bposit32 codes on a sample against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = [
    (128, 256, 128), (1, 1, 16), (7, 9, 32), (129, 257, 144), (300, 520, 1040),
    (256, 512, 2048), (64, 1000, 4096), (513, 130, 64),
]


def _rand_i8(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)


def _np(t, dtype=None):
    a = t.cpu().contiguous().numpy()
    return a.view(dtype) if dtype is not None else a


def _check_all(M, N, K, path=0, row_major=False, seed=0):
    from mosyne_bposit import ops
    A = _rand_i8((M, K), seed)
    B = _rand_i8((N, K), seed + 1)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) * 3 + 0.01
    ws = torch.rand(N, dtype=torch.float32) * 2 + 0.01
    Ad, Bd = A.cuda(), B.cuda()
    for rt in (False, True):
        r = ops.gemm_i8(Ad, Bd, bp32=True, bp16=True, i32=True, y_dtype=torch.float32,
                        x_scale=xs.cuda(), w_scale=ws.cuda(), rtne32=rt, rtne16=rt,
                        row_major=row_major, path=path)
        torch.cuda.synchronize()
        mode = "rtne" if rt else "truncate"
        assert np.array_equal(_np(r["i32"]).astype(np.int64), acc), (M, N, K, path)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32, mode))
        assert np.array_equal(_np(r["bp16"], np.uint16), O.encode_int_array(acc, 0, 16, mode))
        y = O.dequant(acc, xs.numpy(), ws.numpy())
        assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32))
    for ydt in (torch.bfloat16, torch.float16):
        r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=ydt, x_scale=xs.cuda(), w_scale=ws.cuda(),
                        row_major=row_major, path=path)
        y = O.dequant(acc, xs.numpy(), ws.numpy())
        if ydt == torch.bfloat16:
            assert np.array_equal(_np(r["y"].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y))
        else:
            assert np.array_equal(_np(r["y"]).view(np.uint16), y.astype(np.float16).view(np.uint16))
    from mosyne_bposit import _api
    assert _api.last_error() == 0


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_tc_auto(cuda_lib, M, N, K):
    _check_all(M, N, K)


@pytest.mark.parametrize("path", [2, 3, 5])   # one-CTA tile width 128 / 256, CTA pair
def test_gemm_tc_tile_widths(cuda_lib, path):
    _check_all(300, 600, 512, path=path)
    _check_all(1024, 1024, 256, path=path)
    _check_all(64, 200, 160, path=path)
    _check_all(777, 257, 2064, path=path, row_major=True)


def _check_single(M, N, K, tail, row_major, seed=3):
    """Every single-output epilogue of the CTA-pair kernel (bposit32 truncate
    and RTNE, fp32/bf16 dequant, bposit16, INT32), with the last wave cut
    into whole, half or quarter tiles."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((M, K), seed)
    B = _rand_i8((N, K), seed + 1)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) * 3 + 0.01
    ws = torch.rand(N, dtype=torch.float32) * 2 + 0.01
    Ad, Bd, xd, wd = A.cuda(), B.cuda(), xs.cuda(), ws.cuda()
    kw = dict(row_major=row_major, path=5, tail=tail)
    y = O.dequant(acc, xs.numpy(), ws.numpy())
    for rt in (False, True):
        r = ops.gemm_i8(Ad, Bd, bp32=True, rtne32=rt, **kw)
        want = O.encode_int_array(acc, 0, 32, "rtne" if rt else "truncate")
        assert np.array_equal(_np(r["bp32"], np.uint32), want), (M, N, K, tail, rt)
    r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=torch.float32, x_scale=xd, w_scale=wd, **kw)
    assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32)), (M, N, K, tail)
    r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=torch.bfloat16, x_scale=xd, w_scale=wd, **kw)
    assert np.array_equal(_np(r["y"].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y))
    r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=torch.float16, x_scale=xd, w_scale=wd, **kw)
    with np.errstate(over="ignore"):
        assert np.array_equal(_np(r["y"]).view(np.uint16), y.astype(np.float16).view(np.uint16))
    r = ops.gemm_i8(Ad, Bd, bp32=False, bp16=True, **kw)
    assert np.array_equal(_np(r["bp16"], np.uint16), O.encode_int_array(acc, 0, 16, "truncate"))
    r = ops.gemm_i8(Ad, Bd, bp32=False, i32=True, **kw)
    assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
    assert _api.last_error() == 0


# M % 4 == 0 column-major 4-byte outputs go through TMA stores, the others
# through direct stores; N ragged against every cut width.
@pytest.mark.parametrize("tail", [0, 1, 2, 3])
@pytest.mark.parametrize("M,N,K", [(300, 600, 512), (258, 300, 256), (1024, 1000, 256),
                                   (2560, 2304, 128)])
def test_gemm_pair_single_outputs(cuda_lib, M, N, K, tail):
    _check_single(M, N, K, tail, row_major=False)


# row-major outputs: N % 8 == 0 takes TMA stores for 4- and 2-byte outputs,
# N % 4 == 0 for 4-byte ones only, other N direct stores
@pytest.mark.parametrize("tail", [1, 2, 3])
@pytest.mark.parametrize("M,N,K", [(516, 777, 384), (516, 776, 384), (300, 1000, 256),
                                   (2560, 2304, 128), (257, 1028, 128)])
def test_gemm_pair_single_outputs_row_major(cuda_lib, M, N, K, tail):
    _check_single(M, N, K, tail, row_major=True)


def test_gemm_row_major_outputs(cuda_lib):
    _check_all(200, 300, 256, row_major=True)


@pytest.mark.parametrize("M,N,K", [(33, 65, 100), (5, 3, 1), (128, 256, 40)])
def test_gemm_simt_path(cuda_lib, M, N, K):
    _check_all(M, N, K)          # K % 16 != 0 -> CUDA-core path
    if K % 16 == 0:
        _check_all(M, N, K, path=4)


def test_gemm_scalar_scales(cuda_lib):
    from mosyne_bposit import ops
    M, N, K = 130, 250, 192
    A, B = _rand_i8((M, K), 5), _rand_i8((N, K), 6)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.tensor([0.37], dtype=torch.float32)
    ws = torch.tensor([2.5], dtype=torch.float32)
    r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=False, y_dtype=torch.float32, x_scale=xs.cuda(),
                    w_scale=ws.cuda())
    y = O.dequant(acc, np.full(M, 0.37, np.float32), np.full(N, 2.5, np.float32))
    assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("path", [2, 5])   # one-CTA tiles, CTA pairs
def test_gemm_scales_outside_fast_divide_range(cuda_lib, path):
    """Blocks whose scales leave [2^-45, 2^46) take the IEEE divide, the others
    the slow-path-free one: tiny and huge scales (subnormal and infinite
    quotients among the outputs), scattered over rows and columns, fp32 y
    against the oracle's IEEE division bit for bit."""
    from mosyne_bposit import ops
    M, N, K = 300, 520, 256
    A, B = _rand_i8((M, K), 21), _rand_i8((N, K), 22)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) * 3 + 0.01
    ws = torch.rand(N, dtype=torch.float32) * 2 + 0.01
    xs[::37] = 1e-20
    xs[5] = 3e25
    ws[::53] = 2e-19
    ws[100:116] = 1e30
    for row_major in (False, True):
        r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=True, y_dtype=torch.float32, x_scale=xs.cuda(),
                        w_scale=ws.cuda(), row_major=row_major, path=path)
        with np.errstate(over="ignore", under="ignore", divide="ignore", invalid="ignore"):
            y = O.dequant(acc, xs.numpy(), ws.numpy())
        assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32)), row_major
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))


def test_gemm_extreme_values(cuda_lib):
    """All -127 / +127 operands: |acc| = 127^2 K at the top of the int32
    range used, every output the same sign."""
    from mosyne_bposit import ops
    M, N, K = 128, 256, 8192
    A = torch.full((M, K), -127, dtype=torch.int8)
    B = torch.full((N, K), 127, dtype=torch.int8)
    r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=True, i32=True)
    acc = np.full((M, N), -127 * 127 * K, dtype=np.int64)
    assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
    assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))


def test_gemm_full_size_4096(cuda_lib):
    """4096^3 (the headline shape): INT32 equal to cuBLAS's exact integer GEMM;
    bposit32 codes equal to the oracle's on 2^16 sampled outputs and
    consistent with encoding the INT32 output everywhere."""
    from mosyne_bposit import ops
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8, device="cuda")
    B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8, device="cuda")
    r = ops.gemm_i8(A, B, bp32=True, i32=True)
    ref = torch._int_mm(A, B.t())
    assert torch.equal(r["i32"], ref)
    enc = ops.int32_to_bp32(r["i32"].t().contiguous()).t()
    assert torch.equal(enc, r["bp32"])
    rng = np.random.default_rng(1)
    idx = rng.integers(0, M * N, 1 << 16)
    mi, ni = idx // N, idx % N
    acc = ref.cpu().numpy().astype(np.int64)[mi, ni]
    got = r["bp32"].cpu().numpy().view(np.uint32)[mi, ni]
    assert np.array_equal(got, O.encode_int_array(acc, 0, 32))
    from mosyne_bposit import _api
    assert _api.last_error() == 0


def test_gemm_bad_args(cuda_lib):
    from mosyne_bposit import _api
    lib = cuda_lib
    assert lib.mosyne_bposit_gemm_i8(0, 0, 4, 4, 16, 0, 0, 0, 0, 0, 0, 0, 0, 0) == -20
    a = torch.zeros((4, 16), dtype=torch.int8, device="cuda")
    assert lib.mosyne_bposit_gemm_i8(a.data_ptr(), a.data_ptr(), 0, 4, 16, 0, 0, 0, 0, 0, 0, 0,
                                     0, 0) == -20
    # dequant output without scales
    y = torch.empty((4, 4), device="cuda")
    assert lib.mosyne_bposit_gemm_i8(a.data_ptr(), a.data_ptr(), 4, 4, 16, 0, 0, 0, 0,
                                     y.data_ptr(), 0, 0, 0, 0) == -20
    assert _api.last_error() == 0


@pytest.mark.parametrize("M,N,K", [(300, 3000, 256), (64, 200, 512), (1024, 4096, 128),
                                   (2100, 4100, 96), (4096, 1536, 64)])
def test_gemm_host_buffers(cuda_lib, M, N, K):
    """The host-buffer entry point (uploads, GEMM and downloads pipelined over
    blocks of output channels, the first block also cut along M into pieces
    with strided downloads; a ragged last piece and block) returns the
    oracle's INT32 and bposit32 codes, column-major [N, M]."""
    from mosyne_bposit import _api
    A = _rand_i8((M, K), 11).numpy()
    B = _rand_i8((N, K), 12).numpy()
    for rt in (0, _api.RTNE_BP32):
        bp, i32 = _api.gemm_i8_host(A, B, want_i32=True, flags=rt)
        acc = O.gemm_exact(A, B.T)
        assert i32.shape == (M, N) and np.array_equal(i32.astype(np.int64), acc)
        want = O.encode_int_array(acc, 0, 32, "rtne" if rt else "truncate")
        assert np.array_equal(np.asarray(bp).view(np.uint32), want)
    assert _api.last_error() == 0


def test_gemm_host_buffers_from_two_threads(cuda_lib):
    """Host threads calling the host-buffer entry point at once (it shares the
    device's staging buffers, one call at a time) each get their own exact
    result."""
    import threading
    from mosyne_bposit import _api
    cases = [(_rand_i8((300, 256), 31 + i).numpy(), _rand_i8((1500, 256), 41 + i).numpy())
             for i in range(4)]
    results = [None] * len(cases)

    def run(i):
        dev = torch.cuda.current_device()
        torch.cuda.set_device(dev)
        for _ in range(3):
            results[i] = _api.gemm_i8_host(cases[i][0], cases[i][1], want_i32=True)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(cases))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for (A, B), (bp, i32) in zip(cases, results):
        acc = O.gemm_exact(A, B.T)
        assert np.array_equal(i32.astype(np.int64), acc)
        assert np.array_equal(np.asarray(bp).view(np.uint32), O.encode_int_array(acc, 0, 32))
    assert _api.last_error() == 0


@pytest.mark.parametrize("shift", [6, 12, 31])
def test_gemm_scale_shift(cuda_lib, shift):
    """bposit outputs of acc / 2^shift (negative scales included) on every
    path: CTA pair (TMA-store and direct-store epilogues), single CTA, CUDA
    cores, and the generic multi-output epilogue."""
    from mosyne_bposit import _api, ops
    for (M, N, K), path in (((300, 600, 512), 5), ((258, 300, 256), 5), ((64, 200, 160), 0),
                            ((70, 90, 40), 4)):
        A = _rand_i8((M, K), shift)
        B = _rand_i8((N, K), shift + 1)
        acc = O.gemm_exact(A.numpy(), B.numpy().T)
        Ad, Bd = A.cuda(), B.cuda()
        for rt in (False, True):
            mode = "rtne" if rt else "truncate"
            r = ops.gemm_i8(Ad, Bd, bp32=True, rtne32=rt, path=path, scale_shift=shift)
            assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, shift, 32, mode)), \
                (M, N, K, path, rt)
            r = ops.gemm_i8(Ad, Bd, bp32=True, bp16=True, i32=True, rtne32=rt, rtne16=rt, path=path,
                            scale_shift=shift)
            assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, shift, 32, mode))
            assert np.array_equal(_np(r["bp16"], np.uint16), O.encode_int_array(acc, shift, 16, mode))
            assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
    assert _api.last_error() == 0


def test_gemm_bposit8_in_bposit32_out(cuda_lib):
    """bposit8 operands -> int8 decode -> exact GEMM -> bposit32 of acc / 2^12,
    the reference's bposit8 IMMA pipeline, against the oracle."""
    from mosyne_bposit import _api, ops
    g = torch.Generator(device="cpu").manual_seed(88)
    # (both operands decoded in one launch: whole 16-byte vectors, ragged
    # sizes with unaligned tails, K not a multiple of 16 -> CUDA-core GEMM)
    for M, N, K, rm in ((512, 768, 1024, False), (37, 50, 64, False), (300, 257, 2000, True),
                        (129, 65, 72, False), (64, 96, 40, True)):
        A = torch.randint(0, 256, (M, K), generator=g, dtype=torch.int32).to(torch.uint8)
        B = torch.randint(0, 256, (N, K), generator=g, dtype=torch.int32).to(torch.uint8)
        r = ops.gemm_bposit8(A.cuda(), B.cuda(), i32=True, row_major=rm)
        a8 = O.bposit8_to_int8_array(A.numpy())
        b8 = O.bposit8_to_int8_array(B.numpy())
        acc = O.gemm_exact(a8, b8.T)
        assert np.array_equal(_np(r["i32"]).astype(np.int64), acc), (M, N, K)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 12, 32))
        rt = ops.gemm_bposit8(A.cuda(), B.cuda(), rtne32=True)
        assert np.array_equal(_np(rt["bp32"], np.uint32), O.encode_int_array(acc, 12, 32, "rtne"))
    assert _api.last_error() == 0


@pytest.mark.parametrize("split", [2, 3, 5, 7])
@pytest.mark.parametrize("M,N,K,path", [(128, 1100, 2048, 3), (77, 600, 1040, 2), (300, 520, 1536, 3)])
def test_gemm_single_cta_split_k(cuda_lib, M, N, K, path, split):
    """Single-CTA kernel with K cut into slices run as one cluster per tile,
    the exact INT32 partials summed through distributed shared memory: every
    output kind, both layouts, slices of one or two k-blocks."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((M, K), split)
    B = _rand_i8((N, K), split + 10)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) * 3 + 0.01
    ws = torch.rand(N, dtype=torch.float32) * 2 + 0.01
    y = O.dequant(acc, xs.numpy(), ws.numpy())
    Ad, Bd, xd, wd = A.cuda(), B.cuda(), xs.cuda(), ws.cuda()
    for rm in (False, True):
        kw = dict(row_major=rm, path=path, split=split)
        r = ops.gemm_i8(Ad, Bd, bp32=True, **kw)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32)), (rm,)
        r = ops.gemm_i8(Ad, Bd, bp32=True, y_dtype=torch.float32, x_scale=xd, w_scale=wd, **kw)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))
        assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32))
        r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=torch.bfloat16, x_scale=xd, w_scale=wd, **kw)
        assert np.array_equal(_np(r["y"].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y))
        r = ops.gemm_i8(Ad, Bd, bp32=True, bp16=True, i32=True, rtne32=True, **kw)
        assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32, "rtne"))
    # repeated calls
    for _ in range(3):
        r = ops.gemm_i8(Ad, Bd, bp32=False, i32=True, path=path, split=split)
        assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
    assert _api.last_error() == 0


@pytest.mark.parametrize("M,N,K", [(32, 4096, 4096), (128, 4096, 11008), (1, 2048, 8192),
                                   (128, 11008, 2048)])
def test_gemm_decode_shapes_auto_split(cuda_lib, M, N, K):
    """Decode-like shapes (few rows, long K) where the kernel picks K slices
    itself: bposit32 and fp32 outputs against the oracle."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((M, K), 21)
    B = _rand_i8((N, K), 22)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) + 0.5
    ws = torch.rand(N, dtype=torch.float32) + 0.5
    r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=True, y_dtype=torch.float32, x_scale=xs.cuda(),
                    w_scale=ws.cuda(), row_major=True)
    assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))
    y = O.dequant(acc, xs.numpy(), ws.numpy())
    assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32))
    assert _api.last_error() == 0


def test_gemm_fp32_and_bposit32_outputs(cuda_lib):
    """The two-output epilogue (fp32 dequant + bposit32 of the same dot
    products) on both kernels and layouts."""
    from mosyne_bposit import _api, ops
    for (M, N, K), path in (((300, 1000, 512), 5), ((96, 1000, 512), 0), ((128, 11008, 2048), 0)):
        A = _rand_i8((M, K), 4)
        B = _rand_i8((N, K), 5)
        acc = O.gemm_exact(A.numpy(), B.numpy().T)
        xs = torch.rand(M, dtype=torch.float32) + 0.5
        ws = torch.rand(N, dtype=torch.float32) + 0.5
        y = O.dequant(acc, xs.numpy(), ws.numpy())
        for rm in (False, True):
            r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=True, y_dtype=torch.float32, x_scale=xs.cuda(),
                            w_scale=ws.cuda(), row_major=rm, path=path)
            assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32)), (M, rm)
            assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32)), (M, rm)
    assert _api.last_error() == 0


@pytest.mark.parametrize("b,M,N,K", [(3, 300, 260, 128), (4, 64, 96, 64), (2, 512, 512, 256)])
def test_gemm_batched(cuda_lib, b, M, N, K):
    """Independent GEMMs per batch entry (attention scores per head), every
    output kind, both layouts, per-entry and scalar scales."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((b, M, K), 21)
    B = _rand_i8((b, N, K), 22)
    xs = torch.rand(b, M) + 0.5
    ws = torch.rand(b, N) + 0.5
    for rm in (False, True):
        r = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=True, i32=True, y_dtype=torch.float32,
                                x_scale=xs.cuda(), w_scale=ws.cuda(), row_major=rm)
        r2 = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=False, y_dtype=torch.bfloat16,
                                 x_scale=xs.cuda(), w_scale=torch.tensor([0.75]).cuda(),
                                 row_major=rm)
        for h in range(b):
            acc = O.gemm_exact(A[h].numpy(), B[h].numpy().T)
            assert np.array_equal(_np(r["i32"][h]).astype(np.int64), acc), (h, rm)
            assert np.array_equal(_np(r["bp32"][h], np.uint32), O.encode_int_array(acc, 0, 32))
            y = O.dequant(acc, xs[h].numpy(), ws[h].numpy())
            assert np.array_equal(_np(r["y"][h]).view(np.uint32), y.view(np.uint32))
            y2 = O.dequant(acc, xs[h].numpy(), np.full(N, 0.75, np.float32))
            assert np.array_equal(_np(r2["y"][h].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y2))
    assert _api.last_error() == 0


@pytest.mark.parametrize("b,M,N,K", [(3, 300, 260, 128), (5, 512, 700, 256), (2, 1024, 96, 64)])
def test_gemm_batched_one_launch(cuda_lib, b, M, N, K):
    """Batches the CTA-pair kernel takes in one launch (M > 128, one or two
    TMA-stored outputs): bposit32, fp32 + bposit32, bf16, both layouts where
    the strides allow TMA stores, per-entry and scalar scales."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((b, M, K), 31)
    B = _rand_i8((b, N, K), 32)
    xs = torch.rand(b, M) + 0.5
    ws = torch.rand(b, N) + 0.5
    accs = [O.gemm_exact(A[h].numpy(), B[h].numpy().T) for h in range(b)]
    for rm in (False, True):
        r = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=True, row_major=rm)
        r2 = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=True, y_dtype=torch.float32,
                                 x_scale=xs.cuda(), w_scale=ws.cuda(), row_major=rm)
        r3 = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=False, y_dtype=torch.bfloat16,
                                 x_scale=torch.tensor([1.5]).cuda(), w_scale=ws.cuda(),
                                 row_major=rm)
        for h in range(b):
            acc = accs[h]
            want = O.encode_int_array(acc, 0, 32)
            assert np.array_equal(_np(r["bp32"][h], np.uint32), want), (h, rm)
            assert np.array_equal(_np(r2["bp32"][h], np.uint32), want), (h, rm)
            y = O.dequant(acc, xs[h].numpy(), ws[h].numpy())
            assert np.array_equal(_np(r2["y"][h]).view(np.uint32), y.view(np.uint32)), (h, rm)
            y3 = O.dequant(acc, np.full(M, 1.5, np.float32), ws[h].numpy())
            assert np.array_equal(_np(r3["y"][h].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y3))
    assert _api.last_error() == 0


def _check_stream_k(M, N, K, seed=11):
    """The CTA-pair kernel's stream-K phase (k-block ranges of the last tiles
    shared over all pairs, exact INT32 partial tiles combined by the pair
    that owns each tile) against the oracle and against the same kernel
    without it, for every single output and fp32 + bposit32 together."""
    from mosyne_bposit import _api, ops
    A = _rand_i8((M, K), seed)
    B = _rand_i8((N, K), seed + 1)
    acc = O.gemm_exact(A.numpy(), B.numpy().T)
    xs = torch.rand(M, dtype=torch.float32) * 3 + 0.01
    ws = torch.rand(N, dtype=torch.float32) * 2 + 0.01
    Ad, Bd, xd, wd = A.cuda(), B.cuda(), xs.cuda(), ws.cuda()
    y = O.dequant(acc, xs.numpy(), ws.numpy())
    for rm in (False, True):
        kw = dict(row_major=rm, path=5, stream_k=True)
        for rt in (False, True):
            r = ops.gemm_i8(Ad, Bd, bp32=True, rtne32=rt, **kw)
            want = O.encode_int_array(acc, 0, 32, "rtne" if rt else "truncate")
            assert np.array_equal(_np(r["bp32"], np.uint32), want), (M, N, K, rm, rt)
        r = ops.gemm_i8(Ad, Bd, bp32=True, y_dtype=torch.float32, x_scale=xd, w_scale=wd, **kw)
        assert np.array_equal(_np(r["y"]).view(np.uint32), y.view(np.uint32)), (M, N, K, rm)
        assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))
        r = ops.gemm_i8(Ad, Bd, bp32=False, y_dtype=torch.bfloat16, x_scale=xd, w_scale=wd, **kw)
        assert np.array_equal(_np(r["y"].view(torch.int16), np.uint16), O.f32_to_bf16_bits(y))
        r = ops.gemm_i8(Ad, Bd, bp32=False, bp16=True, i32=True, **kw)
        assert np.array_equal(_np(r["i32"]).astype(np.int64), acc)
        assert np.array_equal(_np(r["bp16"], np.uint16), O.encode_int_array(acc, 0, 16))
        r2 = ops.gemm_i8(Ad, Bd, bp32=False, i32=True, **dict(kw, stream_k=False))
        assert np.array_equal(_np(r2["i32"]).astype(np.int64), acc)
    # repeated launches reuse the workspace and its ready flags
    for _ in range(3):
        r = ops.gemm_i8(Ad, Bd, bp32=True, path=5, stream_k=True)
    assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))
    assert _api.last_error() == 0


# (all tiles stream-K, ~14 k-blocks a pair), (whole waves then a stream-K
# phase of one wave plus the partial one), (ragged M, N, K), (fewer tiles
# than pairs, K of 2 k-blocks)
@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (4096, 5120, 1024), (1000, 3000, 4112),
                                   (700, 900, 256), (512, 4608, 8192)])
def test_gemm_pair_stream_k(cuda_lib, M, N, K):
    _check_stream_k(M, N, K)


def test_gemm_batched_stream_k(cuda_lib):
    from mosyne_bposit import ops
    b, M, N, K = 3, 300, 500, 640
    A = _rand_i8((b, M, K), 21)
    B = _rand_i8((b, N, K), 22)
    xs = torch.rand(b, M) + 0.5
    ws = torch.rand(b, N) + 0.5
    r = ops.gemm_i8_batched(A.cuda(), B.cuda(), bp32=True, y_dtype=torch.float32,
                            x_scale=xs.cuda(), w_scale=ws.cuda())
    torch.cuda.synchronize()
    for z in range(b):
        acc = O.gemm_exact(A[z].numpy(), B[z].numpy().T)
        assert np.array_equal(_np(r["bp32"][z], np.uint32), O.encode_int_array(acc, 0, 32))
        y = O.dequant(acc, xs[z].numpy(), ws[z].numpy())
        assert np.array_equal(_np(r["y"][z]).view(np.uint32), y.view(np.uint32))



def test_gemm_sm_count_target(cuda_lib):
    """With an SM-count target the GEMMs launch smaller persistent grids (the
    K-split leaves the other SMs to NCCL); results are unchanged."""
    from mosyne_bposit import _api, ops
    try:
        for target in (40, 7, 2):
            _api.set_sm_count_target(target)
            for (M, N, K) in ((1024, 1500, 512), (100, 700, 1024)):
                A = _rand_i8((M, K), target + M)
                B = _rand_i8((N, K), target + N)
                acc = O.gemm_exact(A.numpy(), B.numpy().T)
                r = ops.gemm_i8(A.cuda(), B.cuda(), bp32=True, i32=True)
                assert np.array_equal(_np(r["i32"]).astype(np.int64), acc), (target, M, N, K)
                assert np.array_equal(_np(r["bp32"], np.uint32), O.encode_int_array(acc, 0, 32))
    finally:
        _api.set_sm_count_target(0)
    assert _api.last_error() == 0
