"""The allocation-free W8A8 entry point, checked on the GPU through the C ABI.

mosyne_bposit_linear_w8a8_noalloc exists for callers that cannot call
cudaMalloc -- e.g. a serving process whose device memory is owned by a
caching allocator or capped by its operator, or a plugin host that forbids raw
device allocations.  It keeps its scratch in a fixed static device array
instead of growing buffers with cudaMalloc.  Its results must equal the
regular mosyne_bposit_linear_w8a8 bit for bit (the tolerance every W8A8 test
here uses), on consecutive calls that reuse the shared array, and it must
not change the device's free memory once its kernels are loaded.

This file sorts last so that a stop-at-first-failure run has already run
every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _case(M, K, N, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    cols = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, cols] *= 20.0
    w = torch.randn(N, K, generator=g) * 0.02          # nn.Linear layout = column-major [K,N]
    return x.t().contiguous().cuda(), w.contiguous().cuda()


def _free_bytes():
    torch.cuda.synchronize()
    free_b, _ = torch.cuda.mem_get_info()
    return free_b


def test_noalloc_matches_regular_entry_point(cuda_lib):
    lib = cuda_lib
    shapes = [(128, 2048, 1100, 0), (77, 320, 300, 1), (2048, 4096, 512, 2)]
    free_after = []
    for M, K, N, seed in shapes:                       # consecutive calls share the scratch
        x_cm, w = _case(M, K, N, seed)
        wq = torch.empty((N, K), dtype=torch.int8, device="cuda")
        ws = torch.empty((N,), dtype=torch.float32, device="cuda")
        assert lib.mosyne_bposit_quantize_weight_per_channel(w.data_ptr(), K, N, wq.data_ptr(),
                                                             ws.data_ptr()) == 0
        y_ref = torch.empty((N, M), dtype=torch.float32, device="cuda")
        assert lib.mosyne_bposit_linear_w8a8(x_cm.data_ptr(), M, K, wq.data_ptr(), ws.data_ptr(),
                                             N, y_ref.data_ptr()) == 0
        y = torch.full((N, M), float("nan"), dtype=torch.float32, device="cuda")
        before = _free_bytes()
        rc = lib.mosyne_bposit_linear_w8a8_noalloc(x_cm.data_ptr(), M, K, wq.data_ptr(),
                                                   ws.data_ptr(), N, y.data_ptr(), None)
        assert rc == 0
        free_after.append((before, _free_bytes()))
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32)), (M, K, N)
    # once the kernels are loaded (first call), calls leave free memory unchanged
    for before, after in free_after[1:]:
        assert after == before


def test_noalloc_rejects_inputs_beyond_its_scratch(cuda_lib):
    lib = cuda_lib
    x = torch.zeros(16, device="cuda")
    w = torch.zeros(16, dtype=torch.int8, device="cuda")
    s = torch.ones(1, device="cuda")
    y = torch.zeros(1, device="cuda")
    # M*K = 2^24 bytes > 8 MiB of int8 scratch; M = 16385 rows > 16384
    assert lib.mosyne_bposit_linear_w8a8_noalloc(x.data_ptr(), 4096, 4096, w.data_ptr(),
                                                 s.data_ptr(), 1, y.data_ptr(), None) == -21
    assert lib.mosyne_bposit_linear_w8a8_noalloc(x.data_ptr(), 16385, 1, w.data_ptr(),
                                                 s.data_ptr(), 1, y.data_ptr(), None) == -21
    assert lib.mosyne_bposit_linear_w8a8_noalloc(x.data_ptr(), 0, 16, w.data_ptr(),
                                                 s.data_ptr(), 1, y.data_ptr(), None) == -20


def _regular_and_noalloc(lib, M, K, N, seed, stream=None):
    x_cm, w = _case(M, K, N, seed)
    wq = torch.empty((N, K), dtype=torch.int8, device="cuda")
    ws = torch.empty((N,), dtype=torch.float32, device="cuda")
    assert lib.mosyne_bposit_quantize_weight_per_channel(w.data_ptr(), K, N, wq.data_ptr(),
                                                         ws.data_ptr()) == 0
    y_ref = torch.empty((N, M), dtype=torch.float32, device="cuda")
    assert lib.mosyne_bposit_linear_w8a8(x_cm.data_ptr(), M, K, wq.data_ptr(), ws.data_ptr(),
                                         N, y_ref.data_ptr()) == 0
    torch.cuda.synchronize()
    y = torch.full((N, M), float("nan"), dtype=torch.float32, device="cuda")
    if stream is None:
        rc = lib.mosyne_bposit_linear_w8a8_noalloc(x_cm.data_ptr(), M, K, wq.data_ptr(),
                                                   ws.data_ptr(), N, y.data_ptr(), None)
    else:
        stream.wait_stream(torch.cuda.current_stream())    # y's fill is done first
        with torch.cuda.stream(stream):
            rc = lib.mosyne_bposit_linear_w8a8_noalloc(x_cm.data_ptr(), M, K, wq.data_ptr(),
                                                       ws.data_ptr(), N, y.data_ptr(),
                                                       stream.cuda_stream)
        stream.synchronize()
    assert rc == 0
    return y, y_ref


def test_noalloc_on_a_caller_stream(cuda_lib):
    s = torch.cuda.Stream()
    for seed in (3, 4):                                 # two calls in a row on that stream
        y, y_ref = _regular_and_noalloc(cuda_lib, 300, 1024, 640, seed, stream=s)
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))


def test_noalloc_at_its_size_limits(cuda_lib):
    # M = 16384 rows and M*K = 8 MiB exactly: the largest accepted input
    y, y_ref = _regular_and_noalloc(cuda_lib, 16384, 512, 256, 5)
    assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))


def test_noalloc_reports_a_wait_that_gave_up(cuda_lib):
    """A bounded device wait on this path that gives up must not go unseen:
    the test hook runs the bounded wait that nothing satisfies against this
    path's error word, and last_error reports -30 once, then clears it."""
    from mosyne_bposit import _api
    lib = cuda_lib
    assert _api.last_error() == 0
    assert lib.mosyne_bposit_debug_noalloc_wait_timeout(2_000_000, None) == 0
    assert _api.last_error() == -30
    assert _api.last_error() == 0
    # the path still works afterwards
    y, y_ref = _regular_and_noalloc(lib, 64, 256, 128, 6)
    assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    assert _api.last_error() == 0

