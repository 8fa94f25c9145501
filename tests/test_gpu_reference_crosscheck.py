"""Cross-check against the reference's own C-ABI library, built for sm_100a
from its single source file by oracle/build_ref.sh (cuBLASLt IMMA inside):
same inputs through both libraries, outputs compared bit for bit."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

REF_SO = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libmosyne_bposit_ref.so"


@pytest.fixture(scope="module")
def ref_lib():
    if not REF_SO.exists():
        pytest.skip("reference library not built (oracle/build_ref.sh)")
    lib = ctypes.CDLL(str(REF_SO))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.mosyne_bposit_init.restype = I
    lib.mosyne_bposit_quantize_weight_per_channel.argtypes = [P, I, I, P, P]
    for n in ("mosyne_bposit_linear_w8a8", "mosyne_bposit_linear_w8a8_bf16_io"):
        getattr(lib, n).argtypes = [P, I, I, P, P, I, P]
        getattr(lib, n).restype = I
    assert lib.mosyne_bposit_init() == 0
    return lib


@pytest.mark.parametrize("M,K,N", [(128, 2048, 11008), (64, 512, 1024), (300, 1000, 777)])
def test_linear_matches_reference_library(cuda_lib, ref_lib, M, K, N):
    from mosyne_bposit import _api
    g = torch.Generator(device="cpu").manual_seed(M)
    x = torch.randn(M, K, generator=g) * 0.7
    w = torch.randn(N, K, generator=g) * 0.02            # nn.Linear layout = col-major [K,N]
    x_cm = x.t().contiguous().cuda()
    w_cm = w.contiguous().cuda()
    outs = []
    for lib in (ref_lib, cuda_lib):
        wq = torch.empty((N, K), dtype=torch.int8, device="cuda")
        ws = torch.empty((N,), dtype=torch.float32, device="cuda")
        assert lib.mosyne_bposit_quantize_weight_per_channel(w_cm.data_ptr(), K, N, wq.data_ptr(),
                                                             ws.data_ptr()) == 0
        y = torch.empty((N, M), dtype=torch.float32, device="cuda")
        assert lib.mosyne_bposit_linear_w8a8(x_cm.data_ptr(), M, K, wq.data_ptr(), ws.data_ptr(),
                                             N, y.data_ptr()) == 0
        torch.cuda.synchronize()
        outs.append((wq.cpu(), ws.cpu(), y.cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32))
    assert torch.equal(outs[0][2].view(torch.int32), outs[1][2].view(torch.int32))
    assert _api.last_error() == 0
