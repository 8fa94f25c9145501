"""Failure detection without a GPU fault: a bounded device-side wait that
nothing satisfies gives up, records the failure in the device error word,
and the host reads it as rc -30; the context stays usable afterwards."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_bounded_wait_reports_timeout(cuda_lib):
    from mosyne_bposit import _api, ops
    assert _api.last_error() == 0
    _api.debug_wait_timeout(2_000_000)          # 2 ms limit
    assert _api.last_error() == -30
    assert _api.last_error() == 0               # reading clears it
    # the context still works
    a = torch.ones((128, 64), dtype=torch.int8, device="cuda")
    r = ops.gemm_i8(a, a, bp32=False, i32=True)
    assert int(r["i32"][0, 0]) == 64
    assert _api.last_error() == 0


def test_bad_arguments_return_codes(cuda_lib):
    lib = cuda_lib
    assert lib.mosyne_bposit_quire_to_bp16(0, 5, 0, 0, 0) == -20
    assert lib.mosyne_bposit_float_to_bposit(0, 0, 0, 0, 8, 0, 0) == -20
    assert lib.mosyne_bposit16_table_host(9, 0) == -20
    assert lib.mosyne_bposit_quantize_weight_per_channel(0, 4, 4, 0, 0) == -1
