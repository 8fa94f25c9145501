"""GPU parity: the W8A8 SwiGLU FFN (kernels/test_ffn_layer_real_qwen.cu:300-334)
through mosyne_bposit_ffn_swiglu_w8a8.

Stages compared with the oracle: the gate/up GEMM's dequantised values enter
silu(g) * u, whose expf the oracle (numpy) cannot reproduce to the last place,
so the activation is compared with a relative tolerance of 1e-5; given the
device's activation, the per-token re-quantisation, the down GEMM and its
dequantisation are bit-exact.  End to end the device FFN tracks the oracle's
W8A8 pipeline, and its distance from the fp32 FFN computed by torch is the
W8A8 quantisation error itself."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ffn_case(M, D, F, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, D, generator=g)
    x[:, torch.randperm(D, generator=g)[: max(1, D // 100)]] *= 20.0
    wg = torch.randn(F, D, generator=g) * 0.02
    wu = torch.randn(F, D, generator=g) * 0.02
    wd = torch.randn(D, F, generator=g) * 0.02
    return x, wg, wu, wd


@pytest.mark.parametrize("M,D,F", [(200, 512, 1024), (64, 256, 512), (300, 1024, 2048)])
def test_ffn_stages(cuda_lib, M, D, F):
    from mosyne_bposit import _api, ops
    x, wg, wu, wd = _ffn_case(M, D, F, M)
    packed = ops.pack_swiglu_weights(wg.cuda(), wu.cuda(), wd.cuda())
    act = torch.empty((M, F), dtype=torch.float32, device="cuda")
    y = ops.ffn_swiglu_w8a8(x.cuda(), packed, out_dtype=torch.float32, act=act)
    torch.cuda.synchronize()
    y_ref, act_ref, _, _ = O.ffn_swiglu_w8a8(x.numpy(), wg.numpy(), wu.numpy(), wd.numpy())
    a = act.cpu().numpy()
    np.testing.assert_allclose(a, act_ref, rtol=1e-5, atol=1e-30)
    # given the device activation, the rest is bit-exact
    hq, hs = O.quant_per_token(a)
    dq, ds = O.quant_per_channel(wd.numpy().T)
    want = O.dequant(O.gemm_exact(hq, dq), hs, ds)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert _api.last_error() == 0


def test_ffn_end_to_end_accuracy_and_dtypes(cuda_lib):
    """End to end the device FFN tracks the oracle's W8A8 pipeline (differences
    come only from expf's last place moving a re-quantisation tie), and its
    error against the fp32 FFN is the W8A8 quantisation error itself."""
    from mosyne_bposit import _api, ops
    M, D, F = 256, 1024, 2752
    F -= F % 32
    x, wg, wu, wd = _ffn_case(M, D, F, 7)
    ref = torch.nn.functional.linear(
        torch.nn.functional.silu(torch.nn.functional.linear(x, wg)) * torch.nn.functional.linear(x, wu),
        wd)
    y_or, *_ = O.ffn_swiglu_w8a8(x.numpy(), wg.numpy(), wu.numpy(), wd.numpy())
    y_or = torch.from_numpy(y_or)
    err_or = float((y_or - ref).norm() / ref.norm())
    packed = ops.pack_swiglu_weights(wg.cuda(), wu.cuda(), wd.cuda())
    y = ops.ffn_swiglu_w8a8(x.cuda(), packed).cpu()
    assert float((y - y_or).norm() / y_or.norm()) < 1e-3
    assert float((y - ref).norm() / ref.norm()) < 1.05 * err_or + 1e-3
    # bf16 activations in, bf16 out: the same pipeline on bf16-rounded inputs
    yb = ops.ffn_swiglu_w8a8(x.bfloat16().cuda(), packed).float().cpu()
    assert yb.dtype == torch.float32 and float((yb - ref).norm() / ref.norm()) < 2 * err_or + 1e-2
    assert _api.last_error() == 0


def test_ffn_bad_args(cuda_lib):
    lib = cuda_lib
    t = torch.zeros(64, device="cuda")
    # F not a multiple of 32
    assert lib.mosyne_bposit_ffn_swiglu_w8a8(t.data_ptr(), 0, 4, 64, t.data_ptr(), t.data_ptr(), 48,
                                             t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, None, 0,
                                             None) == -20
