"""GPU parity of the reference's W8A8 ABI and torch integration.

The nine reference entry points (libmosyne_bposit.cu) are called through the
C ABI with their original column-major layouts and compared bit for bit with
the oracle; BPositLinear reproduces the reference's published cross-GPU probe
hashes (cross_gpu_probe.py) on B200."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import bposit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _inputs(M, K, N, seed=0, outliers=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g, dtype=torch.float32)
    if outliers:
        cols = torch.randperm(K, generator=g)[: max(1, K // 100)]
        x[:, cols] *= 20.0
    w = torch.randn(K, N, generator=g, dtype=torch.float32) * 0.02
    return x, w


def _dev_linear(name, x_cm_dev, M, K, wq, ws, N, y_dev):
    from mosyne_bposit import _api
    getattr(_api, name)(x_cm_dev.data_ptr(), M, K, wq.data_ptr(), ws.data_ptr(), N, y_dev.data_ptr())
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,K,N", [(128, 2048, 11008), (1, 64, 8), (77, 320, 300), (256, 1024, 512)])
def test_reference_abi_fp32(cuda_lib, M, K, N):
    from mosyne_bposit import _api
    x, w = _inputs(M, K, N, seed=M + N, outliers=True)
    y_ref, acc, xq, xs, wq_ref, ws_ref = O.linear_w8a8(x.numpy(), w.numpy())
    w_cm = w.t().contiguous().cuda()                 # column-major [K,N]
    wq = torch.empty((N, K), dtype=torch.int8, device="cuda")
    ws = torch.empty((N,), dtype=torch.float32, device="cuda")
    _api.quantize_weight_per_channel_dev(w_cm.data_ptr(), K, N, wq.data_ptr(), ws.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(wq.cpu().numpy(), wq_ref.T)
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), ws_ref.view(np.uint32))
    x_cm = x.t().contiguous().cuda()                 # column-major [M,K]
    y_cm = torch.empty((N, M), dtype=torch.float32, device="cuda")
    _dev_linear("linear_w8a8_dev", x_cm, M, K, wq, ws, N, y_cm)
    assert np.array_equal(y_cm.t().cpu().numpy().view(np.uint32), y_ref.view(np.uint32))
    # host round trip (uploads and quantises the weight per call)
    y_host = _api.linear_w8a8(x.numpy(), w.numpy())
    assert np.array_equal(y_host.view(np.uint32), y_ref.view(np.uint32))


def test_reference_abi_half_types(cuda_lib):
    M, K, N = 96, 512, 384
    x, w = _inputs(M, K, N, seed=3)
    wq, ws = O.quant_per_channel(w.numpy())
    wqd = torch.from_numpy(np.ascontiguousarray(wq.T)).cuda()
    wsd = torch.from_numpy(ws).cuda()
    for tdt in (torch.bfloat16, torch.float16):
        xh = x.to(tdt)
        xf = xh.to(torch.float32).numpy()             # the values the kernel sees
        xq, xs = O.quant_per_token(xf)
        y_ref = O.dequant(O.gemm_exact(xq, wq), xs, ws)
        x_cm = xh.t().contiguous().cuda()
        y32 = torch.empty((N, M), dtype=torch.float32, device="cuda")
        name = "linear_w8a8_dev_bf16" if tdt == torch.bfloat16 else "linear_w8a8_dev_fp16"
        _dev_linear(name, x_cm, M, K, wqd, wsd, N, y32)
        assert np.array_equal(y32.t().cpu().numpy().view(np.uint32), y_ref.view(np.uint32))
        yh = torch.empty((N, M), dtype=tdt, device="cuda")
        _dev_linear(name + "_io", x_cm, M, K, wqd, wsd, N, yh)
        got = yh.t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        exp = O.f32_to_bf16_bits(y_ref) if tdt == torch.bfloat16 else y_ref.astype(np.float16).view(np.uint16)
        assert np.array_equal(got, exp)


def test_row_major_path_and_bposit_outputs(cuda_lib):
    from mosyne_bposit import ops
    M, K, N = 200, 768, 640
    x, w = _inputs(M, K, N, seed=9, outliers=True)
    y_ref, acc, *_ = O.linear_w8a8(x.numpy(), w.numpy())
    wq, ws = ops.quantize_per_channel(w.t().contiguous().cuda())
    r = ops.linear_w8a8(x.cuda(), wq, ws, bp32=True, bp16=True)
    torch.cuda.synchronize()
    assert np.array_equal(r["y"].cpu().numpy().view(np.uint32), y_ref.view(np.uint32))
    assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(acc, 0, 32))
    assert np.array_equal(r["bp16"].cpu().numpy().view(np.uint16), O.encode_int_array(acc, 0, 16))


def test_per_tensor_quantisation(cuda_lib):
    from mosyne_bposit import ops
    M, K, N = 128, 2048, 1100
    x, w = _inputs(M, K, N, seed=0)
    xq, xs = O.quant_per_tensor(x.numpy())
    wq, ws = O.quant_per_tensor(w.numpy())
    q_d, s_d = ops.quantize_per_tensor(x.cuda())
    assert np.array_equal(q_d.cpu().numpy(), xq)
    assert s_d.cpu().numpy().view(np.uint32)[0] == np.float32(xs).view(np.uint32)
    q_c, s_c = ops.quantize_per_tensor(x.t().contiguous().cuda(), col_major=True)
    assert np.array_equal(q_c.cpu().numpy(), xq)
    wqd, wsd = ops.quantize_per_tensor(w.t().contiguous().cuda())     # [N,K] rows
    assert np.array_equal(wqd.cpu().numpy(), wq.T)
    # more than 2048 rows (warp-per-row kernel, rows walked last to first,
    # a partial last block of rows)
    t = torch.randn(4100, 68, generator=torch.Generator().manual_seed(3))
    tq, ts = O.quant_per_tensor(t.numpy())
    q_t, s_t = ops.quantize_per_tensor(t.cuda())
    assert np.array_equal(q_t.cpu().numpy(), tq)
    q_tc, _ = ops.quantize_per_tensor(t.t().contiguous().cuda(), col_major=True)
    assert np.array_equal(q_tc.cpu().numpy(), tq)
    r = ops.linear_w8a8(x.cuda(), wqd, wsd, per_tensor=True, bp32=True)
    acc = O.gemm_exact(xq, wq)
    y_ref = O.dequant(acc, np.full(M, xs, np.float32), np.full(N, ws, np.float32))
    assert np.array_equal(r["y"].cpu().numpy().view(np.uint32), y_ref.view(np.uint32))
    assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(acc, 0, 32))


@pytest.mark.parametrize("shape,dtype", [
    ((1, 4), torch.float32), ((3, 1000), torch.float32),        # one cluster
    ((128, 2048), torch.float32), ((128, 2048), torch.bfloat16),
    ((512, 1024), torch.float32),                               # the largest one-cluster tensor
    ((512, 1028), torch.float32), ((1000, 4096), torch.float16),  # grid-barrier launch
    ((5, 7), torch.float32), ((3000, 20000), torch.float32),    # two-pass
])
def test_per_tensor_quantiser_paths(cuda_lib, shape, dtype):
    """Every per-tensor quantiser (one cluster for small tensors, one launch
    with a grid barrier, two passes) against the oracle, bit for bit."""
    from mosyne_bposit import _api, ops
    g = torch.Generator().manual_seed(shape[0] * 7 + shape[1])
    t = (torch.randn(*shape, generator=g) * 3).to(dtype)
    if t.numel() > 8:
        t.view(-1)[t.numel() // 3] = 40.0                      # one outlier sets the scale
    ref_q, ref_s = O.quant_per_tensor(t.float().numpy())
    q, s = ops.quantize_per_tensor(t.cuda())
    assert np.array_equal(q.cpu().numpy(), ref_q)
    assert s.cpu().numpy().view(np.uint32)[0] == np.float32(ref_s).view(np.uint32)
    assert _api.last_error() == 0


@pytest.mark.parametrize("M,K", [(96, 1024), (600, 2048)])
def test_per_tensor_one_launch_graph_replays(cuda_lib, M, K):
    """The one-launch per-tensor quantisers (one cluster; a grid barrier whose
    state resets itself): a CUDA graph of the per-tensor linear replayed on
    changing inputs gives each input's exact result, with the two-pass
    quantiser (rows too long for one launch) run between the replays."""
    from mosyne_bposit import _api, ops
    N = 520
    g = torch.Generator().manual_seed(17)
    wq, ws = ops.quantize_per_channel((torch.randn(N, K, generator=g) * 0.02).cuda())
    wq_h, ws_h = wq.cpu().numpy(), ws.cpu().numpy()
    x_buf = torch.empty(M, K, device="cuda")
    xs = [torch.randn(M, K, generator=g) * (1 + 3 * i) for i in range(3)]
    x_buf.copy_(xs[0].cuda())
    ops.linear_w8a8(x_buf, wq, ws, out_dtype=torch.float32, bp32=True, per_tensor=True)  # warm-up
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream), torch.cuda.graph(graph, stream=stream):
        r = ops.linear_w8a8(x_buf, wq, ws, out_dtype=torch.float32, bp32=True, per_tensor=True)
    torch.cuda.synchronize()
    for i, x in enumerate(xs):
        x_buf.copy_(x.cuda())
        graph.replay()
        torch.cuda.synchronize()
        xq, xsc = O.quant_per_tensor(x.numpy())
        acc = O.gemm_exact(xq, wq_h.T)
        y_ref = O.dequant(acc, np.full(M, xsc, np.float32), ws_h)
        assert np.array_equal(r["y"].cpu().numpy().view(np.uint32), y_ref.view(np.uint32)), i
        assert np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(acc, 0, 32))
        big = torch.randn(300, 20000, generator=g)
        q_b, _ = ops.quantize_per_tensor(big.cuda())
        assert np.array_equal(q_b.cpu().numpy(), O.quant_per_tensor(big.numpy())[0])
    del graph
    assert _api.last_error() == 0


def test_per_token_quantiser_layouts(cuda_lib):
    from mosyne_bposit import ops
    # row lengths for every register-resident variant (1, 2, 4, 8, 16 vectors
    # per thread), the two-pass fallback beyond them, odd K, and M % 4 != 0
    # (the column-major scalar kernels) next to M % 4 == 0 (vector kernels)
    for (M, K) in [(1, 16), (3, 5), (130, 1000), (2048, 4096), (132, 2052), (5, 9000),
                   (12, 20000), (64, 1028)]:
        x, _ = _inputs(M, K, 1, seed=M, outliers=True)
        xq, xs = O.quant_per_token(x.numpy())
        for tdt in (torch.float32, torch.bfloat16, torch.float16):
            xt = x.to(tdt)
            xq, xs = O.quant_per_token(xt.to(torch.float32).numpy())
            q1, s1 = ops.quantize_per_token(xt.cuda())
            q2, s2 = ops.quantize_per_token(xt.t().contiguous().cuda(), col_major=True)
            assert np.array_equal(q1.cpu().numpy(), xq) and np.array_equal(q2.cpu().numpy(), xq)
            assert np.array_equal(s1.cpu().numpy().view(np.uint32), xs.view(np.uint32))
            assert np.array_equal(s2.cpu().numpy().view(np.uint32), xs.view(np.uint32))


def test_zero_rows_get_unit_scale(cuda_lib):
    from mosyne_bposit import ops
    x = torch.zeros((4, 64), device="cuda")
    x[2, 5] = 3.0
    q, s = ops.quantize_per_token(x)
    assert s.cpu().tolist() == [1.0, 1.0, np.float32(127.0) / np.float32(3.0), 1.0]


def test_probe_hashes_on_b200(cuda_lib, golden):
    """The reference's cross-GPU probe: BPositLinear fp32 outputs hash to the
    values published for RTX 3090 and RTX 5090."""
    from mosyne_bposit.torch_compat import BPositLinear
    g = golden("probe_hashes.json")
    for key, (M, K, N) in g["shapes"].items():
        gen = torch.Generator(device="cpu").manual_seed(g["seed"])
        x = torch.randn(M, K, generator=gen, dtype=torch.float32) * 0.3
        w = torch.randn(N, K, generator=gen, dtype=torch.float32) * (1.0 / K ** 0.5)
        y = BPositLinear(weight=w.cuda())(x.cuda())
        h = hashlib.sha256(y.detach().cpu().contiguous().numpy().tobytes()).hexdigest()
        assert h == g["hashes"][key], key


def test_torch_device_path_matches_host_path(cuda_lib):
    from mosyne_bposit.torch_compat import BPositLinear
    torch.manual_seed(0)
    M, K, N = 32, 256, 512
    w = torch.randn(N, K) * (1.0 / K ** 0.5)
    x = torch.randn(M, K) * 0.5
    y_dev = BPositLinear(weight=w.cuda())(x.cuda()).cpu()
    y_host = BPositLinear(weight=w)(x)
    assert torch.equal(y_dev, y_host)
    assert "path=device" in repr(BPositLinear(weight=w.cuda()))
    assert "path=host-fallback" in repr(BPositLinear(weight=w))


def test_torch_dtypes_bias_and_error_band(cuda_lib):
    from mosyne_bposit.torch_compat import BPositLinear
    torch.manual_seed(0)
    M, K, N = 64, 512, 1024
    x = torch.randn(2, M // 2, K, device="cuda") * 0.5
    w = torch.randn(N, K, device="cuda") * (1.0 / K ** 0.5)
    b = torch.randn(N, device="cuda")
    mod = BPositLinear(weight=w, bias=b)
    ref = x @ w.t() + b
    y = mod(x)
    assert y.shape == (2, M // 2, N)
    rel = ((y - ref).pow(2).mean().sqrt() / ref.pow(2).mean().sqrt()).item()
    assert rel < 0.05
    yb = mod(x.to(torch.bfloat16))
    yh = mod(x.to(torch.float16))
    yd = mod(x.to(torch.float64))
    assert yb.dtype == torch.bfloat16 and yh.dtype == torch.float16 and yd.dtype == torch.float64
    assert ((y - yb.float()).abs().max() / y.abs().max()).item() < 5e-2
    assert ((y - yh.float()).abs().max() / y.abs().max()).item() < 1e-2


def test_fused_qkv_forward(cuda_lib):
    import torch.nn as nn
    from mosyne_bposit.torch_compat import BPositLinear, FusedQKVProjection
    torch.manual_seed(1)
    q, k, v = nn.Linear(256, 256, bias=False), nn.Linear(256, 64, bias=False), nn.Linear(256, 64, bias=False)
    q, k, v = q.cuda(), k.cuda(), v.cuda()
    f = FusedQKVProjection.from_separate(q_proj=q, k_proj=k, v_proj=v)
    x = torch.randn(8, 256, device="cuda")
    qo, ko, vo = f(x)
    full = BPositLinear(weight=torch.cat([q.weight, k.weight, v.weight]))(x)
    assert torch.equal(torch.cat([qo, ko, vo], dim=-1), full)
    assert qo.shape == (8, 256) and ko.shape == (8, 64) and vo.shape == (8, 64)


def test_not_initialised_and_bad_args(cuda_lib):
    from mosyne_bposit import _api
    lib = cuda_lib
    x = torch.zeros((8, 16), device="cuda")
    wq = torch.zeros((8, 16), dtype=torch.int8, device="cuda")
    ws = torch.ones(8, device="cuda")
    y = torch.empty((8, 8), device="cuda")
    lib.mosyne_bposit_shutdown()
    assert lib.mosyne_bposit_linear_w8a8(x.data_ptr(), 8, 16, wq.data_ptr(), ws.data_ptr(), 8,
                                         y.data_ptr()) == -10
    assert lib.mosyne_bposit_init() == 0
    assert lib.mosyne_bposit_init() == 0          # idempotent
    assert lib.mosyne_bposit_linear_w8a8(x.data_ptr(), 0, 16, wq.data_ptr(), ws.data_ptr(), 8,
                                         y.data_ptr()) == -20
    assert lib.mosyne_bposit_linear_w8a8(x.data_ptr(), 8, 16, wq.data_ptr(), ws.data_ptr(), 8,
                                         y.data_ptr()) == 0
    assert _api.last_error() == 0
