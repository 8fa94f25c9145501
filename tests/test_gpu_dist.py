"""Multi-GPU (world size 2 and every GPU of the box, NCCL, one process per GPU) tests of
mosyne_bposit.dist on the CUDA library: the K-split linear (global row
maxima by all_reduce(MAX), exact INT32 partials by all_reduce(SUM)) and the
column-parallel GEMM with all-gather must equal the one-GPU results bit for
bit, and the oracle; the K-split's reduce-scatter (in chunks, gathered or
kept per rank), its all-reduce form and its INT64 partials (K = 140,000)
equal the exact single-GPU sums.  Skipped on machines with fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parent.parent


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port):
    import datetime
    for p in (str(ROOT), str(ROOT / "mosyne-bposit_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from mosyne_bposit import _api
    _api.load_library(init=True)


def _worker(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from mosyne_bposit import _api, ops
        from mosyne_bposit import dist as D
        from oracle import bposit_oracle as O
        dev = torch.device("cuda", rank)
        report = {}

        # K-split linear: x [M,K] row-major, nn.Linear weight [N,K]
        M, K, N = 96, 3072, 640
        g = torch.Generator(device="cpu").manual_seed(5)
        x = torch.randn(M, K, generator=g)
        x[:, torch.randperm(K, generator=g)[:30]] *= 25.0
        w = torch.randn(N, K, generator=g) * 0.02
        wq, ws = ops.quantize_per_channel(w.to(dev))             # scales of the FULL weight
        k0, k1 = D.shard_range(K, world, rank)
        res = D.ksplit_linear(x[:, k0:k1].contiguous().to(dev), wq[:, k0:k1].contiguous(), ws,
                              bp32=True)
        one = ops.linear_w8a8(x.to(dev), wq, ws, out_dtype=torch.float32, bp32=True)
        torch.cuda.synchronize()
        report["ksplit_y_vs_one_gpu"] = torch.equal(res["y"].contiguous().view(torch.int32).cpu(),
                                                   one["y"].contiguous().view(torch.int32).cpu())
        report["ksplit_bp32_vs_one_gpu"] = torch.equal(res["bp32"].contiguous().cpu(),
                                                      one["bp32"].contiguous().cpu())
        y_ref, acc, *_ = O.linear_w8a8(x.numpy(), w.numpy().T)
        report["ksplit_i32_vs_oracle"] = np.array_equal(
            res["i32"].cpu().numpy().astype(np.int64), acc)
        report["ksplit_y_vs_oracle"] = np.array_equal(
            res["y"].cpu().numpy().view(np.uint32), y_ref.view(np.uint32))

        # column-parallel GEMM with all-gather
        M, K, N = 257, 512, 1000
        A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        n0, n1 = D.shard_range(N, world, rank)
        full = D.nshard_gemm_i8(A.to(dev), B[n0:n1].contiguous().to(dev), bp32=True, gather=True)
        acc = O.gemm_exact(A.numpy(), B.numpy().T)
        report["nshard_bp32_vs_oracle"] = np.array_equal(
            full["bp32"].cpu().numpy().view(np.uint32), O.encode_int_array(acc, 0, 32))
        # K-split variants: reduce-scatter in chunks (gathered and per rank),
        # all-reduce, and INT64 partials beyond the INT32 range
        M, K, N = 200, 2048, 1000
        A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        xs = torch.rand(M, generator=g) + 0.5
        ws_ = torch.rand(N, generator=g) + 0.5
        k0, k1 = D.shard_range(K, world, rank)
        acc = O.gemm_exact(A.numpy(), B.numpy().T)
        want_bp = O.encode_int_array(acc, 0, 32)
        want_y = O.dequant(acc, xs.numpy(), ws_.numpy())
        a_s, b_s = A[:, k0:k1].contiguous().to(dev), B[:, k0:k1].contiguous().to(dev)
        for reduce, chunks in (("scatter", 1), ("scatter", 3), ("all", 2)):
            r = D.ksplit_gemm_i8(a_s, b_s, bp32=True, y_dtype=torch.float32, x_scale=xs.to(dev),
                                 w_scale=ws_.to(dev), reduce=reduce, chunks=chunks)
            report[f"ksplit_{reduce}_{chunks}"] = (
                np.array_equal(r["bp32"].cpu().numpy().view(np.uint32), want_bp)
                and np.array_equal(r["y"].cpu().numpy().view(np.uint32), want_y.view(np.uint32)))
        own = D.ksplit_gemm_i8(a_s, b_s, bp32=True, chunks=3, gather=False)
        per = D.ksplit_layout(N, world, 3)["per"]
        bp = own["bp32"].cpu().numpy().view(np.uint32)
        report["ksplit_owned_columns"] = all(
            np.array_equal(bp[:, j * per:j * per + b - a], want_bp[:, a:b])
            for j, (a, b) in enumerate(own["cols"]))
        Kw = 140_000
        Aw = torch.full((64, Kw), 127, dtype=torch.int8)
        Aw[::2] = -127
        Bw = torch.full((40, Kw), 127, dtype=torch.int8)
        k0, k1 = D.shard_range(Kw, world, rank)
        r = D.ksplit_gemm_i8(Aw[:, k0:k1].contiguous().to(dev), Bw[:, k0:k1].contiguous().to(dev),
                             bp32=True)
        accw = O.gemm_exact(Aw.numpy(), Bw.numpy().T)
        report["ksplit_wide_i64"] = np.array_equal(r["i64"].cpu().numpy(), accw)
        report["ksplit_wide_bp32"] = np.array_equal(r["bp32"].cpu().numpy().view(np.uint32),
                                                    O.encode_int_array(accw, 0, 32))
        report["device_error"] = _api.last_error()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        ok = all(v is True for k, v in report.items() if k != "device_error") and \
            report["device_error"] == 0
        q.put((rank, ok, report))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def _worlds():
    """2 ranks, and every GPU of the box when it has more than two."""
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [2] + ([n] if n > 2 else [])


@pytest.mark.parametrize("world", _worlds())
def test_ksplit_and_nshard_multi_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(ok for _, ok, _ in out), out
