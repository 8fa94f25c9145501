"""Multi-process (world size 2, gloo, CPU) tests of the N-shard and K-split
host logic in mosyne_bposit.dist: shard ranges, global scale reduction,
exact INT32 partial reduction, gathering -- results bit-identical to the
single-process computation.  The per-rank compute steps are stand-ins
(numpy, from the oracle) passed in by the test; on a GPU they are the CUDA
library.  Also: a rank that fails before a collective is detected by the
others through the process group's timeout, without any GPU involved."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

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


def _setup(rank, world, port, timeout_s=60):
    import datetime
    for p in (str(ROOT), str(ROOT / "mosyne-bposit_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _stand_ins():
    from oracle import bposit_oracle as O

    def gemm_i32(A, B):
        acc = O.gemm_exact(A.numpy(), B.numpy().T).astype(np.int32)
        return torch.from_numpy(np.ascontiguousarray(acc.T)).t()

    def epilogue(acc, *, bp32, bp16, y_dtype, x_scale, w_scale, rtne32, rtne16):
        a = acc.numpy().astype(np.int64)
        out = {}
        if bp32:
            out["bp32"] = torch.from_numpy(O.encode_int_array(a, 0, 32, "rtne" if rtne32 else "truncate").view(np.int32))
        if y_dtype is not None:
            out["y"] = torch.from_numpy(O.dequant(a, x_scale.numpy(), w_scale.numpy()))
        return out

    def gemm_full(A, B, *, bp32, bp16, y_dtype, x_scale, w_scale, rtne32, rtne16):
        return epilogue(gemm_i32(A, B), bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale,
                        w_scale=w_scale, rtne32=rtne32, rtne16=rtne16)

    def absmax(x):
        return torch.from_numpy(np.abs(x.numpy()).max(axis=1).astype(np.float32))

    def quant(x, row_max):
        s = O.quant_scale(row_max.numpy())
        return torch.from_numpy(O.quantize(x.numpy(), s[:, None])), torch.from_numpy(s)

    return dict(local_gemm=gemm_i32, local_epilogue=epilogue, gemm_full=gemm_full,
                local_absmax=absmax, local_quant=quant)


def _worker_ksplit(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from mosyne_bposit import dist as D
        from oracle import bposit_oracle as O
        si = _stand_ins()
        M, K, N = 48, 1000, 70
        rng = np.random.default_rng(0)
        x = (rng.standard_normal((M, K)) * np.where(rng.random(K) < 0.02, 20.0, 1.0)).astype(np.float32)
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        wq, ws = O.quant_per_channel(w.T)                      # scales from the FULL weight
        k0, k1 = D.shard_range(K, world, rank)
        res = D.ksplit_linear(torch.from_numpy(x[:, k0:k1].copy()),
                              torch.from_numpy(np.ascontiguousarray(wq.T[:, k0:k1])),
                              torch.from_numpy(ws), bp32=True, **{k: si[k] for k in
                              ("local_gemm", "local_epilogue", "local_absmax", "local_quant")})
        y_ref, acc, *_ = O.linear_w8a8(x, w.T)
        ok = (np.array_equal(res["i32"].numpy().astype(np.int64), acc)
              and np.array_equal(res["y"].numpy().view(np.uint32), y_ref.view(np.uint32))
              and np.array_equal(res["bp32"].numpy().view(np.uint32), O.encode_int_array(acc, 0, 32)))
        q.put((rank, ok, None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def _ksplit_case(M, K, N, seed, extreme=False):
    """Quantised K-split operands (int8 A [M,K], B [N,K]) and scales; with
    ``extreme`` every code is 127, so INT32 sums overflow beyond K = 133,152."""
    rng = np.random.default_rng(seed)
    if extreme:
        A = np.full((M, K), 127, np.int8)
        B = np.full((N, K), 127, np.int8)
        A[::2] = -127
    else:
        A = rng.integers(-127, 128, (M, K), dtype=np.int8)
        B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    xs = (rng.random(M) + 0.5).astype(np.float32)
    ws = (rng.random(N) + 0.5).astype(np.float32)
    return A, B, xs, ws


def _worker_ksplit_variants(rank, world, port, q):
    """reduce-scatter with chunks (gathered and per-rank), all-reduce, and the
    INT64 partials beyond the INT32 limit; every result equals the exact
    single-process one."""
    try:
        _setup(rank, world, port)
        from mosyne_bposit import dist as D
        from oracle import bposit_oracle as O
        si = _stand_ins()
        local = {k: si[k] for k in ("local_gemm", "local_epilogue")}
        report = {}
        for name, (M, K, N, chunks, reduce, extreme) in {
                "scatter_c3": (17, 300, 70, 3, "scatter", False),
                "scatter_c1_uneven": (9, 64, 5, 1, "scatter", False),
                "all_c2": (12, 96, 33, 2, "all", False),
                "wide": (6, 140000, 7, 2, "scatter", True)}.items():
            A, B, xs, ws = _ksplit_case(M, K, N, len(name), extreme)
            k0, k1 = D.shard_range(K, world, rank)
            acc = O.gemm_exact(A, B.T)
            want_bp = O.encode_int_array(acc, 0, 32)
            want_y = O.dequant(acc, xs, ws)
            res = D.ksplit_gemm_i8(torch.from_numpy(A[:, k0:k1].copy()),
                                   torch.from_numpy(B[:, k0:k1].copy()), bp32=True,
                                   y_dtype=torch.float32, x_scale=torch.from_numpy(xs),
                                   w_scale=torch.from_numpy(ws), reduce=reduce, chunks=chunks,
                                   **local)
            key = "i64" if extreme else "i32"
            report[name] = (np.array_equal(res[key].numpy().astype(np.int64), acc)
                            and np.array_equal(res["bp32"].numpy().view(np.uint32), want_bp)
                            and np.array_equal(res["y"].numpy().view(np.uint32),
                                               want_y.view(np.uint32)))
            if reduce == "scatter":
                own = D.ksplit_gemm_i8(torch.from_numpy(A[:, k0:k1].copy()),
                                       torch.from_numpy(B[:, k0:k1].copy()), bp32=True,
                                       reduce=reduce, chunks=chunks, gather=False, **local)
                bp = own["bp32"].numpy().view(np.uint32)
                j, ok = 0, True
                per = D.ksplit_layout(N, world, chunks)["per"]
                for (a, b) in own["cols"]:
                    ok &= np.array_equal(bp[:, j:j + b - a], want_bp[:, a:b])
                    j += per
                report[name + "_owned"] = bool(ok)
        if extreme:
            # the same sums in INT32 would wrap: refused unless wide
            try:
                D.ksplit_gemm_i8(torch.from_numpy(A[:, k0:k1].copy()),
                                 torch.from_numpy(B[:, k0:k1].copy()), wide=False, **local)
                report["refuses_narrow"] = False
            except ValueError:
                report["refuses_narrow"] = True
        q.put((rank, all(report.values()), report))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


def _worker_nshard(rank, world, port, q):
    try:
        _setup(rank, world, port)
        from mosyne_bposit import dist as D
        from oracle import bposit_oracle as O
        si = _stand_ins()
        M, K, N = 33, 256, 101
        rng = np.random.default_rng(1)
        A = rng.integers(-127, 128, (M, K), dtype=np.int8)
        B = rng.integers(-127, 128, (N, K), dtype=np.int8)
        n0, n1 = D.shard_range(N, world, rank)
        res = D.nshard_gemm_i8(torch.from_numpy(A), torch.from_numpy(B[n0:n1].copy()), gather=True,
                               local_gemm=si["gemm_full"])
        acc = O.gemm_exact(A, B.T)
        ok = np.array_equal(res["bp32"].numpy().view(np.uint32), O.encode_int_array(acc, 0, 32))
        q.put((rank, ok, None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, False, repr(e)))


def _worker_dead_rank(rank, world, port, q):
    _setup(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, True, "left before the collective"))
        q.close()
        q.join_thread()
        os._exit(0)                      # leaves between steps; nothing in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, False, "collective completed without the peer"))
    except Exception as e:
        q.put((rank, True, type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_ksplit_bit_identical_to_single_process():
    out = _run(_worker_ksplit)
    assert all(ok for _, ok, _ in out), out


def test_ksplit_reduce_scatter_chunks_and_wide_partials():
    out = _run(_worker_ksplit_variants, timeout=240)
    assert all(ok for _, ok, _ in out), out


def test_ksplit_layout_partitions_columns():
    from mosyne_bposit.dist import ksplit_layout, ksplit_owned_columns
    for N in (1, 7, 70, 1000, 28672):
        for world in (1, 2, 3, 8):
            for chunks in (1, 2, 3, 5):
                L = ksplit_layout(N, world, chunks)
                assert L["padded"] >= N and L["padded"] % world == 0
                spans = sorted(r for k in range(world)
                               for r in ksplit_owned_columns(N, world, k, chunks) if r[1] > r[0])
                assert spans[0][0] == 0 and spans[-1][1] == N
                assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_nshard_gather_bit_identical():
    out = _run(_worker_nshard)
    assert all(ok for _, ok, _ in out), out


def test_peer_failure_detected_by_timeout():
    out = _run(_worker_dead_rank, timeout=90)
    assert all(ok for _, ok, _ in out), out


def test_shard_range_partitions():
    from mosyne_bposit.dist import shard_range
    for total in (1, 7, 4096, 28672):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
