"""Benchmark: fused INT8 GEMM -> INT32 -> bposit32 on B200 (tcgen05).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one launch of the fused GEMM over one batch: the 4096^3 int8
GEMM (A row-major, B column-major, uniform int8 in [-127,127]) whose every
exact INT32 dot product leaves the kernel as a bposit32 code (truncating,
the reference's default), inputs resident in HBM.  Inputs rotate over
enough buffer sets (> 3x the 126 MB L2) that no step reads operands the
previous step left in L2.  The 2048x14336x4096 FFN-gate shape is measured
the same way and reported under "workloads".

N > 1 (torchrun, one rank per GPU): column-parallel N-shard -- each rank
computes its own 4096-column block of an M=4096, K=4096, N=4096*ranks GEMM
(weak scaling, no collective on the data path); time = max over ranks.

Every N also runs the C5 workload (W8A8 16384 x 8192 x 28672, per-token /
per-channel scales, fp32 y + bposit32): N-shard as strong scaling and, at
N > 1, the K-split with an exact INT32 reduce-scatter over NCCL; the
gathered outputs' SHA-256 are compared with the oracle's committed hashes
and with the same problem run on one GPU ("c5_16384x8192x28672").

--impl reference: the reference's CPU path for the same workload on the
host cores (numpy exact integer GEMM + bposit32 encoding of every output,
the oracle's restatement of kernels/bposit16_reference.py), rank 0 only.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT), str(ROOT / "mosyne-bposit_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "bposit-IMMA TPOPS at 4096³ & 2048×14336×4096, % INT8 peak, 1/2/4/8 GPU"
UNIT = "TPOPS"
HEADLINE = ("gemm_4096", 4096, 4096, 4096)
SECOND = ("ffn_gate_2048x14336x4096", 2048, 14336, 4096)
L2_BYTES = 126 * 1024 * 1024
NOMINAL_INT8_TOPS = 4500.0


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": float(d["bf16_tflops"]), "hbm": float(d["hbm_gbs"]), "src": "measured"}
    return {"bf16": 1590.0, "hbm": 6650.0, "src": "fallback"}


def _traffic(workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get(workload)
        if isinstance(v, dict):
            return v.get("dram_bytes_per_launch")
    return None


class Clocks:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws == 1:
        return None, 0, 0, 1
    import datetime

    import torch
    import torch.distributed as dist
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    # stdout carries exactly one JSON line: NCCL's own log lines (its version
    # banner included) go to stderr unless the caller chose a log file
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    return dist, rank, local, ws


def _barrier(dist):
    if dist is not None:
        dist.barrier()


def _max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _all_ranks(dist, v: float) -> list:
    """v of every rank, in rank order (one all-gather)."""
    if dist is None:
        return [v]
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def _time_gemm(M, N, K, steps, warmup, dist, seed, lib_call):
    """Device time (ms) of `steps` back-to-back launches, inputs rotating."""
    import torch
    per_set = M * K + N * K
    nsets = max(2, math.ceil(3 * L2_BYTES / per_set))
    g = torch.Generator(device="cuda").manual_seed(seed)
    As = [torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8, device="cuda") for _ in range(nsets)]
    Bs = [torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8, device="cuda") for _ in range(nsets)]
    out = torch.empty((N, M), dtype=torch.int32, device="cuda")   # column-major [M,N]
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        lib_call(As[i % nsets], Bs[i % nsets], out, stream)
    _barrier(dist)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        lib_call(As[(warmup + i) % nsets], Bs[(warmup + i) % nsets], out, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    _barrier(dist)
    ms = e0.elapsed_time(e1)
    return ms, nsets, out


def _events_ms(fn, steps, warmup, graph=False):
    """Average device time (ms) of fn() over `steps` back-to-back calls on
    the current stream, after `warmup` calls.  With ``graph`` the `steps`
    calls are captured once into a CUDA graph and the graph is replayed
    inside the timed region: calls whose device work is shorter than their
    host-side launch cost are then timed on the device, as a serving loop
    replaying graphs runs them."""
    import torch
    # a graph capture cannot allocate: the first call (scratch buffers) runs
    # before it even with no warm-up requested
    for _ in range(max(warmup, 1 if graph else 0)):
        fn()
    torch.cuda.synchronize()
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for _ in range(steps):
                fn()
        torch.cuda.synchronize()
        g.replay()                                   # warm replay
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if graph:
        g.replay()
    else:
        for _ in range(steps):
            fn()
    e1.record()
    torch.cuda.synchronize()
    if graph:
        del g
    return e0.elapsed_time(e1) / steps


def extra_workloads(steps, warmup, peaks, select=None):
    """The other measured rows of the path, each on inputs larger than L2
    where the roofline is HBM (rotating copies otherwise):
    * c1: W8A8 linear 128x2048x11008 with a per-tensor activation scale,
      fp32 y and bposit32 outputs (HBM-bound: weights dominate);
    * c2: exact sum of 2^24 bposit16 values -> quire256 -> bposit16 (HBM-bound);
    * qkt: 32 heads of 2048x2048x128 QK^T, fp32 scores + bposit32 codes in one
      batched launch (HBM-bound: 1 GiB written per call);
    * ffn: the W8A8 SwiGLU FFN of a 3B model at M=2048 (2048 -> 11008 -> 2048):
      quantise, fused gate/up GEMM with the activation in its epilogue,
      re-quantise, down GEMM (tensor-bound; torch bf16 FFN timed beside it);
    * dec: decode-like GEMMs (M = 32 / 128 rows, K up to 11008) -> bposit32,
      cuBLASLt INT8 beside (HBM-bound: the weights dominate);
    * sq: square GEMMs 1024^3 / 2048^3 / 3072^3 -> bposit32, cuBLASLt INT8 beside;
    * bp8: the bposit8 path at 4096^3 -- decode both operands (bposit8 ->
      int8 fixed point) in one launch and one fused GEMM whose epilogue encodes
      acc / 2^12.
    ``select`` (a set of those names) limits the run to some of them."""
    import torch

    from mosyne_bposit import ops
    out = {}
    hbm = peaks["hbm"]
    want = (lambda k: True) if select is None else (lambda k: k in select)
    g = torch.Generator(device="cuda").manual_seed(0)
    it = [0]
    if want("c1"):
        # rotate weight copies so each call reads its weights from HBM
        M, K, N = 128, 2048, 11008
        x = torch.randn(M, K, device="cuda", generator=g)
        nw = max(2, math.ceil(3 * L2_BYTES / (N * K)))
        ws = []
        for _ in range(nw):
            w = torch.randn(N, K, device="cuda", generator=g) * 0.02
            ws.append(ops.quantize_per_channel(w))

        def c1():
            wq, sc = ws[it[0] % nw]
            it[0] += 1
            ops.linear_w8a8(x, wq, sc, out_dtype=torch.float32, bp32=True, per_tensor=True)
        ms = _events_ms(c1, steps, warmup, graph=True)
        nbytes = M * K * 4 + N * K + N * 4 + M * N * 4 * 2
        out["linear_c1_128x2048x11008_per_tensor"] = {
            "us_per_call": ms * 1e3, "bytes_per_call": nbytes, "achieved_gbs": nbytes / ms / 1e6,
            "frac_of_hbm": nbytes / ms / 1e6 / hbm, "bound": "hbm",
            "outputs": "fp32 y + bposit32, row-major", "weight_copies": nw,
            "timing": "CUDA-graph replay of the calls"}

        def c1_tok():
            wq, sc = ws[it[0] % nw]
            it[0] += 1
            ops.linear_w8a8(x, wq, sc, out_dtype=torch.float32, bp32=True)
        ms = _events_ms(c1_tok, steps, warmup, graph=True)
        out["linear_c1_128x2048x11008_per_token"] = {
            "us_per_call": ms * 1e3, "bytes_per_call": nbytes, "achieved_gbs": nbytes / ms / 1e6,
            "frac_of_hbm": nbytes / ms / 1e6 / hbm, "bound": "hbm",
            "outputs": "fp32 y + bposit32, row-major", "weight_copies": nw,
            "timing": "CUDA-graph replay of the calls"}
        del ws
    if want("c2"):
        # 2^24 codes (32 MiB) of the headline distribution: magnitudes 2^U,
        # U ~ Uniform[-24, 24], random signs, rounded to bposit16 (RTNE);
        # rotated over > 3x L2
        n = 1 << 24
        nc = max(2, math.ceil(3 * L2_BYTES / (2 * n)))
        codes = []
        for _ in range(nc):
            u = torch.rand(n, device="cuda", generator=g, dtype=torch.float64) * 48.0 - 24.0
            sgn = torch.where(torch.rand(n, device="cuda", generator=g) < 0.5, -1.0, 1.0).double()
            codes.append(ops.float_to_bposit(sgn * torch.exp2(u), 16, rtne=True))
        it[0] = 0

        def c2():
            ops.quire_sum_bp16(codes[it[0] % nc])
            it[0] += 1
        ms = _events_ms(c2, steps, warmup, graph=True)
        out["exact_sum_c2_2^24_bposit16"] = {
            "us_per_call": ms * 1e3, "bytes_per_call": 2 * n, "achieved_gbs": 2 * n / ms / 1e6,
            "frac_of_hbm": 2 * n / ms / 1e6 / hbm, "bound": "hbm", "input_copies": nc,
            "inputs": "+-2^U, U ~ Uniform[-24, 24], bposit16 RTNE",
            "timing": "CUDA-graph replay of the calls"}
        small = codes[0][: 1 << 16].clone()
        ms = _events_ms(lambda: ops.quire_sum_bp16(small), steps, warmup, graph=True)
        out["exact_sum_c2_65536_bposit16"] = {
            "us_per_call": ms * 1e3, "bytes_per_call": 2 << 16, "bound": "latency",
            "inputs": "the first 65,536 codes of the 2^24 set",
            "timing": "CUDA-graph replay of the calls"}
        del codes
    if want("qkt"):
        # 32 heads x (2048 x 2048 x 128), fp32 scores + bposit32 codes
        # (output-bound: 1 GiB written per call)
        H, S_, D_ = 32, 2048, 128
        q = torch.randint(-127, 128, (H, S_, D_), device="cuda", generator=g, dtype=torch.int8)
        k = torch.randint(-127, 128, (H, S_, D_), device="cuda", generator=g, dtype=torch.int8)
        qs = torch.rand(H, S_, device="cuda", generator=g) + 0.5
        kscale = torch.rand(H, S_, device="cuda", generator=g) + 0.5
        ms = _events_ms(lambda: ops.gemm_i8_batched(q, k, bp32=True, y_dtype=torch.float32,
                                                    x_scale=qs, w_scale=kscale), steps, warmup)
        qk_bytes = 2 * H * S_ * D_ + 2 * H * S_ * 4 + H * S_ * S_ * 8
        out["qkt_32x2048x2048x128_fp32_bposit32"] = {
            "us_per_call": ms * 1e3, "bytes_per_call": qk_bytes,
            "achieved_gbs": qk_bytes / ms / 1e6, "frac_of_hbm": qk_bytes / ms / 1e6 / hbm,
            "bound": "hbm", "tpops": 2.0 * H * S_ * S_ * D_ / ms / 1e9, "launches_per_call": 1}
        del q, k
    if want("ffn"):
        M, D, F = 2048, 2048, 11008
        xf = torch.randn(M, D, device="cuda", generator=g)
        wg = torch.randn(F, D, device="cuda", generator=g) * 0.02
        wu = torch.randn(F, D, device="cuda", generator=g) * 0.02
        wd = torch.randn(D, F, device="cuda", generator=g) * 0.02
        packed = ops.pack_swiglu_weights(wg, wu, wd)
        ms = _events_ms(lambda: ops.ffn_swiglu_w8a8(xf, packed, out_dtype=torch.float32),
                        steps, warmup)
        xb, wgb, wub, wdb = xf.bfloat16(), wg.bfloat16(), wu.bfloat16(), wd.bfloat16()
        F_ = torch.nn.functional
        bms = _events_ms(lambda: F_.linear(F_.silu(F_.linear(xb, wgb)) * F_.linear(xb, wub), wdb),
                         steps, warmup)
        ffn_ops = 2.0 * M * D * F * 3
        out["ffn_swiglu_3b_2048x2048x11008"] = {
            "us_per_call": ms * 1e3, "tpops": ffn_ops / ms / 1e9,
            "frac_of_int8_peak": ffn_ops / ms / 1e9 / (2.0 * peaks["bf16"]), "bound": "tensor",
            "torch_bf16_us_per_call": bms * 1e3, "launches_per_call": 4}
    if want("dec"):
        # decode-like GEMMs (few rows, long K): the single-CTA kernel slices K
        # over clusters; cuBLASLt INT8 (INT32 out) on the same shapes beside
        from mosyne_bposit import _api
        lib = _api.load_library()
        for (M, N, K) in ((128, 4096, 11008), (32, 4096, 4096), (128, 2048, 8192)):
            ms, _, _ = _time_gemm(M, N, K, steps, warmup, None, 500 + M,
                                  lambda A, B, o, st: _ours(A, B, o, st, lib))
            lms, _, _ = _time_gemm(M, N, K, steps, warmup, None, 600 + M, _cublas_i8)
            out[f"decode_gemm_{M}x{N}x{K}"] = {
                "us_per_launch": ms / steps * 1e3, "tpops": 2.0 * M * N * K / (ms / steps) / 1e9,
                "cublaslt_int8_int32_out_us": lms / steps * 1e3,
                "bytes_per_launch": M * K + N * K + M * N * 4,
                "frac_of_hbm": (M * K + N * K + M * N * 4) / (ms / steps) / 1e6 / hbm,
                "bound": "hbm", "outputs": "bposit32 column-major"}
    if want("sq"):
        # small and mid square GEMMs -> bposit32 beside cuBLASLt INT8 (INT32 out only) in
        # the same process, inputs rotated over > 3x L2
        from mosyne_bposit import _api
        lib = _api.load_library()
        for n in (1024, 2048, 3072):
            ms, _, _ = _time_gemm(n, n, n, steps, warmup, None, 700 + n,
                                  lambda A, B, o, st: _ours(A, B, o, st, lib))
            lms, _, _ = _time_gemm(n, n, n, steps, warmup, None, 800 + n, _cublas_i8)
            ops_ = 2.0 * n ** 3
            out[f"gemm_{n}^3"] = {
                "us_per_launch": ms / steps * 1e3, "tpops": ops_ / (ms / steps) / 1e9,
                "cublaslt_int8_int32_out_tpops": ops_ / (lms / steps) / 1e9,
                "vs_cublaslt": lms / ms, "outputs": "bposit32 column-major"}
    if want("bp8"):
        # bposit8 operands (uniform codes) rotated over > 3x L2
        M = N = K = 4096
        nsets = max(2, math.ceil(3 * L2_BYTES / (M * K + N * K)))
        A8 = [torch.randint(0, 256, (M, K), device="cuda", generator=g, dtype=torch.int32)
              .to(torch.uint8) for _ in range(nsets)]
        B8 = [torch.randint(0, 256, (N, K), device="cuda", generator=g, dtype=torch.int32)
              .to(torch.uint8) for _ in range(nsets)]
        it[0] = 0

        def bp8():
            i = it[0] % nsets
            it[0] += 1
            ops.gemm_bposit8(A8[i], B8[i])
        ms = _events_ms(bp8, steps, warmup)
        out["bposit8_gemm_4096"] = {
            "us_per_call": ms * 1e3, "tpops": 2.0 * M * N * K / ms / 1e9,
            "frac_of_int8_peak": 2.0 * M * N * K / ms / 1e9 / (2.0 * peaks["bf16"]),
            "bound": "tensor", "launches_per_call": 2,
            "steps": "decode A and B in one launch (bposit8 -> int8 x 2^6), GEMM -> bposit32 "
                     "of acc / 2^12"}
        del A8, B8
    return out


def kernel_table(steps, warmup, peaks):
    """Device time and achieved HBM bandwidth of the element-wise and
    quantisation kernels of the path, one call each on inputs larger than
    L2 (so every call reads its input from HBM).  Bytes are the compulsory
    ones: each input read once, each output written once."""
    import torch

    from mosyne_bposit import ops
    hbm = peaks["hbm"]
    g = torch.Generator(device="cuda").manual_seed(7)
    res = {}

    def row(name, fn, nbytes, launches=1, **extra):
        ms = _events_ms(fn, steps, warmup)
        res[name] = {"us_per_call": ms * 1e3, "bytes_per_call": nbytes,
                     "achieved_gbs": nbytes / ms / 1e6, "frac_of_hbm": nbytes / ms / 1e6 / hbm,
                     "launches_per_call": launches, **extra}

    M, K = 8192, 4096                                    # activations, 128 MiB fp32
    x = torch.randn(M, K, device="cuda", generator=g)
    row("quant_per_token_rowmajor_8192x4096_f32", lambda: ops.quantize_per_token(x),
        M * K * 4 + M * K + M * 4)
    xb = x.bfloat16()
    row("quant_per_token_rowmajor_8192x4096_bf16", lambda: ops.quantize_per_token(xb),
        M * K * 2 + M * K + M * 4)
    xc = x.t().contiguous()                              # column-major [M, K] storage
    row("quant_per_token_colmajor_8192x4096_f32",
        lambda: ops.quantize_per_token(xc, col_major=True), M * K * 4 + M * K + M * 4,
        launches=2)
    del xc
    row("quant_per_tensor_8192x4096_f32", lambda: ops.quantize_per_tensor(x),
        M * K * 4 + M * K + 4, launches=2,
        note="absmax pass, then the quantise pass (which also writes the scale): "
             "the input is read twice")
    del x, xb
    N, Kw = 14336, 4096                                  # FFN gate weight, 224 MiB fp32
    w = torch.randn(N, Kw, device="cuda", generator=g) * 0.02
    row("quant_per_channel_14336x4096_f32", lambda: ops.quantize_per_channel(w),
        N * Kw * 4 + N * Kw + N * 4)
    del w
    n = 1 << 25                                          # 32 M elements
    i32 = torch.randint(-(1 << 31), 1 << 31, (n,), device="cuda", generator=g,
                        dtype=torch.int64).to(torch.int32)
    row("int32_to_bp32_2^25", lambda: ops.int32_to_bp32(i32), 8 * n)
    acc = i32[: 8192 * 4096].view(4096, 8192).t()        # logical [8192, 4096], column-major
    xs = torch.rand(8192, device="cuda", generator=g) + 0.5
    wsc = torch.rand(4096, device="cuda", generator=g) + 0.5
    row("epilogue_i32_8192x4096_bp32_f32",
        lambda: ops.epilogue_i32(acc, bp32=True, y_dtype=torch.float32, x_scale=xs, w_scale=wsc),
        8192 * 4096 * 12 + 8192 * 4 + 4096 * 4)
    del i32, acc
    f = torch.randn(n, device="cuda", generator=g)
    row("float_to_bp16_rtne_2^25_f32", lambda: ops.float_to_bposit(f, 16, rtne=True), 6 * n)
    del f
    codes = torch.randint(-(1 << 15), 1 << 15, (n,), device="cuda", generator=g,
                          dtype=torch.int32).to(torch.int16)
    codes2 = torch.randint(-(1 << 15), 1 << 15, (n,), device="cuda", generator=g,
                           dtype=torch.int32).to(torch.int16)
    for op in ("add", "mul", "recip", "sqrt", "log2", "exp2"):
        if op in ("add", "mul"):
            row(f"bposit16_{op}_2^25", lambda op=op: ops.bposit16_op(op, codes, codes2), 6 * n)
        else:
            row(f"bposit16_{op}_2^25", lambda op=op: ops.bposit16_op(op, codes), 4 * n)
    del codes2
    nq = 1 << 22                                         # 4 M quires, 128 MiB
    q = ops.bp16_to_quire(codes[:nq])
    row("bp16_to_quire_2^22", lambda: ops.bp16_to_quire(codes[:nq]), 34 * nq)
    row("quire_to_bp32_2^22", lambda: ops.quire_to_bposit(q, 32), 36 * nq)
    row("quire_to_bp16_rtne_2^22", lambda: ops.quire_to_bposit(q, 16, rtne=True), 34 * nq)
    del q, codes
    ne = 1 << 24                                         # probabilities in (0, 1): 32 MiB of codes
    pc = torch.randint(1, 0x4000, (ne,), device="cuda", generator=g,
                       dtype=torch.int32).to(torch.int16)
    row("shannon_entropy_bp16_2^24", lambda: ops.shannon_entropy_bp16(pc), 2 * ne,
        note="term table bposit16(p * log2(p)) gathered per code, exact quire256 sum")
    del pc
    b8 = torch.randint(0, 256, (1 << 27,), device="cuda", generator=g,
                       dtype=torch.int32).to(torch.uint8)
    row("bposit8_to_int8_2^27", lambda: ops.bposit8_to_int8(b8), 2 << 27)
    del b8
    return res


def _sha256_t(t) -> str:
    """SHA-256 of a device tensor's bytes (copied to the host in 256 MiB pieces)."""
    import hashlib

    import torch
    h = hashlib.sha256()
    flat = t.contiguous().view(torch.uint8).reshape(-1)
    step = 256 << 20
    for i in range(0, flat.numel(), step):
        h.update(flat[i:i + step].cpu().numpy().tobytes())
    return h.hexdigest()


def _api_sm_count() -> int:
    from mosyne_bposit import _api
    return _api.sm_count()


def _c5_golden():
    p = ROOT / "tests" / "golden" / "c5_hashes.json"
    if not p.exists():
        return None
    return json.loads(p.read_text())["rows"].get("16384")


def c2_determinism(dist, ws, rank, runs=5):
    """The determinism headline on every rank's GPU: the exact quire sum of
    the headline's 65,536 bposit16 codes (tests/golden/headline_codes.npy),
    ``runs`` times per GPU; every (GPU, run) bit pattern is gathered and
    compared, and with the published quire word and bposit16 code
    (tests/golden/headline.json)."""
    import numpy as np
    import torch

    from mosyne_bposit import ops
    gdir = ROOT / "tests" / "golden"
    codes = np.load(gdir / "headline_codes.npy")
    h = json.loads((gdir / "headline.json").read_text())
    x = torch.from_numpy(codes.view(np.int16).copy()).cuda()
    words = []
    for _ in range(runs):
        q, b16, b32 = ops.quire_sum_bp16(x)
        words.append(torch.cat([q.view(torch.int32), b16.to(torch.int32), b32]))
    mine = torch.stack(words)                                   # [runs, 10] int32
    if dist is not None:
        allr = [torch.empty_like(mine) for _ in range(ws)]
        dist.all_gather(allr, mine)
        mine = torch.stack(allr)
    pats = mine.reshape(-1, mine.shape[-1]).cpu().numpy()
    uniq = {p.tobytes() for p in pats}
    first = pats[0]
    qw = [f"{int(v):016x}" for v in first[:8].view(np.uint64)]
    b16 = int(np.uint16(first[8] & 0xFFFF))
    return {"gpus": ws, "runs_per_gpu": runs, "patterns_seen": len(uniq),
            "one_bit_pattern": len(uniq) == 1, "quire_words": qw, "bposit16": f"0x{b16:04x}",
            "bposit32": f"0x{int(np.uint32(first[9])):08x}",
            "matches_published": qw == h["quire_words"] and b16 == h["published_bp16"]}


def c5_workload(dist, ws, rank, steps, warmup, chunks=4):
    """C5: W8A8 16384 x 8192 x 28672 with per-token activation and
    per-channel weight scales, fp32 y + bposit32 outputs (column-major), on
    every rank of the job:

    * N-shard (strong scaling): rank r computes output channels
      [N r / p, N (r+1) / p) from the whole activation; no collective.
    * K-split (p > 1): rank r holds K slice r of both operands (global
      scales by all_reduce(MAX)); exact INT32 partials are reduce-scattered
      over NCCL in ``chunks`` chunks, each rank encodes the columns it owns.

    Inputs (numpy seed 0, tests/golden/configs.py) are drawn on rank 0 and
    broadcast.  The timed steps are the GEMM (N-shard) and the whole K-split
    call (partial GEMMs + reduce-scatter + epilogue); quantisation is done
    once beforehand, as a weight-stationary layer does.  After timing, the
    outputs are gathered and their SHA-256 compared with the oracle's
    (tests/golden/c5_hashes.json) and, at p > 1, with the same problem run
    on rank 0's GPU alone."""
    import sys as _sys

    import torch

    from mosyne_bposit import dist as D
    from mosyne_bposit import ops
    _sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import configs
    M, K, N = configs.C5
    dev = torch.device("cuda", torch.cuda.current_device())
    if rank == 0:
        x, w = configs.c5_inputs()
        xd, wd = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
        del x, w
    else:
        xd = torch.empty((M, K), dtype=torch.float32, device=dev)
        wd = torch.empty((N, K), dtype=torch.float32, device=dev)
    if dist is not None:
        dist.broadcast(xd, 0)
        dist.broadcast(wd, 0)
    ops_total = 2.0 * M * N * K
    golden = _c5_golden()
    out = {"shape": [M, K, N], "inputs": "numpy default_rng(0): x ~ N(0,1), w ~ N(0,0.02)",
           "outputs": "fp32 y + bposit32, column-major [M,N]", "ranks": ws}

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        _barrier(dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            r = fn()
        e1.record()
        torch.cuda.synchronize()
        own = e0.elapsed_time(e1) / steps
        return _max_over_ranks(dist, own), own, r

    # ---- N-shard
    n0, n1 = D.shard_range(N, ws, rank)
    xq, xs = ops.quantize_per_token(xd)
    wq, wsc = ops.quantize_per_channel(wd[n0:n1])
    res = {"y": torch.empty((n1 - n0, M), dtype=torch.float32, device=dev).t(),
           "bp32": torch.empty((n1 - n0, M), dtype=torch.int32, device=dev).t()}
    ms, own_ms, _ = timed(lambda: ops.gemm_i8(xq, wq, bp32=True, y_dtype=torch.float32,
                                              x_scale=xs, w_scale=wsc, out=res))
    out["nshard"] = {"ms_per_step": ms, "tpops": ops_total / ms / 1e9, "rank0_ms": own_ms,
                     "per_gpu_columns": n1 - n0}
    hashes = {}
    for k in ("bp32", "y"):
        full = D.gather_columns(res[k]) if dist is not None else res[k]
        if rank == 0:
            hashes[k] = _sha256_t(full.t())
        del full
    if rank == 0:
        out["nshard"]["sha256"] = hashes
        if golden:
            out["nshard"]["bit_identical_to_oracle"] = (hashes["bp32"] == golden["bp32"] and
                                                        hashes["y"] == golden["y_f32"])
    del res, wq
    # ---- K-split
    if dist is not None:
        k0, k1 = D.shard_range(K, ws, rank)
        xq_s, xs_g = D.ksplit_quantize_rows(xd[:, k0:k1].contiguous())
        wq_s, ws_g = D.ksplit_quantize_rows(wd[:, k0:k1].contiguous())

        def kstep():
            return D.ksplit_gemm_i8(xq_s, wq_s, bp32=True, y_dtype=torch.float32, x_scale=xs_g,
                                    w_scale=ws_g, chunks=chunks, gather=False)
        ms_k, own_k, r = timed(kstep)
        # the same with the chunk GEMMs on every SM (no room left for NCCL)
        ms_k_all, _, r_all = timed(lambda: D.ksplit_gemm_i8(
            xq_s, wq_s, bp32=True, y_dtype=torch.float32, x_scale=xs_g, w_scale=ws_g,
            chunks=chunks, gather=False, gemm_sms=1 << 30))
        del r_all
        # the reduce-scatter alone, on buffers of the same size
        L = D.ksplit_layout(N, ws, chunks)
        src = torch.zeros((L["padded"], M), dtype=torch.int32, device=dev)
        dst = torch.empty((L["padded"] // ws, M), dtype=torch.int32, device=dev)
        ms_rs, _, _ = timed(lambda: dist.reduce_scatter_tensor(dst, src))
        del src, dst
        g = D.ksplit_gather(r, N, chunks=chunks, keys=("bp32", "y"))
        kh = {k: _sha256_t(g[k].t()) for k in ("bp32", "y")} if rank == 0 else {}
        del g, r
        out["ksplit"] = {"ms_per_step": ms_k, "tpops": ops_total / ms_k / 1e9, "rank0_ms": own_k,
                         "chunks": chunks, "gemm_sms": _api_sm_count() - D.KSPLIT_NCCL_SMS,
                         "ms_per_step_gemm_on_all_sms": ms_k_all, "reduce_scatter_ms": ms_rs,
                         "reduce_scatter_bytes_per_rank": 4 * L["padded"] * M,
                         "reduce_scatter_busbw_gbs": (ws - 1) / ws * 4 * L["padded"] * M / ms_rs / 1e6,
                         "note": "per step: partial INT32 GEMMs of the K slice on gemm_sms SMs, "
                                 "NCCL int32 reduce-scatter per chunk on the others (overlapping "
                                 "the next chunk's GEMM), fp32 y + bposit32 epilogue of the owned "
                                 "columns on all SMs"}
        if rank == 0:
            out["ksplit"]["sha256"] = kh
            if golden:
                out["ksplit"]["bit_identical_to_oracle"] = (kh["bp32"] == golden["bp32"] and
                                                            kh["y"] == golden["y_f32"])
        del xq_s, wq_s
        # the same problem on rank 0's GPU alone, in this run
        if rank == 0:
            wq1, ws1 = ops.quantize_per_channel(wd)
            r1 = ops.gemm_i8(xq, wq1, bp32=True, y_dtype=torch.float32, x_scale=xs, w_scale=ws1)
            torch.cuda.synchronize()
            one = {"bp32": _sha256_t(r1["bp32"].t()), "y": _sha256_t(r1["y"].t())}
            del r1, wq1
            out["one_gpu_sha256"] = one
            out["bit_identical_to_1gpu"] = {"nshard": hashes == one, "ksplit": kh == one}
        _barrier(dist)
    if rank == 0 and golden:
        out["oracle_sha256"] = {"bp32": golden["bp32"], "y": golden["y_f32"]}
    del xd, wd, xq
    torch.cuda.empty_cache()
    return out


def _ours(A, B, out, stream, lib, flags=0):
    M, K = A.shape
    N = B.shape[0]
    rc = lib.mosyne_bposit_gemm_i8(A.data_ptr(), B.data_ptr(), M, N, K, 0, 0, out.data_ptr(), 0, 0,
                                   0, 0, flags, stream.cuda_stream)
    if rc != 0:
        raise RuntimeError(f"mosyne_bposit_gemm_i8 rc={rc}")


def _cublas_i8(A, B, out, stream):
    import torch
    torch._int_mm(A, B.t())


def _e2e(M, N, K, steps, lib, dist=None, ws=1):
    """Same workload through the host-buffer C entry point: pinned host A, B
    in, host bposit32 out; H2D + GEMM + D2H inside the timed region (wall
    clock, every rank at once between barriers, the slowest rank counts)."""
    import torch
    g = torch.Generator(device="cpu").manual_seed(7)
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).pin_memory()
    B = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).pin_memory()
    out = torch.empty((N, M), dtype=torch.int32).pin_memory()
    for _ in range(2):
        lib.mosyne_bposit_gemm_i8_host(A.data_ptr(), B.data_ptr(), M, N, K, out.data_ptr(), 0, 0)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        rc = lib.mosyne_bposit_gemm_i8_host(A.data_ptr(), B.data_ptr(), M, N, K, out.data_ptr(), 0, 0)
        if rc != 0:
            raise RuntimeError(f"mosyne_bposit_gemm_i8_host rc={rc}")
    torch.cuda.synchronize()
    dt = _max_over_ranks(dist, (time.perf_counter() - t0) / steps)
    return {"value": ws * 2.0 * M * N * K / dt / 1e12, "unit": UNIT, "ms_per_step": dt * 1e3,
            "h2d_bytes_per_step": ws * (M * K + N * K), "d2h_bytes_per_step": ws * 4 * M * N,
            "api": "mosyne_bposit_gemm_i8_host (pinned host buffers; uploads, GEMM and downloads "
                   "pipelined over blocks of output channels)"}


# --------------------------------------------------------------------- CPU port

def _cpu_port_step(A, B, pool):
    """Exact integer GEMM (float64 BLAS, exact for |sums| < 2^53) and the
    bposit32 code of every output, encoded in parallel row blocks."""
    import numpy as np

    from oracle import bposit_oracle as O
    acc = O.gemm_exact(A, B.T)
    chunks = np.array_split(acc, max(1, min(len(acc), os.cpu_count() or 1)))
    list(pool.map(lambda c: O.encode_int_array(c, 0, 32), chunks))
    return acc.size


def _cpu_rows_for(M, N, K, target_s, pool):
    import numpy as np
    rng = np.random.default_rng(0)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    rows = 16
    while True:
        A = rng.integers(-127, 128, (rows, K), dtype=np.int8)
        t0 = time.perf_counter()
        _cpu_port_step(A, B, pool)
        dt = time.perf_counter() - t0
        if dt >= target_s or rows >= M:
            return rows, dt, B
        rows = min(M, rows * 2 if dt < target_s / 4 else int(rows * target_s / max(dt, 1e-3)) + 1)


def cpu_baseline(M, N, K, target_s=3.0, total_s=10.0):
    """Timed oracle port on a bounded row block of the workload, repeated
    for about `total_s` seconds."""
    import numpy as np
    cores = os.cpu_count() or 1
    with cf.ThreadPoolExecutor(cores) as pool:
        rows, dt, B = _cpu_rows_for(M, N, K, target_s, pool)
        A = np.random.default_rng(1).integers(-127, 128, (rows, K), dtype=np.int8)
        reps = max(1, int(total_s / max(dt, 1e-3)))
        t0 = time.perf_counter()
        for _ in range(reps):
            _cpu_port_step(A, B, pool)
        dt = (time.perf_counter() - t0) / reps
    return {"value": 2.0 * rows * N * K / dt / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{rows} of {M} rows of the {M}x{N}x{K} GEMM (all {N} columns, full K), "
                      f"numpy float64-BLAS exact GEMM + vectorised bposit32 encode of every "
                      f"output on {cores} threads; {reps} repetitions, {dt:.2f} s each"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    name, M, N, K = HEADLINE
    import numpy as np
    cores = os.cpu_count() or 1
    with cf.ThreadPoolExecutor(cores) as pool:
        rows, _, B = _cpu_rows_for(M, N, K, 1.5, pool)
        A = np.random.default_rng(2).integers(-127, 128, (rows, K), dtype=np.int8)
        for _ in range(args.warmup):
            _cpu_port_step(A, B, pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _cpu_port_step(A, B, pool)
        dt = (time.perf_counter() - t0) / args.steps
    value = 2.0 * rows * N * K / dt / 1e12
    sample = (f"{rows} of {M} rows of the {M}x{N}x{K} GEMM per step: numpy float64-BLAS exact "
              f"GEMM + vectorised bposit32 encode on {cores} threads")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"int8 GEMM {M}x{N}x{K} -> INT32 -> bposit32 (truncate)",
                       "M": M, "N": N, "K": K, "implementation": "CPU restatement of the "
                       "reference's numpy + bposit16_reference.py path (oracle port)"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch

    from mosyne_bposit import _api
    dist, rank, local, ws = _dist()
    if dist is None:
        torch.cuda.set_device(0)
    lib = _api.load_library(init=True)
    call = lambda A, B, out, st: _ours(A, B, out, st, lib)  # noqa: E731
    name, M, N, K = HEADLINE
    ops = 2.0 * M * N * K
    with Clocks(local) as clk:
        ms, nsets, _ = _time_gemm(M, N, K, args.steps, args.warmup, dist, 100 + rank, call)
    rank_ms = _all_ranks(dist, ms / args.steps)
    ms = _max_over_ranks(dist, ms)
    clocks = clk.summary()
    per_launch_ms = ms / args.steps
    value = ws * ops / (per_launch_ms * 1e-3) / 1e12
    # at N > 1: the same GEMM on rank 0's GPU alone, the other GPUs idle, in this
    # job -- the one-GPU reference of the same box for the weak-scaling ratio
    solo_ms = None
    if dist is not None:
        _barrier(dist)
        if rank == 0:
            solo_ms, _, _ = _time_gemm(M, N, K, args.steps, args.warmup, None, 100, call)
        _barrier(dist)
    # second shape (same method)
    n2, M2, N2, K2 = SECOND
    ms2, nsets2, _ = _time_gemm(M2, N2, K2, args.steps, args.warmup, dist, 200 + rank, call)
    ms2 = _max_over_ranks(dist, ms2)
    v2 = ws * 2.0 * M2 * N2 * K2 / (ms2 / args.steps * 1e-3) / 1e12
    rc = _api.last_error()
    if rc != 0:
        raise RuntimeError(f"device error word set during the timed region (rc={rc})")
    # cuBLASLt INT8 (INT32 out, no bposit) on the same shapes, for context
    lib_ms, _, _ = _time_gemm(M, N, K, args.steps, args.warmup, None, 300 + rank, _cublas_i8)
    lib_ms2, _, _ = _time_gemm(M2, N2, K2, args.steps, args.warmup, None, 400 + rank, _cublas_i8)
    e2e = _e2e(M, N, K, max(3, min(args.steps, 10)), lib, dist, ws)
    c5 = c5_workload(dist, ws, rank, max(3, min(args.steps, 10)), 2)
    c2det = c2_determinism(dist, ws, rank)
    rc = _api.last_error()
    if rc != 0:
        raise RuntimeError(f"device error word set during the C5 runs (rc={rc})")
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return
    peaks = _peaks()
    peak = 2.0 * peaks["bf16"]
    achieved = ops / (per_launch_ms * 1e-3) / 1e12
    lib_tpops = ops / (lib_ms / args.steps * 1e-3) / 1e12
    lib_tpops2 = 2.0 * M2 * N2 * K2 / (lib_ms2 / args.steps * 1e-3) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_launch_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"int8 GEMM {M}x{N}x{K} -> exact INT32 -> bposit32 (truncate), "
                               "A row-major, B column-major, uniform int8 [-127,127]",
                   "M": M, "N": N, "K": K, "outputs": "bposit32 column-major [M,N]",
                   "parallelism": f"N-shard x{ws} (column-parallel, no collective)",
                   "l2": f"inputs rotate over {nsets} buffer sets (> 3x L2), no flush needed"},
        "workloads": {
            name: {"tpops": value, "ms_per_launch": per_launch_ms,
                   "frac_of_int8_peak": achieved / peak,
                   "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
                   "cublaslt_int8_int32_out_tpops": ops / (lib_ms / args.steps * 1e-3) / 1e12},
            n2: {"tpops": v2, "ms_per_launch": ms2 / args.steps,
                 "frac_of_int8_peak": (v2 / ws) / peak,
                 "frac_of_nominal_4500": (v2 / ws) / NOMINAL_INT8_TOPS,
                 "cublaslt_int8_int32_out_tpops": 2.0 * M2 * N2 * K2 / (lib_ms2 / args.steps * 1e-3) / 1e12},
        },
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": _traffic(name),
                     "peak_source": f"2 x {peaks['src']} bf16 dense ({peaks['bf16']} TFLOP/s; "
                                    "sm_100 int8 dense rate = 2x bf16); int8 ops counted as 2MNK",
                     "kernel": "gemm_i8_tcgen05_pair", "algorithmic": f"2*M*N*K = {ops:.4g} ops per launch"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "ms_per_launch_by_rank": rank_ms,
        "same_box_one_gpu_ms_per_launch": None if solo_ms is None else solo_ms / args.steps,
        # per GPU, this build against cuBLASLt INT8 (INT32 out only) on the same GPU
        "tpops_per_gpu": {"4096^3": achieved, "2048x14336x4096": v2 / ws},
        "cublaslt_int8_tpops": {"4096^3": lib_tpops, "2048x14336x4096": lib_tpops2},
        "vs_cublaslt": {"4096^3": achieved / lib_tpops, "2048x14336x4096": (v2 / ws) / lib_tpops2},
        "c5_16384x8192x28672": c5,
    }
    if dist is not None:
        line["c5_tpops"] = {"nshard": c5["nshard"]["tpops"], "ksplit": c5["ksplit"]["tpops"]}
        line["bit_identical_to_1gpu"] = c5.get("bit_identical_to_1gpu")
    else:
        line["c5_tpops"] = {"one_gpu": c5["nshard"]["tpops"]}
    line["c5_bit_identical_to_oracle"] = {k: c5[k].get("bit_identical_to_oracle")
                                          for k in ("nshard", "ksplit") if k in c5}
    line["c2_determinism_every_gpu"] = c2det
    line["e2e"] = e2e
    if ws == 1:
        line["workloads"].update(extra_workloads(args.steps, args.warmup, peaks))
        line["kernels"] = kernel_table(args.steps, args.warmup, peaks)
        line["cpu_baseline"] = cpu_baseline(M, N, K)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_only_c5(args):
    """--only-c5: the C5 workload alone (any N), one JSON line from rank 0."""
    import torch

    from mosyne_bposit import _api
    dist, rank, local, ws = _dist()
    if dist is None:
        torch.cuda.set_device(0)
    _api.load_library(init=True)
    c5 = c5_workload(dist, ws, rank, args.steps, args.warmup, chunks=args.chunks)
    rc = _api.last_error()
    if rank == 0:
        print(json.dumps({"c5_16384x8192x28672": c5, "n_gpus": ws, "device_error": rc}), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_only_gemm(args):
    import torch

    from mosyne_bposit import _api
    torch.cuda.set_device(0)
    lib = _api.load_library(init=True)
    M, N, K = (int(v) for v in args.only_gemm.split(","))
    ms, nsets, _ = _time_gemm(M, N, K, args.steps, args.warmup, None, 1,
                              lambda A, B, out, st: _ours(A, B, out, st, lib, args.gemm_flags))
    rc = _api.last_error()
    per = ms / args.steps
    print(json.dumps({"shape": [M, N, K], "flags": args.gemm_flags, "ms_per_launch": per,
                      "tpops": 2.0 * M * N * K / per / 1e9, "buffer_sets": nsets,
                      "device_error": rc}), flush=True)


def run_tables(args):
    """--workloads / --kernels: only the selected secondary rows (for
    profilers); prints one JSON line."""
    import torch

    from mosyne_bposit import _api
    torch.cuda.set_device(0)
    _api.load_library(init=True)
    peaks = _peaks()
    line = {}
    if args.workloads:
        sel = None if args.workloads == "all" else set(args.workloads.split(","))
        line["workloads"] = extra_workloads(args.steps, args.warmup, peaks, sel)
    if args.kernels:
        line["kernels"] = kernel_table(args.steps, args.warmup, peaks)
    line["device_error"] = _api.last_error()
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--only-gemm", default=None, metavar="M,N,K",
                    help="time only the fused GEMM at this shape (for profilers); prints one line")
    ap.add_argument("--gemm-flags", type=lambda v: int(v, 0), default=0,
                    help="flags word passed to mosyne_bposit_gemm_i8 with --only-gemm "
                         "(e.g. 0x100000 * (1 + cut) pins the last-wave cut)")
    ap.add_argument("--workloads", default=None, metavar="c1,c2,qkt,ffn,dec,sq,bp8|all",
                    help="run only these secondary workloads and print them (for profilers)")
    ap.add_argument("--only-c5", action="store_true",
                    help="run only the C5 16384x8192x28672 workload (N-shard, K-split, hashes)")
    ap.add_argument("--chunks", type=int, default=4, help="K-split reduce-scatter chunks (--only-c5)")
    ap.add_argument("--kernels", action="store_true",
                    help="run only the element-wise / quantiser kernel table (for profilers)")
    args = ap.parse_args()
    if args.warmup < 3 and not (args.workloads or args.kernels):
        args.warmup = 3
    if args.only_gemm:
        run_only_gemm(args)
    elif args.only_c5:
        run_only_c5(args)
    elif args.workloads or args.kernels:
        run_tables(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
