"""Multi-GPU partitionings of the W8A8 / INT8 GEMM path (one process per GPU,
``torch.distributed`` over NCCL for the plumbing).

The reference has no multi-GPU code; these two partitionings keep results
bit-identical to one GPU for any GPU count:

* **N-shard (column-parallel)** -- rank r owns output channels
  ``[N*r//p, N*(r+1)//p)``: a contiguous block of the column-major weight
  ``[K,N]`` (rows of the ``nn.Linear`` weight) and its scales.  Every rank
  sees the whole activation, computes identical per-token scales, and
  produces its own output columns.  No collective on the data path
  (``gather=True`` all-gathers the blocks afterwards).
* **K-split** -- rank r owns a slice of K of both operands.  Activation
  scales must be global: each rank takes its slice's row maxima and an
  ``all_reduce(MAX)`` (exact, order free) gives the global maxima before
  quantising.  Each rank's GEMM yields an exact integer partial of every
  output; the partials are summed exactly over NCCL and the fused epilogue
  (bposit32 / bposit16 / dequant) runs on the sums.  Integer addition is
  associative (two's-complement wrap-around included), so any rank count
  and any reduction order give the same sums: the reference's quire
  argument (docs/whitepaper/mosyne_bposit_whitepaper.tex:495-507) at the
  width the value needs.  The partials travel as INT32 while the total
  fits (127^2 * K < 2^31) and as INT64 lanes beyond that (exact for
  K < 5.7e14).

  The default reduction is a **reduce-scatter**: the partial columns are cut
  into ``chunks`` chunks of ``p`` equal blocks; rank r receives the sums of
  block r of every chunk and encodes only those columns (1/p of the
  epilogue, half the bytes of an all-reduce on the wire).  The GEMM of
  chunk c+1 runs while chunk c is being reduced.  ``reduce="all"`` keeps an
  all-reduce of every partial, after which every rank encodes everything.

The local compute steps are parameters (``local_gemm``, ``local_epilogue``,
``local_quant``, ...) defaulting to the CUDA library; the collective logic
does not care which device the tensors live on.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

MAX_EXACT_K = (2 ** 31 - 1) // (127 * 127)    # INT32 total stays exact up to this K
MAX_EXACT_K_WIDE = (2 ** 63 - 1) // (127 * 127)
# SMs a chunked K-split leaves to NCCL by default (its reduce-scatter kernels)
KSPLIT_NCCL_SMS = 16


def _all_sms(limit) -> None:
    if limit:
        from . import _api
        _api.set_sm_count_target(0)


def shard_range(total: int, world: int, rank: int) -> tuple:
    """Contiguous block of ``total`` owned by ``rank`` (sizes differ by <= 1)."""
    return total * rank // world, total * (rank + 1) // world


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


# ----------------------------------------------------------------- defaults

def _cuda_gemm_i32(A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None):
    from . import ops
    return ops.gemm_i8(A, B, bp32=False, i32=True,
                       out=None if out is None else {"i32": out})["i32"]


def _cuda_epilogue(acc: torch.Tensor, *, bp32: bool, bp16: bool, y_dtype, x_scale, w_scale,
                   rtne32: bool, rtne16: bool) -> dict:
    from . import ops
    fn = ops.epilogue_i64 if acc.dtype == torch.int64 else ops.epilogue_i32
    return fn(acc, bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale, w_scale=w_scale,
              rtne32=rtne32, rtne16=rtne16)


def _cuda_widen(src: torch.Tensor, dst: torch.Tensor, accumulate: bool) -> None:
    from . import ops
    ops.widen_i32(src, dst, accumulate=accumulate)


def _cuda_gemm_full(A, B, *, bp32, bp16, y_dtype, x_scale, w_scale, rtne32, rtne16):
    from . import ops
    return ops.gemm_i8(A, B, bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale,
                       w_scale=w_scale, rtne32=rtne32, rtne16=rtne16)


def _cuda_row_absmax(x):
    from . import ops
    return ops.row_absmax(x)


def _cuda_quant_with_max(x, row_max):
    from . import ops
    return ops.quantize_with_max(x, row_max)


# ----------------------------------------------------------------- N-shard

def nshard_gemm_i8(A: torch.Tensor, B_shard: torch.Tensor, *, bp32: bool = True, bp16: bool = False,
                   y_dtype=None, x_scale=None, w_scale_shard=None, rtne32: bool = False,
                   rtne16: bool = False, gather: bool = False, group=None,
                   local_gemm: Optional[Callable] = None) -> dict:
    """Column-parallel fused GEMM: ``A [M,K]`` on every rank, ``B_shard
    [N_r,K]`` = this rank's output channels.  Returns this rank's ``[M,N_r]``
    outputs, or with ``gather`` the full ``[M,N]`` (all-gathered blocks)."""
    fn = local_gemm or _cuda_gemm_full
    out = fn(A, B_shard, bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale,
             w_scale=w_scale_shard, rtne32=rtne32, rtne16=rtne16)
    if not gather:
        return out
    return {k: gather_columns(t, group=group) for k, t in out.items()}


def gather_columns(t: torch.Tensor, *, group=None) -> torch.Tensor:
    """All-gather column blocks ``[M, N_r]`` (stored column-major, i.e. the
    transpose views of ``[N_r, M]`` tensors) of every rank, in rank order,
    into the full column-major ``[M, N]`` on every rank."""
    world, _ = _world(group)
    store = t.t().contiguous()                       # [N_r, M]
    sizes = [torch.zeros(1, dtype=torch.int64, device=store.device) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([store.shape[0]], dtype=torch.int64, device=store.device),
                    group=group)
    counts = [int(s.item()) for s in sizes]
    mx = max(counts)
    if all(c == mx for c in counts):
        full = torch.empty((world * mx, store.shape[1]), dtype=store.dtype, device=store.device)
        dist.all_gather_into_tensor(full, store, group=group)
        return full.t()
    pad = torch.zeros((mx, store.shape[1]), dtype=store.dtype, device=store.device)
    pad[: store.shape[0]] = store
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0).t()


# ----------------------------------------------------------------- K-split

# total K per (process group, local K slice), checked against the exact limits
_K_TOTALS: dict = {}


def _total_k(k_local: int, device, group) -> int:
    key = (id(group), k_local)
    k_sum = _K_TOTALS.get(key)
    if k_sum is None:                     # once per (group, local K): a host sync
        t = torch.tensor([k_local], dtype=torch.int64, device=device)
        dist.all_reduce(t, group=group)
        k_sum = _K_TOTALS[key] = int(t.item())
    return k_sum


def ksplit_layout(N: int, world: int, chunks: int = 1) -> dict:
    """Column ownership of the reduce-scatter K-split: ``N`` columns padded to
    ``nchunks * world * per`` and cut into ``nchunks`` chunks of ``world``
    blocks of ``per`` columns; rank r owns block r of every chunk."""
    chunks = max(1, int(chunks))
    per = _cdiv(_cdiv(N, chunks), world)
    cw = per * world
    nchunks = _cdiv(N, cw)
    return {"per": per, "chunk": cw, "nchunks": nchunks, "padded": cw * nchunks}


def ksplit_owned_columns(N: int, world: int, rank: int, chunks: int = 1) -> list:
    """The ``(n0, n1)`` column ranges rank ``rank`` owns (ranges may be empty
    at the padded end), in the order of its rows of the reduced buffer."""
    L = ksplit_layout(N, world, chunks)
    out = []
    for c in range(L["nchunks"]):
        a = c * L["chunk"] + rank * L["per"]
        out.append((min(a, N), min(a + L["per"], N)))
    return out


def _local_partial(dst: torch.Tensor, A: torch.Tensor, B: torch.Tensor, wide: bool,
                   local_gemm, local_widen) -> None:
    """Exact partial of ``A [M,K_r] @ B [n,K_r]^T`` into ``dst`` (storage
    ``[n, M]``, int32 or int64).  INT32 pieces of at most MAX_EXACT_K."""
    K = A.shape[1]
    gemm = local_gemm or _cuda_gemm_i32
    if not wide:
        if local_gemm is None:
            _cuda_gemm_i32(A, B, out=dst.t())
        else:
            dst.copy_(gemm(A, B).t())
        return
    tmp = None
    for j, k0 in enumerate(range(0, K, MAX_EXACT_K)):
        k1 = min(K, k0 + MAX_EXACT_K)
        a, b = (A, B) if (k0 == 0 and k1 == K) else (A[:, k0:k1].contiguous(), B[:, k0:k1].contiguous())
        if local_gemm is None:
            if tmp is None:
                tmp = torch.empty(dst.shape, dtype=torch.int32, device=dst.device)
            _cuda_gemm_i32(a, b, out=tmp.t())
            (local_widen or _cuda_widen)(tmp, dst, j > 0)
        else:
            part = gemm(a, b).t().to(torch.int64)
            if j == 0:
                dst.copy_(part)
            else:
                dst.add_(part)


def ksplit_gemm_i8(A_shard: torch.Tensor, B_shard: torch.Tensor, *, bp32: bool = True,
                   bp16: bool = False, y_dtype=None, x_scale=None, w_scale=None,
                   rtne32: bool = False, rtne16: bool = False, group=None,
                   reduce: str = "scatter", chunks: int = 1, gather: bool = True,
                   wide: Optional[bool] = None, local_gemm: Optional[Callable] = None,
                   local_epilogue: Optional[Callable] = None,
                   local_widen: Optional[Callable] = None,
                   gemm_sms: Optional[int] = None) -> dict:
    """K-split fused GEMM: ``A_shard [M,K_r]``, ``B_shard [N,K_r]`` (this
    rank's K slice), global scales ``x_scale [M]`` / ``w_scale [N]`` (or one
    value).  Exact integer partials, summed over the ranks, then the epilogue.

    ``wide`` (default: when 127^2 * K_total >= 2^31) carries INT64 partials.
    ``reduce="scatter"``: see the module docstring; with ``gather`` every rank
    returns the full ``[M,N]`` outputs (the encoded outputs are
    all-gathered), else only its own columns: ``res["cols"]`` lists their
    ``(n0, n1)`` ranges, in order, and the outputs have one column per owned
    column plus padding (``ksplit_layout``).  ``reduce="all"``: every rank
    returns everything.  ``res["i32"]`` / ``res["i64"]`` is the summed
    accumulator of the columns returned.  ``gemm_sms`` (CUDA library only):
    the chunk GEMMs run on at most that many SMs, leaving the rest to NCCL so
    a chunk's reduction overlaps the next chunk's GEMM (default: all SMs with
    one chunk, all but ``KSPLIT_NCCL_SMS`` with more)."""
    world, rank = _world(group)
    k_sum = _total_k(A_shard.shape[1], A_shard.device, group)
    if wide is None:
        wide = k_sum > MAX_EXACT_K
    if not wide and k_sum > MAX_EXACT_K:
        raise ValueError(f"K={k_sum} exceeds {MAX_EXACT_K}: INT32 partial sums could wrap "
                         "(pass wide=True or leave wide unset)")
    if k_sum > MAX_EXACT_K_WIDE:
        raise ValueError(f"K={k_sum} exceeds {MAX_EXACT_K_WIDE}: INT64 sums could wrap")
    M, N = A_shard.shape[0], B_shard.shape[0]
    limit = None
    if local_gemm is None and A_shard.is_cuda:
        from . import _api
        if gemm_sms is None and max(1, chunks) > 1:
            gemm_sms = max(2, _api.sm_count() - KSPLIT_NCCL_SMS)
        if gemm_sms:
            limit = gemm_sms
            _api.set_sm_count_target(limit)
    try:
        return _ksplit_body(A_shard, B_shard, M, N, wide, bp32=bp32, bp16=bp16, y_dtype=y_dtype,
                            x_scale=x_scale, w_scale=w_scale, rtne32=rtne32, rtne16=rtne16,
                            group=group, reduce=reduce, chunks=chunks, gather=gather,
                            local_gemm=local_gemm, local_epilogue=local_epilogue,
                            local_widen=local_widen, world=world, rank=rank, limit=limit)
    finally:
        _all_sms(limit)


def _ksplit_body(A_shard, B_shard, M, N, wide, *, bp32, bp16, y_dtype, x_scale, w_scale, rtne32,
                 rtne16, group, reduce, chunks, gather, local_gemm, local_epilogue, local_widen,
                 world, rank, limit):
    dt = torch.int64 if wide else torch.int32
    acc_key = "i64" if wide else "i32"
    dev = A_shard.device
    epi = local_epilogue or _cuda_epilogue
    kw = dict(bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale, rtne32=rtne32,
              rtne16=rtne16)

    if reduce == "all":
        nchunks = max(1, chunks)
        store = torch.empty((N, M), dtype=dt, device=dev)       # column-major [M,N]
        pending = []
        for c in range(nchunks):
            n0, n1 = shard_range(N, nchunks, c)
            if n1 <= n0:
                continue
            _local_partial(store[n0:n1], A_shard, B_shard[n0:n1], wide, local_gemm, local_widen)
            pending.append(dist.all_reduce(store[n0:n1], op=dist.ReduceOp.SUM, group=group,
                                           async_op=True))
        for work in pending:
            work.wait()
        _all_sms(limit)
        acc = store.t()
        res = epi(acc, w_scale=w_scale, **kw)
        res[acc_key] = acc
        res["cols"] = [(0, N)]
        return res
    if reduce != "scatter":
        raise ValueError("reduce must be 'scatter' or 'all'")

    L = ksplit_layout(N, world, chunks)
    per, cw, nch, Np = L["per"], L["chunk"], L["nchunks"], L["padded"]
    store = torch.empty((Np, M), dtype=dt, device=dev)
    if Np > N:
        store[N:].zero_()                                      # padded columns add zeros
    recv = torch.empty((nch * per, M), dtype=dt, device=dev)
    pending = []
    for c in range(nch):
        c0, c1 = c * cw, min(N, (c + 1) * cw)
        if c1 > c0:
            _local_partial(store[c0:c1], A_shard, B_shard[c0:c1], wide, local_gemm, local_widen)
        pending.append(dist.reduce_scatter_tensor(recv[c * per:(c + 1) * per],
                                                  store[c0:c0 + cw], op=dist.ReduceOp.SUM,
                                                  group=group, async_op=True))
    for work in pending:
        work.wait()
    _all_sms(limit)
    # this rank's columns: block `rank` of every chunk; padded columns get
    # scale 1 (their sums are zero and are dropped)
    ws_own = w_scale
    if y_dtype is not None and w_scale is not None and w_scale.numel() != 1:
        wpad = torch.ones(Np, dtype=w_scale.dtype, device=w_scale.device)
        wpad[:N] = w_scale.reshape(-1)
        ws_own = wpad.view(nch, world, per)[:, rank, :].reshape(-1).contiguous()
    acc_own = recv.t()                                          # logical [M, nch * per]
    res = epi(acc_own, w_scale=ws_own, **kw)
    res[acc_key] = acc_own
    res["cols"] = ksplit_owned_columns(N, world, rank, chunks)
    if not gather:
        return res
    return ksplit_gather(res, N, chunks=chunks, group=group)


def ksplit_gather(res: dict, N: int, *, chunks: int = 1, keys=None, group=None) -> dict:
    """All-gather the per-rank outputs of a reduce-scatter ``ksplit_gemm_i8``
    (``gather=False``) into full column-major ``[M, N]`` tensors on every
    rank (``keys``: which outputs; default all)."""
    world, _ = _world(group)
    L = ksplit_layout(N, world, chunks)
    per, nch, Np = L["per"], L["nchunks"], L["padded"]
    full = {}
    for k, t in res.items():
        if k == "cols" or (keys is not None and k not in keys):
            continue
        st = t.t().contiguous()                                 # [nch * per, M]
        M = st.shape[1]
        allr = torch.empty((world * st.shape[0], M), dtype=st.dtype, device=st.device)
        dist.all_gather_into_tensor(allr, st, group=group)
        # [world, nch, per, M] -> [nch, world, per, M] -> columns in order
        full[k] = allr.view(world, nch, per, M).transpose(0, 1).reshape(Np, M)[:N].t()
    full["cols"] = [(0, N)]
    return full


def ksplit_quantize_rows(x_shard: torch.Tensor, *, group=None,
                         local_absmax: Optional[Callable] = None,
                         local_quant: Optional[Callable] = None):
    """Per-token quantisation of a K-sliced activation with GLOBAL scales:
    local row maxima -> ``all_reduce(MAX)`` -> quantise the local slice.
    Returns (``q_shard [M,K_r]``, ``x_scale [M]``) -- the same codes the
    one-GPU quantiser produces for these columns.  A K-sliced ``nn.Linear``
    weight ``[N,K_r]`` takes the same route (rows = output channels)."""
    row_max = (local_absmax or _cuda_row_absmax)(x_shard)
    dist.all_reduce(row_max, op=dist.ReduceOp.MAX, group=group)
    return (local_quant or _cuda_quant_with_max)(x_shard, row_max)


def ksplit_linear(x_shard: torch.Tensor, w_i8_shard: torch.Tensor, w_scale: torch.Tensor, *,
                  out_dtype=torch.float32, bp32: bool = False, group=None, reduce: str = "scatter",
                  chunks: int = 1, gather: bool = True, **local) -> dict:
    """W8A8 linear with K split across ranks: row-major ``x_shard [M,K_r]``,
    ``w_i8_shard [N,K_r]`` (this rank's K slice of the ``nn.Linear`` weight,
    quantised with scales computed on the FULL weight), ``w_scale [N]``."""
    q, xs = ksplit_quantize_rows(x_shard, group=group,
                                 local_absmax=local.get("local_absmax"),
                                 local_quant=local.get("local_quant"))
    return ksplit_gemm_i8(q, w_i8_shard, bp32=bp32, y_dtype=out_dtype, x_scale=xs,
                          w_scale=w_scale, group=group, reduce=reduce, chunks=chunks,
                          gather=gather, wide=local.get("wide"),
                          local_gemm=local.get("local_gemm"),
                          local_epilogue=local.get("local_epilogue"),
                          local_widen=local.get("local_widen"))


ksplit_quantize_activation = ksplit_quantize_rows
ksplit_quantize_weight = ksplit_quantize_rows
