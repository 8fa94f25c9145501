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
  quantising.  Each rank's GEMM yields an exact INT32 partial; an
  ``all_reduce(SUM)`` on int32 is exact and order independent (two's
  complement addition is associative and the total fits in int32 when
  127^2 * K < 2^31) -- the quire argument at the width the value needs.
  The fused epilogue (bposit32/bposit16/dequant) then runs on the summed
  INT32.

The local compute steps are parameters (``local_gemm``, ``local_epilogue``,
``local_quant``) defaulting to the CUDA library; the collective logic does
not care which device the tensors live on.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

MAX_EXACT_K = (2 ** 31 - 1) // (127 * 127)    # INT32 total stays exact up to this K


def shard_range(total: int, world: int, rank: int) -> tuple:
    """Contiguous block of ``total`` owned by ``rank`` (sizes differ by <= 1)."""
    return total * rank // world, total * (rank + 1) // world


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


# ----------------------------------------------------------------- defaults

def _cuda_gemm_i32(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    from . import ops
    return ops.gemm_i8(A, B, bp32=False, i32=True)["i32"]


def _cuda_epilogue(acc: torch.Tensor, *, bp32: bool, bp16: bool, y_dtype, x_scale, w_scale,
                   rtne32: bool, rtne16: bool) -> dict:
    from . import ops
    return ops.epilogue_i32(acc, bp32=bp32, bp16=bp16, y_dtype=y_dtype, x_scale=x_scale,
                            w_scale=w_scale, rtne32=rtne32, rtne16=rtne16)


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
    world, _ = _world(group)
    full = {}
    for k in sorted(out):
        t = out[k]
        # gather [N_r, M] storage blocks (column-major outputs are N-blocks)
        store = t.t().contiguous()
        sizes = [torch.zeros(1, dtype=torch.int64, device=store.device) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([store.shape[0]], dtype=torch.int64, device=store.device),
                        group=group)
        mx = int(max(s.item() for s in sizes))
        pad = torch.zeros((mx, store.shape[1]), dtype=store.dtype, device=store.device)
        pad[: store.shape[0]] = store
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad, group=group)
        cat = torch.cat([p[: int(s.item())] for p, s in zip(parts, sizes)], dim=0)
        full[k] = cat.t()
    return full


# ----------------------------------------------------------------- K-split

# total K per (process group, local K slice), checked against MAX_EXACT_K
_K_TOTALS: dict = {}


def ksplit_gemm_i8(A_shard: torch.Tensor, B_shard: torch.Tensor, *, bp32: bool = True,
                   bp16: bool = False, y_dtype=None, x_scale=None, w_scale=None,
                   rtne32: bool = False, rtne16: bool = False, group=None, chunks: int = 0,
                   local_gemm: Optional[Callable] = None,
                   local_epilogue: Optional[Callable] = None) -> dict:
    """K-split fused GEMM: ``A_shard [M,K_r]``, ``B_shard [N,K_r]`` (this
    rank's K slice).  Exact INT32 partials, ``all_reduce(SUM)``, then the
    epilogue.  Every rank returns the full ``[M,N]`` outputs, bit-identical
    to the one-GPU result.  ``chunks`` > 1 splits the output channels into
    blocks whose all-reduce is issued as soon as each block's GEMM is done
    (on B200 the GEMM occupies every SM, so NCCL's kernels only run between
    blocks: one block measured faster)."""
    world, _ = _world(group)
    key = (id(group), A_shard.shape[1])
    k_sum = _K_TOTALS.get(key)
    if k_sum is None:                     # once per (group, local K): a host sync
        k_total = torch.tensor([A_shard.shape[1]], dtype=torch.int64, device=A_shard.device)
        dist.all_reduce(k_total, group=group)
        k_sum = _K_TOTALS[key] = int(k_total.item())
    if k_sum > MAX_EXACT_K:
        raise ValueError(f"K={k_sum} exceeds {MAX_EXACT_K}: the INT32 sum could wrap")
    M, N = A_shard.shape[0], B_shard.shape[0]
    nchunks = max(1, chunks)
    gemm = local_gemm or _cuda_gemm_i32
    store = torch.empty((N, M), dtype=torch.int32, device=A_shard.device)   # column-major [M,N]
    pending = []
    for c in range(nchunks):
        n0, n1 = shard_range(N, nchunks, c)
        if n1 <= n0:
            continue
        if local_gemm is None:            # the GEMM writes its block of the sum buffer
            from . import ops
            ops.gemm_i8(A_shard, B_shard[n0:n1], bp32=False, i32=True,
                        out={"i32": store[n0:n1].t()})
        else:
            store[n0:n1] = gemm(A_shard, B_shard[n0:n1]).t()
        pending.append(dist.all_reduce(store[n0:n1], op=dist.ReduceOp.SUM, group=group,
                                       async_op=True))
    for work in pending:
        work.wait()
    acc = store.t()
    res = (local_epilogue or _cuda_epilogue)(acc, bp32=bp32, bp16=bp16, y_dtype=y_dtype,
                                             x_scale=x_scale, w_scale=w_scale, rtne32=rtne32,
                                             rtne16=rtne16)
    res["i32"] = acc
    return res


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
                  out_dtype=torch.float32, bp32: bool = False, group=None, **local) -> dict:
    """W8A8 linear with K split across ranks: row-major ``x_shard [M,K_r]``,
    ``w_i8_shard [N,K_r]`` (this rank's K slice of the ``nn.Linear`` weight,
    quantised with scales computed on the FULL weight), ``w_scale [N]``."""
    q, xs = ksplit_quantize_rows(x_shard, group=group,
                                       local_absmax=local.get("local_absmax"),
                                       local_quant=local.get("local_quant"))
    return ksplit_gemm_i8(q, w_i8_shard, bp32=bp32, y_dtype=out_dtype, x_scale=xs,
                          w_scale=w_scale, group=group, local_gemm=local.get("local_gemm"),
                          local_epilogue=local.get("local_epilogue"))


ksplit_quantize_activation = ksplit_quantize_rows
ksplit_quantize_weight = ksplit_quantize_rows
