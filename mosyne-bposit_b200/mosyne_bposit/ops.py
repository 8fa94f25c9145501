"""Torch-tensor front end of the C ABI (device tensors in, device tensors out).

Every function allocates its outputs with torch on the input's device and
launches on the current torch stream; the work itself is the CUDA library's.
Logical shapes follow the math: a column-major ``[M, N]`` output is returned
as the ``[M, N]`` transpose view of an ``[N, M]`` allocation.
"""
from __future__ import annotations

import torch

from . import _api

_DT = {torch.float32: _api.DT_F32, torch.bfloat16: _api.DT_BF16, torch.float16: _api.DT_F16,
       torch.float64: _api.DT_F64}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("mosyne_bposit ops take CUDA tensors")


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def _out(shape_mn, dtype, device, row_major):
    M, N = shape_mn
    if row_major:
        return torch.empty((M, N), dtype=dtype, device=device)
    return torch.empty((N, M), dtype=dtype, device=device).t()


def gemm_i8(A: torch.Tensor, B: torch.Tensor, *, bp32: bool = True, bp16: bool = False,
            i32: bool = False, y_dtype: torch.dtype | None = None,
            x_scale: torch.Tensor | None = None, w_scale: torch.Tensor | None = None,
            rtne32: bool = False, rtne16: bool = False, row_major: bool = False,
            out: dict | None = None, path: int = 0, tail: int = 0,
            scale_shift: int = 0, split: int = 0, stream_k: bool | None = None) -> dict:
    """Exact ``acc = A @ B^T`` for int8 ``A [M,K]`` and ``B [N,K]`` (both
    K-contiguous) with the requested encodings of every dot product:
    ``bp32``/``bp16`` (bposit of the INT32 value), ``i32``, and ``y`` =
    ``acc / (x_scale[m] * w_scale[n])`` when ``y_dtype`` is given
    (scalar scales broadcast).  ``out`` may pass preallocated tensors.
    ``scale_shift`` makes the bposit outputs encode ``acc / 2^scale_shift``.
    ``path`` and ``tail`` pin the kernel choice (tests): path 1 tensor cores,
    2/3 one-CTA tiles 128/256 wide, 4 CUDA cores, 5 CTA pairs; tail 1/2/3 cuts
    the CTA-pair kernel's last wave into whole/half/quarter tiles (and turns
    its stream-K phase off); ``stream_k`` True/False pins that phase on/off
    (None: the library's default); split (1-7) sets the single-CTA kernel's K
    slices."""
    _need_cuda(A, B, x_scale, w_scale)
    if A.dtype != torch.int8 or B.dtype != torch.int8:
        raise ValueError("A and B must be int8")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
        raise ValueError(f"shape mismatch: A {tuple(A.shape)} vs B {tuple(B.shape)}")
    A = A.contiguous()
    B = B.contiguous()
    M, K = A.shape
    N = B.shape[0]
    res = dict(out or {})
    dev = A.device
    if bp32 and "bp32" not in res:
        res["bp32"] = _out((M, N), torch.int32, dev, row_major)
    if bp16 and "bp16" not in res:
        res["bp16"] = _out((M, N), torch.int16, dev, row_major)
    if i32 and "i32" not in res:
        res["i32"] = _out((M, N), torch.int32, dev, row_major)
    flags = (_api.RTNE_BP32 if rtne32 else 0) | (_api.RTNE_BP16 if rtne16 else 0) | \
        (_api.OUT_ROW_MAJOR if row_major else 0)
    if y_dtype is not None:
        if x_scale is None or w_scale is None:
            raise ValueError("dequantised output needs x_scale and w_scale")
        if x_scale.numel() == 1:
            flags |= _api.XS_SCALAR
        if w_scale.numel() == 1:
            flags |= _api.WS_SCALAR
        if "y" not in res:
            res["y"] = _out((M, N), y_dtype, dev, row_major)
    if not 0 <= scale_shift <= 31:
        raise ValueError("scale_shift must be in 0..31")
    if not 0 <= split <= 7:
        raise ValueError("split must be in 0..7")
    flags |= ((path & 0xF) << 16) | ((tail & 0x3) << 20) | (scale_shift << 24) | (split << 29) | \
        (0 if stream_k is None else (1 << 23 if stream_k else 1 << 22))
    if flags >= 1 << 31:
        flags -= 1 << 32                                   # the C ABI takes a signed int
    _api.gemm_i8_dev(A.data_ptr(), B.data_ptr(), M, N, K,
                     x_scale=_ptr(x_scale), w_scale=_ptr(w_scale),
                     out_bp32=_ptr(res.get("bp32")), out_bp16=_ptr(res.get("bp16")),
                     out_y=_ptr(res.get("y")), y_dtype=_DT[y_dtype] if y_dtype else 0,
                     out_i32=_ptr(res.get("i32")), flags=flags, stream=_stream(A))
    return res


def gemm_i8_batched(A: torch.Tensor, B: torch.Tensor, *, bp32: bool = True, bp16: bool = False,
                    i32: bool = False, y_dtype: torch.dtype | None = None,
                    x_scale: torch.Tensor | None = None, w_scale: torch.Tensor | None = None,
                    rtne32: bool = False, rtne16: bool = False,
                    row_major: bool = False) -> dict:
    """``gemm_i8`` over a batch (attention scores per head): ``A [b,M,K]``,
    ``B [b,N,K]``, scales ``[b,M]`` / ``[b,N]`` (or one value); outputs
    ``[b,M,N]`` (column-major per entry unless ``row_major``)."""
    _need_cuda(A, B, x_scale, w_scale)
    if A.dtype != torch.int8 or B.dtype != torch.int8:
        raise ValueError("A and B must be int8")
    if A.dim() != 3 or B.dim() != 3 or A.shape[0] != B.shape[0] or A.shape[2] != B.shape[2]:
        raise ValueError(f"shape mismatch: A {tuple(A.shape)} vs B {tuple(B.shape)}")
    A = A.contiguous()
    B = B.contiguous()
    b, M, K = A.shape
    N = B.shape[1]
    dev = A.device

    def out(dtype):
        if row_major:
            return torch.empty((b, M, N), dtype=dtype, device=dev)
        return torch.empty((b, N, M), dtype=dtype, device=dev).transpose(1, 2)
    res = {}
    if bp32:
        res["bp32"] = out(torch.int32)
    if bp16:
        res["bp16"] = out(torch.int16)
    if i32:
        res["i32"] = out(torch.int32)
    flags = (_api.RTNE_BP32 if rtne32 else 0) | (_api.RTNE_BP16 if rtne16 else 0) | \
        (_api.OUT_ROW_MAJOR if row_major else 0)
    if y_dtype is not None:
        if x_scale is None or w_scale is None:
            raise ValueError("dequantised output needs x_scale and w_scale")
        x_scale, w_scale = x_scale.contiguous(), w_scale.contiguous()
        if x_scale.numel() == 1:
            flags |= _api.XS_SCALAR
        if w_scale.numel() == 1:
            flags |= _api.WS_SCALAR
        res["y"] = out(y_dtype)
    _api.gemm_i8_batched_dev(A.data_ptr(), B.data_ptr(), b, M, N, K, x_scale=_ptr(x_scale),
                             w_scale=_ptr(w_scale), out_bp32=_ptr(res.get("bp32")),
                             out_bp16=_ptr(res.get("bp16")), out_y=_ptr(res.get("y")),
                             y_dtype=_DT[y_dtype] if y_dtype else 0, out_i32=_ptr(res.get("i32")),
                             flags=flags, stream=_stream(A))
    return res


def quantize_per_token(x: torch.Tensor, *, col_major: bool = False):
    """Per-token int8 quantisation of ``x [M,K]`` -> (``q [M,K]`` K-contiguous,
    ``scale [M]``).  With ``col_major`` the tensor passed is the ``[K, M]``
    storage of a column-major ``[M, K]`` matrix (the reference's layout)."""
    _need_cuda(x)
    x = x.contiguous()
    if col_major:
        K, M = x.shape
        flags = 0
    else:
        M, K = x.shape
        flags = _api.X_ROW_MAJOR
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    _api.quantize_per_token_dev(x.data_ptr(), _DT[x.dtype], M, K, q.data_ptr(), s.data_ptr(),
                                flags=flags, stream=_stream(x))
    return q, s


def quantize_per_channel(w: torch.Tensor):
    """Per-output-channel int8 quantisation of an ``nn.Linear`` weight
    ``w [N,K]`` (= column-major ``[K,N]``) -> (``q [N,K]``, ``scale [N]``)."""
    _need_cuda(w)
    w = w.contiguous()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    s = torch.empty((N,), dtype=torch.float32, device=w.device)
    _api.quantize_weight_per_channel_ex_dev(w.data_ptr(), _DT[w.dtype], K, N, q.data_ptr(),
                                            s.data_ptr(), stream=_stream(w))
    return q, s


def quantize_per_tensor(t: torch.Tensor, *, col_major: bool = False):
    """One-scale int8 quantisation -> (``q`` row-major ``[rows, cols]``,
    ``scale [1]``).  With ``col_major`` the tensor passed is the ``[cols,
    rows]`` storage of a column-major matrix and ``q`` is its transpose."""
    _need_cuda(t)
    t = t.contiguous()
    if col_major:
        cols, rows = t.shape
        flags = 0
    else:
        rows, cols = t.shape
        flags = _api.X_ROW_MAJOR
    q = torch.empty((rows, cols), dtype=torch.int8, device=t.device)
    s = torch.empty((1,), dtype=torch.float32, device=t.device)
    _api.quantize_per_tensor_dev(t.data_ptr(), _DT[t.dtype], rows, cols, q.data_ptr(),
                                 s.data_ptr(), flags=flags, stream=_stream(t))
    return q, s


def row_absmax(x: torch.Tensor) -> torch.Tensor:
    """|max| of every row of a row-major ``x [M,K]`` (fp32 ``[M]``)."""
    _need_cuda(x)
    x = x.contiguous()
    M, K = x.shape
    out = torch.empty((M,), dtype=torch.float32, device=x.device)
    _api.row_absmax_dev(x.data_ptr(), _DT[x.dtype], M, K, out.data_ptr(), flags=_api.X_ROW_MAJOR,
                        stream=_stream(x))
    return out


def quantize_with_max(x: torch.Tensor, row_max: torch.Tensor):
    """Per-token quantisation of row-major ``x [M,K]`` with given row maxima
    -> (``q [M,K]``, ``scale [M]``)."""
    _need_cuda(x, row_max)
    x = x.contiguous()
    M, K = x.shape
    q = torch.empty((M, K), dtype=torch.int8, device=x.device)
    s = torch.empty((M,), dtype=torch.float32, device=x.device)
    _api.quantize_with_max_dev(x.data_ptr(), _DT[x.dtype], M, K, row_max.contiguous().data_ptr(),
                               q.data_ptr(), s.data_ptr(), flags=_api.X_ROW_MAJOR, stream=_stream(x))
    return q, s


def linear_w8a8(x: torch.Tensor, w_i8: torch.Tensor, w_scale: torch.Tensor, *,
                out_dtype: torch.dtype | None = None, y: bool = True, bp32: bool = False,
                bp16: bool = False,
                per_tensor: bool = False, rtne32: bool = False, rtne16: bool = False) -> dict:
    """Row-major W8A8 linear: ``x [M,K]`` (fp32/bf16/fp16) and a pre-quantised
    ``nn.Linear`` weight ``w_i8 [N,K]`` with ``w_scale [N]`` (or ``[1]``).
    Returns ``{"y": [M,N] in out_dtype (default x.dtype; omitted when
    ``y=False``), "bp32"?, "bp16"?}``, all row-major, with no transposes.
    bp32/bp16 encode the raw INT32 dot product (no scales)."""
    _need_cuda(x, w_i8, w_scale)
    x = x.contiguous()
    M, K = x.shape
    N = w_i8.shape[0]
    if w_i8.shape[1] != K:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} vs w {tuple(w_i8.shape)}")
    out_dtype = out_dtype or x.dtype
    res = {}
    if y:
        res["y"] = torch.empty((M, N), dtype=out_dtype, device=x.device)
    if bp32:
        res["bp32"] = torch.empty((M, N), dtype=torch.int32, device=x.device)
    if bp16:
        res["bp16"] = torch.empty((M, N), dtype=torch.int16, device=x.device)
    flags = _api.X_ROW_MAJOR | _api.OUT_ROW_MAJOR | (_api.X_PER_TENSOR if per_tensor else 0) | \
        (_api.WS_SCALAR if w_scale.numel() == 1 and N != 1 else 0) | \
        (_api.RTNE_BP32 if rtne32 else 0) | (_api.RTNE_BP16 if rtne16 else 0)
    _api.linear_w8a8_ex_dev(x.data_ptr(), _DT[x.dtype], M, K, w_i8.data_ptr(),
                            w_scale.data_ptr(), N, y=_ptr(res.get("y")),
                            y_dtype=_DT[out_dtype] if "y" in res else 0,
                            y_bp32=_ptr(res.get("bp32")), y_bp16=_ptr(res.get("bp16")),
                            flags=flags, stream=_stream(x))
    return res


def quire_sum_bp16(x: torch.Tensor, *, rtne16: bool = False, rtne32: bool = False,
                   max_blocks: int = 0):
    """Exact sum of bposit16 codes (int16/uint16 tensor) ->
    (quire words int64 [4], bposit16 code, bposit32 code) as device tensors."""
    _need_cuda(x)
    x = x.contiguous()
    q = torch.empty((4,), dtype=torch.int64, device=x.device)
    b16 = torch.empty((1,), dtype=torch.int16, device=x.device)
    b32 = torch.empty((1,), dtype=torch.int32, device=x.device)
    flags = (_api.RTNE_BP16 if rtne16 else 0) | (_api.RTNE_BP32 if rtne32 else 0) | \
        ((max_blocks & 0xFFFF) << 16)
    _api.quire_sum_bp16_dev(x.data_ptr(), x.numel(), q_out=q.data_ptr(), bp16_out=b16.data_ptr(),
                            bp32_out=b32.data_ptr(), flags=flags, stream=_stream(x))
    return q, b16, b32


def shannon_entropy_bp16(p: torch.Tensor, *, rtne32: bool = False, rtne16: bool = False,
                         max_blocks: int = 0):
    """Shannon entropy H = -sum p log2(p) of bposit16 probabilities (int16 or
    uint16 codes), every term p * log2(p) taken from the bposit16 term table
    and summed exactly -> (quire words int64 [4], bposit32 code, bposit16 code)
    as device tensors (kernels/shannon_entropy_bposit16.cu:63-119; the
    reference returns the bposit32 code)."""
    _need_cuda(p)
    p = p.contiguous()
    q = torch.empty((4,), dtype=torch.int64, device=p.device)
    b32 = torch.empty((1,), dtype=torch.int32, device=p.device)
    b16 = torch.empty((1,), dtype=torch.int16, device=p.device)
    flags = (_api.RTNE_BP16 if rtne16 else 0) | (_api.RTNE_BP32 if rtne32 else 0) | \
        ((max_blocks & 0xFFFF) << 16)
    _api.shannon_entropy_bp16_dev(p.data_ptr(), p.numel(), q_out=q.data_ptr(),
                                  bp32_out=b32.data_ptr(), bp16_out=b16.data_ptr(), flags=flags,
                                  stream=_stream(p))
    return q, b32, b16


def fp32_atomic_sum(x: torch.Tensor) -> torch.Tensor:
    """The non-deterministic IEEE control: fp32 atomicAdd of every element."""
    _need_cuda(x)
    acc = torch.zeros((1,), dtype=torch.float32, device=x.device)
    _api.fp32_atomic_sum_dev(x.contiguous().data_ptr(), x.numel(), acc.data_ptr(),
                             stream=_stream(x))
    return acc


def quire_to_bposit(q: torch.Tensor, nbits: int = 16, *, rtne: bool = False) -> torch.Tensor:
    """``q [n, 4]`` int64 quire words -> bposit16 (int16) or bposit32 (int32)."""
    _need_cuda(q)
    q = q.contiguous()
    n = q.shape[0]
    out = torch.empty((n,), dtype=torch.int16 if nbits == 16 else torch.int32, device=q.device)
    _api.quire_to_bposit_dev(q.data_ptr(), n, out.data_ptr(), nbits, rtne=rtne, stream=_stream(q))
    return out


def bp16_to_quire(x: torch.Tensor) -> torch.Tensor:
    _need_cuda(x)
    x = x.contiguous()
    out = torch.empty((x.numel(), 4), dtype=torch.int64, device=x.device)
    _api.bp16_to_quire_dev(x.data_ptr(), x.numel(), out.data_ptr(), stream=_stream(x))
    return out


def int32_to_bp32(x: torch.Tensor, scale_shift: int = 0, *, rtne: bool = False) -> torch.Tensor:
    _need_cuda(x)
    x = x.contiguous()
    out = torch.empty_like(x, dtype=torch.int32)
    _api.int32_to_bp32_dev(x.data_ptr(), x.numel(), scale_shift, out.data_ptr(), rtne=rtne,
                           stream=_stream(x))
    return out


def bposit8_to_int8(x: torch.Tensor) -> torch.Tensor:
    """bposit8 codes (uint8 or int8 tensor) -> int8 fixed point with 6
    fraction bits, clamp(floor(value * 64)) -- the decode pass of the
    bposit8 IMMA path; the result feeds ``gemm_i8``."""
    _need_cuda(x)
    if x.dtype not in (torch.uint8, torch.int8):
        raise ValueError("bposit8 codes must be uint8 or int8")
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    _api.bposit8_to_int8_dev(x.data_ptr(), x.numel(), out.data_ptr(), stream=_stream(x))
    return out


def pack_swiglu_weights(w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> dict:
    """Quantise an FFN's ``nn.Linear`` weights per output channel for
    ``ffn_swiglu_w8a8``: gate and up ``[F, D]`` are interleaved in blocks of 32
    channels into one ``[2F, D]`` int8 matrix (and ``[2F]`` scales) so a
    single GEMM produces both; down ``[D, F]`` is quantised as is."""
    _need_cuda(w_gate, w_up, w_down)
    F, D = w_gate.shape
    if w_up.shape != (F, D) or w_down.shape != (D, F):
        raise ValueError("expected w_gate, w_up [F, D] and w_down [D, F]")
    if F % 32:
        raise ValueError("F must be a multiple of 32")
    qg, sg = quantize_per_channel(w_gate)
    qu, su = quantize_per_channel(w_up)
    qd, sd = quantize_per_channel(w_down)
    w_gu = torch.stack((qg.view(F // 32, 32, D), qu.view(F // 32, 32, D)), 1).reshape(2 * F, D)
    s_gu = torch.stack((sg.view(F // 32, 32), su.view(F // 32, 32)), 1).reshape(2 * F)
    return {"w_gu_i8": w_gu.contiguous(), "w_gu_scale": s_gu.contiguous(), "w_down_i8": qd,
            "w_down_scale": sd, "F": F, "D": D}


def ffn_swiglu_w8a8(x: torch.Tensor, packed: dict, *, out_dtype: torch.dtype | None = None,
                    act: torch.Tensor | None = None) -> torch.Tensor:
    """W8A8 SwiGLU FFN ``down(silu(gate(x)) * up(x))`` on row-major ``x [M, D]``
    with weights from ``pack_swiglu_weights``; ``act`` (fp32 ``[M, F]``) may
    receive the activation.  Returns ``y [M, D]`` in ``out_dtype`` (default
    ``x.dtype``)."""
    _need_cuda(x)
    x = x.contiguous()
    M, D = x.shape
    if D != packed["D"]:
        raise ValueError(f"x has {D} features, the FFN expects {packed['D']}")
    F = packed["F"]
    out_dtype = out_dtype or x.dtype
    y = torch.empty((M, D), dtype=out_dtype, device=x.device)
    if act is not None and (act.dtype != torch.float32 or act.shape != (M, F) or
                            not act.is_contiguous()):
        raise ValueError("act must be a contiguous fp32 [M, F] tensor")
    _api.ffn_swiglu_w8a8_dev(x.data_ptr(), _DT[x.dtype], M, D, packed["w_gu_i8"].data_ptr(),
                             packed["w_gu_scale"].data_ptr(), F, packed["w_down_i8"].data_ptr(),
                             packed["w_down_scale"].data_ptr(), y.data_ptr(), _DT[out_dtype],
                             act=act.data_ptr() if act is not None else 0, stream=_stream(x))
    return y


def gemm_bposit8(A: torch.Tensor, B: torch.Tensor, *, bp32: bool = True, i32: bool = False,
                 rtne32: bool = False, row_major: bool = False) -> dict:
    """bposit8 in, bposit32 out (the reference's IMMA path for bposit8
    tensors, kernels/test_mera_isometry_imma.cu:224-352): ``A [M,K]`` and
    ``B [N,K]`` bposit8 codes are decoded to int8 with 6 fraction bits, the
    exact INT32 GEMM runs on the tensor cores and the epilogue encodes
    ``acc / 2^12`` to bposit32 (``i32`` returns the raw accumulator).  Both
    operands are decoded in one launch into library scratch."""
    _need_cuda(A, B)
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[1]:
        raise ValueError(f"shape mismatch: A {tuple(A.shape)} vs B {tuple(B.shape)}")
    A = A.contiguous()
    B = B.contiguous()
    M, K = A.shape
    N = B.shape[0]
    res = {}
    if bp32:
        res["bp32"] = _out((M, N), torch.int32, A.device, row_major)
    if i32:
        res["i32"] = _out((M, N), torch.int32, A.device, row_major)
    flags = (_api.RTNE_BP32 if rtne32 else 0) | (_api.OUT_ROW_MAJOR if row_major else 0)
    _api.gemm_bposit8_dev(A.data_ptr(), B.data_ptr(), M, N, K, out_bp32=_ptr(res.get("bp32")),
                          out_i32=_ptr(res.get("i32")), flags=flags, stream=_stream(A))
    return res


def float_to_bposit(x: torch.Tensor, nbits: int = 16, *, rtne: bool = False) -> torch.Tensor:
    _need_cuda(x)
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.int16 if nbits == 16 else torch.int32, device=x.device)
    _api.float_to_bposit_dev(x.data_ptr(), _DT[x.dtype], x.numel(), out.data_ptr(), nbits,
                             rtne=rtne, stream=_stream(x))
    return out


def epilogue_i32(acc: torch.Tensor, *, bp32: bool = True, bp16: bool = False,
                 y_dtype: torch.dtype | None = None, x_scale: torch.Tensor | None = None,
                 w_scale: torch.Tensor | None = None, rtne32: bool = False,
                 rtne16: bool = False) -> dict:
    """Epilogue over a logical ``[M,N]`` INT32 accumulator stored column-major
    (i.e. ``acc`` is the transpose view of an ``[N, M]`` tensor)."""
    _need_cuda(acc, x_scale, w_scale)
    M, N = acc.shape
    store = acc.t()
    if not store.is_contiguous():
        store = store.contiguous()
    res = {}
    if bp32:
        res["bp32"] = _out((M, N), torch.int32, acc.device, False)
    if bp16:
        res["bp16"] = _out((M, N), torch.int16, acc.device, False)
    flags = (_api.RTNE_BP32 if rtne32 else 0) | (_api.RTNE_BP16 if rtne16 else 0)
    if y_dtype is not None:
        res["y"] = _out((M, N), y_dtype, acc.device, False)
        if x_scale.numel() == 1:
            flags |= _api.XS_SCALAR
        if w_scale.numel() == 1:
            flags |= _api.WS_SCALAR
    _api.epilogue_i32_dev(store.data_ptr(), M, N, x_scale=_ptr(x_scale), w_scale=_ptr(w_scale),
                          out_bp32=_ptr(res.get("bp32")), out_bp16=_ptr(res.get("bp16")),
                          out_y=_ptr(res.get("y")), y_dtype=_DT[y_dtype] if y_dtype else 0,
                          flags=flags, stream=_stream(acc))
    return res


def epilogue_i64(acc: torch.Tensor, *, bp32: bool = True, bp16: bool = False,
                 y_dtype: torch.dtype | None = None, x_scale: torch.Tensor | None = None,
                 w_scale: torch.Tensor | None = None, rtne32: bool = False,
                 rtne16: bool = False, scale_shift: int = 0) -> dict:
    """``epilogue_i32`` over an INT64 accumulator (a logical ``[M,N]`` stored
    column-major): the exact sum of partials that may not fit INT32."""
    _need_cuda(acc, x_scale, w_scale)
    if acc.dtype != torch.int64:
        raise ValueError("acc must be int64")
    M, N = acc.shape
    store = acc.t()
    if not store.is_contiguous():
        store = store.contiguous()
    res = {}
    if bp32:
        res["bp32"] = _out((M, N), torch.int32, acc.device, False)
    if bp16:
        res["bp16"] = _out((M, N), torch.int16, acc.device, False)
    if not 0 <= scale_shift <= 31:
        raise ValueError("scale_shift must be in 0..31")
    flags = (_api.RTNE_BP32 if rtne32 else 0) | (_api.RTNE_BP16 if rtne16 else 0) | \
        (scale_shift << 24)
    if y_dtype is not None:
        if x_scale is None or w_scale is None:
            raise ValueError("dequantised output needs x_scale and w_scale")
        res["y"] = _out((M, N), y_dtype, acc.device, False)
        if x_scale.numel() == 1:
            flags |= _api.XS_SCALAR
        if w_scale.numel() == 1:
            flags |= _api.WS_SCALAR
    _api.epilogue_i64_dev(store.data_ptr(), M, N, x_scale=_ptr(x_scale), w_scale=_ptr(w_scale),
                          out_bp32=_ptr(res.get("bp32")), out_bp16=_ptr(res.get("bp16")),
                          out_y=_ptr(res.get("y")), y_dtype=_DT[y_dtype] if y_dtype else 0,
                          flags=flags, stream=_stream(acc))
    return res


def widen_i32(src: torch.Tensor, dst: torch.Tensor | None = None, *,
              accumulate: bool = False) -> torch.Tensor:
    """``dst = src`` (or ``dst += src`` with ``accumulate``) as INT64, element
    by element over same-shaped contiguous tensors; returns ``dst``."""
    _need_cuda(src, dst)
    if src.dtype != torch.int32 or not src.is_contiguous():
        raise ValueError("src must be a contiguous int32 tensor")
    if dst is None:
        if accumulate:
            raise ValueError("accumulate needs dst")
        dst = torch.empty(src.shape, dtype=torch.int64, device=src.device)
    if dst.dtype != torch.int64 or not dst.is_contiguous() or dst.numel() != src.numel():
        raise ValueError("dst must be a contiguous int64 tensor of src's size")
    _api.widen_i32_dev(src.data_ptr(), src.numel(), dst.data_ptr(), accumulate=accumulate,
                       stream=_stream(src))
    return dst


def bposit16_op(op: str, a: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """Element-wise bposit16 ALU: add, mul, mul_exact (binary); neg,
    neg_ones_complement, recip, sqrt, log2, exp2 (unary)."""
    _need_cuda(a, b)
    a = a.contiguous()
    out = torch.empty_like(a, dtype=torch.int16)
    if b is None:
        _api.bposit16_unary_dev(op, a.data_ptr(), a.numel(), out.data_ptr(), stream=_stream(a))
    else:
        b = b.contiguous()
        if b.numel() != a.numel():
            raise ValueError("operands differ in size")
        _api.bposit16_binary_dev(op, a.data_ptr(), b.data_ptr(), a.numel(), out.data_ptr(),
                                 stream=_stream(a))
    return out
