"""ctypes binding of libmosyne_bposit.so (B200 / sm_100a build).

Mirrors the reference's Python API (packages/mosyne_bposit/src/mosyne_bposit/
_api.py:21-248): the same function names, argument order, validation
messages (raised before the library loads) and ``RuntimeError`` on a
non-zero return code.  The functions after ``shutdown`` expose this build's
additional C entry points (fused GEMM, quantisers, quire sums, bposit
encoders, bposit16 ALU).

There is no CPU fallback: every call runs the CUDA library, and a missing
library raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_SO_NAME = "libmosyne_bposit.so"
_lib = None

# dtype codes and flags (include/mosyne_bposit.h)
DT_F32, DT_BF16, DT_F16, DT_F64 = 0, 1, 2, 3
RTNE_BP32 = 0x1
RTNE_BP16 = 0x2
XS_SCALAR = 0x4
WS_SCALAR = 0x8
OUT_ROW_MAJOR = 0x10
X_ROW_MAJOR = 0x20
X_PER_TENSOR = 0x40

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t


def library_path() -> Path:
    """Return the absolute path the .so should live at (next to this module)."""
    return _HERE / _SO_NAME


def _resolve_library() -> Path:
    env = os.environ.get("MOSYNE_BPOSIT_SO")
    return Path(env) if env else library_path()


_SIGS = {
    # reference ABI (libmosyne_bposit.cu:95-495)
    "mosyne_bposit_init": (_I, []),
    "mosyne_bposit_shutdown": (None, []),
    "mosyne_bposit_linear_w8a8_host": (_I, [ctypes.POINTER(ctypes.c_float), _I, _I,
                                            ctypes.POINTER(ctypes.c_float), _I,
                                            ctypes.POINTER(ctypes.c_float)]),
    "mosyne_bposit_quantize_weight_per_channel": (_I, [_P, _I, _I, _P, _P]),
    "mosyne_bposit_linear_w8a8": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_linear_w8a8_bf16": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_linear_w8a8_bf16_io": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_linear_w8a8_fp16": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_linear_w8a8_fp16_io": (_I, [_P, _I, _I, _P, _P, _I, _P]),
    # additions
    "mosyne_bposit_version": (ctypes.c_char_p, []),
    "mosyne_bposit_last_error": (_I, []),
    "mosyne_bposit_set_sm_count_target": (_I, [_I]),
    "mosyne_bposit_debug_wait_timeout": (_I, [ctypes.c_ulonglong, _P]),
    "mosyne_bposit_gemm_i8": (_I, [_P, _P, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _I, _P]),
    "mosyne_bposit_gemm_i8_host": (_I, [_P, _P, _I, _I, _I, _P, _P, _I]),
    "mosyne_bposit_gemm_i8_batched": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P,
                                           _I, _P]),
    "mosyne_bposit_linear_w8a8_ex": (_I, [_P, _I, _I, _I, _P, _P, _I, _P, _I, _P, _P, _I, _P]),
    "mosyne_bposit_quantize_per_token": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_quantize_per_tensor": (_I, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_quantize_weight_per_channel_ex": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "mosyne_bposit_row_absmax": (_I, [_P, _I, _I, _I, _P, _I, _P]),
    "mosyne_bposit_quantize_with_max": (_I, [_P, _I, _I, _I, _P, _P, _P, _I, _P]),
    "mosyne_bposit_quire_sum_bp16": (_I, [_P, _SZ, _P, _P, _P, _I, _P]),
    "mosyne_bposit_fp32_atomic_sum": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit_shannon_entropy_bp16": (_I, [_P, _SZ, _P, _P, _P, _I, _P]),
    # kernels/shannon_entropy_bposit16.cu:124: the reference's entropy symbol
    "shannon_entropy_bposit16_cuda": (_I, [_P, _SZ, _P]),
    "mosyne_bposit_quire_to_bp16": (_I, [_P, _SZ, _P, _I, _P]),
    "mosyne_bposit_quire_to_bp32": (_I, [_P, _SZ, _P, _I, _P]),
    "mosyne_bposit_bp16_to_quire": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit_int32_to_bp32": (_I, [_P, _SZ, _I, _P, _I, _P]),
    "mosyne_bposit_bposit8_to_int8": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit_gemm_bposit8": (_I, [_P, _P, _I, _I, _I, _P, _P, _I, _P]),
    "mosyne_bposit_ffn_swiglu_w8a8": (_I, [_P, _I, _I, _I, _P, _P, _I, _P, _P, _P, _I, _P, _I, _P]),
    "mosyne_bposit_float_to_bposit": (_I, [_P, _I, _SZ, _P, _I, _I, _P]),
    "mosyne_bposit_epilogue_i32": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P]),
    "mosyne_bposit_epilogue_i64": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _I, _I, _P]),
    "mosyne_bposit_widen_i32": (_I, [_P, _SZ, _P, _I, _P]),
    "mosyne_bposit16_add": (_I, [_P, _P, _SZ, _P, _P]),
    "mosyne_bposit16_mul": (_I, [_P, _P, _SZ, _P, _P]),
    "mosyne_bposit16_mul_exact": (_I, [_P, _P, _SZ, _P, _P]),
    "mosyne_bposit16_neg": (_I, [_P, _SZ, _P, _I, _P]),
    "mosyne_bposit16_recip": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit16_sqrt": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit16_log2": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit16_exp2": (_I, [_P, _SZ, _P, _P]),
    "mosyne_bposit16_table_host": (_I, [_I, _P]),
    "mosyne_bposit_debug_alu_check": (_I, [_I, _P]),
    "mosyne_bposit_linear_w8a8_noalloc": (_I, [_P, _I, _I, _P, _P, _I, _P, _P]),
    "mosyne_bposit_debug_noalloc_wait_timeout": (_I, [ctypes.c_ulonglong, _P]),
}


def load_library(init: bool = False) -> ctypes.CDLL:
    """Load the shared library and declare every exported signature.  With
    ``init`` it also runs ``mosyne_bposit_init`` (which needs a GPU)."""
    global _lib
    if _lib is None:
        p = _resolve_library()
        if not p.exists():
            raise RuntimeError(
                f"libmosyne_bposit.so not found at {p}. "
                f"Run `mosyne-bposit-build` (python mosyne-bposit_b200/build.py; requires nvcc) "
                f"or set MOSYNE_BPOSIT_SO to a prebuilt .so path."
            )
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    if init:
        rc = _lib.mosyne_bposit_init()
        if rc != 0:
            raise RuntimeError(f"mosyne_bposit_init failed (rc={rc})")
    return _lib


def _ensure_library() -> ctypes.CDLL:
    return load_library(init=True)


def _check(rc: int, name: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{name} failed (rc={rc})")


def linear_w8a8(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Compute ``y = x @ w`` via the W8A8 bposit pipeline (reference
    _api.py:91-119).  Row-major numpy ``x (M, K)`` and ``w (K, N)`` in, a
    row-major float32 ``(M, N)`` out; per-channel weight scales and
    per-token activation scales, exact INT32 accumulation."""
    if x.ndim != 2 or w.ndim != 2:
        raise ValueError(f"x and w must be 2-D (got x.shape={x.shape}, w.shape={w.shape})")
    if x.shape[1] != w.shape[0]:
        raise ValueError(
            f"shape mismatch: x.shape[1]={x.shape[1]} != w.shape[0]={w.shape[0]}"
        )
    lib = _ensure_library()
    M, K = x.shape
    _, N = w.shape
    x_cm = np.asfortranarray(x.astype(np.float32, copy=False))
    w_cm = np.asfortranarray(w.astype(np.float32, copy=False))
    y_cm = np.zeros((M, N), dtype=np.float32, order="F")
    fp = ctypes.POINTER(ctypes.c_float)
    rc = lib.mosyne_bposit_linear_w8a8_host(
        x_cm.ctypes.data_as(fp), M, K, w_cm.ctypes.data_as(fp), N, y_cm.ctypes.data_as(fp))
    if rc != 0:
        raise RuntimeError(f"mosyne_bposit_linear_w8a8_host failed (rc={rc})")
    return np.ascontiguousarray(y_cm)


def quantize_weight_per_channel_dev(w_fp32_dev_ptr: int, K: int, N: int,
                                    w_i8_dev_ptr: int, w_scale_dev_ptr: int) -> None:
    """Column-major fp32 ``[K, N]`` device weight -> int8 ``[K, N]`` plus
    ``w_scale[N]`` (reference _api.py:122-141)."""
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quantize_weight_per_channel(w_fp32_dev_ptr, K, N, w_i8_dev_ptr,
                                                         w_scale_dev_ptr),
           "mosyne_bposit_quantize_weight_per_channel")


def _linear_dev(name, x, M, K, w, ws, N, y):
    lib = _ensure_library()
    _check(getattr(lib, name)(x, M, K, w, ws, N, y), name)


def linear_w8a8_dev(x_fp32_dev_ptr: int, M: int, K: int, w_i8_dev_ptr: int,
                    w_scale_dev_ptr: int, N: int, y_fp32_dev_ptr: int) -> None:
    """Device-pointer W8A8 linear, fp32 column-major x and y (reference
    _api.py:144-165)."""
    _linear_dev("mosyne_bposit_linear_w8a8", x_fp32_dev_ptr, M, K, w_i8_dev_ptr,
                w_scale_dev_ptr, N, y_fp32_dev_ptr)


def linear_w8a8_dev_bf16(x_bf16_dev_ptr: int, M: int, K: int, w_i8_dev_ptr: int,
                         w_scale_dev_ptr: int, N: int, y_fp32_dev_ptr: int) -> None:
    """bf16 x, fp32 y (reference _api.py:168-184)."""
    _linear_dev("mosyne_bposit_linear_w8a8_bf16", x_bf16_dev_ptr, M, K, w_i8_dev_ptr,
                w_scale_dev_ptr, N, y_fp32_dev_ptr)


def linear_w8a8_dev_bf16_io(x_bf16_dev_ptr: int, M: int, K: int, w_i8_dev_ptr: int,
                            w_scale_dev_ptr: int, N: int, y_bf16_dev_ptr: int) -> None:
    """bf16 x and y (reference _api.py:187-204)."""
    _linear_dev("mosyne_bposit_linear_w8a8_bf16_io", x_bf16_dev_ptr, M, K, w_i8_dev_ptr,
                w_scale_dev_ptr, N, y_bf16_dev_ptr)


def linear_w8a8_dev_fp16(x_fp16_dev_ptr: int, M: int, K: int, w_i8_dev_ptr: int,
                         w_scale_dev_ptr: int, N: int, y_fp32_dev_ptr: int) -> None:
    """fp16 x, fp32 y (reference _api.py:207-222)."""
    _linear_dev("mosyne_bposit_linear_w8a8_fp16", x_fp16_dev_ptr, M, K, w_i8_dev_ptr,
                w_scale_dev_ptr, N, y_fp32_dev_ptr)


def linear_w8a8_dev_fp16_io(x_fp16_dev_ptr: int, M: int, K: int, w_i8_dev_ptr: int,
                            w_scale_dev_ptr: int, N: int, y_fp16_dev_ptr: int) -> None:
    """fp16 x and y (reference _api.py:225-241)."""
    _linear_dev("mosyne_bposit_linear_w8a8_fp16_io", x_fp16_dev_ptr, M, K, w_i8_dev_ptr,
                w_scale_dev_ptr, N, y_fp16_dev_ptr)


def shutdown() -> None:
    """Free GPU resources held by the library.  Safe to call multiple times."""
    global _lib
    if _lib is not None:
        _lib.mosyne_bposit_shutdown()


# ---------------------------------------------------------------------------
# Additional device-pointer entry points (integer addresses, stream handles)
# ---------------------------------------------------------------------------


def version() -> str:
    return load_library().mosyne_bposit_version().decode()


def set_sm_count_target(sms: int) -> None:
    """GEMMs of the current device use at most ``sms`` SMs (0: all)."""
    _check(_ensure_library().mosyne_bposit_set_sm_count_target(int(sms)),
           "mosyne_bposit_set_sm_count_target")


def sm_count() -> int:
    import torch
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def last_error() -> int:
    """Synchronise and return the device error word as a return code
    (0 ok, -30 a device-side wait gave up)."""
    return _ensure_library().mosyne_bposit_last_error()


def debug_wait_timeout(limit_ns: int = 1_000_000, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_debug_wait_timeout(limit_ns, stream), "mosyne_bposit_debug_wait_timeout")


def gemm_i8_dev(A: int, B: int, M: int, N: int, K: int, *, x_scale: int = 0, w_scale: int = 0,
                out_bp32: int = 0, out_bp16: int = 0, out_y: int = 0, y_dtype: int = DT_F32,
                out_i32: int = 0, flags: int = 0, stream: int = 0) -> None:
    """Fused INT8 GEMM (A [M,K], B [N,K], both K-contiguous) with any of the
    bposit32 / bposit16 / dequant / INT32 outputs."""
    lib = _ensure_library()
    _check(lib.mosyne_bposit_gemm_i8(A, B, M, N, K, x_scale, w_scale, out_bp32, out_bp16, out_y,
                                     y_dtype, out_i32, flags, stream), "mosyne_bposit_gemm_i8")


def gemm_i8_batched_dev(A: int, B: int, batch: int, M: int, N: int, K: int, *, x_scale: int = 0,
                        w_scale: int = 0, out_bp32: int = 0, out_bp16: int = 0, out_y: int = 0,
                        y_dtype: int = DT_F32, out_i32: int = 0, flags: int = 0,
                        stream: int = 0) -> None:
    """``batch`` independent fused GEMMs of one shape, operands and outputs
    contiguous per batch entry."""
    lib = _ensure_library()
    _check(lib.mosyne_bposit_gemm_i8_batched(A, B, batch, M, N, K, x_scale, w_scale, out_bp32,
                                             out_bp16, out_y, y_dtype, out_i32, flags, stream),
           "mosyne_bposit_gemm_i8_batched")


def gemm_i8_host(A: np.ndarray, B: np.ndarray, *, want_i32: bool = False, flags: int = 0):
    """Host-buffer GEMM: int8 ``A (M, K)`` and ``B (N, K)`` (K contiguous)
    -> column-major bposit32 codes ``(M, N)`` (and INT32 if asked), as
    row-major numpy arrays."""
    A = np.ascontiguousarray(A, dtype=np.int8)
    B = np.ascontiguousarray(B, dtype=np.int8)
    M, K = A.shape
    N = B.shape[0]
    if B.shape[1] != K:
        raise ValueError(f"shape mismatch: A.shape[1]={K} != B.shape[1]={B.shape[1]}")
    lib = _ensure_library()
    bp = np.empty((N, M), dtype=np.uint32)
    i32 = np.empty((N, M), dtype=np.int32) if want_i32 else None
    _check(lib.mosyne_bposit_gemm_i8_host(A.ctypes.data, B.ctypes.data, M, N, K, bp.ctypes.data,
                                          i32.ctypes.data if want_i32 else 0, flags),
           "mosyne_bposit_gemm_i8_host")
    return (bp.T, i32.T) if want_i32 else bp.T


def linear_w8a8_ex_dev(x: int, x_dtype: int, M: int, K: int, w_i8: int, w_scale: int, N: int, *,
                       y: int = 0, y_dtype: int = DT_F32, y_bp32: int = 0, y_bp16: int = 0,
                       flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_linear_w8a8_ex(x, x_dtype, M, K, w_i8, w_scale, N, y, y_dtype,
                                            y_bp32, y_bp16, flags, stream),
           "mosyne_bposit_linear_w8a8_ex")


def quantize_per_token_dev(x: int, x_dtype: int, M: int, K: int, x_i8: int, x_scale: int, *,
                           flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quantize_per_token(x, x_dtype, M, K, x_i8, x_scale, flags, stream),
           "mosyne_bposit_quantize_per_token")


def quantize_per_tensor_dev(t: int, dtype: int, rows: int, cols: int, q: int, scale: int, *,
                            flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quantize_per_tensor(t, dtype, rows, cols, q, scale, flags, stream),
           "mosyne_bposit_quantize_per_tensor")


def quantize_weight_per_channel_ex_dev(w: int, dtype: int, K: int, N: int, w_i8: int,
                                       w_scale: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quantize_weight_per_channel_ex(w, dtype, K, N, w_i8, w_scale, stream),
           "mosyne_bposit_quantize_weight_per_channel_ex")


def row_absmax_dev(x: int, x_dtype: int, M: int, K: int, row_max: int, *, flags: int = 0,
                   stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_row_absmax(x, x_dtype, M, K, row_max, flags, stream),
           "mosyne_bposit_row_absmax")


def quantize_with_max_dev(x: int, x_dtype: int, M: int, K: int, row_max: int, x_i8: int,
                          x_scale: int, *, flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quantize_with_max(x, x_dtype, M, K, row_max, x_i8, x_scale, flags,
                                               stream), "mosyne_bposit_quantize_with_max")


def quire_sum_bp16_dev(x: int, n: int, *, q_out: int = 0, bp16_out: int = 0, bp32_out: int = 0,
                       flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_quire_sum_bp16(x, n, q_out, bp16_out, bp32_out, flags, stream),
           "mosyne_bposit_quire_sum_bp16")


def shannon_entropy_bp16_dev(p: int, n: int, *, q_out: int = 0, bp32_out: int = 0,
                             bp16_out: int = 0, flags: int = 0, stream: int = 0) -> None:
    """H = -sum p log2(p) of n bposit16 codes at device address ``p``
    (kernels/shannon_entropy_bposit16.cu:63-119), asynchronous on ``stream``."""
    lib = _ensure_library()
    _check(lib.mosyne_bposit_shannon_entropy_bp16(p, n, q_out, bp32_out, bp16_out, flags, stream),
           "mosyne_bposit_shannon_entropy_bp16")


def fp32_atomic_sum_dev(x: int, n: int, acc: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_fp32_atomic_sum(x, n, acc, stream), "mosyne_bposit_fp32_atomic_sum")


def quire_to_bposit_dev(q: int, n: int, out: int, nbits: int = 16, *, rtne: bool = False,
                        stream: int = 0) -> None:
    lib = _ensure_library()
    fn = lib.mosyne_bposit_quire_to_bp16 if nbits == 16 else lib.mosyne_bposit_quire_to_bp32
    _check(fn(q, n, out, int(rtne), stream), f"mosyne_bposit_quire_to_bp{nbits}")


def bp16_to_quire_dev(x: int, n: int, out: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_bp16_to_quire(x, n, out, stream), "mosyne_bposit_bp16_to_quire")


def int32_to_bp32_dev(x: int, n: int, scale_shift: int, out: int, *, rtne: bool = False,
                      stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_int32_to_bp32(x, n, scale_shift, out, int(rtne), stream),
           "mosyne_bposit_int32_to_bp32")


def ffn_swiglu_w8a8_dev(x: int, x_dtype: int, M: int, D: int, w_gu_i8: int, w_gu_scale: int,
                        F: int, w_down_i8: int, w_down_scale: int, y: int, y_dtype: int, *,
                        act: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_ffn_swiglu_w8a8(x, x_dtype, M, D, w_gu_i8, w_gu_scale, F, w_down_i8,
                                             w_down_scale, y, y_dtype, act, 0, stream),
           "mosyne_bposit_ffn_swiglu_w8a8")


def gemm_bposit8_dev(A: int, B: int, M: int, N: int, K: int, *, out_bp32: int = 0,
                     out_i32: int = 0, flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_gemm_bposit8(A, B, M, N, K, out_bp32, out_i32, flags, stream),
           "mosyne_bposit_gemm_bposit8")


def bposit8_to_int8_dev(x: int, n: int, out: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_bposit8_to_int8(x, n, out, stream), "mosyne_bposit_bposit8_to_int8")


def float_to_bposit_dev(x: int, dtype: int, n: int, out: int, nbits: int = 16, *,
                        rtne: bool = False, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_float_to_bposit(x, dtype, n, out, nbits, int(rtne), stream),
           "mosyne_bposit_float_to_bposit")


def epilogue_i32_dev(acc: int, M: int, N: int, *, x_scale: int = 0, w_scale: int = 0,
                     out_bp32: int = 0, out_bp16: int = 0, out_y: int = 0, y_dtype: int = DT_F32,
                     flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_epilogue_i32(acc, M, N, x_scale, w_scale, out_bp32, out_bp16, out_y,
                                          y_dtype, flags, stream), "mosyne_bposit_epilogue_i32")


def epilogue_i64_dev(acc: int, M: int, N: int, *, x_scale: int = 0, w_scale: int = 0,
                     out_bp32: int = 0, out_bp16: int = 0, out_y: int = 0, y_dtype: int = DT_F32,
                     flags: int = 0, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_epilogue_i64(acc, M, N, x_scale, w_scale, out_bp32, out_bp16, out_y,
                                          y_dtype, flags, stream), "mosyne_bposit_epilogue_i64")


def widen_i32_dev(src: int, n: int, dst: int, *, accumulate: bool = False, stream: int = 0) -> None:
    lib = _ensure_library()
    _check(lib.mosyne_bposit_widen_i32(src, n, dst, 1 if accumulate else 0, stream),
           "mosyne_bposit_widen_i32")


_ALU1 = {"recip": "mosyne_bposit16_recip", "sqrt": "mosyne_bposit16_sqrt",
         "log2": "mosyne_bposit16_log2", "exp2": "mosyne_bposit16_exp2"}
_ALU2 = {"add": "mosyne_bposit16_add", "mul": "mosyne_bposit16_mul",
         "mul_exact": "mosyne_bposit16_mul_exact"}


def bposit16_unary_dev(op: str, a: int, n: int, out: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    if op in ("neg", "neg_ones_complement"):
        _check(lib.mosyne_bposit16_neg(a, n, out, int(op != "neg"), stream), "mosyne_bposit16_neg")
        return
    name = _ALU1[op]
    _check(getattr(lib, name)(a, n, out, stream), name)


def bposit16_binary_dev(op: str, a: int, b: int, n: int, out: int, *, stream: int = 0) -> None:
    lib = _ensure_library()
    name = _ALU2[op]
    _check(getattr(lib, name)(a, b, n, out, stream), name)


def debug_alu_check(op: str) -> tuple:
    """Exhaustive check of the bposit16 ALU's 32-bit forms against their int64
    forms over all 2^32 code pairs ("add", "mul_exact", "quire_sum" or "mul"),
    or the GEMM epilogues' divisions against the IEEE division on 2^32
    pseudo-random operand pairs ("dequant_div", "silu_div"), and that divide's
    reciprocal step on every normal divisor in its range ("div_reciprocal"),
    or the exact sum's per-code decode against the quire image of every
    bposit16 code ("sum_decode"): returns (mismatches, first mismatching
    pair, operand or code, or None)."""
    out = np.zeros(2, dtype=np.uint64)
    idx = ("add", "mul_exact", "quire_sum", "mul", "dequant_div", "silu_div",
           "div_reciprocal", "sum_decode").index(op)
    _check(_ensure_library().mosyne_bposit_debug_alu_check(idx, out.ctypes.data),
           "mosyne_bposit_debug_alu_check")
    first = int(out[1])
    return int(out[0]), (None if first == 2 ** 64 - 1 else first)


def bposit16_table(which: str) -> np.ndarray:
    """Copy one device-resident ALU table (log2/exp2/sqrt/recip) to the host."""
    idx = ("log2", "exp2", "sqrt", "recip").index(which)
    out = np.empty(65536, dtype=np.uint16)
    _check(_ensure_library().mosyne_bposit16_table_host(idx, out.ctypes.data),
           "mosyne_bposit16_table_host")
    return out
