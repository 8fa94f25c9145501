"""mosyne_bposit.torch_compat -- drop-in PyTorch integration.

Same public API and behaviour as the reference module
(packages/mosyne_bposit/src/mosyne_bposit/torch_compat.py:82-448):

``BPositLinear(weight, bias=None)``
    ``nn.Module`` that quantises an ``nn.Linear`` weight once (per-output-
    channel int8) and runs the W8A8 pipeline in ``forward``.  CUDA-resident
    weights stay on the device; CUDA inputs take the device path.

``replace_linear_modules(model, predicate=None, narrow_n_threshold=None,
skip_kv_proj=False)``
    Swap ``nn.Linear`` children for ``BPositLinear`` with the reference's
    three filters.

``FusedQKVProjection``
    Q/K/V projections concatenated into one wider ``BPositLinear``; here
    ``forward`` is implemented (one GEMM, then the output split).

Device path (torch_compat.py:166-211 in the reference): the reference
transposes x into a column-major copy, calls the C ABI, and transposes y
back (two extra passes).  This build quantises the row-major x directly and
writes the row-major y from the GEMM epilogue (no transposes), on the current
torch stream; the numbers are the same bit for bit.
"""
from __future__ import annotations

from typing import Callable, Optional

try:
    import torch
    import torch.nn as nn
except ImportError as e:  # pragma: no cover - only without torch
    raise ImportError(
        "mosyne_bposit.torch_compat requires PyTorch. "
        "Install with `pip install mosyne-bposit[torch]` or `pip install torch`."
    ) from e

from . import ops
from ._api import linear_w8a8


class BPositLinear(nn.Module):
    """Drop-in W8A8 replacement for ``nn.Linear`` on the B200 bposit pipeline.

    Parameters
    ----------
    weight : Tensor ``(out_features, in_features)``, any dtype castable to fp32.
    bias : optional Tensor ``(out_features,)``.
    """

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> None:
        super().__init__()
        if weight.ndim != 2:
            raise ValueError(f"weight must be 2-D (got shape {tuple(weight.shape)})")
        K = weight.shape[1]
        N = weight.shape[0]
        self.in_features = K
        self.out_features = N
        self._cuda_device: Optional[torch.device] = None
        if weight.is_cuda:
            # [N, K] row-major is the column-major [K, N] layout the kernels read.
            w_fp32 = weight.detach().to(torch.float32).contiguous()
            w_i8, w_scale = ops.quantize_per_channel(w_fp32)
            self.register_buffer("_w_i8_buf", w_i8, persistent=False)
            self.register_buffer("_w_scale_buf", w_scale, persistent=False)
            self.register_buffer(
                "_w_fp32_buf", weight.detach().to(torch.float32).t().contiguous().cpu(),
                persistent=False)
            self._cuda_device = weight.device
        else:
            w_fp32 = weight.detach().to(torch.float32).t().contiguous().cpu()
            self.register_buffer("_w_fp32_buf", w_fp32, persistent=False)
            self._w_i8_buf = None
            self._w_scale_buf = None
        if bias is not None:
            self.register_buffer("_b_fp32_buf", bias.detach().to(torch.float32).contiguous(),
                                 persistent=False)
        else:
            self._b_fp32_buf = None

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "BPositLinear":
        return cls(weight=linear.weight, bias=linear.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        K = orig_shape[-1]
        if K != self.in_features:
            raise ValueError(
                f"input last dim {K} does not match in_features {self.in_features}")
        x_flat = x.reshape(-1, K)
        N = self.out_features
        if (x_flat.is_cuda and self._w_i8_buf is not None and self._w_scale_buf is not None
                and x_flat.device == self._cuda_device):
            if x_flat.dtype in (torch.bfloat16, torch.float16, torch.float32):
                y = ops.linear_w8a8(x_flat, self._w_i8_buf, self._w_scale_buf)["y"]
            else:
                y = ops.linear_w8a8(x_flat.to(torch.float32), self._w_i8_buf,
                                    self._w_scale_buf)["y"].to(x.dtype)
        else:
            # host-pointer entry point (uploads and quantises the weight per call)
            x_np = x_flat.detach().to(torch.float32).cpu().numpy()
            y_np = linear_w8a8(x_np, self._w_fp32_buf.numpy())
            y = torch.from_numpy(y_np).to(x.device).to(x.dtype)
        if self._b_fp32_buf is not None:
            y = y + self._b_fp32_buf.to(y.device).to(y.dtype)
        return y.reshape(*orig_shape[:-1], N)

    def extra_repr(self) -> str:
        path = "device" if self._w_i8_buf is not None else "host-fallback"
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"has_bias={self._b_fp32_buf is not None}, dtype=W8A8(bposit-IMMA), "
                f"path={path}")


_KV_PROJ_LEAVES = ("k_proj", "v_proj")


def _is_kv_proj(full_name: str) -> bool:
    """True iff the leaf of ``full_name`` is ``k_proj`` or ``v_proj``."""
    return full_name.rsplit(".", 1)[-1] in _KV_PROJ_LEAVES


def replace_linear_modules(
    model: nn.Module,
    predicate: Optional[Callable[[str, nn.Linear], bool]] = None,
    narrow_n_threshold: Optional[int] = None,
    skip_kv_proj: bool = False,
) -> nn.Module:
    """Replace every ``nn.Linear`` in *model* with a ``BPositLinear``.

    A module is skipped if ``predicate(name, linear)`` is falsy, if its
    ``out_features`` is below ``narrow_n_threshold``, or (``skip_kv_proj``)
    if its qualified name ends in ``.k_proj`` / ``.v_proj``
    (reference torch_compat.py:243-319).  Returns the modified model."""
    targets = []
    for qual_name, module in model.named_modules():
        for attr, child in module._modules.items():
            if isinstance(child, nn.Linear) and not isinstance(child, BPositLinear):
                full = f"{qual_name}.{attr}" if qual_name else attr
                if predicate is not None and not predicate(full, child):
                    continue
                if narrow_n_threshold is not None and child.out_features < narrow_n_threshold:
                    continue
                if skip_kv_proj and _is_kv_proj(full):
                    continue
                targets.append((module, attr, child))
    for parent, attr, lin in targets:
        setattr(parent, attr, BPositLinear.from_linear(lin))
    return model


class FusedQKVProjection(nn.Module):
    """Q, K and V projections as one wider ``BPositLinear`` (reference
    torch_compat.py:322-437, where ``forward`` is not implemented).  One
    GEMM over ``[q_out + k_out + v_out, in_features]``; ``forward`` returns
    ``(q, k, v)`` views of its output."""

    def __init__(self, q_out: int, k_out: int, v_out: int, in_features: int) -> None:
        super().__init__()
        if q_out <= 0 or k_out <= 0 or v_out <= 0:
            raise ValueError("q_out / k_out / v_out must be positive")
        if in_features <= 0:
            raise ValueError("in_features must be positive")
        self.q_out = q_out
        self.k_out = k_out
        self.v_out = v_out
        self.in_features = in_features
        self.out_features = q_out + k_out + v_out
        self._fused: Optional[BPositLinear] = None

    @classmethod
    def from_separate(cls, q_proj: nn.Linear, k_proj: nn.Linear,
                      v_proj: nn.Linear) -> "FusedQKVProjection":
        in_f = q_proj.in_features
        if k_proj.in_features != in_f or v_proj.in_features != in_f:
            raise ValueError(
                f"q/k/v in_features mismatch: q={q_proj.in_features}, "
                f"k={k_proj.in_features}, v={v_proj.in_features}")
        has_bias = q_proj.bias is not None
        if (k_proj.bias is not None) != has_bias or (v_proj.bias is not None) != has_bias:
            raise ValueError(
                "all three of q/k/v_proj must agree on bias presence "
                "(common case is no bias; FusedQKVProjection won't "
                "interleave bias-yes and bias-no projections)")
        fused = cls(q_out=q_proj.out_features, k_out=k_proj.out_features,
                    v_out=v_proj.out_features, in_features=in_f)
        cat_w = torch.cat([q_proj.weight, k_proj.weight, v_proj.weight], dim=0)
        cat_b = torch.cat([q_proj.bias, k_proj.bias, v_proj.bias], dim=0) if has_bias else None
        fused._fused = BPositLinear(weight=cat_w, bias=cat_b)
        return fused

    def forward(self, x: torch.Tensor):
        if self._fused is None:
            raise RuntimeError("FusedQKVProjection has no weights; build it with from_separate()")
        y = self._fused(x)
        return tuple(y.split([self.q_out, self.k_out, self.v_out], dim=-1))

    def extra_repr(self) -> str:
        return (f"q_out={self.q_out}, k_out={self.k_out}, v_out={self.v_out}, "
                f"in_features={self.in_features}, out_features={self.out_features}, "
                f"materialised={self._fused is not None}")


__all__ = ["BPositLinear", "FusedQKVProjection", "replace_linear_modules"]
