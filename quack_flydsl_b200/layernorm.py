"""LayerNorm behind the reference's Python API.

The reference has no ``quack/layernorm.py``: ``layernorm_fwd`` / ``layernorm_bwd`` live in
quack/rmsnorm.py:1625-1724 and drive the RMSNorm kernels with ``is_layernorm=True``; there is
no autograd wrapper.  This module re-exports those two entry points with the same signatures and
checks (including the fp32-only weight/bias assertion of ``layernorm_fwd``) and adds
``layernorm()``, an autograd-enabled wrapper that also accepts 16-bit weight and bias.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from quack_flydsl_b200.rmsnorm import (
    _SUPPORTED,
    _ensure_contiguous,
    _finalize_partials,
    _rmsnorm_bwd,
    _rmsnorm_fwd,
)
from quack_flydsl_b200.rmsnorm_config import get_sm_count


def layernorm_fwd(
    x: Tensor,
    weight: Tensor,
    bias: Optional[Tensor] = None,
    eps: float = 1e-6,
    return_rstd: bool = False,
    return_mean: bool = False,
):
    """LayerNorm forward.  x: (M, N); weight (and bias): (N,) float32.  Returns ``out`` followed
    by ``rstd`` and / or ``mean`` (fp32, (M,)) when requested."""
    assert x.dim() == 2, "Input must be 2D"
    assert weight.dim() == 1, "Weight must be 1D"
    assert x.dtype in _SUPPORTED, "Unsupported dtype"
    assert weight.dtype == torch.float32, "Weight must be float32"
    if bias is not None:
        assert bias.dim() == 1, "Bias must be 1D"
        assert bias.dtype == torch.float32, "Bias must be float32"
    M = x.shape[0]
    out = torch.empty_like(x)
    rstd = torch.empty(M, device=x.device, dtype=torch.float32) if return_rstd else None
    mean = torch.empty(M, device=x.device, dtype=torch.float32) if return_mean else None
    _rmsnorm_fwd(x, weight, out, bias, rstd, mean, None, None, eps, True)
    if return_rstd and return_mean:
        return out, rstd, mean
    if return_rstd:
        return out, rstd
    if return_mean:
        return out, mean
    return out


def _layernorm_bwd_impl(x, weight, dout, rstd, mean, has_bias, param_dtype):
    N = x.size(-1)
    dx = torch.empty_like(x)
    sm_count = get_sm_count(N, x.device, x.dtype)
    dw_partial = torch.empty(sm_count, N, device=x.device, dtype=torch.float32)
    db_partial = torch.empty(sm_count, N, device=x.device, dtype=torch.float32) if has_bias else None
    if x.numel() > 0:
        _rmsnorm_bwd(x, weight, dout, rstd, dx, dw_partial, db_partial, None, None, sm_count,
                     mean=mean, is_layernorm=True)
        dw = _finalize_partials(dw_partial, param_dtype)
        db = _finalize_partials(db_partial, param_dtype) if has_bias else None
    else:
        dw = torch.zeros(N, device=x.device, dtype=param_dtype)
        db = torch.zeros(N, device=x.device, dtype=param_dtype) if has_bias else None
    return dx, dw, db


def layernorm_bwd(
    x: Tensor,
    weight: Tensor,
    dout: Tensor,
    rstd: Tensor,
    mean: Tensor,
    has_bias: bool = True,
) -> Tuple[Tensor, Tensor, Optional[Tensor]]:
    """LayerNorm backward from the saved rstd and mean.  Returns (dx, dw, db); db is None when
    ``has_bias`` is False.  dw / db are reduced in fp32 (per-CTA partials, then a fixed-order
    column sum) and returned in ``weight.dtype``."""
    assert x.dim() == 2, "Input must be 2D"
    assert weight.dim() == 1, "Weight must be 1D"
    return _layernorm_bwd_impl(x, weight, dout, rstd, mean, has_bias, weight.dtype)


class LayerNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        x = _ensure_contiguous(x)
        M = x.shape[0]
        out = torch.empty_like(x)
        need_grad = any(ctx.needs_input_grad[:3])
        rstd = torch.empty(M, device=x.device, dtype=torch.float32) if need_grad else None
        mean = torch.empty(M, device=x.device, dtype=torch.float32) if need_grad else None
        _rmsnorm_fwd(x, weight, out, bias, rstd, mean, None, None, eps, True)
        ctx.save_for_backward(x, weight, rstd, mean)
        ctx.has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, dout):
        x, weight, rstd, mean = ctx.saved_tensors
        dout = _ensure_contiguous(dout)
        dx, dw, db = _layernorm_bwd_impl(x, weight, dout, rstd, mean, ctx.has_bias, weight.dtype)
        return dx, dw, db, None


def layernorm(x: Tensor, weight: Tensor, bias: Optional[Tensor] = None, eps: float = 1e-5) -> Tensor:
    """LayerNorm over the last dimension with autograd.  x: (..., N); weight / bias: (N,) in
    float32, float16 or bfloat16."""
    assert weight is not None and weight.dim() == 1, "Weight must be 1D"
    shape = x.shape
    out = LayerNormFunction.apply(x.reshape(-1, shape[-1]), weight, bias, eps)
    return out.reshape(shape)
