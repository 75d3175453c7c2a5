"""Oracle: RMSNorm / LayerNorm forward and backward on CPU.  Test infrastructure only.

Follows the reference's PyTorch reference functions rmsnorm_ref (quack/rmsnorm.py:563-575),
rmsnorm_bwd_ref (:578-594), layernorm_ref (:1727-1730), layernorm_rstd_ref (:1733-1737),
layernorm_mean_ref (:1740-1741).  What those do not return is restated from the kernel math:
rstd (quack/rmsnorm.py:311,324), the residual gradient (:1132-1140), LayerNorm backward
(:1128-1131) and db (:1143-1144).
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor


def _up(t: Optional[Tensor], dt) -> Optional[Tensor]:
    return None if t is None else t.detach().to(dt)


def rmsnorm_ref(x, w=None, bias=None, residual=None, eps=1e-6, weight_offset=0.0,
                out_dtype=None, residual_dtype=None, compute_dtype=torch.float32):
    """Returns out, or (out, residual_out) when a residual is given or residual_dtype is set.
    All math in ``compute_dtype`` on the (already rounded) inputs; outputs are rounded once."""
    h = _up(x, compute_dtype)
    if residual is not None:
        h = h + _up(residual, compute_dtype)
    ms = (h * h).mean(dim=-1, keepdim=True)
    y = h / torch.sqrt(ms + eps)
    if w is not None:
        y = y * (_up(w, compute_dtype) + weight_offset)
    if bias is not None:
        y = y + _up(bias, compute_dtype)
    out = y.to(out_dtype or x.dtype)
    if residual is None and residual_dtype is None:
        return out
    res_dt = residual_dtype or (residual.dtype if residual is not None else x.dtype)
    return out, h.to(res_dt)


def rmsnorm_rstd_ref(x, residual=None, eps=1e-6, compute_dtype=torch.float32):
    h = _up(x, compute_dtype)
    if residual is not None:
        h = h + _up(residual, compute_dtype)
    return (1.0 / torch.sqrt((h * h).mean(dim=-1) + eps)).to(torch.float32)


def rmsnorm_bwd_ref(x, w, dout, rstd, weight_offset=0.0, dresidual_out=None, has_bias=False,
                    compute_dtype=torch.float32):
    """x is the pre-norm input (x + residual when there was a residual).
    Returns (dx, dw, db) as ``compute_dtype`` tensors (dw / db None when absent); the caller
    rounds.  dx already includes ``dresidual_out``."""
    xf = _up(x, compute_dtype)
    dy = _up(dout, compute_dtype)
    r = _up(rstd, compute_dtype).unsqueeze(-1)
    xhat = xf * r
    wdy = dy * (_up(w, compute_dtype) + weight_offset) if w is not None else dy
    c1 = (xhat * wdy).mean(dim=-1, keepdim=True)
    dx = (wdy - xhat * c1) * r
    if dresidual_out is not None:
        dx = dx + _up(dresidual_out, compute_dtype)
    lead = tuple(range(dy.dim() - 1)) if w is None or w.dim() == 1 else (0,)
    dw = (dy * xhat).sum(dim=lead) if w is not None else None
    db = dy.sum(dim=lead) if has_bias else None
    return dx, dw, db


def _ln_stats(x):
    """Row mean and biased variance in float64: inputs with a large common offset (the reference's
    ragged-N known-answer case has x ~ 1000 +- 1) lose digits in an fp32 running sum, and the
    oracle should be the exact answer, not one particular summation order."""
    xd = x.detach().to(torch.float64)
    mu = xd.mean(dim=-1, keepdim=True)
    var = ((xd - mu) ** 2).mean(dim=-1, keepdim=True)
    return mu, var


def layernorm_mean_ref(x, compute_dtype=torch.float32):
    return _ln_stats(x)[0].squeeze(-1).to(torch.float32)


def layernorm_rstd_ref(x, eps=1e-6, compute_dtype=torch.float32):
    _, var = _ln_stats(x)
    return (1.0 / torch.sqrt(var.squeeze(-1) + eps)).to(torch.float32)


def layernorm_ref(x, w, bias=None, eps=1e-6, compute_dtype=torch.float32):
    mu, var = _ln_stats(x)
    xhat = ((x.detach().to(torch.float64) - mu) / torch.sqrt(var + eps)).to(compute_dtype)
    y = xhat * _up(w, compute_dtype)
    if bias is not None:
        y = y + _up(bias, compute_dtype)
    return y.to(x.dtype)


def layernorm_bwd_ref(x, w, dout, rstd, mean, has_bias=True, compute_dtype=torch.float32):
    """Returns (dx, dw, db) in ``compute_dtype``."""
    dy = _up(dout, compute_dtype)
    r = _up(rstd, compute_dtype).unsqueeze(-1)
    # centre in float64 (see _ln_stats), then continue in compute_dtype
    xc = x.detach().to(torch.float64) - mean.detach().to(torch.float64).unsqueeze(-1)
    xhat = xc.to(compute_dtype) * r
    wdy = dy * _up(w, compute_dtype)
    c1 = (xhat * wdy).mean(dim=-1, keepdim=True)
    c2 = wdy.mean(dim=-1, keepdim=True)
    dx = (wdy - c2 - xhat * c1) * r
    dw = (dy * xhat).sum(dim=0)
    db = dy.sum(dim=0) if has_bias else None
    return dx, dw, db
