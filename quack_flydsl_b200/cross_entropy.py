"""Cross-entropy loss behind the reference's Python API.

Host-side mirror of quack/cross_entropy.py: ops ``quack::cross_entropy_fwd_out`` (:312-364) and
``quack::cross_entropy_bwd_out`` (:618-628), ``cross_entropy_fwd`` (:367-390),
``cross_entropy_bwd`` (:631-662), ``CrossEntropyFunction`` (:665-712) and ``cross_entropy``
(:715-765), including the ``lse_partial`` mode, class weights, ``ignore_index`` and the in-place
backward.
"""

from __future__ import annotations

from ctypes import byref
from typing import Literal, Optional

import torch
from torch import Tensor

from quack_flydsl_b200 import _C
from quack_flydsl_b200.dsl import kernel_op

_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32)


def _rows(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 or t.size(-1) == 1 else t.contiguous()


def _num_classes(x, target_logit, weight) -> int:
    """Upper bound of valid class ids: what the kernel may index weight / target_logit with."""
    if weight is not None:
        return weight.numel()
    if target_logit is not None:
        return target_logit.size(1) if target_logit.dim() == 2 else 0
    return x.size(1)


def _fill_ce_fwd(a, x, target, target_logit, loss, lse, dx, weight, ignore_index, col_offset=0):
    a.x, a.target, a.weight = _C.ptr(x), _C.ptr(target), _C.ptr(weight)
    a.loss, a.lse, a.dx = _C.ptr(loss), _C.ptr(lse), _C.ptr(dx)
    a.M, a.N = x.shape
    a.x_row_stride = x.stride(0)
    a.dx_row_stride = dx.stride(0) if dx is not None else 0
    a.col_offset = int(col_offset)
    a.ignore_index = int(ignore_index)
    a.num_classes = _num_classes(x, target_logit, weight)
    a.x_dtype = _C.float_code(x)
    a.target_dtype = _C.INDEX_CODES[target.dtype]
    a.weight_dtype = _C.float_code(weight)
    if target_logit is not None:
        a.target_logit = _C.ptr(target_logit)
        a.target_logit_dtype = _C.float_code(target_logit)
        a.target_logit_ndim = target_logit.dim()
        a.target_logit_row_stride = target_logit.stride(0) if target_logit.dim() == 2 else 0
    cfg = _C.env_cfg("ce_fwd")
    if cfg is not None:
        a.cfg = cfg


@kernel_op("quack::cross_entropy_fwd_out", mutates_args={"loss", "lse", "dx"})
def cross_entropy_fwd_out(
    x: Tensor,
    target: Tensor,
    target_logit: Optional[Tensor],
    loss: Tensor,
    lse: Optional[Tensor],
    dx: Optional[Tensor],
    weight: Optional[Tensor],
    ignore_index: int = -100,
) -> None:
    """Per-row loss (fp32), optional log-sum-exp and optional gradient w.r.t. the logits.

    x: (M, N) logits; target: (M,) int32/int64; target_logit: optional (M, K) or (M,) tensor the
    target logit is read from instead of x; weight: optional (N,) class weights.  Rows whose
    target equals ``ignore_index`` get loss 0 and a zero dx row.  dx may be x itself."""
    assert x.dim() == 2, "Input must be 2D"
    assert target.dim() == 1, "Target must be 1D"
    assert x.dtype in _SUPPORTED, "Unsupported input dtype"
    assert target.dtype in (torch.int32, torch.int64), "Target must be int32 or int64"
    if target_logit is not None:
        assert target_logit.dtype in _SUPPORTED
        assert target_logit.dim() in (1, 2)
    if weight is not None:
        assert weight.is_floating_point() and weight.dtype in _SUPPORTED, "weight must be a floating-point tensor"
    assert x.shape[0] == target.shape[0], "Batch dimensions must match"
    for name, t in (("mX", x), ("mTarget", target), ("mLoss", loss)):
        _C.require_cuda(t, name)
    if x.size(0) == 0:
        return
    assert loss.dtype == torch.float32 and loss.is_contiguous()
    if loss.numel() != x.size(0):
        raise ValueError(f"Mismatched mLoss.shape[0]: expected {x.size(0)}, got {loss.numel()}")
    x_ = _rows(x)
    target_ = target.contiguous()
    tl_ = None
    if target_logit is not None:
        tl_ = _rows(target_logit) if target_logit.dim() == 2 else target_logit.contiguous()
    w_ = weight.contiguous() if weight is not None else None
    # The gradient kernel reads the log-sum-exp back, so a dx request needs an lse buffer.
    lse_ = lse
    if lse_ is None and dx is not None:
        lse_ = torch.empty_like(loss)
    if lse_ is not None:
        assert lse_.dtype == torch.float32 and lse_.is_contiguous()
        if lse_.numel() != x.size(0):
            raise ValueError(f"Mismatched mLSE.shape[0]: expected {x.size(0)}, got {lse_.numel()}")
    dx_ = dx
    if dx is not None:
        assert dx.shape == x.shape and dx.dtype == x.dtype
        if dx.stride(-1) != 1:
            dx_ = torch.empty_like(dx, memory_format=torch.contiguous_format)
    a = _C.CeFwdArgs()
    _fill_ce_fwd(a, x_, target_, tl_, loss, lse_, dx_, w_, ignore_index)
    _C.launch(_C.lib().qb_ce_fwd, a, x_, "cross_entropy_fwd")
    if dx is not None and dx_ is not dx:
        dx.copy_(dx_)


def cross_entropy_fwd(
    x: Tensor,
    target: Tensor,
    target_logit: Optional[Tensor] = None,
    weight: Optional[Tensor] = None,
    ignore_index: int = -100,
    return_lse: bool = False,
    return_dx: bool = False,
    inplace_backward: bool = False,
):
    """Returns loss, plus lse and / or dx when requested (dx is x itself with
    ``inplace_backward``)."""
    M = x.size(0)
    loss = torch.empty(M, device=x.device, dtype=torch.float32)
    lse = torch.empty(M, device=x.device, dtype=torch.float32) if return_lse else None
    dx = (x if inplace_backward else torch.empty_like(x)) if return_dx else None
    cross_entropy_fwd_out(x, target, target_logit, loss, lse, dx, weight, ignore_index)
    if return_lse and return_dx:
        return loss, lse, dx
    if return_lse:
        return loss, lse
    if return_dx:
        return loss, dx
    return loss


def _cross_entropy_backward(x, target, dloss, lse, dx, weight=None, ignore_index=-100) -> None:
    assert x.dim() == 2, "Input must be 2D"
    assert target.dim() == 1, "Target must be 1D"
    assert dloss.dim() == 1, "dloss must be 1D"
    assert lse.dim() == 1, "lse must be 1D"
    assert x.shape[0] == target.shape[0], "Batch dimensions must match"
    assert x.shape[0] == dloss.shape[0], "Batch dimensions must match"
    assert x.shape[0] == lse.shape[0], "Batch dimensions must match"
    assert x.dtype in _SUPPORTED, "Unsupported input dtype"
    assert target.dtype in (torch.int32, torch.int64), "Target must be int32 or int64"
    if weight is not None:
        assert weight.is_cuda, "weight must be on CUDA device"
        assert weight.is_floating_point(), "weight must be a floating-point tensor"
    for name, t in (("mX", x), ("mTarget", target), ("mdLoss", dloss), ("mLSE", lse), ("mdX", dx)):
        _C.require_cuda(t, name)
    if x.size(0) == 0:
        return
    assert dx.shape == x.shape
    x_ = _rows(x)
    dx_ = dx if dx.stride(-1) == 1 else torch.empty_like(dx, memory_format=torch.contiguous_format)
    dloss_ = dloss if dloss.dtype == torch.float32 else dloss.float()
    lse_ = lse.contiguous() if lse.dtype == torch.float32 else lse.float().contiguous()
    w_ = weight.contiguous() if weight is not None else None
    if w_ is not None and w_.dtype not in _SUPPORTED:
        w_ = w_.float()
    target_ = target.contiguous()
    a = _C.CeBwdArgs()
    a.x, a.target, a.dloss, a.lse = _C.ptr(x_), _C.ptr(target_), _C.ptr(dloss_), _C.ptr(lse_)
    a.weight, a.dx = _C.ptr(w_), _C.ptr(dx_)
    a.M, a.N = x_.shape
    a.x_row_stride, a.dx_row_stride = x_.stride(0), dx_.stride(0)
    a.dloss_stride = dloss_.stride(0)  # 0 for an expanded scalar
    a.col_offset = 0
    a.ignore_index = int(ignore_index)
    a.num_classes = w_.numel() if w_ is not None else x_.size(1)
    a.x_dtype, a.dx_dtype = _C.float_code(x_), _C.float_code(dx_)
    a.target_dtype = _C.INDEX_CODES[target_.dtype]
    a.weight_dtype = _C.float_code(w_)
    cfg = _C.env_cfg("ce_bwd")
    if cfg is not None:
        a.cfg = cfg
    _C.launch(_C.lib().qb_ce_bwd, a, x_, "cross_entropy_bwd")
    if dx_ is not dx:
        dx.copy_(dx_)


@kernel_op("quack::cross_entropy_bwd_out", mutates_args={"dx"})
def cross_entropy_bwd_out(
    x: Tensor,
    target: Tensor,
    dloss: Tensor,
    lse: Tensor,
    dx: Tensor,
    weight: Optional[Tensor] = None,
    ignore_index: int = -100,
) -> None:
    """dx = (softmax(x) - onehot(target)) * dloss * weight[target], from the saved lse."""
    _cross_entropy_backward(x, target, dloss, lse, dx, weight, ignore_index)


def cross_entropy_bwd(
    x: Tensor,
    target: Tensor,
    dloss: Tensor,
    lse: Tensor,
    weight: Optional[Tensor] = None,
    ignore_index: int = -100,
    inplace_backward: bool = False,
) -> Tensor:
    """Returns dx; with ``inplace_backward`` (eager only) the gradient overwrites x and x is
    returned.  Under torch.compile the out-of-place op is used, as in the reference."""
    if inplace_backward and not torch.compiler.is_compiling():
        _cross_entropy_backward(x=x, target=target, dloss=dloss, lse=lse, dx=x, weight=weight,
                                ignore_index=ignore_index)
        return x
    dx = torch.empty_like(x)
    cross_entropy_bwd_out(x=x, target=target, dloss=dloss, lse=lse, dx=dx, weight=weight,
                          ignore_index=ignore_index)
    return dx


class CrossEntropyFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, target, lse_partial=None, weight=None, ignore_index=-100,
                inplace_backward=False):
        if lse_partial is None:
            loss, lse = cross_entropy_fwd(x, target, weight=weight, ignore_index=ignore_index,
                                          return_lse=True)
        else:
            # Partial log-sum-exps already reduce blocks of columns: the row's lse is the lse of
            # the partials, and the target logit still comes from x.
            loss, lse = cross_entropy_fwd(lse_partial, target, target_logit=x, weight=weight,
                                          ignore_index=ignore_index, return_lse=True)
        ctx.save_for_backward(x, target, lse, weight)
        ctx.ignore_index = ignore_index
        ctx.inplace_backward = inplace_backward
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x, target, lse, weight = ctx.saved_tensors
        dx = cross_entropy_bwd(x, target, dloss, lse, weight=weight,
                               ignore_index=ctx.ignore_index,
                               inplace_backward=ctx.inplace_backward)
        return dx, None, None, None, None, None


def cross_entropy(
    x: Tensor,
    target: Tensor,
    lse_partial: Optional[Tensor] = None,
    weight: Optional[Tensor] = None,
    ignore_index: int = -100,
    reduction: Literal["none", "mean", "sum"] = "mean",
    inplace_backward: bool = False,
) -> Tensor:
    """Cross-entropy loss with autograd.  x: (M, N) logits; target: (M,) class ids.
    ``reduction``: "none" -> (M,) fp32 losses, "sum", or "mean" over the non-ignored rows
    (weighted by ``weight[target]`` when class weights are given)."""
    loss = CrossEntropyFunction.apply(x, target, lse_partial, weight, ignore_index,
                                      inplace_backward)
    if reduction == "mean":
        if weight is not None:
            valid = target != ignore_index
            denom = (weight[target.clamp(min=0)] * valid).sum()
            return loss.sum() / denom
        return loss.sum() / (target != ignore_index).sum().float()
    if reduction == "sum":
        return loss.sum()
    if reduction == "none":
        return loss
    raise ValueError(
        f"Invalid reduction mode: {reduction}. Expected one of 'none', 'mean', or 'sum'"
    )
