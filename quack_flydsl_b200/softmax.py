"""Softmax over the last dimension behind the reference's Python API.

Host-side mirror of quack/softmax.py: ops ``quack::_softmax_fwd`` (:193-207) and
``quack::_softmax_backward`` (:373-391), ``softmax_fwd`` / ``softmax_bwd`` (:210-213, :394-397),
``SoftmaxFunction`` (:400-411) and ``softmax`` (:414-423).
"""

from __future__ import annotations

from ctypes import byref

import torch

from quack_flydsl_b200 import _C
from quack_flydsl_b200.dsl import kernel_op

_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32)


def _rows(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 or t.size(-1) == 1 else t.contiguous()


@kernel_op("quack::_softmax_fwd", mutates_args={"out"})
def _softmax_fwd(x: torch.Tensor, out: torch.Tensor) -> None:
    """out = softmax(x, dim=-1) for a 2-D x; out is pre-allocated with x's shape."""
    assert x.dim() == 2, "Input must be 2D"
    assert x.dtype in _SUPPORTED, "Unsupported dtype"
    assert out.shape == x.shape and out.dtype in _SUPPORTED
    if not (x.is_cuda and out.is_cuda):
        _C.require_cuda(x, "mX")
        _C.require_cuda(out, "mO")
    if x.numel() == 0:
        return
    x_ = _rows(x)
    out_ = out if out.stride(-1) == 1 else torch.empty_like(out, memory_format=torch.contiguous_format)
    a = _C.SoftmaxFwdArgs()
    a.x, a.out = _C.ptr(x_), _C.ptr(out_)
    a.M, a.N = x_.shape
    a.x_row_stride, a.out_row_stride = x_.stride(0), out_.stride(0)
    a.x_dtype, a.out_dtype = _C.float_code(x_), _C.float_code(out_)
    cfg = _C.env_cfg("softmax_fwd")
    if cfg is not None:
        a.cfg = cfg
    _C.launch(_C.lib().qb_softmax_fwd, a, x_, "softmax_fwd")
    if out_ is not out:
        out.copy_(out_)


def softmax_fwd(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    _softmax_fwd(x, out)
    return out


@kernel_op("quack::_softmax_backward", mutates_args={"dx"})
def _softmax_backward(dy: torch.Tensor, y: torch.Tensor, dx: torch.Tensor) -> None:
    """dx = y * (dy - sum(dy * y, dim=-1)) for 2-D dy and y (the saved softmax output)."""
    assert dy.dim() == 2, "dy must be 2D"
    assert y.dim() == 2, "y must be 2D"
    assert dy.shape == y.shape, "dy and y must have same shape"
    assert dy.dtype in _SUPPORTED, "Unsupported dtype"
    assert y.dtype == dy.dtype, "dy and y must have same dtype"
    assert dx.shape == dy.shape and dx.dtype in _SUPPORTED
    if not (dy.is_cuda and y.is_cuda and dx.is_cuda):
        for name, t in (("mdY", dy), ("mY", y), ("mdX", dx)):
            _C.require_cuda(t, name)
    if dy.numel() == 0:
        return
    dy_, y_ = _rows(dy), _rows(y)
    dx_ = dx if dx.stride(-1) == 1 else torch.empty_like(dx, memory_format=torch.contiguous_format)
    a = _C.SoftmaxBwdArgs()
    a.dy, a.y, a.dx = _C.ptr(dy_), _C.ptr(y_), _C.ptr(dx_)
    a.M, a.N = dy_.shape
    a.dy_row_stride, a.y_row_stride, a.dx_row_stride = dy_.stride(0), y_.stride(0), dx_.stride(0)
    a.dy_dtype, a.y_dtype, a.dx_dtype = _C.float_code(dy_), _C.float_code(y_), _C.float_code(dx_)
    cfg = _C.env_cfg("softmax_bwd")
    if cfg is not None:
        a.cfg = cfg
    _C.launch(_C.lib().qb_softmax_bwd, a, dy_, "softmax_bwd")
    if dx_ is not dx:
        dx.copy_(dx_)


def softmax_bwd(dy: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    dx = torch.empty_like(dy)
    _softmax_backward(dy, y, dx)
    return dx


class SoftmaxFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = softmax_fwd(x)
        ctx.save_for_backward(y)  # the backward needs only the output
        return y

    @staticmethod
    def backward(ctx, dy):
        (y,) = ctx.saved_tensors
        return softmax_bwd(dy, y)


def softmax(x: torch.Tensor) -> torch.Tensor:
    """Softmax over the last dimension of a 2-D tensor, with autograd."""
    return SoftmaxFunction.apply(x)
