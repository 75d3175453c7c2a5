"""Top-k (optionally followed by a softmax over the k values) behind the reference's Python API.

Host-side mirror of quack/topk.py: ops ``quack::_topk_fwd`` (:234-254) and ``quack::_topk_bwd``
(:461-491), ``topk_fwd`` (:257-272), ``topk_bwd`` (:494-516), ``TopKFunction`` (:519-535) and
``topk`` (:538-549).  The forward keeps the reference's contract (N and k powers of two,
N <= 4096, k <= 128); values and indices are exact: no mantissa bits are spent on the index.
"""

from __future__ import annotations

from ctypes import byref
from typing import Optional

import torch

from quack_flydsl_b200 import _C
from quack_flydsl_b200.dsl import kernel_op

_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32)


def _is_pow2(v: int) -> bool:
    return v > 0 and (v & (v - 1)) == 0


@kernel_op("quack::_topk_fwd", mutates_args={"values", "indices"})
def _topk_fwd(x: torch.Tensor, k: int, softmax: bool, values: torch.Tensor,
              indices: torch.Tensor) -> None:
    """values (M, k), indices (M, k) int32 = the k largest entries of every row of x (M, N),
    largest first; with ``softmax`` the values are replaced by their softmax."""
    assert x.dim() == 2, "Input must be 2D"
    assert x.dtype in _SUPPORTED, "Unsupported dtype"
    assert k > 0 and k <= x.shape[1], "k must be positive and <= N"
    N = x.shape[1]
    assert _is_pow2(N), "N must be a power of 2"
    assert _is_pow2(k), "k must be a power of 2"
    assert k <= 128
    assert N <= 4096
    assert values.shape == (x.shape[0], k) and values.dtype == x.dtype and values.is_contiguous()
    assert indices.shape == (x.shape[0], k) and indices.dtype == torch.int32 and indices.is_contiguous()
    for name, t in (("mX", x), ("mValues", values), ("mIndices", indices)):
        _C.require_cuda(t, name)
    if x.numel() == 0:
        return
    x_ = x if x.stride(-1) == 1 else x.contiguous()
    a = _C.TopkFwdArgs()
    a.x, a.values, a.indices = _C.ptr(x_), _C.ptr(values), _C.ptr(indices)
    a.M, a.N = x_.shape
    a.k = int(k)
    a.x_row_stride = x_.stride(0)
    a.x_dtype = _C.float_code(x_)
    a.softmax = int(bool(softmax))
    with _C.device_of(x_):
        _C.check(_C.lib().qb_topk_fwd(byref(a), _C.stream_of(x_)), "topk_fwd")


def topk_fwd(x: torch.Tensor, k: int, softmax: bool = False):
    """Returns (values (M, k) in x.dtype, indices (M, k) int32)."""
    M = x.size(0)
    values = torch.empty((M, k), dtype=x.dtype, device=x.device)
    indices = torch.empty((M, k), dtype=torch.int32, device=x.device)
    _topk_fwd(x, k, softmax, values, indices)
    return values, indices


@kernel_op("quack::_topk_bwd", mutates_args={"dx"})
def _topk_bwd(dvalues: torch.Tensor, values: Optional[torch.Tensor], indices: torch.Tensor, k: int,
              softmax: bool, dx: torch.Tensor) -> None:
    """dx (M, N) = the upstream gradients scattered to their columns, zero elsewhere (every row of
    dx is written completely); with ``softmax`` the gradients first pass through the softmax
    Jacobian of the saved ``values``."""
    assert dvalues.dim() == 2, "dvalues must be 2D"
    if values is not None:
        assert values.dim() == 2, "values must be 2D"
    assert indices.dim() == 2, "indices must be 2D"
    assert dvalues.dtype in _SUPPORTED, "Unsupported dtype"
    assert dx.dim() == 2 and dx.dtype in _SUPPORTED
    if softmax:
        assert values is not None, "values are required for the softmax backward"
    for name, t in (("mdValues", dvalues), ("mIndices", indices), ("mdX", dx)):
        _C.require_cuda(t, name)
    if dvalues.numel() == 0:
        return
    assert indices.dtype == torch.int32
    dv = dvalues.contiguous()
    vals = values.contiguous() if values is not None else None
    idx = indices.contiguous()
    dx_ = dx if dx.stride(-1) == 1 else torch.empty_like(dx, memory_format=torch.contiguous_format)
    a = _C.TopkBwdArgs()
    a.dvalues, a.values, a.indices, a.dx = _C.ptr(dv), _C.ptr(vals), _C.ptr(idx), _C.ptr(dx_)
    a.M, a.N = dx_.shape
    a.k = dv.shape[1]
    a.dx_row_stride = dx_.stride(0)
    a.dvalues_dtype, a.values_dtype, a.dx_dtype = _C.float_code(dv), _C.float_code(vals), _C.float_code(dx_)
    a.softmax = int(bool(softmax))
    with _C.device_of(dx_):
        _C.check(_C.lib().qb_topk_bwd(byref(a), _C.stream_of(dx_)), "topk_bwd")
    if dx_ is not dx:
        dx.copy_(dx_)


def topk_bwd(dvalues: torch.Tensor, values: Optional[torch.Tensor], indices: torch.Tensor, N: int,
             softmax: bool = False) -> torch.Tensor:
    """Returns dx (M, N) in dvalues.dtype."""
    M, k = dvalues.shape
    # the kernel writes every row completely, so no zero-fill pass is needed first
    dx = torch.empty((M, N), dtype=dvalues.dtype, device=dvalues.device)
    _topk_bwd(dvalues, values, indices, k, softmax, dx)
    return dx


class TopKFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, k: int, softmax: bool = False):
        values, indices = topk_fwd(x, k, softmax=softmax)
        ctx.save_for_backward(values if softmax else None, indices)
        ctx.k = k
        ctx.N = x.shape[1]
        ctx.softmax = softmax
        ctx.mark_non_differentiable(indices)
        ctx.set_materialize_grads(False)
        return values, indices

    @staticmethod
    def backward(ctx, dvalues: torch.Tensor, dindices_: Optional[torch.Tensor] = None):
        values, indices = ctx.saved_tensors
        if dvalues is None:
            return None, None, None
        dx = topk_bwd(dvalues, values, indices, N=ctx.N, softmax=ctx.softmax)
        return dx, None, None


def topk(x: torch.Tensor, k: int, softmax: bool = False):
    """Top-k over the last dimension of a 2-D tensor with autograd: returns (values, indices),
    values sorted in descending order (softmaxed over the k entries if ``softmax``)."""
    return TopKFunction.apply(x, k, softmax)
