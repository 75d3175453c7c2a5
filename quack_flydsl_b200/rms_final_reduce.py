"""rstd from partial sums of squares, behind the reference's Python API.

Host-side mirror of quack/rms_final_reduce.py: op ``quack::rms_final_reduce_out`` (:138-153) and
``rms_final_reduce`` (:156-166).  The kernel is the finalising step of a GEMM + RMSNorm pipeline:
the GEMM epilogue leaves one partial sum of squares per (row, column tile); this reduces them and
applies ``rsqrt(sum * scale + eps)``.
"""

from __future__ import annotations

from ctypes import byref

import torch
from torch import Tensor

from quack_flydsl_b200 import _C
from quack_flydsl_b200.dsl import kernel_op

_SUPPORTED = (torch.float16, torch.bfloat16, torch.float32)


@kernel_op("quack::rms_final_reduce_out", mutates_args=("rstd",), device_types="cuda")
def _rms_final_reduce_out(x: Tensor, rstd: Tensor, scale: float, eps: float) -> None:
    """rstd[m] = rsqrt(sum_n(x[m, n]) * scale + eps); rstd is a pre-allocated fp32 vector."""
    assert x.dim() == 2, "Input must be 2D"
    assert x.dtype in _SUPPORTED, "Unsupported dtype"
    assert rstd.dtype == torch.float32 and rstd.shape == (x.shape[0],)
    _C.require_cuda(x, "mX")
    _C.require_cuda(rstd, "mRstd")
    if x.shape[0] == 0:
        return
    assert x.shape[1] > 0, "rows must not be empty"
    x_ = x if x.stride(-1) == 1 or x.size(-1) == 1 else x.contiguous()
    rstd_ = rstd if rstd.is_contiguous() else torch.empty_like(rstd, memory_format=torch.contiguous_format)
    a = _C.RmsFinalReduceArgs()
    a.x, a.rstd = _C.ptr(x_), _C.ptr(rstd_)
    a.M, a.N = x_.shape
    a.x_row_stride = x_.stride(0)
    a.scale, a.eps = float(scale), float(eps)
    a.x_dtype = _C.float_code(x_)
    with _C.device_of(x_):
        _C.check(_C.lib().qb_rms_final_reduce(byref(a), _C.stream_of(x_)), "rms_final_reduce")
    if rstd_ is not rstd:
        rstd.copy_(rstd_)


def rms_final_reduce(x: Tensor, scale: float, eps: float = 1e-6) -> Tensor:
    """rstd[m] = rsqrt(sum_n(x[m, n]) * scale + eps) for a 2-D x of partial sums of squares;
    ``scale`` is typically 1 / (number of columns the sums were taken over)."""
    assert x.ndim == 2
    rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    _rms_final_reduce_out(x, rstd, scale, eps)
    return rstd
