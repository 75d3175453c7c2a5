"""Linear layer + cross-entropy without materialising the full logits, behind the reference API.

Host-side mirror of quack/linear_cross_entropy.py: ``linear_cross_entropy_func`` (:15-28),
``linear_cross_entropy_func_ref`` (:31-40), ``chunked_linear_cross_entropy_fwd`` (:43-111),
``ChunkedLinearCrossEntropyFunction`` (:114-192), ``chunked_linear_cross_entropy`` (:195-222) and
``LinearCrossEntropy`` (:225-276).

Per chunk of rows: logits = x_chunk @ W^T (cuBLAS through ``torch.mm``), then ONE launch of the
cross-entropy kernel that writes the loss and overwrites the logits with their gradient
(``quack::cross_entropy_fwd_out`` with ``dx`` aliasing the logits), then dx_chunk = dlogits @ W and
dW += dlogits^T @ x_chunk, again through cuBLAS.  The reference routes the three matrix products
through its own GEMM stack (quack/gemm_interface.py); plain library GEMMs stand in for it here
and fp32 accumulation of dW across chunks is kept.
"""

from __future__ import annotations

from typing import Literal, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor
from torch.amp import custom_bwd, custom_fwd

from quack_flydsl_b200.cross_entropy import cross_entropy, cross_entropy_fwd_out

__all__ = [
    "linear_cross_entropy_func", "linear_cross_entropy_func_ref", "chunked_linear_cross_entropy_fwd",
    "ChunkedLinearCrossEntropyFunction", "chunked_linear_cross_entropy", "LinearCrossEntropy",
]


def linear_fwd_convert_type(*tensors):
    """Casts to the autocast dtype when autocast is on (reference: quack/linear.py:24-28)."""
    if torch.is_autocast_enabled():
        dtype = torch.get_autocast_dtype("cuda")
        tensors = tuple(t.to(dtype=dtype) for t in tensors)
    return tensors


def linear_cross_entropy_func(
    x: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["none", "mean", "sum"] = "mean",
    inplace_backward: bool = False,
) -> Tensor:
    """Unchunked form: full logits through ``F.linear``, then the cross-entropy kernels."""
    y = F.linear(x, weight, bias)
    batch_shape = y.shape[:-1]
    loss = cross_entropy(y.reshape(-1, y.shape[-1]), target.reshape(-1), ignore_index=ignore_index,
                         reduction=reduction, inplace_backward=inplace_backward)
    return loss.reshape(batch_shape) if reduction == "none" else loss


def linear_cross_entropy_func_ref(
    x: Tensor,
    weight: Tensor,
    bias: Optional[Tensor],
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["none", "mean", "sum"] = "mean",
) -> Tensor:
    y = F.linear(x, weight, bias)
    return F.cross_entropy(y, target, ignore_index=ignore_index, reduction=reduction)


def _mm_f32(a: Tensor, b: Tensor, out: Tensor) -> None:
    """out (fp32) = a @ b for 16-bit or fp32 operands."""
    if a.dtype == torch.float32:
        torch.mm(a, b, out=out)
    else:
        torch.mm(a, b, out_dtype=torch.float32, out=out)


def _addmm_f32(acc: Tensor, a: Tensor, b: Tensor) -> None:
    """acc (fp32) += a @ b for 16-bit or fp32 operands."""
    if a.dtype == torch.float32:
        torch.addmm(acc, a, b, out=acc)
    else:
        torch.addmm(acc, a, b, out_dtype=torch.float32, out=acc)


def chunked_linear_cross_entropy_fwd(
    x: Tensor,  # (B*L, d)
    weight: Tensor,  # (V, d)
    target: Tensor,  # (B*L,)
    chunk_size: int = 4096,
    ignore_index: int = -100,
    tuned: bool = True,
):
    """Returns ``(loss, dx, dw, last_dlogits_chunk, last_x_chunk)``: per-row loss (fp32), the
    gradient of the summed loss w.r.t. x, the fp32 weight gradient accumulated over all chunks
    but the last (None for a single chunk), and the last chunk's logit gradient and input, whose
    contribution to dw is added in the backward pass together with the upstream scale."""
    del tuned  # accepted for signature compatibility: there is nothing to autotune here
    B_L, d = x.shape
    V, _ = weight.shape
    device = x.device
    num_chunks = (B_L + chunk_size - 1) // chunk_size
    assert chunk_size % 8 == 0, "chunk_size must be multiple of 8"
    assert B_L % 8 == 0
    loss = torch.empty(B_L, device=device, dtype=torch.float32)
    logits_buf = torch.empty((min(chunk_size, B_L), V), device=device, dtype=x.dtype)
    dx = torch.empty_like(x)
    dw = torch.empty_like(weight, dtype=torch.float32) if num_chunks > 1 else None
    last_dlogits_chunk = None
    last_x_chunk = None
    chunks = zip(*(t.split(chunk_size) for t in (x, target, loss, dx)))
    for i, (x_chunk, target_chunk, loss_chunk, dx_chunk) in enumerate(chunks):
        chunk_len = x_chunk.shape[0]
        logits_chunk = logits_buf[:chunk_len]
        torch.mm(x_chunk, weight.mT, out=logits_chunk)
        dlogits_chunk = logits_chunk  # the gradient overwrites the logits
        cross_entropy_fwd_out(logits_chunk, target_chunk, None, loss_chunk, None, dlogits_chunk,
                              None, ignore_index)
        torch.mm(dlogits_chunk, weight, out=dx_chunk)
        if i == num_chunks - 1:
            last_dlogits_chunk = dlogits_chunk
            last_x_chunk = x_chunk
        elif i == 0:
            _mm_f32(dlogits_chunk.T, x_chunk, dw)
        else:
            _addmm_f32(dw, dlogits_chunk.T, x_chunk)
    return loss, dx, dw, last_dlogits_chunk, last_x_chunk


class ChunkedLinearCrossEntropyFunction(torch.autograd.Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, weight, target, ignore_index=-100, reduction="mean", chunk_size=4096,
                tuned=True):
        """Computes the loss and, already here, dx and (most of) dw; backward only scales them."""
        ctx.weight_dtype = weight.dtype
        x, weight = linear_fwd_convert_type(x, weight)
        batch_shape = x.shape[:-1]
        x = x.reshape(-1, x.shape[-1])
        loss, dx, dw, last_dlogits_chunk, last_x_chunk = chunked_linear_cross_entropy_fwd(
            x, weight, target.reshape(-1), chunk_size, ignore_index, tuned=tuned
        )
        loss_sum = loss.sum()
        loss_scale = None if reduction == "sum" else 1.0 / (target != ignore_index).sum().float()
        ctx.save_for_backward(dx, dw, last_dlogits_chunk, last_x_chunk, loss_scale)
        ctx.batch_shape = batch_shape
        return loss_sum if loss_scale is None else loss_sum * loss_scale

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dloss):
        dx, dw, last_dlogits_chunk, last_x_chunk, loss_scale = ctx.saved_tensors
        if loss_scale is not None:
            dloss = dloss * loss_scale
        dx.mul_(dloss)
        dx = dx.reshape(*ctx.batch_shape, dx.shape[-1])
        # dw = dloss * (dw + last_dlogits^T @ last_x), accumulated in fp32
        if dw is None:
            dw = torch.empty((last_dlogits_chunk.shape[1], last_x_chunk.shape[1]),
                             device=dx.device, dtype=torch.float32)
            _mm_f32(last_dlogits_chunk.T, last_x_chunk, dw)
        else:
            _addmm_f32(dw, last_dlogits_chunk.T, last_x_chunk)
        dw = dw.mul_(dloss).to(ctx.weight_dtype)
        return dx, dw, None, None, None, None, None


def chunked_linear_cross_entropy(
    x: Tensor,
    weight: Tensor,
    target: Tensor,
    chunk_size: int = 4096,
    ignore_index: int = -100,
    reduction: Literal["mean", "sum"] = "mean",
    tuned: bool = True,
) -> Tensor:
    """Cross-entropy of ``x @ weight.T`` against ``target`` with autograd support, processing
    ``chunk_size`` rows at a time so that only a (chunk_size, V) block of logits ever exists.
    x: (..., d) with a multiple of 8 rows; weight: (V, d); target: (...,)."""
    if reduction not in ["mean", "sum"]:
        raise ValueError(f"Invalid reduction: {reduction}")
    return ChunkedLinearCrossEntropyFunction.apply(x, weight, target, ignore_index, reduction,
                                                   chunk_size, tuned)


class LinearCrossEntropy(nn.Linear):
    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 ignore_index: int = -100, reduction: Literal["none", "mean", "sum"] = "mean",
                 chunk_size: Optional[int] = None, inplace_backward: bool = False,
                 tuned: bool = True, device=None, dtype=None) -> None:
        super().__init__(in_features, out_features, bias=bias, device=device, dtype=dtype)
        self.ignore_index = ignore_index
        self.reduction = reduction
        self.chunk_size = chunk_size
        self.inplace_backward = inplace_backward
        self.tuned = tuned

    def forward(self, input: Tensor, target: Tensor) -> Tensor:
        if (
            self.bias is None
            and input.is_cuda
            and input.stride(-1) == 1
            and self.in_features % 8 == 0
            and self.out_features % 8 == 0
            and input.shape[:-1].numel() % 8 == 0
            and self.chunk_size is not None
            and self.chunk_size % 8 == 0
            and self.reduction in ["mean", "sum"]
        ):
            return chunked_linear_cross_entropy(input, self.weight, target,
                                                chunk_size=self.chunk_size,
                                                ignore_index=self.ignore_index,
                                                reduction=self.reduction, tuned=self.tuned)
        return linear_cross_entropy_func(input, self.weight, self.bias, target,
                                         ignore_index=self.ignore_index, reduction=self.reduction,
                                         inplace_backward=self.inplace_backward)
