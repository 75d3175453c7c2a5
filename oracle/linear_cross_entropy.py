"""Oracle: linear layer + cross-entropy and the rstd finalisation of a GEMM + RMSNorm pipeline,
on CPU.  Test infrastructure only.

``linear_cross_entropy_ref`` restates what the reference's test oracle computes
(quack/linear_cross_entropy.py:31-40: ``F.cross_entropy(F.linear(x, weight), target)`` on
upcast inputs, tests/test_linear_cross_entropy.py:33-35) together with its gradients, written
out instead of taken through autograd.  ``rms_final_reduce_ref`` is the closed form the
reference's test uses (tests/test_linear.py:793-803).
"""

from __future__ import annotations

import torch

from oracle.cross_entropy import cross_entropy_bwd_ref


def linear_cross_entropy_ref(x, weight, target, ignore_index=-100, reduction="mean",
                             compute_dtype=torch.float64):
    """Returns (loss, dx, dw) of ``reduce(cross_entropy(x @ weight.T, target))`` for 2-D x (M, d),
    weight (V, d), target (M,); loss is a scalar for "mean" / "sum" and (M,) for "none" (then the
    gradients are those of the sum)."""
    xf = x.detach().to(compute_dtype)
    wf = weight.detach().to(compute_dtype)
    logits = xf @ wf.T
    t = target.detach().long()
    m = logits.max(dim=-1).values
    lse = m + torch.log(torch.exp(logits - m.unsqueeze(-1)).sum(dim=-1))
    ok = t != ignore_index
    safe = torch.where(ok, t, torch.zeros_like(t))
    loss = torch.where(ok, lse - logits.gather(1, safe.unsqueeze(1)).squeeze(1), torch.zeros_like(lse))
    valid = target != ignore_index
    scale = 1.0 / valid.sum().to(compute_dtype) if reduction == "mean" else torch.ones((), dtype=compute_dtype)
    dloss = torch.full((x.shape[0],), 1.0, dtype=compute_dtype) * scale
    dlogits = cross_entropy_bwd_ref(logits, target, dloss, lse,
                                    ignore_index=ignore_index, compute_dtype=compute_dtype)
    dx = dlogits @ wf
    dw = dlogits.T @ xf
    if reduction == "none":
        return loss, dx, dw
    return loss.sum() * scale, dx, dw


def rms_final_reduce_ref(x, scale, eps=1e-6):
    """rstd[m] = rsqrt(sum_n x[m, n] * scale + eps), fp32."""
    return torch.rsqrt(x.detach().float().sum(dim=-1) * scale + eps)
