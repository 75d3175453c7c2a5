"""Oracle: cross-entropy forward / backward and the vocabulary-sharded combine on CPU.
Test infrastructure only.

The reference's tests compare against ``F.cross_entropy(reduction="none", ignore_index, weight)``
on fp32 logits and ``torch.logsumexp`` (tests/test_cross_entropy.py:51,64-66,288); per-row
semantics restated from the kernel (quack/cross_entropy.py:227-265 forward incl. fused dx,
:500-546 backward): ignored rows give loss 0 and a zero gradient row, lse is still produced,
class weights scale both loss and gradient by w[target].
"""

from __future__ import annotations

from typing import Optional

import torch


def cross_entropy_ref(x, target, weight=None, ignore_index=-100, target_logit=None,
                      compute_dtype=torch.float32):
    """Returns (loss, lse), both fp32 of shape (M,)."""
    xf = x.detach().to(compute_dtype)
    t = target.detach().long()
    m = xf.max(dim=-1).values
    lse = m + torch.log(torch.exp(xf - m.unsqueeze(-1)).sum(dim=-1))
    valid = t != ignore_index
    safe = torch.where(valid, t, torch.zeros_like(t))
    if target_logit is None:
        tl = xf.gather(1, safe.unsqueeze(1)).squeeze(1)
    else:
        tlf = target_logit.detach().to(compute_dtype)
        tl = tlf.gather(1, safe.unsqueeze(1)).squeeze(1) if tlf.dim() == 2 else tlf
    loss = lse - tl
    if weight is not None:
        loss = loss * weight.detach().to(compute_dtype)[safe]
    loss = torch.where(valid, loss, torch.zeros_like(loss))
    return loss.to(torch.float32), lse.to(torch.float32)


def cross_entropy_bwd_ref(x, target, dloss, lse, weight=None, ignore_index=-100,
                          compute_dtype=torch.float32, col_offset=0):
    """dx = (exp(x - lse) - onehot(target)) * dloss * w[target]; zero rows where ignored.
    With ``col_offset`` the columns of x are global classes col_offset .. col_offset + N - 1."""
    xf = x.detach().to(compute_dtype)
    t = target.detach().long()
    M, N = xf.shape
    p = torch.exp(xf - lse.detach().to(compute_dtype).unsqueeze(-1))
    valid = t != ignore_index
    cols = torch.arange(N, device=xf.device).unsqueeze(0) + col_offset
    onehot = (cols == t.unsqueeze(1)) & valid.unsqueeze(1)
    g = dloss.detach().to(compute_dtype).expand(M).clone()
    if weight is not None:
        safe = torch.where(valid, t, torch.zeros_like(t))
        g = g * weight.detach().to(compute_dtype)[safe]
    g = torch.where(valid, g, torch.zeros_like(g))
    return ((p - onehot.to(compute_dtype)) * g.unsqueeze(-1)).to(x.dtype)


def cross_entropy_shard_stats_ref(x_shard, target, col_offset, ignore_index=-100,
                                  compute_dtype=torch.float32):
    """Per-row (max, sum exp(x - max), target logit or 0) of one vocabulary shard."""
    xf = x_shard.detach().to(compute_dtype)
    t = target.detach().long()
    N = xf.shape[1]
    m = xf.max(dim=-1).values
    s = torch.exp(xf - m.unsqueeze(-1)).sum(dim=-1)
    local = t - col_offset
    owned = (t != ignore_index) & (local >= 0) & (local < N)
    safe = torch.where(owned, local, torch.zeros_like(local))
    tl = torch.where(owned, xf.gather(1, safe.unsqueeze(1)).squeeze(1), torch.zeros_like(m))
    return torch.stack([m, s, tl]).to(torch.float32)


def cross_entropy_combine_ref(stats, target, weight=None, ignore_index=-100):
    """stats: (G, 3, M).  m = max_g m_g; s = sum_g s_g exp(m_g - m); t = sum_g t_g."""
    st = stats.detach().to(torch.float32)
    t = target.detach().long()
    m = st[:, 0].max(dim=0).values
    s = (st[:, 1] * torch.exp(st[:, 0] - m.unsqueeze(0))).sum(dim=0)
    tl = st[:, 2].sum(dim=0)
    lse = m + torch.log(s)
    valid = t != ignore_index
    loss = lse - tl
    if weight is not None:
        safe = torch.where(valid, t, torch.zeros_like(t))
        loss = loss * weight.detach().float()[safe]
    return torch.where(valid, loss, torch.zeros_like(loss)), lse
