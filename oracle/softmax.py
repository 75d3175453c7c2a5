"""Oracle: softmax forward / backward on CPU.  Test infrastructure only.

The reference's tests take ``torch.nn.functional.softmax`` and autograd through it as ground
truth (tests/test_softmax.py:53-57); the arithmetic therefore lives in PyTorch (installed wheel,
torch 2.11.0, not part of the reference tree).  This file restates the textbook formulas the
kernels implement (quack/softmax.py:141-176 forward, :330-353 backward) and is pinned against
fixtures generated with those PyTorch calls.
"""

from __future__ import annotations

import torch


def softmax_ref(x, compute_dtype=torch.float32):
    xf = x.detach().to(compute_dtype)
    m = xf.max(dim=-1, keepdim=True).values
    e = torch.exp(xf - m)
    return (e / e.sum(dim=-1, keepdim=True)).to(x.dtype)


def softmax_bwd_ref(dy, y, compute_dtype=torch.float32):
    """dx = y * (dy - sum(dy * y)) from the saved (rounded) output y."""
    dyf = dy.detach().to(compute_dtype)
    yf = y.detach().to(compute_dtype)
    dot = (dyf * yf).sum(dim=-1, keepdim=True)
    return (yf * (dyf - dot)).to(dy.dtype)
