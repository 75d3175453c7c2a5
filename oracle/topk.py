"""CPU oracle of top-k (+ softmax over the k values).  TEST INFRASTRUCTURE ONLY.

The reference has no reference function for this op; its test compares with ``torch.topk``
(largest, sorted) followed by ``torch.softmax`` over the k values in fp32
(tests/test_topk.py:40-43) and builds the expected input gradient by scattering
(tests/test_topk.py:62-64,75-80).  Restated here with a stable descending sort, which also fixes
the order of equal values (smaller column first: what the kernels produce).
"""

from __future__ import annotations

import torch


def topk_ref(x, k: int, softmax: bool = False):
    """Returns (values (M, k) in x.dtype, indices (M, k) int32), largest first."""
    xs = x.detach()
    order = torch.sort(xs.float(), dim=-1, descending=True, stable=True).indices[:, :k]
    values = torch.gather(xs, 1, order)
    if softmax:
        values = torch.softmax(values.float(), dim=-1).to(x.dtype)
    return values, order.to(torch.int32)


def topk_bwd_ref(dvalues, values, indices, N: int, softmax: bool = False):
    """dx (M, N) fp32: dvalues scattered to ``indices`` (through the softmax Jacobian of the saved
    ``values`` when the forward applied a softmax)."""
    g = dvalues.detach().float()
    if softmax:
        y = values.detach().float()
        g = y * (g - (g * y).sum(dim=-1, keepdim=True))
    dx = torch.zeros(dvalues.shape[0], N, dtype=torch.float32)
    dx.scatter_(1, indices.long(), g)
    return dx
