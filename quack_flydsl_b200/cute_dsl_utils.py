"""The one helper of quack/cute_dsl_utils.py that callers of the row-reduction path use.

The reference module is mostly CuTe-DSL plumbing (argument structs, compile helpers); nothing of
that exists here because nothing is compiled at run time.  ``get_device_capacity``
(quack/cute_dsl_utils.py:115-137) is kept because user code and the reference's own tests branch
on it.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple, Union

import torch


def get_device_capacity(device: Union[torch.device, torch.Tensor, None] = None) -> Tuple[int, int]:
    """(major, minor) compute capability of ``device`` (a device, a tensor, or the current CUDA
    device).  ``QUACK_ARCH`` (e.g. ``sm_100`` or ``100``) overrides the query, as in the reference."""
    arch = os.environ.get("QUACK_ARCH")
    if arch:
        digits = "".join(ch for ch in arch if ch.isdigit())
        if len(digits) >= 2:
            return int(digits[:-1]), int(digits[-1])
    if isinstance(device, torch.Tensor):
        device = device.device
    return tuple(torch.cuda.get_device_capability(device))
