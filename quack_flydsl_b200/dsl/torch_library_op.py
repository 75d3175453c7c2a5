"""``kernel_op``: registers an output-mutating launcher as a ``torch.library`` custom op.

Same contract as the reference's ``cute_op`` (quack/dsl/torch_library_op.py:29-99), which it
replaces name for name (``cute_op`` stays available as an alias):

* the op only mutates pre-allocated tensors and returns ``None``;
* its fake (meta) implementation does nothing, so tracing never runs the launcher;
* called eagerly, the Python body runs directly and skips the dispatcher (the dispatcher +
  functionalisation cost is of the order of the kernels' own run time); under ``torch.compile``
  the call is routed through the registered op so that it becomes a graph node.
"""

from __future__ import annotations

import functools
from typing import Any, Callable, Iterable, Optional, Union

import torch

__all__ = ["kernel_op", "cute_op"]


class _DirectWhenEager:
    """What ``kernel_op`` returns: callable like the body, attribute access like the CustomOpDef."""

    def __init__(self, op_def, body: Callable):
        self._custom_op = op_def
        self._init_fn = body
        functools.update_wrapper(self, body)

    def __call__(self, *args, **kwargs):
        # Dynamo folds is_compiling() to True while tracing, so compiled graphs take the first
        # branch and eager code the second.
        if torch.compiler.is_compiling():
            return self._custom_op(*args, **kwargs)
        return self._init_fn(*args, **kwargs)

    def __getattr__(self, item):
        # Reached only for names not found on the wrapper itself.
        return getattr(self.__dict__["_custom_op"], item)


def kernel_op(
    name: str,
    *,
    mutates_args: Union[str, Iterable[str]],
    schema: Optional[str] = None,
    device_types: Optional[Union[str, Iterable[str]]] = None,
) -> Callable[[Callable], Any]:
    """Decorator. ``name`` is ``"namespace::op"``; ``schema`` must be given when an optional tensor
    is mutated (PyTorch cannot infer that alias annotation)."""

    def register(body: Callable) -> _DirectWhenEager:
        options: dict = {"mutates_args": mutates_args}
        if schema is not None:
            options["schema"] = schema
        if device_types is not None:
            options["device_types"] = device_types
        op_def = torch.library.custom_op(name, body, **options)

        def _nothing(*args, **kwargs):
            return None

        op_def.register_fake(_nothing)
        return _DirectWhenEager(op_def, body)

    return register


cute_op = kernel_op
