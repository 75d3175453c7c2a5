"""Alias package: ``import quack`` resolves to the B200-native implementation in
``quack_flydsl_b200`` so that code written against the reference package
(``from quack import rmsnorm``, ``from quack.rmsnorm import rmsnorm_fwd`` ...) runs unchanged."""

import importlib as _importlib
import sys as _sys

import quack_flydsl_b200 as _impl
from quack_flydsl_b200 import *  # noqa: F401,F403
from quack_flydsl_b200 import __all__, __version__  # noqa: F401

for _name in ("rmsnorm", "rmsnorm_config", "layernorm", "softmax", "cross_entropy", "rounding",
              "sharded", "linear_cross_entropy", "rms_final_reduce", "cute_dsl_utils", "topk", "dsl",
              "dsl.torch_library_op"):
    _sys.modules[f"quack.{_name}"] = _importlib.import_module(f"quack_flydsl_b200.{_name}")
