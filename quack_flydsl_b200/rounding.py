"""``RoundingMode`` is exported by the reference's top-level package (quack/__init__.py:21) for its
GEMM epilogues (quack/rounding.py).  The row-reduction kernels always round to nearest even; the
enum exists so that ``from quack import RoundingMode`` keeps working."""

import enum


class RoundingMode(enum.IntEnum):
    RN = 0  # round to nearest even (the only mode the row-reduction kernels use)
    RS = 1  # stochastic rounding (GEMM epilogues only; not used on this path)
