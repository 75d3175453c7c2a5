"""B200-native (sm_100a) row-reduction kernels behind the QuACK Python API.

RMSNorm, LayerNorm, softmax and cross-entropy, forward and backward.  The public names and
signatures are those of the reference package (quack/__init__.py:18-29); ``import quack`` also
works through the thin alias package at the repository root.
"""

__version__ = "0.6.1+b200"

from quack_flydsl_b200.rmsnorm import rmsnorm  # noqa: E402
from quack_flydsl_b200.layernorm import layernorm  # noqa: E402
from quack_flydsl_b200.softmax import softmax  # noqa: E402
from quack_flydsl_b200.cross_entropy import cross_entropy  # noqa: E402
from quack_flydsl_b200.rounding import RoundingMode  # noqa: E402

__all__ = ["rmsnorm", "layernorm", "softmax", "cross_entropy", "RoundingMode"]
