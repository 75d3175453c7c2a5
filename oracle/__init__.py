"""CPU oracle for the row-reduction hot path.  TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU, fp32 by default) restatement of what the reference computes for RMSNorm,
LayerNorm, softmax and cross-entropy, forward and backward.  Only the test-suite, the smoke
check and the CPU-baseline / reference arm of the benchmark may import this package; the
product (``quack_flydsl_b200``) never does and has no CPU path.

Parity pinning: ``tests/test_oracle_golden.py`` checks every function here against fixtures in
``tests/golden/`` that were produced by the reference's own PyTorch reference functions
(AST-extracted from quack/rmsnorm.py:563-594,1727-1741 and executed on CPU) and by the PyTorch
calls the reference's tests use as ground truth (``F.softmax``, ``F.cross_entropy``,
``torch.logsumexp``, ``F.layer_norm`` + autograd; tests/test_softmax.py:53,
tests/test_cross_entropy.py:51,288, tests/test_layernorm.py:64-74), and against the reference
tests' closed-form known answers.
"""

from oracle.norm import (  # noqa: F401
    layernorm_bwd_ref,
    layernorm_mean_ref,
    layernorm_ref,
    layernorm_rstd_ref,
    rmsnorm_bwd_ref,
    rmsnorm_ref,
    rmsnorm_rstd_ref,
)
from oracle.softmax import softmax_bwd_ref, softmax_ref  # noqa: F401
from oracle.cross_entropy import (  # noqa: F401
    cross_entropy_bwd_ref,
    cross_entropy_combine_ref,
    cross_entropy_ref,
    cross_entropy_shard_stats_ref,
)
from oracle.linear_cross_entropy import linear_cross_entropy_ref, rms_final_reduce_ref  # noqa: F401
from oracle.topk import topk_bwd_ref, topk_ref  # noqa: F401
from oracle.util import bf16_ulp_diff, make_config_inputs  # noqa: F401
