"""CPU tests of the host-side mirror of the reference API: argument validation raises the
reference's exception types and messages before anything touches CUDA, allocation / aliasing
rules, launch-plan tables, the alias package."""

import pytest
import torch

import importlib

import quack
from quack_flydsl_b200 import sharded

# The package re-exports functions named like its submodules (as the reference does), so the
# modules themselves are fetched by name.
ce_mod = importlib.import_module("quack_flydsl_b200.cross_entropy")
ln_mod = importlib.import_module("quack_flydsl_b200.layernorm")
rn_mod = importlib.import_module("quack_flydsl_b200.rmsnorm")
sm_mod = importlib.import_module("quack_flydsl_b200.softmax")
from quack_flydsl_b200.rmsnorm_config import (
    RmsNormBwdConfig,
    RmsNormFwdConfig,
    get_all_bwd_configs,
    get_all_fwd_configs,
)


def test_alias_package_exposes_reference_names():
    assert quack.__all__ == ["rmsnorm", "layernorm", "softmax", "cross_entropy", "RoundingMode"]
    from quack.rmsnorm import (  # noqa: F401
        QuackRMSNorm, RMSNormFunction, _compile_rmsnorm_fwd, rmsnorm, rmsnorm_bwd,
        rmsnorm_bwd_tuned, rmsnorm_fwd, rmsnorm_fwd_tuned,
    )
    from quack.layernorm import layernorm, layernorm_bwd, layernorm_fwd  # noqa: F401
    from quack.softmax import softmax, softmax_bwd, softmax_fwd  # noqa: F401
    from quack.cross_entropy import (  # noqa: F401
        cross_entropy, cross_entropy_bwd, cross_entropy_fwd, cross_entropy_fwd_out,
    )
    from quack.rmsnorm_config import RmsNormFwdConfig as C  # noqa: F401
    assert quack.rmsnorm is rn_mod.rmsnorm


def test_rmsnorm_validation_messages():
    # reference: tests/test_rmsnorm.py:337-380
    x = torch.randn(32, 1024, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"Mismatched mW.shape\[0\]"):
        rn_mod.rmsnorm(x, torch.randn(512))
    with pytest.raises(ValueError, match="expected device_type=cuda"):
        rn_mod.rmsnorm(x, torch.randn(1024))
    with pytest.raises(AssertionError, match="Unsupported dtype"):
        rn_mod.rmsnorm(x.double(), torch.randn(1024))
    with pytest.raises(AssertionError, match="Weight must be float32, float16 or bfloat16"):
        rn_mod.rmsnorm(x, torch.randn(1024, dtype=torch.float64))
    with pytest.raises(AssertionError, match="weight_offset requires a weight"):
        rn_mod.rmsnorm_fwd(x, None, weight_offset=1.0)
    with pytest.raises(RuntimeError, match="requires a config"):
        rn_mod.rmsnorm_fwd_tuned.fn(x, None, torch.empty_like(x))
    with pytest.raises(RuntimeError, match="requires a config"):
        rn_mod.rmsnorm_bwd_tuned.fn(x, None, x, torch.empty(32), torch.empty_like(x), None)


def test_layernorm_validation_messages():
    # reference: tests/test_layernorm.py:142-181
    w = torch.randn(1024)
    with pytest.raises(AssertionError, match="Input must be 2D"):
        ln_mod.layernorm_fwd(torch.randn(2, 32, 1024, dtype=torch.float16), w)
    x = torch.randn(32, 1024, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"Mismatched mW.shape\[0\]"):
        ln_mod.layernorm_fwd(x, torch.randn(512))
    with pytest.raises(ValueError, match="expected device_type=cuda"):
        ln_mod.layernorm_fwd(x, w)
    with pytest.raises(AssertionError, match="Unsupported dtype"):
        ln_mod.layernorm_fwd(x.double(), w)
    with pytest.raises(AssertionError, match="Weight must be float32"):
        ln_mod.layernorm_fwd(x, w.half())
    with pytest.raises(AssertionError, match="Bias must be float32"):
        ln_mod.layernorm_fwd(x, w, bias=w.half())


def test_softmax_and_ce_validation_messages():
    with pytest.raises(AssertionError, match="Input must be 2D"):
        sm_mod.softmax_fwd(torch.randn(2, 3, 8))
    with pytest.raises(AssertionError, match="Unsupported dtype"):
        sm_mod.softmax_fwd(torch.randn(3, 8, dtype=torch.float64))
    with pytest.raises(ValueError, match="expected device_type=cuda"):
        sm_mod.softmax_fwd(torch.randn(3, 8))
    with pytest.raises(AssertionError, match="dy and y must have same shape"):
        sm_mod.softmax_bwd(torch.randn(3, 8), torch.randn(3, 16))
    x = torch.randn(4, 16)
    t = torch.randint(0, 16, (4,))
    with pytest.raises(AssertionError, match="Target must be int32 or int64"):
        ce_mod.cross_entropy_fwd(x, t.float())
    with pytest.raises(AssertionError, match="Target must be 1D"):
        ce_mod.cross_entropy_fwd(x, t.unsqueeze(0))
    with pytest.raises(AssertionError, match="Unsupported input dtype"):
        ce_mod.cross_entropy_fwd(x.double(), t)
    with pytest.raises(ValueError, match="expected device_type=cuda"):
        ce_mod.cross_entropy_fwd(x, t)


def test_device_check_precedes_empty_early_out():
    x = torch.empty(0, 4096, dtype=torch.bfloat16)
    w = torch.randn(4096)
    with pytest.raises(ValueError, match="expected device_type=cuda"):
        rn_mod.rmsnorm_fwd(x, w)  # device validation precedes the empty early-out, as with TVM-FFI


def test_config_dataclasses_and_search_spaces():
    f = RmsNormFwdConfig(num_threads=128, threads_per_row=32, cluster_n=2, reload_from="smem",
                         delay_w_load=True)
    b = RmsNormBwdConfig(num_threads=128, threads_per_row=32, cluster_n=2, reload_wdy=None,
                         reload_x=None, use_tma=False, smem_stages=2)
    with pytest.raises(Exception):
        f.num_threads = 1  # frozen
    assert b.smem_stages == 2
    assert all(c.threads_per_row <= c.num_threads for c in get_all_fwd_configs())
    assert len(get_all_bwd_configs()) > len(get_all_fwd_configs())
    h = RmsNormFwdConfig.from_analytical_heuristic(8192, 16)
    assert (h.num_threads, h.threads_per_row, h.cluster_n) == (128, 128, 1)
    assert RmsNormFwdConfig.from_analytical_heuristic(65536, 16).cluster_n == 4
    assert RmsNormFwdConfig.from_analytical_heuristic(262144, 16).cluster_n == 16
    hb = RmsNormBwdConfig.from_analytical_heuristic(8192, 16, 16)
    assert (hb.num_threads, hb.threads_per_row, hb.cluster_n) == (128, 128, 1)
    assert RmsNormBwdConfig.from_analytical_heuristic(262144, 16, 16).cluster_n == 16
    # short rows: several rows per CTA
    hs = RmsNormFwdConfig.from_analytical_heuristic(256, 16)
    assert hs.threads_per_row < hs.num_threads
    # RMSNorm at hidden sizes 1024 ... 4096 (16-bit, with residual): four chunks per thread
    for n, tpr in ((4096, 128), (2048, 64), (1024, 32)):
        hf = RmsNormFwdConfig.from_analytical_heuristic(n, 16)
        assert (hf.num_threads, hf.threads_per_row, hf.cluster_n) == (128, tpr, 1), (n, hf)
    # LayerNorm and rows that do not fill such a tile keep eight chunks per thread
    assert RmsNormFwdConfig.from_analytical_heuristic(4096, 16, is_layernorm=True).threads_per_row == 64
    assert RmsNormFwdConfig.from_analytical_heuristic(3072, 16).threads_per_row == 64


def test_selection_cache_counts_specialisations():
    c = rn_mod._SelectionCache()
    c.note(("a", 1))
    c.note(("a", 1))
    c.note(("b", 2))
    assert c.cache_info().currsize == 2 and c.cache_info().hits == 1
    c.cache_clear()
    assert c.cache_info().currsize == 0


def test_row_and_vocab_shards_cover_everything():
    for M, G in [(32768, 8), (10, 4), (3, 8), (65536, 2)]:
        spans = [sharded.row_shard(M, r, G) for r in range(G)]
        assert spans[0][0] == 0 and spans[-1][1] == M
        assert all(spans[i][1] == spans[i + 1][0] for i in range(G - 1))
    for N, G in [(128256, 8), (128256, 2), (1000, 4), (8, 8)]:
        spans = [sharded.vocab_shard(N, r, G) for r in range(G)]
        assert spans[0][0] == 0 and spans[-1][1] == N
        assert all(spans[i][1] == spans[i + 1][0] for i in range(G - 1))
        assert all(b % 8 == 0 for b, _ in spans)
    assert sharded.vocab_shard(128256, 3, 8) == (3 * 16032, 4 * 16032)


def test_row_stride_helper():
    x = torch.empty(8, 576)[:, :512]
    assert rn_mod._row_stride(x) == 576
    y = torch.empty(4, 6, 64)
    assert rn_mod._row_stride(y) == 64
    assert rn_mod._row_stride(y[:, :3]) is None  # (4, 3, 64) view: rows not uniformly strided
    assert rn_mod._row_stride(torch.empty(8, 64).t()) is None


def test_get_sm_count_pure_python_estimate(monkeypatch):
    """Inside torch.compile traces get_sm_count cannot ask the library; the pure-Python estimate
    gives one persistent CTA (two of 128 threads) per SM, or the clusters resident at once."""
    import types

    from quack_flydsl_b200 import rmsnorm_config as rc

    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda device: types.SimpleNamespace(multi_processor_count=148))
    monkeypatch.setattr(torch.compiler, "is_compiling", lambda: True)
    assert rc.get_sm_count(4096, "cuda", torch.bfloat16) == 296     # 128-thread CTAs, two per SM
    assert rc.get_sm_count(8192, "cuda", torch.bfloat16) == 296
    assert rc.get_sm_count(16384, "cuda", torch.bfloat16) == 148    # one 256-thread CTA per SM
    assert rc.get_sm_count(32768, "cuda", torch.bfloat16) == 74     # clusters of two such CTAs
    assert rc.get_sm_count(65536, "cuda", torch.bfloat16) == 32     # clusters of 8
    assert rc.get_sm_count(131072, "cuda", torch.bfloat16) == 15    # clusters of 16
    assert rc.get_sm_count(262144, "cuda", torch.bfloat16) == 7    # clusters of 16 CTAs of 256 threads
    assert rc.get_sm_count(8192, "cuda", torch.float32) == 148
    assert rc.get_sm_count(4096, "cuda", torch.float32) == 296
