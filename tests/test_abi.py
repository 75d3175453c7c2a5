"""CPU-only checks of the C-ABI library: it loads without a GPU, exports every symbol that
include/quack_b200.h declares, agrees with the ctypes binding on every struct layout, and
reports (rather than crashes on) calls that cannot run."""

import ctypes
import re
from pathlib import Path

import pytest

from quack_flydsl_b200 import _C

ROOT = Path(__file__).resolve().parents[1]


def _declared_symbols():
    text = (ROOT / "include" / "quack_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qb_[a-z_0-9]+)\s*\(", text)))


def test_header_symbols_are_exported():
    lib = _C.lib()
    declared = _declared_symbols()
    assert len(declared) >= 13
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert sorted(_C.EXPORTED_SYMBOLS) == sorted(n for n in declared)


def test_struct_layouts_match():
    lib = _C.lib()
    assert lib.qb_abi_version() == _C.QB_ABI_VERSION
    for code, struct in _C._SIZEOF_CODES.items():
        assert lib.qb_sizeof_args(code) == ctypes.sizeof(struct), struct.__name__
    assert lib.qb_sizeof_args(99) == -1


def test_null_and_bad_arguments_are_reported_not_fatal():
    lib = _C.lib()
    assert lib.qb_norm_fwd(None, None) == _C.QB_ERR_INVALID
    assert "null" in _C.last_error()
    a = _C.SoftmaxFwdArgs()
    assert lib.qb_softmax_fwd(ctypes.byref(a), None) == _C.QB_ERR_INVALID
    b = _C.CeFwdArgs()
    b.x, b.target, b.M, b.N = 16, 16, 4, 8  # dx without lse
    b.dx, b.loss = 16, 16
    assert lib.qb_ce_fwd(ctypes.byref(b), None) == _C.QB_ERR_INVALID
    assert "lse" in _C.last_error()
    c = _C.ColsumArgs()
    assert lib.qb_colsum(ctypes.byref(c), None) == _C.QB_ERR_INVALID


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv("QUACK_B200_LIB", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_C, "_LIB", None)
    with pytest.raises(ImportError, match="no fallback"):
        _C.lib()


def test_env_launch_override(monkeypatch):
    monkeypatch.setenv("QUACK_B200_CFG", "norm_fwd:512:512:1:296;norm_bwd:256:256:1:0:3")
    f = _C.env_cfg("norm_fwd")
    assert (f.num_threads, f.threads_per_row, f.cluster_n, f.max_ctas, f.stages) == (512, 512, 1, 296, 0)
    b = _C.env_cfg("norm_bwd")
    assert (b.num_threads, b.stages) == (256, 3)
    assert _C.env_cfg("softmax_fwd") is None
