"""GPU parity tests of softmax forward / backward against the CPU oracle, after the reference's
tests/test_softmax.py, plus the benchmark row sweep (N = 4096 ... 131072) at reduced M."""

import importlib

import pytest
import torch

import oracle
from _util import assert_close_to_oracle, oracle_device, to

pytestmark = pytest.mark.gpu

sm = importlib.import_module("quack_flydsl_b200.softmax")
DEV = "cuda"
TOL = {torch.bfloat16: 1e-2, torch.float16: 1e-3, torch.float32: 1e-4}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [192, 256, 760, 1024, 1128, 4096, 16384, 32768, 65536, 131072, 262144])
@pytest.mark.parametrize("M", [1, 199])
def test_softmax(M, N, dtype):
    x = (0.1 * torch.randn(M, N, device=DEV)).to(dtype).requires_grad_()
    out = sm.softmax(x)
    dy = torch.randn_like(out)
    (dx,) = torch.autograd.grad(out, x, grad_outputs=dy)
    assert out.shape == x.shape and out.dtype == dtype and dx.dtype == dtype
    ref = oracle.softmax_ref(x.detach().cpu().float())
    assert_close_to_oracle(out, ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], what="y")
    sums = out.float().sum(-1)
    torch.testing.assert_close(sums, torch.ones_like(sums), atol=1e-4 if dtype == torch.float32 else 4e-3, rtol=0)
    assert (out >= 0).all() and (out <= 1).all()
    dx_ref = oracle.softmax_bwd_ref(dy.cpu().float(), out.detach().cpu().float())
    assert_close_to_oracle(dx, dx_ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], max_ulp=None, what="dx")


@pytest.mark.parametrize("N", [4096, 16384, 65536, 131072])
def test_softmax_config_row_sweep(N):
    """Benchmark softmax sweep (x = 3 * N(0,1) bf16, dy ~ N(0,1)) at reduced M."""
    M = 2 ** 24 // N
    d = oracle.make_config_inputs(f"c4:{N}", rows=M, device=DEV)
    y = sm.softmax_fwd(d["x"])
    assert_close_to_oracle(y, oracle.softmax_ref(d["x"].cpu().float()), torch.bfloat16, what="y")
    dx = sm.softmax_bwd(d["dy"], y)
    dx_ref = oracle.softmax_bwd_ref(d["dy"].cpu().float(), y.cpu().float())
    assert_close_to_oracle(dx, dx_ref, torch.bfloat16, max_ulp=None, what="dx")
    # rows of dx sum to ~0 (softmax Jacobian annihilates constants)
    assert (dx.float().sum(-1).abs() <= 3e-2).all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_softmax_extreme_values(dtype):
    M, N = 16, 1024
    for v in (10.0, -10.0):
        out = sm.softmax(torch.full((M, N), v, device=DEV, dtype=dtype))
        torch.testing.assert_close(out, torch.full_like(out, 1.0 / N), atol=1e-3, rtol=1e-3)
    x = torch.zeros((M, N), device=DEV, dtype=dtype)
    x[:, 0] = 10.0
    x[:, 1:] = -10.0
    out = sm.softmax(x)
    assert (out[:, 0] > 0.99).all() and (out[:, 1:] < 0.01).all()


def test_softmax_shift_invariance_and_masked_inputs():
    x = torch.randn(8, 512, device=DEV)
    torch.testing.assert_close(sm.softmax(x), sm.softmax(x + 100.0), atol=1e-6, rtol=1e-6)
    # -inf entries (attention-style masks) get probability exactly 0
    x[:, 100:] = float("-inf")
    y = sm.softmax(x)
    assert (y[:, 100:] == 0).all()
    torch.testing.assert_close(y[:, :100].cpu(), oracle.softmax_ref(x[:, :100].cpu()), atol=1e-6, rtol=1e-5)


def test_softmax_golden_fixtures(softmax_ce_golden):
    for c in softmax_ce_golden["softmax"]:
        x, dy = c["x"].to(DEV), c["dy"].to(DEV)
        y = sm.softmax_fwd(x)
        dt = x.dtype
        assert_close_to_oracle(y, c["y"].float(), dt, atol=TOL[dt], rtol=TOL[dt], max_ulp=1, what="y")
        dx = sm.softmax_bwd(dy, c["y"].to(DEV))
        assert_close_to_oracle(dx, c["dx"].float(), dt, atol=TOL[dt], rtol=TOL[dt], max_ulp=None, what="dx")


def test_softmax_strided_rows_and_mixed_dtype_op():
    base = torch.randn(33, 1100, device=DEV, dtype=torch.bfloat16)
    x = base[:, :1024]
    y = sm.softmax_fwd(x)
    assert_close_to_oracle(y, oracle.softmax_ref(x.cpu().float()), torch.bfloat16, what="y")
    out32 = torch.empty(33, 1024, device=DEV, dtype=torch.float32)
    sm._softmax_fwd(x, out32)  # op accepts an output dtype different from the input's
    torch.testing.assert_close(out32.cpu(), oracle.softmax_ref(x.cpu().float()), atol=1e-6, rtol=1e-5)


def test_softmax_empty():
    x = torch.empty(0, 4096, device=DEV, dtype=torch.bfloat16)
    assert sm.softmax_fwd(x).shape == x.shape
    assert sm.softmax_bwd(x, x).shape == x.shape


def test_softmax_torch_compile_fullgraph():
    torch._dynamo.reset()
    x = (0.1 * torch.randn(199, 1024, device=DEV)).bfloat16().requires_grad_()
    fn = torch.compile(sm.softmax, fullgraph=True)
    out = fn(x)
    dy = torch.randn_like(out)
    (dx,) = torch.autograd.grad(out, x, grad_outputs=dy)
    assert_close_to_oracle(out, oracle.softmax_ref(x.detach().cpu().float()), torch.bfloat16, what="y")
    dx_ref = oracle.softmax_bwd_ref(dy.cpu().float(), out.detach().cpu().float())
    assert_close_to_oracle(dx, dx_ref, torch.bfloat16, max_ulp=None, what="dx")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_softmax_streamed_long_rows_match_cluster_path(dtype, monkeypatch):
    """Rows longer than one CTA's registers take the streamed two-pass kernels when there are
    at least as many rows as SMs; flag bit 1 forces the cluster kernels.  Both must agree with
    the oracle and with each other, on strided rows with a ragged chunk count."""
    M, N = 300, 65536 + 8 * 5
    base = (2.0 * torch.randn(M, N + 64, device=DEV)).to(dtype)
    x = base[:, :N]
    x[3, 1000:] = float("-inf")  # masked tail
    dy = torch.randn(M, N, device=DEV).to(dtype)
    y_s = sm.softmax_fwd(x)
    dx_s = sm.softmax_bwd(dy, y_s)
    monkeypatch.setenv("QUACK_B200_CFG", "softmax_fwd:0:0:0:0:0:2;softmax_bwd:0:0:0:0:0:2")
    y_c = sm.softmax_fwd(x)
    dx_c = sm.softmax_bwd(dy, y_s)
    assert not torch.equal(y_c, torch.zeros_like(y_c))
    monkeypatch.delenv("QUACK_B200_CFG")
    ref = oracle.softmax_ref(x.cpu().float())
    for y in (y_s, y_c):
        assert_close_to_oracle(y, ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], what="y")
    assert (y_s[3, 1000:] == 0).all()
    dx_ref = oracle.softmax_bwd_ref(dy.cpu().float(), y_s.cpu().float())
    for dx in (dx_s, dx_c):
        assert_close_to_oracle(dx, dx_ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], max_ulp=None, what="dx")
    if dtype == torch.bfloat16:
        assert oracle.bf16_ulp_diff(y_s.cpu(), y_c.cpu()).max() <= 1
    # explicit thread counts / chunks in flight of the streamed kernels
    for spec in ("softmax_fwd:512:0:0:0:4;softmax_bwd:512:0:0:0:2", "softmax_fwd:256:0:0:148:8;softmax_bwd:1024:0:0:0:4"):
        monkeypatch.setenv("QUACK_B200_CFG", spec)
        y = sm.softmax_fwd(x)
        dx = sm.softmax_bwd(dy, y_s)
        monkeypatch.delenv("QUACK_B200_CFG")
        assert_close_to_oracle(y, ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], what="y")
        assert_close_to_oracle(dx, dx_ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], max_ulp=None, what="dx")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_softmax_cluster_register_kernel_variants(dtype, monkeypatch):
    """Long rows split over a thread-block cluster with the slices held in registers
    (softmax_cluster.cu): every instantiated geometry -- small CTAs without prefetch, large CTAs
    with the next row in flight, the three-buffer pipeline, cluster sizes that are not powers of
    two (N = 40960 -> 5 CTAs), a ragged last slice, fewer rows than clusters -- against the
    oracle, forward and backward, and bit-identical results from run to run."""
    from quack_flydsl_b200 import _C

    flag = 128  # QB_FLAG_CLUSTER_REGS
    fwd_cfgs = ["128:0:0:0:16:{f}:1", "256:0:0:0:8:{f}:1", "512:0:0:0:4:{f}:2", "1024:0:0:0:2:{f}:2",
                "512:0:0:0:2:{f}:3", "256:0:0:0:8:{f}:2"]
    bwd_cfgs = ["128:0:0:0:8:{f}:1", "256:0:0:0:4:{f}:1", "512:0:0:0:2:{f}:2", "1024:0:0:0:2:{f}:2",
                "256:0:0:0:2:{f}:3", "512:0:0:0:4:{f}:2"]
    for M, N in [(150, 65536), (301, 40960), (149, 40008), (200, 32768 + 8)]:
        x = (3.0 * torch.randn(M, N, device=DEV)).to(dtype)
        x[1, 100:] = float("-inf")
        dy = torch.randn(M, N, device=DEV).to(dtype)
        ref = oracle.softmax_ref(x.cpu().float())
        y0 = sm.softmax_fwd(x)
        dx_ref = oracle.softmax_bwd_ref(dy.cpu().float(), y0.cpu().float())
        ran = 0
        for c in fwd_cfgs:
            monkeypatch.setenv("QUACK_B200_CFG", "softmax_fwd:" + c.format(f=flag))
            y = torch.full_like(x, float("nan"))
            try:
                sm._softmax_fwd(x, y)
            except ValueError:
                continue  # the geometry cannot hold this row (more than 16 CTAs)
            finally:
                monkeypatch.delenv("QUACK_B200_CFG")
            if "softmax_cluster_kernel" not in _C.last_kernel():
                continue  # fell through to another kernel: capacity
            ran += 1
            assert_close_to_oracle(y, ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], what=f"y {c} {M}x{N}")
            assert (y[1, 100:] == 0).all()
        for c in bwd_cfgs:
            monkeypatch.setenv("QUACK_B200_CFG", "softmax_bwd:" + c.format(f=flag))
            dx = torch.full_like(x, float("nan"))
            dx2 = torch.full_like(x, float("nan"))
            try:
                sm._softmax_backward(dy, y0, dx)
                sm._softmax_backward(dy, y0, dx2)
            except ValueError:
                continue
            finally:
                monkeypatch.delenv("QUACK_B200_CFG")
            if "softmax_cluster_kernel" not in _C.last_kernel():
                continue
            ran += 1
            assert_close_to_oracle(dx, dx_ref, dtype, atol=TOL[dtype], rtol=TOL[dtype], max_ulp=None,
                                   what=f"dx {c} {M}x{N}")
            assert torch.equal(dx, dx2)
        assert ran >= 4, f"the cluster kernel did not serve {M}x{N} {dtype}"
    # the default backward for long rows is this kernel; no wait may have timed out
    dx = sm.softmax_bwd(dy, y0)
    assert "softmax_cluster_kernel" in _C.last_kernel()
    assert _C.ring_timeouts() == 0
