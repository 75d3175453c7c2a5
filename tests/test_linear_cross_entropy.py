"""GPU parity tests of the chunked linear + cross-entropy path and of rms_final_reduce against
the CPU oracle, after the reference's tests/test_linear_cross_entropy.py and
tests/test_linear.py:790-803."""

import importlib

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

lce = importlib.import_module("quack_flydsl_b200.linear_cross_entropy")
rfr = importlib.import_module("quack_flydsl_b200.rms_final_reduce")
DEV = "cuda"


def _check_against_oracle(x, weight, target, loss, ignore_index, reduction):
    """The reference's criterion (tests/test_linear_cross_entropy.py:41-48): the error against an
    exact evaluation may be at most a small multiple of the error of the same computation done
    by PyTorch in the input precision."""
    loss_ref, dx_ref, dw_ref = oracle.linear_cross_entropy_ref(
        x.detach().cpu(), weight.detach().cpu(), target.cpu(), ignore_index=ignore_index,
        reduction=reduction)
    x_pt = x.detach().clone().requires_grad_()
    w_pt = weight.detach().clone().requires_grad_()
    loss_pt = lce.linear_cross_entropy_func_ref(x_pt, w_pt, None, target, ignore_index=ignore_index,
                                                reduction=reduction)
    loss_pt.backward()
    err = lambda a, b: (a.detach().double().cpu() - b.double()).abs().max().item()  # noqa: E731
    assert err(loss, loss_ref) < 3 * err(loss_pt, loss_ref) + 1e-5
    assert err(x.grad, dx_ref) < 2 * err(x_pt.grad, dx_ref) + 1e-4
    assert err(weight.grad, dw_ref) < 2 * err(w_pt.grad, dw_ref) + 1e-4


@pytest.mark.parametrize("reduction", ["mean", "sum"])
@pytest.mark.parametrize("V", [32000, 50264, 128256])
@pytest.mark.parametrize("d", [768, 1024])
@pytest.mark.parametrize("B_L", [8, 16, 24])
def test_chunked_linear_cross_entropy(B_L, d, V, reduction):
    x = (torch.randn(B_L, d, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    weight = (torch.randn(V, d, device=DEV, dtype=torch.bfloat16) / d ** 0.5).requires_grad_()
    target = torch.randint(0, V, (B_L,), device=DEV, dtype=torch.int64)
    loss = lce.chunked_linear_cross_entropy(x, weight, target, chunk_size=16, reduction=reduction,
                                            tuned=False)
    loss.backward()
    _check_against_oracle(x, weight, target, loss, -100, reduction)


@pytest.mark.parametrize("reduction", ["mean", "sum"])
@pytest.mark.parametrize("chunk_size", [256, 1024])
def test_chunked_linear_cross_entropy_ignore_index(reduction, chunk_size):
    B_L, d, V = 1024, 512, 2048
    ignore_index = V - 1
    x = (torch.randn(B_L, d, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    weight = (torch.randn(V, d, device=DEV, dtype=torch.bfloat16) / d ** 0.5).requires_grad_()
    target = torch.randint(0, V, (B_L,), device=DEV, dtype=torch.int64)
    target[torch.rand(B_L, device=DEV) < 0.2] = ignore_index
    loss = lce.chunked_linear_cross_entropy(x, weight, target, chunk_size=chunk_size,
                                            ignore_index=ignore_index, reduction=reduction, tuned=False)
    loss.backward()
    _check_against_oracle(x, weight, target, loss, ignore_index, reduction)


def test_chunked_linear_cross_entropy_vocabulary_rows_single_launch_path():
    """Chunks with at least as many rows as SMs and a 32K vocabulary take the single-launch
    loss + dx kernel inside the chunk loop (three chunks, the last one ragged)."""
    B_L, d, V, chunk = 640, 256, 32768, 256
    x = (torch.randn(B_L, d, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    weight = (torch.randn(V, d, device=DEV, dtype=torch.bfloat16) / d ** 0.5).requires_grad_()
    target = torch.randint(0, V, (B_L,), device=DEV, dtype=torch.int64)
    target[::7] = -100
    loss = lce.chunked_linear_cross_entropy(x, weight, target, chunk_size=chunk, reduction="mean")
    loss.backward()
    _check_against_oracle(x, weight, target, loss, -100, "mean")


def test_chunked_linear_cross_entropy_golden_fixtures(linear_ce_golden):
    for c in linear_ce_golden["linear_cross_entropy"]:
        x = c["x"].detach().to(DEV).requires_grad_()
        w = c["weight"].detach().to(DEV).requires_grad_()
        t = c["target"].to(DEV)
        loss = lce.chunked_linear_cross_entropy(x, w, t, chunk_size=8, ignore_index=c["ignore_index"],
                                                reduction=c["reduction"])
        loss.backward()
        tol = 2e-2 if x.dtype == torch.bfloat16 else 1e-4
        torch.testing.assert_close(loss.float().cpu(), c["loss"], atol=tol, rtol=tol)
        torch.testing.assert_close(x.grad.float().cpu(), c["dx"], atol=tol, rtol=tol)
        torch.testing.assert_close(w.grad.float().cpu(), c["dw"], atol=tol, rtol=tol)


def test_chunked_linear_cross_entropy_rejects_bad_reduction():
    x = torch.randn(8, 64, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(128, 64, device=DEV, dtype=torch.bfloat16)
    t = torch.randint(0, 128, (8,), device=DEV)
    with pytest.raises(ValueError, match="Invalid reduction"):
        lce.chunked_linear_cross_entropy(x, w, t, reduction="none")


@pytest.mark.parametrize("chunk_size", [None, 64])
def test_linear_cross_entropy_module(chunk_size):
    torch.manual_seed(0)
    mod = lce.LinearCrossEntropy(256, 1024, bias=False, chunk_size=chunk_size, device=DEV,
                                 dtype=torch.bfloat16)
    x = (torch.randn(4, 32, 256, device=DEV, dtype=torch.bfloat16) * 0.1).requires_grad_()
    target = torch.randint(0, 1024, (4, 32), device=DEV)
    loss = mod(x, target.reshape(-1) if chunk_size is None else target)
    loss.backward()
    loss_ref, dx_ref, dw_ref = oracle.linear_cross_entropy_ref(
        x.detach().reshape(-1, 256).cpu(), mod.weight.detach().cpu(), target.reshape(-1).cpu())
    torch.testing.assert_close(loss.double().cpu(), loss_ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(x.grad.reshape(-1, 256).double().cpu(), dx_ref, atol=2e-3, rtol=5e-2)
    torch.testing.assert_close(mod.weight.grad.double().cpu(), dw_ref, atol=2e-3, rtol=5e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [1, 4, 8, 16, 64, 128, 100, 2051])
@pytest.mark.parametrize("M", [1, 37, 960, 1920])
def test_rms_final_reduce(M, N, dtype):
    scale, eps = 1.0 / 4096, 1e-6
    x = torch.randn((M, N), device=DEV, dtype=dtype).abs()  # partial sums are non-negative
    rstd = rfr.rms_final_reduce(x, scale=scale, eps=eps)
    ref = oracle.rms_final_reduce_ref(x.cpu(), scale, eps)
    assert rstd.dtype == torch.float32 and rstd.shape == (M,)
    torch.testing.assert_close(rstd.cpu(), ref, atol=1e-5, rtol=1e-5)


def test_rms_final_reduce_strided_rows_empty_and_fixtures(linear_ce_golden):
    base = torch.rand(50, 40, device=DEV)
    x = base[:, :24]
    torch.testing.assert_close(rfr.rms_final_reduce(x, 0.5).cpu(),
                               oracle.rms_final_reduce_ref(x.cpu(), 0.5), atol=1e-5, rtol=1e-5)
    assert rfr.rms_final_reduce(torch.empty(0, 8, device=DEV), 1.0).shape == (0,)
    for c in linear_ce_golden["rms_final_reduce"]:
        got = rfr.rms_final_reduce(c["x"].to(DEV), c["scale"], c["eps"])
        torch.testing.assert_close(got.cpu(), c["rstd"], atol=1e-5, rtol=1e-5)
