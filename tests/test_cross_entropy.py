"""GPU parity tests of cross-entropy forward / backward against the CPU oracle, after the
reference's tests/test_cross_entropy.py: class weights, ignore_index, lse_partial mode, fused dx,
in-place backward, reductions, stride-0 dloss; fp32 loss / lse are held to rtol 1e-5."""

import importlib
import math

import pytest
import torch

import oracle
from _util import assert_close_to_oracle

pytestmark = pytest.mark.gpu

ce = importlib.import_module("quack_flydsl_b200.cross_entropy")
DEV = "cuda"
ATOL, RTOL = 5e-5, 1e-5


def _dx_tol(dtype):
    return {torch.float32: (ATOL, RTOL), torch.float16: (1e-3, 2e-3), torch.bfloat16: (1e-2, 1.6e-2)}[dtype]


@pytest.mark.parametrize("has_weight", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [192, 668, 1024, 1128, 4096, 32768, 128256, 262144])
@pytest.mark.parametrize("M", [1, 289])
def test_cross_entropy(M, N, dtype, has_weight):
    x = (0.1 * torch.randn(M, N, device=DEV)).to(dtype).requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV, dtype=torch.int64)
    weight = (torch.rand(N, device=DEV) + 0.1) if has_weight else None
    wc = None if weight is None else weight.cpu()
    for masked in (False, True):
        t = target.clone()
        if masked:
            mask = torch.rand(M, device=DEV) < 0.3
            t[mask] = -100
        xi = x.detach().clone().requires_grad_()
        loss = ce.cross_entropy(xi, t, weight=weight, reduction="none", ignore_index=-100)
        dloss = torch.randn_like(loss)
        (dx,) = torch.autograd.grad(loss, xi, grad_outputs=dloss)
        assert loss.shape == (M,) and loss.dtype == torch.float32 and dx.shape == x.shape
        loss_ref, lse_ref = oracle.cross_entropy_ref(xi.detach().cpu(), t.cpu(), weight=wc)
        torch.testing.assert_close(loss.detach().cpu(), loss_ref, atol=ATOL, rtol=RTOL)
        assert (loss >= 0).all() and torch.isfinite(loss).all()
        if masked:
            assert (loss[mask] == 0).all(), "loss must be exactly 0 for ignored rows"
            assert (dx[mask] == 0).all(), "gradient rows must be exactly 0 for ignored rows"
        dx_ref = oracle.cross_entropy_bwd_ref(xi.detach().cpu().float(), t.cpu(), dloss.cpu(), lse_ref, weight=wc)
        at, rt = _dx_tol(dtype)
        assert_close_to_oracle(dx, dx_ref, dtype, atol=at, rtol=rt, max_ulp=None, what="dx")


def test_cross_entropy_config_shape_fp32_outputs():
    """Benchmark shape family (bf16 logits = 2 * N(0,1), N = 128256, int64 targets, 5 %
    ignored, mean reduction) on a row slice the CPU oracle handles; loss and lse to rtol 1e-5."""
    M = 512
    d = oracle.make_config_inputs("c5", rows=M, device=DEV)
    x, t = d["x"].requires_grad_(), d["target"]
    loss_rows, lse = ce.cross_entropy_fwd(x.detach(), t, return_lse=True)
    loss_ref, lse_ref = oracle.cross_entropy_ref(x.detach().cpu(), t.cpu())
    torch.testing.assert_close(lse.cpu(), lse_ref, atol=0, rtol=1e-5)
    torch.testing.assert_close(loss_rows.cpu(), loss_ref, atol=1e-6, rtol=1e-5)
    loss = ce.cross_entropy(x, t, reduction="mean")
    loss.backward()
    n_valid = int((t != -100).sum())
    torch.testing.assert_close(loss.detach().cpu(), loss_ref.sum() / n_valid, atol=0, rtol=1e-5)
    dloss = torch.full((M,), 1.0 / n_valid)
    dx_ref = oracle.cross_entropy_bwd_ref(x.detach().cpu().float(), t.cpu(), dloss, lse_ref)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, what="dlogits")
    assert (x.grad[t == -100] == 0).all()


def test_cross_entropy_lse_partial():
    # reference: tests/test_cross_entropy.py:91-124
    M, N = 1024, 128256
    x = (0.1 * torch.randn(M, N, device=DEV)).bfloat16().requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV)
    with torch.no_grad():
        lse_partial = x.view(M, N // 128, 128).float().logsumexp(dim=-1)
    loss = ce.cross_entropy(x, target, lse_partial=lse_partial, reduction="none")
    dloss = torch.randn_like(loss)
    (dx,) = torch.autograd.grad(loss, x, grad_outputs=dloss)
    loss_ref, lse_ref = oracle.cross_entropy_ref(x.detach().cpu(), target.cpu())
    torch.testing.assert_close(loss.detach().cpu(), loss_ref, atol=ATOL, rtol=RTOL)
    dx_ref = oracle.cross_entropy_bwd_ref(x.detach().cpu().float(), target.cpu(), dloss.cpu(), lse_ref)
    assert_close_to_oracle(dx, dx_ref, torch.bfloat16, atol=1e-2, rtol=1.6e-2, max_ulp=None, what="dx")


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_cross_entropy_extreme_values(dtype):
    M, N = 16, 1024
    target = torch.randint(0, N, (M,), device=DEV)
    want = torch.full((M,), math.log(N), device=DEV)
    for v in (10.0, -10.0):
        loss = ce.cross_entropy_fwd(torch.full((M, N), v, device=DEV, dtype=dtype), target)
        torch.testing.assert_close(loss, want, atol=1e-5, rtol=1e-5)
    x = torch.full((M, N), -10.0, device=DEV, dtype=dtype)
    x[torch.arange(M), target] = 10.0
    assert (ce.cross_entropy_fwd(x, target) < 1.0).all()


def test_cross_entropy_numerical_stability_and_edge_targets():
    M, N = 8, 512
    x = torch.randn(M, N, device=DEV)
    target = torch.randint(0, N, (M,), device=DEV)
    torch.testing.assert_close(ce.cross_entropy_fwd(x, target), ce.cross_entropy_fwd(x + 100.0, target),
                               atol=1e-5, rtol=1e-5)
    for t in (torch.zeros(M, dtype=torch.int64), torch.full((M,), N - 1)):
        loss = ce.cross_entropy_fwd(x, t.to(DEV))
        torch.testing.assert_close(loss.cpu(), oracle.cross_entropy_ref(x.cpu(), t)[0], atol=1e-5, rtol=1e-5)
    # int32 targets
    loss32 = ce.cross_entropy_fwd(x, target.int())
    assert torch.equal(loss32, ce.cross_entropy_fwd(x, target))


def test_cross_entropy_ignore_index_edge_cases():
    M, N = 16, 1024
    x = 0.1 * torch.randn(M, N, device=DEV)
    loss = ce.cross_entropy_fwd(x, torch.zeros(M, device=DEV, dtype=torch.int64), ignore_index=0)
    assert (loss == 0).all()
    t = torch.randint(0, N, (M,), device=DEV)
    loss = ce.cross_entropy_fwd(x, t, ignore_index=-1)
    torch.testing.assert_close(loss.cpu(), oracle.cross_entropy_ref(x.cpu(), t.cpu(), ignore_index=-1)[0],
                               atol=1e-5, rtol=1e-5)
    # lse is still produced for ignored rows
    t[0] = -100
    loss, lse = ce.cross_entropy_fwd(x, t, return_lse=True)
    assert loss[0] == 0
    torch.testing.assert_close(lse.cpu(), oracle.cross_entropy_ref(x.cpu(), t.cpu())[1], atol=0, rtol=1e-5)


@pytest.mark.parametrize("inplace_backward", [False, True])
@pytest.mark.parametrize("has_weight", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [192, 1024, 32768, 128256])
@pytest.mark.parametrize("M", [1, 77])
def test_cross_entropy_fwd_with_grad(M, N, dtype, has_weight, inplace_backward):
    # reference: tests/test_cross_entropy.py:230-314 (fused dx; identity of the in-place buffer)
    x = (0.1 * torch.randn(M, N, device=DEV)).to(dtype)
    target = torch.randint(0, N, (M,), device=DEV)
    target[torch.rand(M, device=DEV) < 0.2] = -100
    weight = (torch.rand(N, device=DEV) + 0.1) if has_weight else None
    x_copy = x.clone()
    x_cpu = x.cpu()
    loss, lse, dx = ce.cross_entropy_fwd(x_copy, target, weight=weight, return_lse=True, return_dx=True,
                                         inplace_backward=inplace_backward)
    assert (dx is x_copy) == inplace_backward
    wc = None if weight is None else weight.cpu()
    loss_ref, lse_ref = oracle.cross_entropy_ref(x_cpu, target.cpu(), weight=wc)
    torch.testing.assert_close(loss.cpu(), loss_ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(lse.cpu(), lse_ref, atol=ATOL, rtol=RTOL)
    dx_ref = oracle.cross_entropy_bwd_ref(x_cpu.float(), target.cpu(), torch.ones(M), lse_ref, weight=wc)
    at, rt = _dx_tol(dtype)
    assert_close_to_oracle(dx, dx_ref, dtype, atol=at, rtol=rt, max_ulp=None, what="dx")
    assert (dx[target == -100] == 0).all()
    # loss-only call with return_dx and no lse request
    loss2, dx2 = ce.cross_entropy_fwd(x.clone(), target, weight=weight, return_dx=True)
    assert torch.equal(loss2, loss) and torch.equal(dx2, dx)


def test_cross_entropy_inplace_backward_autograd():
    M, N = 77, 4096
    x = (0.1 * torch.randn(M, N, device=DEV)).bfloat16().requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV)
    x_ref = x.detach().cpu().clone()
    loss = ce.cross_entropy(x, target, reduction="sum", inplace_backward=True)
    loss.backward()
    # the backward kernel overwrote the logits with the gradient (autograd may hand out a copy of
    # the returned tensor as .grad, so compare contents, not identity)
    assert torch.equal(x.detach(), x.grad)
    _, lse_ref = oracle.cross_entropy_ref(x_ref, target.cpu())
    dx_ref = oracle.cross_entropy_bwd_ref(x_ref.float(), target.cpu(), torch.ones(M), lse_ref)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, atol=1e-2, rtol=1.6e-2, max_ulp=None, what="dx")


@pytest.mark.parametrize("reduction", ["none", "mean", "sum"])
@pytest.mark.parametrize("has_weight", [False, True])
def test_cross_entropy_reductions(reduction, has_weight):
    # reference: tests/test_cross_entropy.py:337-368
    M, N = 289, 1024
    x = torch.randn(M, N, device=DEV).requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV)
    target[::7] = -100
    weight = (torch.rand(N, device=DEV) + 0.1) if has_weight else None
    got = ce.cross_entropy(x, target, weight=weight, reduction=reduction)
    loss_ref, _ = oracle.cross_entropy_ref(x.detach().cpu(), target.cpu(), weight=None if weight is None else weight.cpu())
    valid = (target != -100).cpu()
    if reduction == "none":
        want = loss_ref
    elif reduction == "sum":
        want = loss_ref.sum()
    elif has_weight:
        want = loss_ref.sum() / weight.cpu()[target.cpu().clamp(min=0)][valid].sum()
    else:
        want = loss_ref.sum() / valid.sum()
    torch.testing.assert_close(got.detach().cpu(), want, atol=1e-4, rtol=1e-5)
    with pytest.raises(ValueError, match="Invalid reduction mode"):
        ce.cross_entropy(x, target, reduction="max")


def test_cross_entropy_stride0_dloss():
    # reference: tests/test_cross_entropy.py:371-387: loss.sum().backward() hands an expanded scalar
    M, N = 64, 2048
    x = torch.randn(M, N, device=DEV).requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV)
    lse = torch.logsumexp(x.detach(), -1)
    dloss = torch.tensor(0.5, device=DEV).expand(M)
    assert dloss.stride(0) == 0
    dx = ce.cross_entropy_bwd(x.detach(), target, dloss, lse)
    dx_ref = oracle.cross_entropy_bwd_ref(x.detach().cpu(), target.cpu(), torch.full((M,), 0.5), lse.cpu())
    torch.testing.assert_close(dx.cpu(), dx_ref, atol=ATOL, rtol=1e-4)


def test_cross_entropy_golden_fixtures(softmax_ce_golden):
    for c in softmax_ce_golden["cross_entropy"]:
        x, t = c["x"].to(DEV), c["target"].to(DEV)
        w = None if c["weight"] is None else c["weight"].to(DEV)
        loss, lse = ce.cross_entropy_fwd(x, t, weight=w, return_lse=True)
        torch.testing.assert_close(loss.cpu(), c["loss"], atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse.cpu(), c["lse"], atol=ATOL, rtol=RTOL)
        dx = ce.cross_entropy_bwd(x, t, c["dloss"].to(DEV), lse, weight=w)
        at, rt = _dx_tol(x.dtype)
        assert_close_to_oracle(dx, c["dx"].float(), x.dtype, atol=at, rtol=rt, max_ulp=None, what="dx")


def test_cross_entropy_empty():
    x = torch.empty(0, 1024, device=DEV, dtype=torch.bfloat16)
    t = torch.empty(0, device=DEV, dtype=torch.int64)
    loss, lse, dx = ce.cross_entropy_fwd(x, t, return_lse=True, return_dx=True)
    assert loss.shape == (0,) and lse.shape == (0,) and dx.shape == (0, 1024)
    assert ce.cross_entropy_bwd(x, t, loss, lse).shape == (0, 1024)


def test_cross_entropy_torch_compile_fullgraph():
    torch._dynamo.reset()
    M, N = 289, 4096
    x = (0.1 * torch.randn(M, N, device=DEV)).bfloat16().requires_grad_()
    target = torch.randint(0, N, (M,), device=DEV)
    target[::5] = -100
    fn = torch.compile(ce.cross_entropy, fullgraph=True)
    loss = fn(x, target, reduction="none", inplace_backward=True)  # compiled: out-of-place gradient
    dloss = torch.randn_like(loss)
    (dx,) = torch.autograd.grad(loss, x, grad_outputs=dloss)
    loss_ref, lse_ref = oracle.cross_entropy_ref(x.detach().cpu(), target.cpu())
    torch.testing.assert_close(loss.detach().cpu(), loss_ref, atol=ATOL, rtol=RTOL)
    dx_ref = oracle.cross_entropy_bwd_ref(x.detach().cpu().float(), target.cpu(), dloss.cpu(), lse_ref)
    assert_close_to_oracle(dx, dx_ref, torch.bfloat16, atol=1e-2, rtol=1.6e-2, max_ulp=None, what="dx")


@pytest.mark.parametrize("inplace_backward", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [32768, 40008, 128256])
def test_cross_entropy_fwd_with_grad_single_launch(N, dtype, inplace_backward, monkeypatch):
    """With at least as many rows as SMs and vocabulary-sized rows, loss + lse + dx come from one
    launch that streams every row twice.  It must agree with the oracle and with the two-kernel
    path (flag bit 1), with class weights, ignored rows and the in-place gradient buffer."""
    M = 300
    x = (2.0 * torch.randn(M, N, device=DEV)).to(dtype)
    target = torch.randint(0, N, (M,), device=DEV)
    target[torch.rand(M, device=DEV) < 0.2] = -100
    target[0], target[1] = 0, N - 1  # first and last column carry the one-hot term
    weight = torch.rand(N, device=DEV) + 0.1
    x_cpu = x.cpu()
    x_work = x.clone()
    loss, lse, dx = ce.cross_entropy_fwd(x_work, target, weight=weight, return_lse=True, return_dx=True,
                                         inplace_backward=inplace_backward)
    assert (dx is x_work) == inplace_backward
    monkeypatch.setenv("QUACK_B200_CFG", "ce_fwd:0:0:0:0:0:2")
    loss2, lse2, dx2 = ce.cross_entropy_fwd(x.clone(), target, weight=weight, return_lse=True, return_dx=True)
    monkeypatch.delenv("QUACK_B200_CFG")
    loss_ref, lse_ref = oracle.cross_entropy_ref(x_cpu, target.cpu(), weight=weight.cpu())
    for l, s in ((loss, lse), (loss2, lse2)):
        torch.testing.assert_close(l.cpu(), loss_ref, atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(s.cpu(), lse_ref, atol=ATOL, rtol=RTOL)
    dx_ref = oracle.cross_entropy_bwd_ref(x_cpu.float(), target.cpu(), torch.ones(M), lse_ref, weight=weight.cpu())
    at, rt = _dx_tol(dtype)
    for d in (dx, dx2):
        assert_close_to_oracle(d, dx_ref, dtype, atol=at, rtol=rt, max_ulp=None, what="dx")
        assert (d[target == -100] == 0).all()
    # explicit CTA sizes of the single-launch kernel
    for threads in (256, 512, 1024):
        monkeypatch.setenv("QUACK_B200_CFG", f"ce_fwd:{threads}")
        l3, s3, d3 = ce.cross_entropy_fwd(x.clone(), target, weight=weight, return_lse=True, return_dx=True)
        monkeypatch.delenv("QUACK_B200_CFG")
        torch.testing.assert_close(s3.cpu(), lse_ref, atol=ATOL, rtol=RTOL)
        assert_close_to_oracle(d3, dx_ref, dtype, atol=at, rtol=rt, max_ulp=None, what="dx")
