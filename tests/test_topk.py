"""Top-k (+ softmax) forward / backward: the CPU oracle against the torch.topk fixtures (CPU), and
the CUDA kernels against the oracle (GPU), after the reference's tests/test_topk.py."""

import importlib

import pytest
import torch

import oracle
from conftest import GOLDEN

DEV = "cuda"
TOL = {torch.bfloat16: (1e-2, 1e-2), torch.float16: (1e-3, 1e-3), torch.float32: (1e-6, 1e-6)}


@pytest.fixture(scope="module")
def topk_golden():
    return torch.load(GOLDEN / "topk_golden.pt", weights_only=True)


def test_topk_oracle_matches_torch_fixtures(topk_golden):
    for c in topk_golden["topk"]:
        vals, idx = oracle.topk_ref(c["x"], c["k"], c["softmax"])
        assert vals.dtype == c["values"].dtype and idx.dtype == torch.int32
        atol, rtol = TOL[vals.dtype]
        torch.testing.assert_close(vals, c["values"], atol=atol if c["softmax"] else 0, rtol=rtol if c["softmax"] else 0)
        # equal values may be listed in another order by torch.topk: compare the gathered values
        assert torch.equal(torch.gather(c["x"], 1, idx.long()), torch.gather(c["x"], 1, c["indices"].long()))
        dx = oracle.topk_bwd_ref(c["dvalues"], c["values"], c["indices"], c["x"].shape[1], c["softmax"])
        torch.testing.assert_close(dx.to(c["dx"].dtype), c["dx"], atol=atol, rtol=rtol)


def test_topk_oracle_ties_prefer_the_smaller_column():
    x = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0, 0.0, 2.0, 1.0]])
    vals, idx = oracle.topk_ref(x, 4)
    assert vals.tolist() == [[3.0, 3.0, 3.0, 2.0]] and idx.tolist() == [[1, 2, 4, 3]]


# ------------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------------
def _topk_mod():
    return importlib.import_module("quack_flydsl_b200.topk")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N,k", [(64, 16), (128, 32), (256, 16), (512, 32), (1024, 32), (4096, 32),
                                 (4096, 64), (4096, 128), (2048, 64), (32, 1), (8, 8), (4096, 1), (2048, 4)])
@pytest.mark.parametrize("M", [1, 37, 199])
@pytest.mark.parametrize("softmax", [False, True])
def test_topk_matches_oracle(M, N, k, dtype, softmax):
    tk = _topk_mod()
    x = torch.randn(M, N, device=DEV).to(dtype).requires_grad_()
    vals, idx = tk.topk(x, k, softmax=softmax)
    assert vals.shape == (M, k) and vals.dtype == dtype and idx.dtype == torch.int32
    ref_vals, ref_idx = oracle.topk_ref(x.detach().cpu(), k, softmax)
    # indices are exact, ties included (smaller column first)
    assert torch.equal(idx.cpu(), ref_idx)
    if softmax:
        atol, rtol = TOL[dtype]
        torch.testing.assert_close(vals.detach().cpu(), ref_vals, atol=atol, rtol=rtol)
        s = vals.detach().float().sum(-1)
        torch.testing.assert_close(s, torch.ones_like(s), atol=1e-2, rtol=0)
    else:
        assert torch.equal(vals.detach().cpu(), ref_vals)  # selected values are copied, not recomputed
        assert (vals[:, :-1] >= vals[:, 1:]).all()
    dvalues = torch.randn(M, k, device=DEV).to(dtype)
    vals.backward(dvalues)
    dx_ref = oracle.topk_bwd_ref(dvalues.cpu(), vals.detach().cpu(), idx.cpu(), N, softmax)
    atol, rtol = TOL[dtype]
    torch.testing.assert_close(x.grad.float().cpu(), dx_ref, atol=max(atol, 1e-6), rtol=rtol)
    # everything outside the k columns is exactly zero
    mask = torch.ones(M, N, dtype=torch.bool)
    mask.scatter_(1, idx.cpu().long(), False)
    assert (x.grad.cpu()[mask] == 0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_topk_ties_and_special_values(dtype):
    tk = _topk_mod()
    # many equal values: exact agreement with the stable-sort oracle, indices included
    x = torch.randint(-3, 4, (64, 1024), device=DEV).to(dtype)
    x[0, :] = 1.0
    x[1, ::2] = float("-inf")
    x[2, 5] = float("inf")
    for k in (1, 16, 128):
        vals, idx = tk.topk_fwd(x, k)
        rv, ri = oracle.topk_ref(x.cpu(), k)
        assert torch.equal(vals.cpu(), rv) and torch.equal(idx.cpu(), ri)
    # negative zero sorts below positive zero; both are zeros to a comparison on values
    z = torch.zeros(2, 64, device=DEV, dtype=dtype)
    z[0, 10] = -0.0
    vals, idx = tk.topk_fwd(z, 8)
    assert (vals == 0).all()


@pytest.mark.gpu
def test_topk_golden_fixtures(topk_golden):
    tk = _topk_mod()
    for c in topk_golden["topk"]:
        x = c["x"].to(DEV)
        vals, idx = tk.topk_fwd(x, c["k"], softmax=c["softmax"])
        atol, rtol = TOL[x.dtype]
        torch.testing.assert_close(vals.cpu(), c["values"], atol=atol if c["softmax"] else 0,
                                   rtol=rtol if c["softmax"] else 0)
        assert torch.equal(torch.gather(c["x"], 1, idx.cpu().long()), torch.gather(c["x"], 1, c["indices"].long()))
        dx = tk.topk_bwd(c["dvalues"].to(DEV), c["values"].to(DEV) if c["softmax"] else None,
                         c["indices"].to(DEV), x.shape[1], softmax=c["softmax"])
        torch.testing.assert_close(dx.cpu(), c["dx"], atol=max(atol, 1e-6), rtol=rtol)


@pytest.mark.gpu
def test_topk_strided_rows_compile_and_errors():
    tk = _topk_mod()
    base = torch.randn(50, 1024 + 64, device=DEV).to(torch.bfloat16)
    x = base[:, :1024]  # row stride 1088 elements
    vals, idx = tk.topk_fwd(x, 32)
    rv, ri = oracle.topk_ref(x.cpu(), 32)
    assert torch.equal(vals.cpu(), rv) and torch.equal(idx.cpu(), ri)
    fn = torch.compile(tk.topk, fullgraph=True)
    xg = torch.randn(9, 512, device=DEV, requires_grad=True)
    v, i = fn(xg, 16, softmax=True)
    v.sum().backward()
    assert xg.grad is not None and torch.isfinite(xg.grad).all()
    with pytest.raises(AssertionError):
        tk.topk_fwd(torch.randn(4, 100, device=DEV), 4)  # N not a power of two
    with pytest.raises(AssertionError):
        tk.topk_fwd(torch.randn(4, 8192, device=DEV), 4)  # N > 4096
    # empty batch: no launch
    v, i = tk.topk_fwd(torch.empty(0, 4096, device=DEV, dtype=torch.bfloat16), 8)
    assert v.shape == (0, 8) and i.shape == (0, 8)
    dx = tk.topk_bwd(torch.empty(0, 8, device=DEV, dtype=torch.bfloat16), None,
                     torch.empty(0, 8, device=DEV, dtype=torch.int32), N=4096)
    assert dx.shape == (0, 4096)
