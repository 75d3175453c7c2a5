"""qb_norm_bwd_static: norm backward with the partial-sum workspace inside the library.

Collected last on purpose (file name): the entry point shares one device array between all its
calls, so it is exercised both in a fresh process (this file alone) and after every other test has
used the GPU.  Everything goes through the C ABI with raw pointers; the expected values come from
the stock entry points (qb_norm_bwd + qb_colsum) on the same inputs.
"""

from ctypes import byref

import pytest
import torch

import oracle
from quack_flydsl_b200 import _C

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = (16 << 20) // 4
MIN_PARTIALS = 64


def _fill_bwd(a, x, w, dout, rstd, mean, dx, is_layernorm):
    M, N = x.shape
    a.x, a.weight, a.dout, a.rstd, a.mean = (_C.ptr(x), _C.ptr(w), _C.ptr(dout), _C.ptr(rstd),
                                             _C.ptr(mean))
    a.dx = _C.ptr(dx)
    a.M, a.H, a.N = M, 1, N
    a.x_row_stride = a.dout_row_stride = a.dx_row_stride = N
    a.x_dtype = a.dout_dtype = a.dx_dtype = _C.float_code(x)
    a.weight_dtype = _C.float_code(w)
    a.is_layernorm = int(is_layernorm)


def _stock(x, w, dout, rstd, mean, is_layernorm, want_db):
    """dx, dw, db from the existing entry points with a torch-allocated workspace."""
    M, N = x.shape
    lib = _C.lib()
    stream = _C.stream_of(x)
    P = lib.qb_norm_bwd_num_partials(N, _C.float_code(x), int(is_layernorm), -1)
    assert P > 0
    dx = torch.empty_like(x)
    dwp = torch.empty(P, N, device=x.device, dtype=torch.float32)
    dbp = torch.empty(P, N, device=x.device, dtype=torch.float32) if want_db else None
    a = _C.NormBwdArgs()
    _fill_bwd(a, x, w, dout, rstd, mean, dx, is_layernorm)
    a.dw_partial, a.db_partial, a.num_partials = _C.ptr(dwp), _C.ptr(dbp), P
    _C.check(lib.qb_norm_bwd(byref(a), stream), "qb_norm_bwd")
    outs = []
    for part in (dwp, dbp):
        if part is None:
            outs.append(None)
            continue
        out = torch.empty(N, device=x.device, dtype=w.dtype)
        c = _C.ColsumArgs()
        c.partial, c.out, c.out_f32 = _C.ptr(part), _C.ptr(out), None
        c.P, c.cols, c.out_dtype = P, N, _C.float_code(out)
        _C.check(lib.qb_colsum(byref(c), stream), "qb_colsum")
        outs.append(out)
    return dx, outs[0], outs[1]


def _static(x, w, dout, rstd, mean, is_layernorm, want_db):
    N = x.shape[1]
    dx = torch.empty_like(x)
    dw = torch.empty(N, device=x.device, dtype=w.dtype)
    db = torch.empty(N, device=x.device, dtype=w.dtype) if want_db else None
    s = _C.NormBwdStaticArgs()
    _fill_bwd(s.bwd, x, w, dout, rstd, mean, dx, is_layernorm)
    s.dw, s.db, s.param_dtype = _C.ptr(dw), _C.ptr(db), _C.float_code(w)
    rc = _C.lib().qb_norm_bwd_static(byref(s), _C.stream_of(x))
    return rc, dx, dw, db


def _inputs(M, N, dtype, is_layernorm, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, N, device="cuda", dtype=torch.float32, generator=g).to(dtype)
    dout = torch.randn(M, N, device="cuda", dtype=torch.float32, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(N, device="cuda", dtype=torch.float32, generator=g))
    xf = x.float()
    if is_layernorm:
        mean = xf.mean(dim=1)
        rstd = torch.rsqrt(xf.var(dim=1, unbiased=False) + 1e-6)
    else:
        mean = None
        rstd = torch.rsqrt(xf.square().mean(dim=1) + 1e-6)
    return x, w, dout, rstd, mean


def _assert_param_grad_close(got, ref, M):
    # Both sides sum fp32 partials in a fixed order but may split rows over a different number of
    # persistent CTAs (the built-in workspace caps it), so allow fp32 re-association of M terms
    # plus one rounding to the parameter dtype.
    eps_out = torch.finfo(ref.dtype).eps
    scale = ref.float().abs().max().clamp_min(1.0)
    tol = float(scale) * (eps_out + 1e-6 * max(1.0, M ** 0.5))
    assert torch.isfinite(got.float()).all()
    assert (got.float() - ref.float()).abs().max().item() <= tol


@pytest.mark.parametrize(
    "M,N,dtype,wdtype,is_layernorm",
    [
        (4096, 4096, torch.bfloat16, torch.bfloat16, False),
        (2000, 8192, torch.bfloat16, torch.float32, False),
        (1024, 4096, torch.bfloat16, torch.float32, True),
        (777, 1000, torch.float32, torch.float32, True),
        (64, 32768, torch.float16, torch.float16, True),
    ],
)
def test_static_workspace_matches_stock_entry_points(M, N, dtype, wdtype, is_layernorm):
    want_db = is_layernorm
    for call in range(2):  # two calls in a row: the second one finds the first one's leftovers
        x, w, dout, rstd, mean = _inputs(M, N, dtype, is_layernorm, seed=100 + call)
        w = w.to(wdtype)
        dx_ref, dw_ref, db_ref = _stock(x, w, dout, rstd, mean, is_layernorm, want_db)
        rc, dx, dw, db = _static(x, w, dout, rstd, mean, is_layernorm, want_db)
        assert rc == 0, _C.lib().qb_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(dx, dx_ref)  # dx does not depend on the workspace at all
        _assert_param_grad_close(dw, dw_ref, M)
        if want_db:
            _assert_param_grad_close(db, db_ref, M)


def test_static_workspace_ignores_stale_contents_of_other_shapes():
    # a large shape first, then a small one whose slices overlap the large one's leftovers
    big = _inputs(512, 16384, torch.bfloat16, True, seed=7)
    rc, *_ = _static(*big[:1], big[1].float(), *big[2:], True, True)
    assert rc == 0
    x, w, dout, rstd, mean = _inputs(300, 512, torch.bfloat16, True, seed=8)
    w = w.float()
    dx_ref, dw_ref, db_ref = _stock(x, w, dout, rstd, mean, True, True)
    rc, dx, dw, db = _static(x, w, dout, rstd, mean, True, True)
    assert rc == 0, _C.lib().qb_last_error().decode()
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref)
    _assert_param_grad_close(dw, dw_ref, 300)
    _assert_param_grad_close(db, db_ref, 300)


def test_static_workspace_does_not_allocate():
    x, w, dout, rstd, mean = _inputs(1024, 2048, torch.bfloat16, False, seed=3)
    w = w.float()
    _static(x, w, dout, rstd, mean, False, False)  # set-up call
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    s = _C.NormBwdStaticArgs()
    _fill_bwd(s.bwd, x, w, dout, rstd, mean, dx, False)
    s.dw, s.db, s.param_dtype = _C.ptr(dw), None, _C.float_code(w)
    torch_before = torch.cuda.memory_allocated()
    for _ in range(3):
        assert _C.lib().qb_norm_bwd_static(byref(s), _C.stream_of(x)) == 0
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == torch_before
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after >= free_before  # no driver-level allocation either


def test_static_workspace_rejects_rows_beyond_its_capacity():
    N = SCRATCH_FLOATS // MIN_PARTIALS  # fits with one gradient buffer, not with two
    x, w, dout, rstd, mean = _inputs(8, N, torch.bfloat16, True, seed=5)
    w = w.float()
    rc, *_ = _static(x, w, dout, rstd, mean, True, True)
    assert rc == -2
    msg = _C.lib().qb_last_error().decode()
    assert "workspace" in msg and "limit" in msg
    rc, dx, dw, _ = _static(x, w, dout, rstd, mean, True, False)
    assert rc == 0, _C.lib().qb_last_error().decode()
    dx_ref, dw_ref, _ = _stock(x, w, dout, rstd, mean, True, False)
    torch.cuda.synchronize()
    assert torch.equal(dx, dx_ref)
    _assert_param_grad_close(dw, dw_ref, 8)


def test_static_workspace_against_the_cpu_oracle():
    """Not only against the stock CUDA entry points: dx, dw and db of the no-allocation entry point
    against the CPU oracle's LayerNorm backward on the same inputs."""
    M, N = 1500, 2048
    x, w, dout, rstd, mean = _inputs(M, N, torch.bfloat16, True, seed=11)
    for call in range(2):
        rc, dx, dw, db = _static(x, w, dout, rstd, mean, True, True)
        assert rc == 0, _C.lib().qb_last_error().decode()
        torch.cuda.synchronize()
        dx_ref, dw_ref, db_ref = oracle.layernorm_bwd_ref(x.cpu(), w.cpu(), dout.cpu(), rstd.cpu(), mean.cpu())
        scale = float(dx_ref.abs().max())
        assert (dx.float().cpu() - dx_ref).abs().max().item() <= 2.0**-7 * scale
        # fp32 parameter gradients: fp32 accumulation over M rows on both sides
        assert (dw.cpu() - dw_ref).abs().max().item() <= 5e-6 * M**0.5 * max(1.0, float(dw_ref.abs().max()))
        assert (db.cpu() - db_ref).abs().max().item() <= 5e-6 * M**0.5 * max(1.0, float(db_ref.abs().max()))


def test_static_workspace_per_head_and_bias_only():
    """H > 1 (one weight row per head: the partial slices are (P, H, N)) and a call that wants db
    but not dw."""
    M, H, N = 333, 4, 256
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(M, H, N, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(M, H, N, device="cuda", generator=g).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(H, N, device="cuda", generator=g)
    rstd = torch.rsqrt(x.float().square().mean(dim=-1) + 1e-6)  # (M, H)

    def call(want_dw, want_db):
        dx = torch.empty_like(x)
        dw = torch.empty(H, N, device="cuda") if want_dw else None
        db = torch.empty(H, N, device="cuda") if want_db else None
        s = _C.NormBwdStaticArgs()
        a = s.bwd
        a.x, a.weight, a.dout, a.rstd, a.dx = _C.ptr(x), _C.ptr(w if want_dw else None), _C.ptr(dout), _C.ptr(rstd), _C.ptr(dx)
        a.M, a.H, a.N = M, H, N
        a.x_row_stride = a.dout_row_stride = a.dx_row_stride = N
        a.x_dtype = a.dout_dtype = a.dx_dtype = _C.float_code(x)
        a.weight_dtype = _C.float_code(w)
        s.dw, s.db, s.param_dtype = _C.ptr(dw), _C.ptr(db), _C.QB_F32
        rc = _C.lib().qb_norm_bwd_static(byref(s), _C.stream_of(x))
        assert rc == 0, _C.lib().qb_last_error().decode()
        torch.cuda.synchronize()
        return dx, dw, db

    for _ in range(2):
        dx, dw, db = call(True, True)
        xhat = x.float() * rstd[..., None]
        dw_ref = (dout.float() * xhat).sum(0)
        db_ref = dout.float().sum(0)
        torch.testing.assert_close(dw, dw_ref, atol=2e-3, rtol=1e-4)
        torch.testing.assert_close(db, db_ref, atol=2e-3, rtol=1e-4)
        wdy = dout.float() * w
        dx_ref = (wdy - xhat * (xhat * wdy).mean(-1, keepdim=True)) * rstd[..., None]
        assert (dx.float() - dx_ref).abs().max().item() <= 2.0**-7 * float(dx_ref.abs().max())
        _, dw2, db2 = call(False, True)
        assert dw2 is None
        torch.testing.assert_close(db2, db_ref, atol=2e-3, rtol=1e-4)


def test_static_workspace_residual_gradient_and_empty_batch():
    """The residual-gradient streams (dresidual_out added into dx, dresidual written in its own
    dtype) and M == 0, where dw / db must come back as zeros without touching the workspace."""
    M, N = 257, 1024
    x, w, dout, rstd, _ = _inputs(M, N, torch.bfloat16, False, seed=31)
    dres_out = torch.randn(M, N, device="cuda")  # fp32 residual stream
    dx = torch.empty_like(x)
    dres = torch.empty_like(dres_out)
    dw = torch.empty(N, device="cuda")
    s = _C.NormBwdStaticArgs()
    _fill_bwd(s.bwd, x, w, dout, rstd, None, dx, False)
    s.bwd.dresidual_out, s.bwd.dresidual = _C.ptr(dres_out), _C.ptr(dres)
    s.bwd.dresidual_out_row_stride = s.bwd.dresidual_row_stride = N
    s.bwd.dresidual_out_dtype = s.bwd.dresidual_dtype = _C.QB_F32
    s.dw, s.db, s.param_dtype = _C.ptr(dw), None, _C.QB_F32
    for _ in range(2):
        assert _C.lib().qb_norm_bwd_static(byref(s), _C.stream_of(x)) == 0, _C.lib().qb_last_error().decode()
        torch.cuda.synchronize()
        xhat = x.float() * rstd[:, None]
        wdy = dout.float() * w
        ref = (wdy - xhat * (xhat * wdy).mean(-1, keepdim=True)) * rstd[:, None] + dres_out
        torch.testing.assert_close(dres, ref, atol=1e-4, rtol=1e-4)
        assert (dx.float() - ref).abs().max().item() <= 2.0**-7 * float(ref.abs().max())
        torch.testing.assert_close(dw, (dout.float() * xhat).sum(0), atol=2e-3, rtol=1e-4)
    # empty batch
    e = torch.empty(0, N, device="cuda", dtype=torch.bfloat16)
    dw.fill_(7.0)
    db = torch.full((N,), 7.0, device="cuda")
    s2 = _C.NormBwdStaticArgs()
    _fill_bwd(s2.bwd, e, w, e, rstd[:0], None, e, False)
    s2.dw, s2.db, s2.param_dtype = _C.ptr(dw), _C.ptr(db), _C.QB_F32
    # data_ptr() of an empty tensor is 0: give the entry point non-null dummies for the row tensors
    s2.bwd.x = s2.bwd.dout = s2.bwd.dx = _C.ptr(x)
    s2.bwd.rstd = _C.ptr(rstd)
    assert _C.lib().qb_norm_bwd_static(byref(s2), _C.stream_of(x)) == 0, _C.lib().qb_last_error().decode()
    torch.cuda.synchronize()
    assert (dw == 0).all() and (db == 0).all()
