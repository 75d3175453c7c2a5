"""GPU parity tests of LayerNorm forward / backward against the CPU oracle, after the reference's
tests/test_layernorm.py (parametrisation, tolerances, ragged-N known-answer regression)."""

import importlib

import pytest
import torch

import oracle
from _util import assert_close_to_oracle

pytestmark = pytest.mark.gpu

ln = importlib.import_module("quack_flydsl_b200.layernorm")
DEV = "cuda"


@pytest.mark.parametrize("has_bias", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [256, 512, 760, 1024, 1128, 2048, 4096, 8192, 16384, 32768, 65536,
                               131072, 262144])
@pytest.mark.parametrize("M", [1, 37, 199, 4096])
def test_layernorm_forward_backward(M, N, dtype, has_bias):
    if M == 4096 and N > 16384:
        pytest.skip("covered by smaller M and by the full-size configuration test")
    if M == 37 and N not in (256, 1128, 32768):
        pytest.skip("same tile choice as M=199")
    eps = 1e-6
    x = torch.randn(M, N, device=DEV, dtype=dtype)
    w = torch.randn(N, device=DEV, dtype=torch.float32)
    out, rstd, mean = ln.layernorm_fwd(x, w, eps=eps, return_rstd=True, return_mean=True)
    assert out.shape == x.shape and out.dtype == dtype
    assert rstd.shape == (M,) and rstd.dtype == torch.float32
    assert mean.shape == (M,) and mean.dtype == torch.float32
    xc, wc = x.cpu(), w.cpu()
    ref = oracle.layernorm_ref(xc.float(), wc, eps=eps)
    assert_close_to_oracle(out, ref, dtype, atol={torch.float32: 1e-4}.get(dtype), what="out")
    torch.testing.assert_close(rstd.cpu(), oracle.layernorm_rstd_ref(xc, eps=eps), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(mean.cpu(), oracle.layernorm_mean_ref(xc), atol=1e-5, rtol=1e-5)
    if N > 128 * 1024 and dtype == torch.float32:
        return  # fp32 backward is limited to N <= 128K, as in the reference
    dout = torch.randn_like(x)
    dx, dw, db = ln.layernorm_bwd(x, w, dout, rstd, mean, has_bias=has_bias)
    assert dx.shape == x.shape and dx.dtype == dtype
    assert dw.shape == (N,) and dw.dtype == torch.float32
    dx_ref, dw_ref, db_ref = oracle.layernorm_bwd_ref(xc, wc, dout.cpu(), rstd.cpu(), mean.cpu(), has_bias)
    assert_close_to_oracle(dx, dx_ref, dtype, atol={torch.float32: 2e-4}.get(dtype), max_ulp=None, what="dx")
    sum_atol = 5e-6 * (M ** 0.5) * 4 if dtype == torch.float32 else 1e-3 * (M ** 0.5)
    torch.testing.assert_close(dw.cpu(), dw_ref, atol=sum_atol, rtol=1e-3)
    if has_bias:
        assert db.shape == (N,) and db.dtype == torch.float32
        torch.testing.assert_close(db.cpu(), db_ref, atol=sum_atol, rtol=1e-3)
    else:
        assert db is None


def test_layernorm_fwd_return_arity():
    M, N = 37, 1024
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, device=DEV, dtype=torch.float32)
    out_r, rstd_only = ln.layernorm_fwd(x, w, return_rstd=True, return_mean=False)
    assert out_r.shape == x.shape and rstd_only.shape == (M,) and rstd_only.dtype == torch.float32
    out_m, mean_only = ln.layernorm_fwd(x, w, return_rstd=False, return_mean=True)
    assert out_m.shape == x.shape and mean_only.shape == (M,)
    out_only = ln.layernorm_fwd(x, w)
    assert isinstance(out_only, torch.Tensor) and out_only.shape == x.shape


def test_layernorm_ragged_n_known_answer(norm_golden):
    """Closed-form input of the reference's regression test (tests/test_layernorm.py:121-139):
    padding lanes of a ragged row must not enter the variance."""
    c = norm_golden["layernorm_ragged_known_answer"]
    x, w = c["x"].to(DEV), c["w"].to(DEV)
    out, rstd, mean = ln.layernorm_fwd(x, w, eps=c["eps"], return_rstd=True, return_mean=True)
    torch.testing.assert_close(out.cpu(), oracle.layernorm_ref(c["x"], c["w"], eps=c["eps"]), atol=2e-4, rtol=1e-4)
    torch.testing.assert_close(rstd.cpu(), oracle.layernorm_rstd_ref(c["x"], eps=c["eps"]), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(mean.cpu(), oracle.layernorm_mean_ref(c["x"]), atol=1e-5, rtol=1e-5)
    # and the committed outputs of the reference's own CPU functions
    torch.testing.assert_close(out.cpu(), c["out"], atol=4e-4, rtol=1e-4)
    torch.testing.assert_close(rstd.cpu(), c["rstd"], atol=1e-5, rtol=1e-4)


def test_layernorm_golden_fixtures(norm_golden):
    for c in norm_golden["layernorm"]:
        x, w, dout = c["x"].to(DEV), c["w"].to(DEV), c["dout"].to(DEV)
        out, rstd, mean = ln.layernorm_fwd(x, w, eps=c["eps"], return_rstd=True, return_mean=True)
        dt = x.dtype
        assert_close_to_oracle(out, c["out"].float(), dt, atol={torch.float32: 2e-5}.get(dt), max_ulp=1, what="out")
        torch.testing.assert_close(rstd.cpu(), c["rstd"], atol=0, rtol=1e-5)
        dx, dw, db = ln.layernorm_bwd(x, w, dout, rstd, mean)
        assert_close_to_oracle(dx, c["dx"].float(), dt, atol={torch.float32: 5e-5}.get(dt), max_ulp=None, what="dx")
        torch.testing.assert_close(dw.cpu(), c["dw"], atol=1e-3, rtol=1e-3)
        torch.testing.assert_close(db.cpu(), c["db"], atol=1e-3, rtol=1e-3)


def test_layernorm_autograd_bf16_params_config_shape():
    """Shape family of the LayerNorm benchmark configuration (bf16 x, weight and bias, eps 1e-5,
    x ~ N(0.5, 1)) through the autograd wrapper, on a row slice the CPU oracle handles."""
    M, N, eps = 2048, 4096, 1e-5
    d = oracle.make_config_inputs("c3", rows=M, device=DEV)
    x = d["x"].requires_grad_()
    w = d["weight"].requires_grad_()
    b = d["bias"].requires_grad_()
    out = ln.layernorm(x, w, b, eps=eps)
    out.backward(d["dout"])
    xc, wc, bc = x.detach().cpu(), w.detach().cpu(), b.detach().cpu()
    assert_close_to_oracle(out.detach(), oracle.layernorm_ref(xc.float(), wc, bias=bc, eps=eps), torch.bfloat16, what="out")
    rstd, mean = oracle.layernorm_rstd_ref(xc, eps=eps), oracle.layernorm_mean_ref(xc)
    dx_ref, dw_ref, db_ref = oracle.layernorm_bwd_ref(xc, wc, d["dout"].cpu(), rstd, mean)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, max_ulp=None, what="dx")
    assert w.grad.dtype == torch.bfloat16 and b.grad.dtype == torch.bfloat16
    for g, r in ((w.grad, dw_ref), (b.grad, db_ref)):
        torch.testing.assert_close(g.float().cpu(), r.bfloat16().float(),
                                   atol=2 * 2 ** -8 * float(r.abs().max()), rtol=1e-2)


def test_layernorm_full_size_config_properties():
    """Benchmark shape bf16 [65536, 4096] at full size: statistics against the fp32 formulas
    on the GPU, outputs through size-independent properties."""
    M, N, eps = 65536, 4096, 1e-5
    g = torch.Generator(device=DEV).manual_seed(0)
    x = (0.5 + torch.randn(M, N, device=DEV, generator=g)).bfloat16()
    w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).bfloat16()
    b = (0.1 * torch.randn(N, device=DEV, generator=g)).bfloat16()
    dout = torch.randn(M, N, device=DEV, generator=g).bfloat16()
    out = torch.empty_like(x)
    rstd = torch.empty(M, device=DEV)
    mean = torch.empty(M, device=DEV)
    ln._rmsnorm_fwd(x, w, out, b, rstd, mean, None, None, eps, True)
    torch.testing.assert_close(mean, oracle.layernorm_mean_ref(x), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(rstd, oracle.layernorm_rstd_ref(x, eps=eps), atol=0, rtol=1e-5)
    assert_close_to_oracle(out[:4096], oracle.layernorm_ref(x[:4096].float(), w, bias=b, eps=eps), torch.bfloat16, what="out")
    dx, dw, db = ln._layernorm_bwd_impl(x, w, dout, rstd, mean, True, torch.bfloat16)
    # LayerNorm gradient rows sum to zero and are orthogonal to the centred input
    s = dx.float().sum(-1)
    assert (s.abs() <= 2e-3 * dx.float().abs().sum(-1)).all()
    torch.testing.assert_close(db.float(), dout.float().sum(0).bfloat16().float(), atol=4.0, rtol=2e-2)
    dx_ref, _, _ = oracle.layernorm_bwd_ref(x[:2048], w, dout[:2048], rstd[:2048], mean[:2048])
    assert_close_to_oracle(dx[:2048], dx_ref, torch.bfloat16, max_ulp=None, what="dx")
    # bitwise reproducible dw / db
    dx2, dw2, db2 = ln._layernorm_bwd_impl(x, w, dout, rstd, mean, True, torch.bfloat16)
    assert torch.equal(dw, dw2) and torch.equal(db, db2) and torch.equal(dx, dx2)


def test_layernorm_empty():
    x = torch.empty(0, 1024, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(1024, device=DEV)
    out, rstd, mean = ln.layernorm_fwd(x, w, return_rstd=True, return_mean=True)
    assert out.shape == (0, 1024)
    dx, dw, db = ln.layernorm_bwd(x, w, torch.empty_like(x), rstd, mean)
    assert (dw == 0).all() and (db == 0).all()


rnm = importlib.import_module("quack_flydsl_b200.rmsnorm")


@pytest.mark.parametrize("force", [False, True])
def test_norm_forward_streamed_long_rows(force, monkeypatch):
    """Long rows with at least one row per SM take the streamed two-pass forward kernels (flag
    bit 4 forces them for shorter rows too).  RMSNorm with and without a residual, LayerNorm with
    bias, parameters in the input dtype and in fp32, a ragged chunk count, and a large common
    offset for the one-pass LayerNorm statistics."""
    M = 160
    N = 4104 if force else 65536 + 8 * 3
    if force:
        monkeypatch.setenv("QUACK_B200_CFG", "norm_fwd:0:0:0:0:0:16")
    g = torch.Generator(device=DEV).manual_seed(3)
    for dtype, wdtype in ((torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
                          (torch.float32, torch.float32)):
        x = torch.randn(M, N, device=DEV, generator=g).to(dtype)
        res = torch.randn(M, N, device=DEV, generator=g).to(dtype)
        w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(wdtype)
        b = (0.1 * torch.randn(N, device=DEV, generator=g)).to(wdtype)
        xc, rc, wc, bc = x.cpu(), res.cpu(), w.cpu(), b.cpu()
        # RMSNorm, no residual
        out, _, rstd = rnm.rmsnorm_fwd(x, w, store_rstd=True)
        assert_close_to_oracle(out, oracle.rmsnorm_ref(xc, wc, out_dtype=torch.float32), dtype,
                               atol={torch.float32: 2e-5}.get(dtype), what="rms out")
        torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd_ref(xc), atol=0, rtol=1e-5)
        # RMSNorm + residual (+ bias)
        out, res_out, rstd = rnm.rmsnorm_fwd(x, w, bias=b, residual=res, store_rstd=True)
        ref_out, ref_h = oracle.rmsnorm_ref(xc, wc, bias=bc, residual=rc, out_dtype=torch.float32,
                                            residual_dtype=torch.float32)
        assert torch.equal(res_out.cpu(), ref_h.to(dtype))
        assert_close_to_oracle(out, ref_out, dtype, atol={torch.float32: 2e-5}.get(dtype), what="rms+res out")
        torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd_ref(xc, residual=rc), atol=0, rtol=1e-5)
        # LayerNorm with bias through the op (any parameter dtype)
        o = torch.empty_like(x)
        rs, mn = torch.empty(M, device=DEV), torch.empty(M, device=DEV)
        rnm._rmsnorm_fwd(x, w, o, b, rs, mn, None, None, 1e-5, True)
        assert_close_to_oracle(o, oracle.layernorm_ref(xc, wc, bc, eps=1e-5), dtype,
                               atol={torch.float32: 2e-5}.get(dtype), what="ln out")
        torch.testing.assert_close(rs.cpu(), oracle.layernorm_rstd_ref(xc, eps=1e-5), atol=0, rtol=1e-5)
        torch.testing.assert_close(mn.cpu(), oracle.layernorm_mean_ref(xc), atol=1e-6, rtol=1e-5)
    # large common offset: x = 1000 + row * 100 + small pattern (fp32)
    cols = torch.arange(N, device=DEV, dtype=torch.float32)
    rows = torch.arange(M, device=DEV, dtype=torch.float32).unsqueeze(1)
    x = 1000.0 + rows * 100.0 + ((cols % 17) - 8.0) / 8.0
    w = torch.ones(N, device=DEV)
    o = torch.empty_like(x)
    rs, mn = torch.empty(M, device=DEV), torch.empty(M, device=DEV)
    rnm._rmsnorm_fwd(x, w, o, None, rs, mn, None, None, 1e-5, True)
    torch.testing.assert_close(mn.cpu(), oracle.layernorm_mean_ref(x.cpu()), atol=0, rtol=1e-6)
    torch.testing.assert_close(rs.cpu(), oracle.layernorm_rstd_ref(x.cpu(), eps=1e-5), atol=0, rtol=2e-4)
    torch.testing.assert_close(o.cpu(), oracle.layernorm_ref(x.cpu(), w.cpu(), eps=1e-5), atol=5e-3, rtol=1e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [64, 128, 256, 512, 768, 1024, 2048, 4096, 6144, 8192, 16384])
def test_layernorm_statistics_one_pass_and_centred_rows_mixed(N, dtype):
    """The register kernel takes sum and sum of squares in one pass and falls back to the centred
    second pass for rows whose mean is large against their spread.  Rows of both kinds alternate
    here, so that they meet inside one CTA and -- for rows narrower than a warp -- inside one
    warp; constant rows (variance 0), an all-zero row and rows scaled far down are included.
    rstd must hold rtol 1e-5 against the oracle on every row, whichever branch it took."""
    M = 301
    g = torch.Generator(device=DEV).manual_seed(N)
    x = torch.randn(M, N, device=DEV, generator=g)
    x[::3] += 50.0          # mean^2 >> var: centred pass
    x[1::7] *= 1e-3         # tiny spread around 0: one pass
    x[2::11] = x[2::11] * 1e-3 + 7.0   # tiny spread around 7: centred pass
    x[5] = 3.0              # constant row
    x[6] = 0.0              # zero row
    x = x.to(dtype)
    w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(dtype)
    b = (0.1 * torch.randn(N, device=DEV, generator=g)).to(dtype)
    out = torch.empty_like(x)
    rstd, mean = torch.empty(M, device=DEV), torch.empty(M, device=DEV)
    rnm._rmsnorm_fwd(x, w, out, b, rstd, mean, None, None, 1e-5, True)
    xc = x.cpu()
    torch.testing.assert_close(mean.cpu(), oracle.layernorm_mean_ref(xc), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(rstd.cpu(), oracle.layernorm_rstd_ref(xc, eps=1e-5), atol=0, rtol=1e-5)
    ref = oracle.layernorm_ref(xc, w.cpu(), b.cpu(), eps=1e-5).float()
    assert torch.isfinite(out.float()).all()
    # rows with a tiny spread amplify the rounding of the mean by rstd (up to 316): compare the
    # ordinary rows tightly and all rows against the bound that amplification allows
    plain = torch.ones(M, dtype=torch.bool)
    plain[1::7] = False; plain[2::11] = False; plain[5] = False; plain[6] = False
    assert_close_to_oracle(out[plain.to(DEV)], ref[plain], dtype, atol={torch.float32: 1e-4}.get(dtype), what="out")
    tol = 2e-3 if dtype == torch.float32 else 5e-2
    assert float((out.cpu().float() - ref).abs().max()) <= tol * max(1.0, float(ref.abs().max()))


def test_norm_forward_long_rows_residual_out_in_place():
    """residual_out may be the residual buffer itself (in-place residual stream update); long rows
    must then not take the kernel that reads the inputs a second time."""
    M, N = 160, 65536
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(M, N, device=DEV, generator=g).bfloat16()
    res = torch.randn(M, N, device=DEV, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).bfloat16()
    ref_out, ref_h = oracle.rmsnorm_ref(x.cpu(), w.cpu(), residual=res.cpu(), out_dtype=torch.float32,
                                        residual_dtype=torch.float32)
    out = torch.empty_like(x)
    rstd = torch.empty(M, device=DEV)
    rnm._rmsnorm_fwd(x, w, out, None, rstd, None, res, res, 1e-6)  # residual_out is residual
    assert torch.equal(res.cpu(), ref_h.bfloat16())
    assert_close_to_oracle(out, ref_out, torch.bfloat16, what="out")


@pytest.mark.parametrize("N", [12288, 16384])
@pytest.mark.parametrize("pdtype", [torch.bfloat16, torch.float16])
def test_norm_forward_packed_parameter_staging(N, pdtype):
    """Rows whose fp32 weight + bias slices no longer fit the shared-memory staging keep 16-bit
    parameters packed there; LayerNorm and RMSNorm with bias, weight_offset included."""
    M = 200
    dtype = pdtype
    g = torch.Generator(device=DEV).manual_seed(7)
    x = (0.5 + torch.randn(M, N, device=DEV, generator=g)).to(dtype)
    w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(pdtype)
    b = (0.1 * torch.randn(N, device=DEV, generator=g)).to(pdtype)
    xc, wc, bc = x.cpu(), w.cpu(), b.cpu()
    o = torch.empty_like(x)
    rs, mn = torch.empty(M, device=DEV), torch.empty(M, device=DEV)
    rnm._rmsnorm_fwd(x, w, o, b, rs, mn, None, None, 1e-5, True)
    assert_close_to_oracle(o, oracle.layernorm_ref(xc, wc, bc, eps=1e-5), dtype, what="ln out")
    torch.testing.assert_close(rs.cpu(), oracle.layernorm_rstd_ref(xc, eps=1e-5), atol=0, rtol=1e-5)
    rnm._rmsnorm_fwd(x, w, o, b, rs, None, None, None, 1e-6, False, 0.5)
    ref = oracle.rmsnorm_ref(xc, wc, bias=bc, weight_offset=0.5, out_dtype=torch.float32)
    assert_close_to_oracle(o, ref, dtype, what="rms out")
    rnm._rmsnorm_fwd(x, None, o, b, rs, mn, None, None, 1e-5, True)  # bias only
    ref = oracle.layernorm_ref(xc, torch.ones(N), bc, eps=1e-5)
    assert_close_to_oracle(o, ref, dtype, what="ln bias-only out")
