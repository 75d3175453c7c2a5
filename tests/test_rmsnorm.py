"""GPU parity tests of RMSNorm forward / backward: the sm_100a kernels, called through the C ABI
behind the reference's Python API, against the CPU oracle.  Parametrisation and tolerances follow
the reference's tests/test_rmsnorm.py; bf16 outputs are additionally held to <= 2 bf16 ulp and
fp32 rstd to rtol 1e-5."""

import importlib

import pytest
import torch

import oracle
from _util import ATOL, assert_close_to_oracle, oracle_device, to

pytestmark = pytest.mark.gpu

rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
from quack_flydsl_b200.rmsnorm_config import RmsNormBwdConfig, RmsNormFwdConfig  # noqa: E402

DEV = "cuda"


def _check_fwd_bwd(M, N, dtype, wdtype, weight_offset=0.0, has_bias=False, has_residual=False):
    x = torch.randn(M, N, device=DEV, dtype=dtype, requires_grad=True)
    w = None
    if wdtype is not None:
        w = torch.randn(N, device=DEV, dtype=wdtype)
        if weight_offset:
            w = 0.1 * w
        w.requires_grad_()
    b = torch.randn(N, device=DEV, dtype=wdtype, requires_grad=True) if has_bias else None
    res = torch.randn(M, N, device=DEV, dtype=dtype, requires_grad=True) if has_residual else None
    out = rn.rmsnorm(x, w, bias=b, residual=res, weight_offset=weight_offset)
    assert out.shape == x.shape and out.dtype == dtype
    dout = torch.randn_like(out)
    out.backward(dout)

    dev = oracle_device(x)
    xo, wo, bo, ro, do = to(dev, x, w, b, res, dout)
    ref = oracle.rmsnorm_ref(xo, wo, bias=bo, residual=ro, weight_offset=weight_offset,
                             out_dtype=torch.float32, residual_dtype=torch.float32 if has_residual else None)
    ref_out, ref_h = ref if has_residual else (ref, xo.float())
    assert_close_to_oracle(out.detach(), ref_out, dtype, what="out")
    # backward consumes the pre-norm sum rounded to the residual dtype, like the kernel does
    x_pre = ref_h.to(dtype) if has_residual else xo
    rstd = oracle.rmsnorm_rstd_ref(x_pre)
    dx_ref, dw_ref, db_ref = oracle.rmsnorm_bwd_ref(x_pre, wo, do, rstd, weight_offset=weight_offset,
                                                     has_bias=has_bias)
    assert x.grad.dtype == dtype
    assert_close_to_oracle(x.grad, dx_ref, dtype, max_ulp=None, what="dx")
    if has_residual:
        assert_close_to_oracle(res.grad, dx_ref, dtype, max_ulp=None, what="dresidual")
    if w is not None:
        assert w.grad.dtype == wdtype
        if wdtype == torch.float32:
            atol = 5e-6 * (M ** 0.5) if dtype == torch.float32 else 2e-3 * (M ** 0.5)
        else:
            atol = 2 * torch.finfo(wdtype).eps * float(dw_ref.abs().max())
        torch.testing.assert_close(w.grad.float().cpu(), dw_ref.to(wdtype).float().cpu(), atol=atol, rtol=1e-3)
    if has_bias:
        atol = 2 * torch.finfo(wdtype).eps * float(db_ref.abs().max()) + 1e-4 * (M ** 0.5)
        torch.testing.assert_close(b.grad.float().cpu(), db_ref.to(wdtype).float().cpu(), atol=atol, rtol=1e-3)


@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32, None])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("N", [192, 256, 760, 1024, 1128, 4096, 8192, 32768, 131072, 262144])
@pytest.mark.parametrize("M", [1, 199, 8192])
def test_rmsnorm_forward_backward(M, N, dtype, wdtype):
    if M == 8192 and N > 32768:
        pytest.skip("covered by M=199 and by the full-size configuration test")
    if N > 128 * 1024 and dtype == torch.float32:
        # fp32 backward is limited to N <= 128K, as in the reference (quack/rmsnorm.py:637-639)
        x = torch.randn(M, N, device=DEV, dtype=dtype)
        w = torch.randn(N, device=DEV, dtype=wdtype) if wdtype is not None else None
        out = rn.rmsnorm(x, w)
        assert_close_to_oracle(out, oracle.rmsnorm_ref(x.cpu(), None if w is None else w.cpu(),
                                                       out_dtype=torch.float32), dtype, what="out")
        return
    _check_fwd_bwd(M, N, dtype, wdtype)


@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [1024, 4096, 32768])
@pytest.mark.parametrize("M", [1, 199])
def test_rmsnorm_weight_offset(M, N, dtype, wdtype):
    _check_fwd_bwd(M, N, dtype, wdtype, weight_offset=1.0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [256, 1128, 8192])
def test_rmsnorm_bias_and_residual(N, dtype):
    _check_fwd_bwd(199, N, dtype, torch.float32, has_bias=True)
    _check_fwd_bwd(199, N, dtype, dtype, has_residual=True)
    _check_fwd_bwd(64, N, dtype, dtype, has_bias=True, has_residual=True)


def test_rmsnorm_rstd_rtol_1e5_and_residual_out():
    M, N = 257, 8192
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(N, device=DEV)).bfloat16()
    out, res_out, rstd = rn.rmsnorm_fwd(x, w, residual=res, store_rstd=True)
    ref_out, ref_h = oracle.rmsnorm_ref(x.cpu(), w.cpu(), residual=res.cpu(), out_dtype=torch.float32,
                                        residual_dtype=torch.float32)
    assert torch.equal(res_out.cpu(), ref_h.to(torch.bfloat16))  # x + residual rounded once
    torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd_ref(x.cpu(), residual=res.cpu()),
                               atol=0, rtol=1e-5)
    assert_close_to_oracle(out, ref_out, torch.bfloat16, what="out")


def test_rmsnorm_residual_dtype_fp32_is_bit_exact():
    # reference: tests/test_rmsnorm.py:559-593
    M, N = 64, 4096
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    res = torch.randn(M, N, device=DEV, dtype=torch.float32)
    w = torch.randn(N, device=DEV, dtype=torch.float32)
    out, res_out, _ = rn.rmsnorm_fwd(x, w, residual=res, residual_dtype=torch.float32)
    assert res_out.dtype == torch.float32
    assert torch.equal(res_out, x.float() + res)
    ref_out, _ = oracle.rmsnorm_ref(x.cpu(), w.cpu(), residual=res.cpu(), out_dtype=torch.float32)
    assert_close_to_oracle(out, ref_out, torch.bfloat16, what="out")
    # no residual but a different residual dtype: residual_out is x cast
    _, res_out2, _ = rn.rmsnorm_fwd(x, w, residual_dtype=torch.float32)
    assert torch.equal(res_out2, x.float())
    # no residual, same dtype: x itself is handed back
    _, res_out3, _ = rn.rmsnorm_fwd(x, w)
    assert res_out3 is x


def test_rmsnorm_prenorm_backward_through_both_outputs():
    # reference: tests/test_rmsnorm.py:461-502
    M, N = 199, 1024
    dtype = torch.bfloat16
    x = torch.randn(M, N, device=DEV, dtype=dtype, requires_grad=True)
    res = torch.randn(M, N, device=DEV, dtype=dtype, requires_grad=True)
    w = torch.randn(N, device=DEV, dtype=torch.float32, requires_grad=True)
    out, res_out = rn.rmsnorm(x, w, residual=res, prenorm=True)
    g1, g2 = torch.randn_like(out), torch.randn_like(res_out)
    torch.autograd.backward([out, res_out], [g1, g2])
    h = (x.detach().float() + res.detach().float()).to(dtype).cpu()
    rstd = oracle.rmsnorm_rstd_ref(h)
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(h, w.detach().cpu(), g1.cpu(), rstd, dresidual_out=g2.cpu())
    assert_close_to_oracle(x.grad, dx_ref, dtype, max_ulp=None, what="dx")
    assert torch.equal(x.grad, res.grad)
    torch.testing.assert_close(w.grad.cpu(), dw_ref, atol=2e-3 * M ** 0.5, rtol=1e-3)
    # prenorm=False returns only out
    assert isinstance(rn.rmsnorm(x, w, residual=res, prenorm=False), torch.Tensor)


def test_rmsnorm_amp_bf16_dout_fp32_x():
    # reference: tests/test_rmsnorm.py:505-518: dx keeps x's dtype when dout is narrower
    M, N = 128, 2048
    x = torch.randn(M, N, device=DEV, dtype=torch.float32)
    w = torch.randn(N, device=DEV, dtype=torch.float32)
    dout = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    rstd = oracle.rmsnorm_rstd_ref(x.cpu()).to(DEV)
    dx, dw, _, _ = rn.rmsnorm_bwd(x, w, dout, rstd)
    assert dx.dtype == torch.float32 and dw.dtype == torch.float32
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(x.cpu(), w.cpu(), dout.cpu(), rstd.cpu())
    torch.testing.assert_close(dx.cpu(), dx_ref, atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(dw.cpu(), dw_ref, atol=5e-6 * M ** 0.5 * 10, rtol=1e-3)


def test_rmsnorm_dresidual_other_dtype_is_separate_buffer():
    M, N = 96, 1024
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    dout = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    dres_out = torch.randn(M, N, device=DEV, dtype=torch.float32)
    rstd = oracle.rmsnorm_rstd_ref(x.cpu()).to(DEV)
    dx, dw, db, dres = rn.rmsnorm_bwd(x, w, dout, rstd, dresidual_out=dres_out, has_residual=True)
    assert dres is not dx and dres.dtype == torch.float32 and dx.dtype == torch.bfloat16 and db is None
    dx_ref, _, _ = oracle.rmsnorm_bwd_ref(x.cpu(), w.cpu(), dout.cpu(), rstd.cpu(), dresidual_out=dres_out.cpu())
    torch.testing.assert_close(dres.cpu(), dx_ref, atol=1e-4, rtol=1e-4)
    assert_close_to_oracle(dx, dx_ref, torch.bfloat16, max_ulp=None, what="dx")


def test_rmsnorm_strided_rows_and_noncontiguous_grad():
    # reference: tests/test_rmsnorm.py:147-165, 264-291 (ld = 576 for N = 512)
    M, N, ld = 77, 512, 576
    base = torch.randn(M, ld, device=DEV, dtype=torch.bfloat16)
    x = base[:, :N].detach().requires_grad_()
    assert x.stride(0) == ld
    w = torch.randn(N, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out = rn.rmsnorm(x, w)
    ref = oracle.rmsnorm_ref(x.detach().cpu(), w.detach().cpu(), out_dtype=torch.float32)
    assert_close_to_oracle(out.detach(), ref, torch.bfloat16, what="out")
    g = torch.randn(N, M, device=DEV, dtype=torch.bfloat16).t()  # non-contiguous upstream grad
    out.backward(g)
    rstd = oracle.rmsnorm_rstd_ref(x.detach().cpu())
    dx_ref, _, _ = oracle.rmsnorm_bwd_ref(x.detach().cpu(), w.detach().cpu(), g.cpu(), rstd)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, max_ulp=None, what="dx")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [64, 128])
def test_rmsnorm_per_head(D, dtype):
    # reference: tests/test_rmsnorm.py:210-261 (QK-norm: x (B, S, H, D), weight (H, D))
    B, S, H = 2, 37, 6
    x = torch.randn(B, S, H, D, device=DEV, dtype=dtype, requires_grad=True)
    w = torch.randn(H, D, device=DEV, dtype=torch.float32, requires_grad=True)
    out = rn.rmsnorm(x, w)
    assert out.shape == x.shape
    ref = oracle.rmsnorm_ref(x.detach().cpu(), w.detach().cpu(), out_dtype=torch.float32)
    assert_close_to_oracle(out.detach(), ref, dtype, what="out")
    dout = torch.randn_like(out)
    out.backward(dout)
    xf = x.detach().cpu().reshape(-1, H, D)
    rstd = oracle.rmsnorm_rstd_ref(xf)
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(xf, w.detach().cpu(), dout.cpu().reshape(-1, H, D), rstd)
    assert_close_to_oracle(x.grad.reshape(-1, H, D), dx_ref, dtype, max_ulp=None, what="dx")
    assert w.grad.shape == (H, D)
    torch.testing.assert_close(w.grad.cpu(), dw_ref, atol=2e-3 * (B * S) ** 0.5, rtol=1e-3)


def test_rmsnorm_3d_input_and_module():
    x = torch.randn(2, 32, 1024, device=DEV, dtype=torch.float16)
    w = torch.randn(1024, device=DEV, dtype=torch.float32)
    out = rn.rmsnorm(x, w)
    assert out.shape == x.shape and out.dtype == x.dtype
    mod = rn.QuackRMSNorm(1024, eps=1e-6, device=DEV, dtype=torch.bfloat16)
    xb = torch.randn(4, 7, 1024, device=DEV, dtype=torch.bfloat16)
    ref = oracle.rmsnorm_ref(xb.cpu(), mod.weight.detach().cpu(), out_dtype=torch.float32)
    assert_close_to_oracle(mod(xb).detach(), ref, torch.bfloat16, what="module out")


def test_rmsnorm_empty_inputs():
    # reference: tests/test_rmsnorm.py:596-633
    N = 1024
    x = torch.empty(0, N, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    out, res_out, rstd = rn.rmsnorm_fwd(x, w, store_rstd=True)
    assert out.shape == (0, N) and rstd.shape == (0,) and res_out is x
    dx, dw, db, dres = rn.rmsnorm_bwd(x, w, torch.empty_like(x), rstd, has_bias=True)
    assert dx.shape == (0, N) and (dw == 0).all() and (db == 0).all() and dres is None


def test_rmsnorm_specialisation_counter():
    # reference: tests/test_rmsnorm.py:383-422 (there: JIT cache entries)
    rn._compile_rmsnorm_fwd.cache_clear()
    M, N = 32, 1024
    w = torch.randn(N, device=DEV)
    rn.rmsnorm_fwd(torch.randn(M, N, device=DEV, dtype=torch.float16), w)
    assert rn._compile_rmsnorm_fwd.cache_info().currsize == 1
    rn.rmsnorm_fwd(torch.randn(2 * M, N, device=DEV, dtype=torch.float16), w)
    assert rn._compile_rmsnorm_fwd.cache_info().currsize == 1
    rn.rmsnorm_fwd(torch.randn(M, 2 * N, device=DEV, dtype=torch.float16), torch.randn(2 * N, device=DEV))
    assert rn._compile_rmsnorm_fwd.cache_info().currsize == 2
    rn.rmsnorm_fwd(torch.randn(M, N, device=DEV, dtype=torch.float32), w)
    assert rn._compile_rmsnorm_fwd.cache_info().currsize == 3


@pytest.mark.parametrize("threads_per_row", [32, 64])
def test_rmsnorm_degenerate_cluster_config_is_clamped(threads_per_row):
    # reference: tests/test_rmsnorm.py:644-728
    M, N = 256, 256
    dtype = torch.bfloat16
    x = torch.randn(M, N, device=DEV, dtype=dtype)
    w = torch.randn(N, device=DEV, dtype=dtype) * 0.1
    out = torch.empty_like(x)
    rstd = torch.empty(M, device=DEV, dtype=torch.float32)
    fcfg = RmsNormFwdConfig(num_threads=128, threads_per_row=threads_per_row, cluster_n=2,
                            reload_from=None, delay_w_load=False)
    rn.rmsnorm_fwd_tuned.fn(x, w, out, bias=None, rstd=rstd, mean=None, residual=None,
                            residual_out=None, eps=1e-6, is_layernorm=False, per_head=False, config=fcfg)
    torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd_ref(x.cpu()), atol=0, rtol=1e-5)
    assert_close_to_oracle(out, oracle.rmsnorm_ref(x.cpu(), w.cpu(), out_dtype=torch.float32), dtype, what="out")
    dout = torch.randn(M, N, device=DEV, dtype=dtype)
    dx = torch.empty_like(x)
    sm_count = torch.cuda.get_device_properties(DEV).multi_processor_count * 2
    dw_partial = torch.empty((sm_count, N), device=DEV, dtype=torch.float32)
    bcfg = RmsNormBwdConfig(num_threads=128, threads_per_row=threads_per_row, cluster_n=2,
                            reload_wdy=None, reload_x=None, use_tma=False, smem_stages=2)
    rn.rmsnorm_bwd_tuned.fn(x, w, dout, rstd, dx, dw_partial=dw_partial, db_partial=None,
                            dresidual_out=None, dresidual=None, sm_count=sm_count, per_head=False,
                            has_dw_partial=True, has_db_partial=False, config=bcfg)
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(x.cpu(), w.cpu(), dout.cpu(), rstd.cpu())
    assert_close_to_oracle(dx, dx_ref, dtype, max_ulp=None, what="dx")
    torch.testing.assert_close(dw_partial.sum(0).cpu(), dw_ref, atol=2e-3 * M ** 0.5, rtol=1e-3)


@pytest.mark.parametrize("cluster_n", [1, 2, 4])
@pytest.mark.parametrize("num_threads,threads_per_row", [(128, 32), (128, 128), (256, 128), (512, 512)])
def test_rmsnorm_explicit_configs(num_threads, threads_per_row, cluster_n):
    # reference: tests/test_rmsnorm.py:741-843 (explicit-config plumbing)
    M, N = 1024, 4096
    dtype = torch.bfloat16
    x = torch.randn(M, N, device=DEV, dtype=dtype)
    w = torch.randn(N, device=DEV, dtype=dtype) * 0.1
    out = torch.empty_like(x)
    rstd = torch.empty(M, device=DEV, dtype=torch.float32)
    fcfg = RmsNormFwdConfig(num_threads, threads_per_row, cluster_n)
    rn.rmsnorm_fwd_tuned.fn(x, w, out, rstd=rstd, config=fcfg)
    assert_close_to_oracle(out, oracle.rmsnorm_ref(x.cpu(), w.cpu(), out_dtype=torch.float32), dtype, what="out")
    dout = torch.randn_like(x)
    dx = torch.empty_like(x)
    P = 148
    dw_partial = torch.empty((P, N), device=DEV, dtype=torch.float32)
    for stages in (1, 2, 4):
        bcfg = RmsNormBwdConfig(num_threads, threads_per_row, cluster_n, smem_stages=stages)
        try:
            rn.rmsnorm_bwd_tuned.fn(x, w, dout, rstd, dx, dw_partial=dw_partial, sm_count=P, config=bcfg)
        except ValueError as e:  # a config whose per-thread slice cannot fit is rejected, not run
            assert "does not fit" in str(e)
            continue
        dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(x.cpu(), w.cpu(), dout.cpu(), rstd.cpu())
        assert_close_to_oracle(dx, dx_ref, dtype, max_ulp=None, what=f"dx stages={stages}")
        torch.testing.assert_close(dw_partial.sum(0).cpu(), dw_ref, atol=2e-3 * M ** 0.5, rtol=1e-3)


def test_rmsnorm_backward_is_bitwise_deterministic():
    M, N = 4096, 8192
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(N, device=DEV, dtype=torch.bfloat16)
    dout = torch.randn_like(x)
    rstd = torch.rsqrt(x.float().square().mean(-1) + 1e-6)
    a = rn.rmsnorm_bwd(x, w, dout, rstd, has_bias=True)
    b = rn.rmsnorm_bwd(x, w, dout, rstd, has_bias=True)
    for u, v in zip(a[:3], b[:3]):
        assert torch.equal(u, v)


def test_rmsnorm_full_size_config_roundtrip_properties():
    """Headline benchmark shape (bf16 [32768, 8192] + residual) at full size: checked through
    size-independent properties and against the fp32 formulas evaluated on the GPU."""
    M, N = 32768, 8192
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16, generator=g)
    res = torch.randn(M, N, device=DEV, dtype=torch.bfloat16, generator=g)
    w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).bfloat16()
    dout = torch.randn(M, N, device=DEV, dtype=torch.bfloat16, generator=g)
    out, res_out, rstd = rn.rmsnorm_fwd(x, w, residual=res, store_rstd=True)
    ref_out, ref_h = oracle.rmsnorm_ref(x, w, residual=res, out_dtype=torch.float32, residual_dtype=torch.float32)
    assert torch.equal(res_out, ref_h.to(torch.bfloat16))
    torch.testing.assert_close(rstd, oracle.rmsnorm_rstd_ref(x, residual=res), atol=0, rtol=1e-5)
    assert_close_to_oracle(out, ref_out, torch.bfloat16, what="out")
    del ref_out, ref_h
    # scale covariance: rmsnorm(2h) == rmsnorm(h) up to eps (property, no oracle needed)
    out2, _, _ = rn.rmsnorm_fwd(res_out * 2, w)
    out1, _, _ = rn.rmsnorm_fwd(res_out, w)
    assert (oracle.bf16_ulp_diff(out1[:4096], out2[:4096]) <= 1).all()
    dx, dw, _, dres = rn.rmsnorm_bwd(res_out, w, dout, rstd, has_residual=True)
    assert dres is dx
    # each dx row is orthogonal to its x row (sum_j dx_j * x_j == 0 for RMSNorm)
    dot = (dx.float() * res_out.float()).sum(-1)
    scale = (dx.float().abs() * res_out.float().abs()).sum(-1)
    assert (dot.abs() <= 2e-3 * scale).all()
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(res_out[:2048], w, dout[:2048], rstd[:2048])
    assert_close_to_oracle(dx[:2048], dx_ref, torch.bfloat16, max_ulp=None, what="dx")
    xhat = res_out.float() * rstd.unsqueeze(1)
    dw_full = (dout.float() * xhat).sum(0)
    torch.testing.assert_close(dw.float(), dw_full.bfloat16().float(),
                               atol=2 * 2 ** -8 * float(dw_full.abs().max()), rtol=1e-2)


def test_rmsnorm_torch_compile_fullgraph():
    torch._dynamo.reset()
    M, N = 199, 1024
    x = torch.randn(M, N, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(N, device=DEV, dtype=torch.float32, requires_grad=True)
    fn = torch.compile(rn.rmsnorm, fullgraph=True)
    out = fn(x, w)
    dout = torch.randn_like(out)
    out.backward(dout)
    ref = oracle.rmsnorm_ref(x.detach().cpu(), w.detach().cpu(), out_dtype=torch.float32)
    assert_close_to_oracle(out.detach(), ref, torch.bfloat16, what="out")
    rstd = oracle.rmsnorm_rstd_ref(x.detach().cpu())
    dx_ref, dw_ref, _ = oracle.rmsnorm_bwd_ref(x.detach().cpu(), w.detach().cpu(), dout.cpu(), rstd)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, max_ulp=None, what="dx")
    torch.testing.assert_close(w.grad.cpu(), dw_ref, atol=2e-3 * M ** 0.5, rtol=1e-3)


@pytest.mark.parametrize("N", [131072, 262144])
def test_rmsnorm_large_tensor(N):
    """More than 2**32 elements per tensor (reference: tests/test_rmsnorm.py:294-335): 64-bit row
    offsets in the kernels.  Checked in row blocks against the fp32 formulas on the GPU."""
    M = 32 * 1024
    need = 2 * M * N * 2 + (2 << 30)
    torch.cuda.empty_cache()
    if need > torch.cuda.mem_get_info()[0] * 0.9:
        pytest.skip("not enough free device memory")
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    for blk in x.chunk(16):
        blk.copy_(torch.randn(blk.shape, device=DEV, generator=g))
    w = torch.randn(N, device=DEV, generator=g)
    out = rn.rmsnorm(x, w, eps=1e-5)
    # first, middle and last row blocks (the last one lies beyond 2**32 elements)
    for lo in (0, M // 2 - 64, M - 128):
        xs = x[lo:lo + 128]
        ref = oracle.rmsnorm_ref(xs, w, eps=1e-5, out_dtype=torch.float32)
        assert_close_to_oracle(out[lo:lo + 128], ref, torch.bfloat16, what=f"out rows {lo}..")
    del out, x


def test_rmsnorm_compile_2d_then_4d():
    """torch.compile(rmsnorm) called with a 2-D input and then, without a dynamo reset, with a 4-D
    per-head input plus bias and residual (reference: tests/test_rmsnorm.py:168-207)."""
    torch._dynamo.reset()
    f = torch.compile(rn.rmsnorm, fullgraph=True)
    x = torch.randn(32, 256, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(256, device=DEV, requires_grad=True)
    out = f(x, w, eps=1e-5)
    out.sum().backward()
    ref = oracle.rmsnorm_ref(x.detach().cpu(), w.detach().cpu(), eps=1e-5, out_dtype=torch.float32)
    assert_close_to_oracle(out.detach(), ref, torch.bfloat16, what="out 2d")
    rstd = oracle.rmsnorm_rstd_ref(x.detach().cpu(), eps=1e-5)
    dx_ref, _, _ = oracle.rmsnorm_bwd_ref(x.detach().cpu(), w.detach().cpu(), torch.ones(32, 256), rstd)
    assert_close_to_oracle(x.grad, dx_ref, torch.bfloat16, max_ulp=None, what="dx 2d")

    x4 = torch.randn(2, 16, 4, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w2 = torch.randn(4, 64, device=DEV, requires_grad=True)
    b2 = torch.randn(4, 64, device=DEV, requires_grad=True)
    r4 = torch.randn(2, 16, 4, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out2 = f(x4, w2, bias=b2, residual=r4, eps=1e-6)
    out2.sum().backward()
    # per-head oracle: head h of every token uses row h of the (4, 64) parameters
    xr, rr = x4.detach().cpu().float().requires_grad_(), r4.detach().cpu().float().requires_grad_()
    wr, br = w2.detach().cpu().clone().requires_grad_(), b2.detach().cpu().clone().requires_grad_()
    h = xr.bfloat16().float() + rr.bfloat16().float()
    o_ref = h * torch.rsqrt(h.square().mean(-1, keepdim=True) + 1e-6) * wr + br
    o_ref.sum().backward()
    assert_close_to_oracle(out2.detach(), o_ref.detach(), torch.bfloat16, what="out 4d")
    torch.testing.assert_close(x4.grad.float().cpu(), xr.grad, atol=1e-1, rtol=1e-2)
    torch.testing.assert_close(r4.grad.float().cpu(), rr.grad, atol=1e-1, rtol=1e-2)
    torch.testing.assert_close(w2.grad.cpu(), wr.grad, atol=2e-2 * 32 ** 0.5, rtol=1e-2)
    torch.testing.assert_close(b2.grad.cpu(), br.grad, atol=2e-2 * 32 ** 0.5, rtol=1e-2)


@pytest.mark.parametrize("is_layernorm", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [1536, 2560, 3072, 3584, 5120, 7168, 10240, 14336])
def test_norm_backward_rows_of_three_five_six_seven_chunks(N, dtype, is_layernorm, monkeypatch):
    """Hidden sizes whose 16-byte chunk count is 3, 5, 6 or 7 times the threads of a row are served
    by backward kernels with exactly that many chunks per thread (no padding chunks).  dx against
    the oracle, dw / db against its column sums, for several rows per CTA and a single row; the
    padded 8-chunk kernel (flag bit 1) must give bit-identical dx."""
    from quack_flydsl_b200 import _C
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    g = torch.Generator(device=DEV).manual_seed(N)
    for M in (333, 1):
        x = (0.3 + torch.randn(M, N, device=DEV, generator=g)).to(dtype)
        w = (1 + 0.1 * torch.randn(N, device=DEV, generator=g)).to(dtype)
        dout = torch.randn(M, N, device=DEV, generator=g).to(dtype)
        xc = x.cpu()
        if is_layernorm:
            rstd_c, mean_c = oracle.layernorm_rstd_ref(xc, eps=1e-5), oracle.layernorm_mean_ref(xc)
            dx_ref, dw_ref, db_ref = oracle.layernorm_bwd_ref(xc, w.cpu(), dout.cpu(), rstd_c, mean_c)
        else:
            rstd_c, mean_c = oracle.rmsnorm_rstd_ref(xc, eps=1e-6), None
            dx_ref, dw_ref, db_ref = oracle.rmsnorm_bwd_ref(xc, w.cpu(), dout.cpu(), rstd_c)
        rstd = rstd_c.to(DEV)
        mean = mean_c.to(DEV) if is_layernorm else None
        P = get_sm_count(N, torch.device(DEV), dtype)
        results = {}
        for padded in (False, True):
            dx = torch.full_like(x, 7.0)
            dwp = torch.full((P, N), 7.0, device=DEV)
            dbp = torch.full((P, N), 7.0, device=DEV) if is_layernorm else None
            if padded:
                monkeypatch.setenv("QUACK_B200_CFG", "norm_bwd:0:0:0:0:0:1")
            else:
                monkeypatch.delenv("QUACK_B200_CFG", raising=False)
            rn._rmsnorm_bwd(x, w, dout, rstd, dx, dwp, dbp, None, None, P, mean, is_layernorm)
            results[padded] = (dx, dwp.sum(0), dbp.sum(0) if is_layernorm else None, _C.last_kernel())
        monkeypatch.delenv("QUACK_B200_CFG", raising=False)
        dx, dw, db, kernel = results[False]
        assert torch.equal(dx, results[True][0]), (kernel, results[True][3])
        assert_close_to_oracle(dx, dx_ref, dtype, max_ulp=None, what="dx")
        sum_atol = 1e-3 * (M ** 0.5) * 4
        torch.testing.assert_close(dw.cpu(), dw_ref.float(), atol=sum_atol, rtol=1e-2)
        if is_layernorm:
            torch.testing.assert_close(db.cpu(), db_ref.float(), atol=sum_atol, rtol=1e-2)
