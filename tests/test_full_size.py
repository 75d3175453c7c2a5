"""Parity at the exact benchmark sizes.

The five benchmark configurations at full size: RMSNorm fp32 [4096, 4096] (the CPU-runnable case),
LayerNorm bf16 [65536, 4096] forward and backward, the softmax sweep at M * N = 2^31 elements for
N = 4096 / 16384 / 65536 / 131072, and cross-entropy on bf16 [16384, 128256] logits (2.1e9
elements: element offsets beyond 2^31).  Inputs are seeded synthetic tensors with the benchmark's
value distributions, generated on the device (a CPU generator would need minutes for 2^31 values).

What is compared: blocks of rows at the start, in the middle and at the END of every tensor go
to the CPU oracle (bf16 results within 2 bf16 ulp, fp32 row statistics rtol 1e-5); per-row
statistics, parameter gradients and size-independent properties (rows of softmax sum to 1, rows of
dx sum to 0, ignored rows are exactly 0) are checked over the whole tensor against the oracle
formulas evaluated on the device in fp32 / fp64."""

import importlib

import pytest
import torch

import oracle
from _util import assert_close_to_oracle

pytestmark = pytest.mark.gpu

rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
ln = importlib.import_module("quack_flydsl_b200.layernorm")
sm = importlib.import_module("quack_flydsl_b200.softmax")
ce = importlib.import_module("quack_flydsl_b200.cross_entropy")
DEV = "cuda"
BF = torch.bfloat16


def _need_gb(gb):
    free, _ = torch.cuda.mem_get_info()
    if free < gb * 2**30:
        pytest.skip(f"needs {gb} GiB of free device memory")


def _randn(shape, scale=1.0, shift=0.0, dtype=BF, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    out = torch.empty(shape, device=DEV, dtype=dtype)
    rows = max(1, (1 << 26) // shape[-1])  # fp32 staging of 64 Mi elements at a time
    for r0 in range(0, shape[0], rows):
        blk = torch.randn((min(rows, shape[0] - r0),) + tuple(shape[1:]), device=DEV, generator=g)
        out[r0:r0 + rows] = (blk * scale + shift).to(dtype)
    return out


def _blocks(M, rows):
    """Row ranges at the start, in the middle and at the end of a tensor of M rows."""
    rows = min(rows, M)
    starts = sorted({0, max(0, M // 2 - rows // 2), M - rows})
    return [slice(s, s + rows) for s in starts]


def test_c1_rmsnorm_fp32_4096x4096_exact():
    d = oracle.make_config_inputs("c1", device=DEV)
    out, _, rstd = rn.rmsnorm_fwd(d["x"], d["weight"], eps=d["eps"], store_rstd=True)
    ref = oracle.rmsnorm_ref(d["x"].cpu(), d["weight"].cpu(), eps=d["eps"])
    torch.testing.assert_close(out.cpu(), ref, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(rstd.cpu(), oracle.rmsnorm_rstd_ref(d["x"].cpu(), eps=d["eps"]),
                               atol=0, rtol=1e-5)


def test_c3_layernorm_full_size_all_outputs():
    _need_gb(6)
    M, N, eps = 65536, 4096, 1e-5
    x = _randn((M, N), shift=0.5, seed=1)
    w = (1 + 0.1 * torch.randn(N, device=DEV)).to(BF)
    b = (0.1 * torch.randn(N, device=DEV)).to(BF)
    dout = _randn((M, N), seed=2)
    out = torch.empty_like(x)
    rstd, mean = torch.empty(M, device=DEV), torch.empty(M, device=DEV)
    rn._rmsnorm_fwd(x, w, out, b, rstd, mean, None, None, eps, True)
    # all rows of out / rstd / mean against the oracle formulas on the device (chunks of 4096 rows)
    for r0 in range(0, M, 4096):
        xs = x[r0:r0 + 4096]
        ref = oracle.layernorm_ref(xs, w, b, eps=eps, compute_dtype=torch.float32)
        d = oracle.bf16_ulp_diff(out[r0:r0 + 4096], ref)
        assert int(d.max()) <= 2 or float((out[r0:r0 + 4096].float() - ref.float()).abs()[
            (d > 2).to(DEV)].max()) < 1e-4, f"rows {r0}: {int(d.max())} ulp"
        torch.testing.assert_close(rstd[r0:r0 + 4096], oracle.layernorm_rstd_ref(xs, eps=eps), atol=0, rtol=1e-5)
        torch.testing.assert_close(mean[r0:r0 + 4096], oracle.layernorm_mean_ref(xs), atol=1e-6, rtol=1e-5)
    # row blocks against the CPU oracle
    for blk in _blocks(M, 512):
        ref = oracle.layernorm_ref(x[blk].cpu(), w.cpu(), b.cpu(), eps=eps)
        assert_close_to_oracle(out[blk], ref.float(), BF, what=f"out rows {blk}")
    dx, dw, db = ln._layernorm_bwd_impl(x, w, dout, rstd, mean, True, BF)
    # dw / db against fp64 column sums over ALL rows (device, chunked)
    dw_ref = torch.zeros(N, device=DEV, dtype=torch.float64)
    db_ref = torch.zeros(N, device=DEV, dtype=torch.float64)
    for r0 in range(0, M, 8192):
        xs, ds = x[r0:r0 + 8192].double(), dout[r0:r0 + 8192].double()
        xhat = (xs - mean[r0:r0 + 8192, None].double()) * rstd[r0:r0 + 8192, None].double()
        dw_ref += (ds * xhat).sum(0)
        db_ref += ds.sum(0)
    # fp32 accumulation over 65536 rows, then one rounding to bf16
    for got, ref, name in ((dw, dw_ref, "dw"), (db, db_ref, "db")):
        scale = float(ref.abs().max())
        err = (got.double() - ref).abs().max().item()
        assert err <= scale * 2.0**-8 + 0.05, f"{name}: max error {err} (scale {scale})"
    for blk in _blocks(M, 512):
        dx_ref, _, _ = oracle.layernorm_bwd_ref(x[blk].cpu(), w.cpu(), dout[blk].cpu(), rstd[blk].cpu(),
                                                mean[blk].cpu())
        assert_close_to_oracle(dx[blk], dx_ref.float(), BF, max_ulp=None, what=f"dx rows {blk}")
    # rows of dx sum to ~0 and are orthogonal to xhat (LayerNorm's two projections)
    for r0 in range(0, M, 8192):
        assert float(dx[r0:r0 + 8192].float().sum(-1).abs().max()) < 0.5


@pytest.mark.parametrize("N", [4096, 16384, 65536, 131072])
def test_c4_softmax_full_size(N):
    _need_gb(18)
    M = 2**31 // N
    x = _randn((M, N), scale=3.0, seed=3)
    y = sm.softmax_fwd(x)
    rows_per = max(1, 2**21 // N)
    for blk in _blocks(M, rows_per):
        assert_close_to_oracle(y[blk], oracle.softmax_ref(x[blk].cpu().float()), BF, what=f"y rows {blk}")
    step = max(1, 2**27 // N)
    for r0 in range(0, M, step):
        s = y[r0:r0 + step].float().sum(-1)
        torch.testing.assert_close(s, torch.ones_like(s), atol=6e-3, rtol=0)
    dy = _randn((M, N), seed=4)
    dx = sm.softmax_bwd(dy, y)
    del x
    for blk in _blocks(M, rows_per):
        ref = oracle.softmax_bwd_ref(dy[blk].cpu().float(), y[blk].cpu().float())
        assert_close_to_oracle(dx[blk], ref, BF, max_ulp=None, what=f"dx rows {blk}")
    for r0 in range(0, M, step):
        assert float(dx[r0:r0 + step].float().sum(-1).abs().max()) < 5e-2


def test_c5_cross_entropy_full_size():
    _need_gb(14)
    M, N = 16384, 128256
    x = _randn((M, N), scale=2.0, seed=5)
    g = torch.Generator(device=DEV).manual_seed(6)
    target = torch.randint(0, N, (M,), device=DEV, generator=g)
    target[torch.rand(M, device=DEV, generator=g) < 0.05] = -100
    target[-1] = N - 1   # the very last logit of the tensor is a target
    target[-2] = -100    # and the row before it is ignored
    loss, lse = ce.cross_entropy_fwd(x, target, return_lse=True)
    # every row: lse / loss against fp64 on the device
    lse_ref = torch.empty(M, device=DEV, dtype=torch.float64)
    for r0 in range(0, M, 512):
        lse_ref[r0:r0 + 512] = torch.logsumexp(x[r0:r0 + 512].double(), dim=-1)
    valid = target != -100
    tl = x[torch.arange(M, device=DEV), target.clamp(min=0)].double()
    loss_ref = torch.where(valid, lse_ref - tl, torch.zeros_like(lse_ref))
    torch.testing.assert_close(lse.double(), lse_ref, atol=0, rtol=1e-5)
    torch.testing.assert_close(loss.double(), loss_ref, atol=2e-5, rtol=1e-5)
    assert (loss[~valid] == 0).all()
    count = int(valid.sum())
    dloss = torch.full((M,), 1.0 / count, device=DEV)
    blocks = _blocks(M, 24)
    refs = []
    for blk in blocks:  # CPU oracle on row blocks (start, middle, end)
        l_ref, lse_cpu = oracle.cross_entropy_ref(x[blk].cpu(), target[blk].cpu())
        torch.testing.assert_close(loss[blk].cpu(), l_ref, atol=2e-5, rtol=1e-5)
        refs.append(oracle.cross_entropy_bwd_ref(x[blk].cpu().float(), target[blk].cpu(), dloss[blk].cpu(),
                                                 lse_cpu))
    # backward from the saved lse
    dx = ce.cross_entropy_bwd(x, target, dloss, lse)
    for blk, ref in zip(blocks, refs):
        assert_close_to_oracle(dx[blk], ref, BF, what=f"ce_bwd dx rows {blk}")
    assert (dx[~valid] == 0).all()
    del dx
    # loss + lse + dx in one launch (upstream gradient 1), out of place and in place
    refs1 = [oracle.cross_entropy_bwd_ref(x[blk].cpu().float(), target[blk].cpu(), torch.ones(24),
                                          lse[blk].cpu()) for blk in blocks]
    loss2, lse2, dx2 = ce.cross_entropy_fwd(x, target, return_lse=True, return_dx=True)
    torch.testing.assert_close(loss2, loss, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(lse2, lse, atol=1e-6, rtol=1e-6)
    for blk, ref in zip(blocks, refs1):
        assert_close_to_oracle(dx2[blk], ref, BF, what=f"ce_fwd dx rows {blk}")
    assert (dx2[~valid] == 0).all()
    keep = [dx2[blk].clone() for blk in blocks]
    del dx2
    loss3, dx3 = ce.cross_entropy_fwd(x, target, return_dx=True, inplace_backward=True)
    assert dx3 is x
    torch.testing.assert_close(loss3, loss, atol=1e-6, rtol=1e-6)
    for blk, k in zip(blocks, keep):
        assert torch.equal(dx3[blk], k), f"in-place dx differs from out-of-place dx in rows {blk}"
