"""Pins the CPU oracle: every oracle function against the fixtures produced by the reference's
own PyTorch reference functions / ground-truth calls (tests/golden/make_golden.py) and against
the closed-form known answers of the reference's tests."""

import math

import torch

import oracle

TOL = {torch.float32: (1e-5, 1e-5), torch.float16: (2e-3, 2e-3), torch.bfloat16: (1.6e-2, 1.6e-2)}


def _close(a, b, dt=None, atol=None, rtol=None):
    at, rt = TOL[dt or a.dtype]
    torch.testing.assert_close(a.float(), b.float(), atol=atol or at, rtol=rtol or rt)


def test_rmsnorm_oracle_matches_reference_functions(norm_golden):
    for c in norm_golden["rmsnorm"]:
        got = oracle.rmsnorm_ref(c["x"], c["w"], bias=c["b"], residual=c["res"], eps=c["eps"],
                                 weight_offset=c["weight_offset"])
        out, res_out = got if c["res"] is not None else (got, None)
        # same formula, same fp32 arithmetic: outputs agree to the last rounding
        assert out.dtype == c["out"].dtype
        _close(out, c["out"], atol=1e-6 if out.dtype == torch.float32 else None)
        if res_out is not None:
            assert torch.equal(res_out, c["res_out"])  # x + residual rounded once: bit exact
        x_pre = c["x"] if c["res"] is None else c["res_out"]
        rstd = oracle.rmsnorm_rstd_ref(x_pre, eps=c["eps"])
        torch.testing.assert_close(rstd, c["rstd"], atol=0, rtol=1e-6)
        dx, dw, _ = oracle.rmsnorm_bwd_ref(x_pre, c["w"], c["dout"], c["rstd"],
                                           weight_offset=c["weight_offset"])
        _close(dx.to(c["dx"].dtype), c["dx"], atol=1e-6 if c["dx"].dtype == torch.float32 else None)
        if c["w"] is not None:
            _close(dw.to(c["dw"].dtype), c["dw"], atol=1e-5 if c["dw"].dtype == torch.float32 else None)


def test_layernorm_oracle_matches_reference_functions(norm_golden):
    for c in norm_golden["layernorm"]:
        out = oracle.layernorm_ref(c["x"], c["w"], eps=c["eps"])
        dt = c["x"].dtype
        _close(out, c["out"], atol=2e-5 if dt == torch.float32 else None)
        torch.testing.assert_close(oracle.layernorm_rstd_ref(c["x"], eps=c["eps"]), c["rstd"],
                                   atol=0, rtol=1e-6)
        torch.testing.assert_close(oracle.layernorm_mean_ref(c["x"]), c["mean"], atol=1e-7, rtol=1e-6)
        dx, dw, db = oracle.layernorm_bwd_ref(c["x"], c["w"], c["dout"], c["rstd"], c["mean"])
        _close(dx.to(dt), c["dx"], atol=2e-5 if dt == torch.float32 else None)
        torch.testing.assert_close(dw, c["dw"], atol=2e-4, rtol=1e-4)
        torch.testing.assert_close(db, c["db"], atol=1e-5, rtol=1e-5)


def test_layernorm_ragged_known_answer(norm_golden):
    # closed-form input of the reference's ragged-N regression (tests/test_layernorm.py:121-139)
    c = norm_golden["layernorm_ragged_known_answer"]
    M, N = 3, 769
    cols = torch.arange(N, dtype=torch.float32)
    rows = torch.arange(M, dtype=torch.float32).unsqueeze(1)
    x = 1000.0 + rows * 100.0 + ((cols % 17) - 8.0) / 8.0
    assert torch.equal(x, c["x"])
    # The fixture's `out` is the reference's layernorm_ref evaluated on CPU, i.e. F.layer_norm with
    # fp32 moments of values ~1000 +- 1; it carries ~1e-4 of summation error itself, the oracle
    # (float64 moments) does not.
    torch.testing.assert_close(oracle.layernorm_ref(x, c["w"], eps=c["eps"]), c["out"], atol=3e-4, rtol=0)
    torch.testing.assert_close(oracle.layernorm_rstd_ref(x, eps=c["eps"]), c["rstd"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(oracle.layernorm_mean_ref(x), c["mean"], atol=1e-5, rtol=1e-5)
    # independent closed form: the row offset does not change the variance
    r = ((cols % 17) - 8.0) / 8.0
    var = ((r - r.mean()) ** 2).mean().double()
    want = 1.0 / math.sqrt(var + 1e-5)
    assert abs(oracle.layernorm_rstd_ref(x, eps=1e-5, compute_dtype=torch.float64)[0].item() - want) < 1e-4


def test_softmax_oracle_matches_torch(softmax_ce_golden):
    for c in softmax_ce_golden["softmax"]:
        y = oracle.softmax_ref(c["x"])
        _close(y, c["y"], atol=1e-7 if y.dtype == torch.float32 else None)
        dx = oracle.softmax_bwd_ref(c["dy"], c["y"])
        _close(dx, c["dx"], atol=1e-6 if dx.dtype == torch.float32 else 2e-3)


def test_softmax_known_answers():
    # constant rows -> 1/N; shift invariance (tests/test_softmax.py:79-88, 99-110)
    for v in (10.0, -10.0):
        y = oracle.softmax_ref(torch.full((4, 1024), v))
        torch.testing.assert_close(y, torch.full_like(y, 1 / 1024), atol=1e-9, rtol=1e-6)
    x = torch.randn(8, 512)
    torch.testing.assert_close(oracle.softmax_ref(x), oracle.softmax_ref(x + 100.0), atol=1e-6, rtol=1e-6)


def test_cross_entropy_oracle_matches_torch(softmax_ce_golden):
    for c in softmax_ce_golden["cross_entropy"]:
        loss, lse = oracle.cross_entropy_ref(c["x"], c["target"], weight=c["weight"])
        torch.testing.assert_close(loss, c["loss"], atol=5e-6, rtol=1e-6)
        torch.testing.assert_close(lse, c["lse"], atol=5e-6, rtol=1e-6)
        assert (loss[c["target"] == -100] == 0).all()
        dx = oracle.cross_entropy_bwd_ref(c["x"], c["target"], c["dloss"], lse, weight=c["weight"])
        _close(dx, c["dx"], atol=1e-6 if dx.dtype == torch.float32 else None)
        assert (dx[c["target"] == -100] == 0).all()


def test_cross_entropy_known_answers():
    # equal logits -> log N; all ignored -> exactly 0 (tests/test_cross_entropy.py:136-147, 208-212)
    M, N = 16, 1024
    t = torch.randint(0, N, (M,))
    for v in (10.0, -10.0):
        loss, lse = oracle.cross_entropy_ref(torch.full((M, N), v), t)
        torch.testing.assert_close(loss, torch.full((M,), math.log(N)), atol=1e-5, rtol=1e-6)
    loss, _ = oracle.cross_entropy_ref(torch.randn(M, N), torch.zeros(M, dtype=torch.long), ignore_index=0)
    assert (loss == 0).all()


def test_sharded_combine_equals_unsharded():
    M, N, G = 11, 1000, 4
    x = 2 * torch.randn(M, N)
    t = torch.randint(0, N, (M,))
    t[3] = -100
    w = torch.rand(N) + 0.1
    per = -(-N // G)
    stats = torch.stack([oracle.cross_entropy_shard_stats_ref(x[:, g * per:(g + 1) * per], t, g * per)
                         for g in range(G)])
    loss, lse = oracle.cross_entropy_combine_ref(stats, t, weight=w)
    loss_ref, lse_ref = oracle.cross_entropy_ref(x, t, weight=w)
    torch.testing.assert_close(loss, loss_ref, atol=2e-6, rtol=1e-6)
    torch.testing.assert_close(lse, lse_ref, atol=2e-6, rtol=1e-6)
    # the local backward pieces concatenate to the full gradient
    dl = torch.randn(M)
    dx = torch.cat([oracle.cross_entropy_bwd_ref(x[:, g * per:(g + 1) * per], t, dl, lse_ref, weight=w,
                                                 col_offset=g * per) for g in range(G)], dim=1)
    torch.testing.assert_close(dx, oracle.cross_entropy_bwd_ref(x, t, dl, lse_ref, weight=w))


def test_bf16_ulp_distance():
    a = torch.tensor([1.0, -1.0, 0.0, 3.0], dtype=torch.bfloat16)
    b = torch.tensor([1.0078125, -1.0078125, 0.0, 3.0], dtype=torch.bfloat16)
    assert oracle.bf16_ulp_diff(a, b).tolist() == [1, 1, 0, 0]


def test_linear_cross_entropy_oracle_matches_reference_function(linear_ce_golden):
    # fixtures: the reference's linear_cross_entropy_func_ref + autograd on fp32-upcast inputs
    for c in linear_ce_golden["linear_cross_entropy"]:
        loss, dx, dw = oracle.linear_cross_entropy_ref(
            c["x"].float(), c["weight"].float(), c["target"], ignore_index=c["ignore_index"],
            reduction=c["reduction"])
        torch.testing.assert_close(loss.float(), c["loss"], atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(dx.float(), c["dx"], atol=1e-6, rtol=1e-4)
        torch.testing.assert_close(dw.float(), c["dw"], atol=1e-6, rtol=1e-4)


def test_rms_final_reduce_oracle_matches_closed_form(linear_ce_golden):
    for c in linear_ce_golden["rms_final_reduce"]:
        got = oracle.rms_final_reduce_ref(c["x"], c["scale"], c["eps"])
        torch.testing.assert_close(got, c["rstd"], atol=0, rtol=1e-6)
    # a single partial sum per row: rstd = rsqrt(x * scale + eps)
    x = torch.tensor([[4.0], [0.0]])
    torch.testing.assert_close(oracle.rms_final_reduce_ref(x, 0.25, 0.0)[0], torch.tensor(1.0))
    torch.testing.assert_close(oracle.rms_final_reduce_ref(x, 0.25, 1e-6)[1], torch.tensor(1000.0), rtol=1e-5, atol=0)
