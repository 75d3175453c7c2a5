"""Helpers shared by the GPU parity tests."""

import torch

import oracle

# reference test tolerances (tests/test_rmsnorm.py:22-26, tests/test_softmax.py:16-21)
ATOL = {torch.bfloat16: 1e-1, torch.float16: 1e-2, torch.float32: 1e-4}


def oracle_device(*tensors, limit=48 * 2**20):
    """The oracle runs on the CPU for everything it finishes in seconds; for the few huge cases the
    same plain-PyTorch fp32 formulas are evaluated on the GPU instead."""
    n = max(t.numel() for t in tensors if t is not None)
    return "cpu" if n <= limit else "cuda"


def to(dev, *tensors):
    return [None if t is None else t.detach().to(dev) for t in tensors]


# Elements that passed only through the absolute floor below, over all calls of this process
# (reported by the ``floor_report`` fixture at the end of a test session).
FLOOR_STATS = {"elements": 0, "floored": 0}
MAX_FLOOR_FRACTION = 1e-4


def assert_close_to_oracle(got, ref_f32, dtype, atol=None, rtol=1e-3, max_ulp=2, what=""):
    """got: kernel output (any float dtype); ref_f32: oracle result before the final rounding.
    bf16: at most ``max_ulp`` bf16 ulps from the rounded oracle value; elements further away must
    be within an absolute floor of 1e-5 * max|ref| (results of a cancellation), and at most
    MAX_FLOOR_FRACTION of a tensor's elements may take that exit.  Other dtypes: the reference
    tests' atol / rtol.  Returns the number of elements that needed the floor."""
    ref = ref_f32.to(got.device)
    assert got.shape == ref.shape, f"{what}: shape {tuple(got.shape)} vs {tuple(ref.shape)}"
    assert got.dtype == dtype, f"{what}: dtype {got.dtype} vs {dtype}"
    assert torch.isfinite(got.float()).all(), f"{what}: non-finite values"
    if dtype == torch.bfloat16 and max_ulp is not None:
        want = ref.to(torch.bfloat16)
        floored = 0
        for g, w in zip(got.reshape(-1).split(1 << 24), want.reshape(-1).split(1 << 24)):
            d = oracle.bf16_ulp_diff(g, w)
            bad = d > max_ulp
            if bad.any():
                # An output that is itself the result of a cancellation (x_hat * w + b ~ 0, or
                # x - mean ~ 0) carries the fp32 rounding noise of its operands, which can be many
                # ulps of the tiny result: such elements are held to an absolute floor instead.
                floor = 1e-5 * max(1.0, float(ref.abs().max()))
                big = bad & ((g.float() - w.float()).abs().cpu() > floor)
                assert not big.any(), (
                    f"{what}: {int(big.sum())} elements differ by more than {max_ulp} bf16 ulp "
                    f"(max {int(d[big].max())}) and by more than {floor:.1e}")
                floored += int(bad.sum())
        FLOOR_STATS["elements"] += got.numel()
        FLOOR_STATS["floored"] += floored
        assert floored <= max(2, MAX_FLOOR_FRACTION * got.numel()), (
            f"{what}: {floored} of {got.numel()} elements are more than {max_ulp} bf16 ulp off and "
            f"pass only through the absolute floor")
        return floored
    else:
        a = ATOL[dtype] if atol is None else atol
        if atol is None and dtype != torch.float32:
            # gradients: two roundings of the largest magnitude instead of the reference's flat atol
            a = min(a, 2 * torch.finfo(dtype).eps * max(float(ref.abs().max()), 1e-3))
            rtol = max(rtol, 2 * torch.finfo(dtype).eps)
        for g, w in zip(got.reshape(-1).split(1 << 24), ref.reshape(-1).split(1 << 24)):
            torch.testing.assert_close(g.float(), w.to(dtype).float(), atol=a, rtol=rtol, msg=lambda m: f"{what}: {m}")
    return 0
