"""CPU tests of the op wrapper, after the reference's tests/test_torch_library_op.py:63-236: the
fake implementation never runs the body, eager calls bypass the dispatcher, compiled graphs go
through the registered op, attribute access reaches the CustomOpDef."""

import torch

from quack_flydsl_b200.dsl import cute_op, kernel_op

CALLS = {"body": 0}


@kernel_op("quack_b200_test::scale_into", mutates_args={"out"})
def scale_into(x: torch.Tensor, out: torch.Tensor, k: float = 2.0) -> None:
    CALLS["body"] += 1
    out.copy_(x * k)


def test_alias_is_same_decorator():
    assert cute_op is kernel_op


def test_eager_runs_body_directly():
    CALLS["body"] = 0
    x = torch.arange(6.0)
    out = torch.empty_like(x)
    assert scale_into(x, out, 3.0) is None
    assert CALLS["body"] == 1
    torch.testing.assert_close(out, x * 3)


def test_registered_op_exists_and_mutates():
    x = torch.arange(4.0)
    out = torch.zeros_like(x)
    torch.ops.quack_b200_test.scale_into(x, out, 2.0)
    torch.testing.assert_close(out, x * 2)
    # attribute access falls through to the CustomOpDef
    assert scale_into._opoverload is torch.ops.quack_b200_test.scale_into.default
    assert scale_into.__name__ == "scale_into"


def test_fake_is_a_noop():
    from torch._subclasses.fake_tensor import FakeTensorMode

    CALLS["body"] = 0
    with FakeTensorMode():
        x = torch.empty(8)
        out = torch.empty(8)
        torch.ops.quack_b200_test.scale_into(x, out, 2.0)
    assert CALLS["body"] == 0


def test_compile_routes_through_the_op():
    def f(x):
        out = torch.empty_like(x)
        scale_into(x, out, 4.0)
        return out + 1

    CALLS["body"] = 0
    g = torch.compile(f, fullgraph=True, backend="aot_eager")
    x = torch.arange(5.0)
    torch.testing.assert_close(g(x), x * 4 + 1)
    assert CALLS["body"] == 1  # once at run time, never while tracing
    x2 = torch.arange(7.0)  # dynamic shape re-use
    torch.testing.assert_close(g(x2), x2 * 4 + 1)


def test_hot_path_ops_are_registered():
    import quack_flydsl_b200.cross_entropy  # noqa: F401
    import quack_flydsl_b200.rmsnorm  # noqa: F401
    import quack_flydsl_b200.softmax  # noqa: F401

    for name in ("_rmsnorm_fwd", "_rmsnorm_bwd", "_softmax_fwd", "_softmax_backward",
                 "cross_entropy_fwd_out", "cross_entropy_bwd_out", "_norm_bwd_colsum"):
        assert hasattr(torch.ops.quack, name), name
    schema = str(torch.ops.quack._rmsnorm_fwd.default._schema)
    assert "Tensor(a2!) out" in schema and "Tensor(a7!)? residual_out" in schema
    schema = str(torch.ops.quack._rmsnorm_bwd.default._schema)
    assert "Tensor(a5!)? dw_partial" in schema and "int? sm_count=None" in schema
