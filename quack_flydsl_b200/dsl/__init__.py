from quack_flydsl_b200.dsl.torch_library_op import cute_op, kernel_op

__all__ = ["cute_op", "kernel_op"]
