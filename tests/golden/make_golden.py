"""Generates tests/golden/*.pt: inputs and outputs of the reference's own CPU-runnable code.

Run in a container where the reference tree is mounted (default /root/reference):

    python tests/golden/make_golden.py [--reference /root/reference]

What is executed:
* ``rmsnorm_ref``, ``rmsnorm_bwd_ref``, ``layernorm_ref``, ``layernorm_rstd_ref``,
  ``layernorm_mean_ref`` -- the FunctionDef nodes are cut out of the reference's
  ``quack/rmsnorm.py`` with ``ast`` (the module itself cannot be imported without its CuTe-DSL
  dependency) and executed unmodified in a namespace that only holds ``torch``;
* the PyTorch calls the reference's tests use as ground truth for the ops that have no
  reference function: ``F.layer_norm`` + autograd (tests/test_layernorm.py:64-74), ``F.softmax``
  + autograd (tests/test_softmax.py:53-57), ``F.cross_entropy`` / ``torch.logsumexp`` + autograd
  (tests/test_cross_entropy.py:51,64-66,288).
Inputs are stored next to the outputs, so the fixtures do not depend on RNG reproducibility.
"""

from __future__ import annotations

import argparse
import ast
from pathlib import Path

import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
WANTED = ("rmsnorm_ref", "rmsnorm_bwd_ref", "layernorm_ref", "layernorm_rstd_ref",
          "layernorm_mean_ref")


def load_reference_functions(ref_root: Path) -> dict:
    src = (ref_root / "quack" / "rmsnorm.py").read_text()
    tree = ast.parse(src)
    ns = {"torch": torch, "Tensor": torch.Tensor}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in WANTED:
            code = compile(ast.Module(body=[node], type_ignores=[]), f"reference:{node.name}", "exec")
            exec(code, ns)
    missing = [n for n in WANTED if n not in ns]
    if missing:
        raise RuntimeError(f"reference functions not found: {missing}")
    return {n: ns[n] for n in WANTED}


def gen_norm(ref) -> dict:
    g = torch.Generator().manual_seed(0)
    cases = []
    for M, N, dt, wdt, has_res, has_bias, off in [
        (7, 48, torch.float32, torch.float32, False, False, 0.0),
        (5, 192, torch.bfloat16, torch.float32, True, False, 0.0),
        (3, 760, torch.float16, torch.bfloat16, True, True, 0.0),
        (4, 1128, torch.bfloat16, torch.bfloat16, False, True, 1.0),
        (2, 2048, torch.bfloat16, torch.bfloat16, True, False, 0.0),
        (6, 769, torch.float32, None, False, False, 0.0),
    ]:
        x = torch.randn(M, N, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(N, generator=g)).to(wdt) if wdt is not None else None
        b = (0.1 * torch.randn(N, generator=g)).to(wdt) if has_bias and wdt is not None else None
        res = torch.randn(M, N, generator=g).to(dt) if has_res else None
        dout = torch.randn(M, N, generator=g).to(dt)
        eps = 1e-6
        fwd = ref["rmsnorm_ref"](x, w, bias=b, residual=res, eps=eps, weight_offset=off)
        out, res_out = fwd if has_res else (fwd, None)
        x_pre = x if res is None else res_out
        rstd = torch.rsqrt(x_pre.float().square().mean(dim=-1) + eps)
        dx, dw = ref["rmsnorm_bwd_ref"](x_pre, w, dout.float(), rstd, eps=eps, weight_offset=off)
        cases.append(dict(x=x, w=w, b=b, res=res, dout=dout, eps=eps, weight_offset=off, out=out,
                          res_out=res_out, rstd=rstd, dx=dx, dw=dw))
    return {"rmsnorm": cases}


def gen_layernorm(ref) -> dict:
    g = torch.Generator().manual_seed(1)
    cases = []
    for M, N, dt in [(7, 48, torch.float32), (5, 256, torch.bfloat16), (3, 1128, torch.float16),
                     (9, 1024, torch.float32)]:
        x = torch.randn(M, N, generator=g).to(dt)
        w = torch.randn(N, generator=g)
        dout = torch.randn(M, N, generator=g).to(dt)
        eps = 1e-6
        out = ref["layernorm_ref"](x, w, eps=eps)
        rstd = ref["layernorm_rstd_ref"](x, eps=eps)
        mean = ref["layernorm_mean_ref"](x)
        # backward ground truth as the reference test builds it: autograd through F.layer_norm
        xr = x.float().requires_grad_()
        wr = w.clone().requires_grad_()
        br = torch.zeros(N, requires_grad=True)
        F.layer_norm(xr, (N,), wr, br, eps=eps).backward(dout.float())
        cases.append(dict(x=x, w=w, dout=dout, eps=eps, out=out, rstd=rstd, mean=mean,
                          dx=xr.grad.to(dt), dw=wr.grad, db=br.grad))
    # closed-form known-answer input of tests/test_layernorm.py:121-139
    M, N, eps = 3, 769, 1e-5
    cols = torch.arange(N, dtype=torch.float32)
    rows = torch.arange(M, dtype=torch.float32).unsqueeze(1)
    x = 1000.0 + rows * 100.0 + ((cols % 17) - 8.0) / 8.0
    w = torch.ones(N)
    cases_ka = dict(x=x, w=w, eps=eps, out=ref["layernorm_ref"](x, w, eps=eps),
                    rstd=ref["layernorm_rstd_ref"](x, eps=eps), mean=ref["layernorm_mean_ref"](x))
    return {"layernorm": cases, "layernorm_ragged_known_answer": cases_ka}


def gen_softmax() -> dict:
    g = torch.Generator().manual_seed(2)
    cases = []
    for M, N, dt, scale in [(5, 192, torch.float32, 0.1), (3, 760, torch.bfloat16, 0.1),
                            (2, 4096, torch.float16, 0.1), (4, 1024, torch.bfloat16, 3.0)]:
        x = (scale * torch.randn(M, N, generator=g)).to(dt)
        dy = torch.randn(M, N, generator=g).to(dt)
        xr = x.clone().requires_grad_()
        y = F.softmax(xr, dim=-1)
        (dx,) = torch.autograd.grad(y, xr, grad_outputs=dy)
        cases.append(dict(x=x, dy=dy, y=y.detach(), dx=dx))
    return {"softmax": cases}


def gen_cross_entropy() -> dict:
    g = torch.Generator().manual_seed(3)
    cases = []
    for M, N, dt, has_w, ign in [(9, 192, torch.float32, False, False),
                                 (7, 668, torch.bfloat16, True, True),
                                 (5, 1128, torch.float16, False, True),
                                 (3, 4096, torch.bfloat16, True, False)]:
        x = (0.1 * torch.randn(M, N, generator=g)).to(dt)
        target = torch.randint(0, N, (M,), generator=g)
        if ign:
            target[torch.rand(M, generator=g) < 0.3] = -100
            target[0] = -100
        w = (torch.rand(N, generator=g) + 0.1) if has_w else None
        dloss = torch.randn(M, generator=g)
        xr = x.float().requires_grad_()
        loss = F.cross_entropy(xr, target, weight=w, reduction="none", ignore_index=-100)
        (dx,) = torch.autograd.grad(loss, xr, grad_outputs=dloss)
        lse = torch.logsumexp(x.float(), dim=-1)
        cases.append(dict(x=x, target=target, weight=w, dloss=dloss, loss=loss.detach(), lse=lse,
                          dx=dx.to(dt)))
    return {"cross_entropy": cases}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    args = ap.parse_args()
    torch.manual_seed(0)
    torch.set_num_threads(1)  # fixed summation order in the generating run
    ref = load_reference_functions(Path(args.reference))
    torch.save({**gen_norm(ref), **gen_layernorm(ref)}, HERE / "norm_golden.pt")
    torch.save({**gen_softmax(), **gen_cross_entropy()}, HERE / "softmax_ce_golden.pt")
    for f in ("norm_golden.pt", "softmax_ce_golden.pt"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
