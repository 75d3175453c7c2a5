"""Generates tests/golden/*.pt: inputs and outputs of the reference's own CPU-runnable code.

Run where a checkout of the reference project is available:

    python tests/golden/make_golden.py --reference <path to the reference tree>

What is executed:
* ``rmsnorm_ref``, ``rmsnorm_bwd_ref``, ``layernorm_ref``, ``layernorm_rstd_ref``,
  ``layernorm_mean_ref`` -- the FunctionDef nodes are cut out of the reference's
  ``quack/rmsnorm.py`` with ``ast`` (the module itself cannot be imported without its CuTe-DSL
  dependency) and executed unmodified in a namespace that only holds ``torch``;
* the PyTorch calls the reference's tests use as ground truth for the ops that have no
  reference function: ``F.layer_norm`` + autograd (tests/test_layernorm.py:64-74), ``F.softmax``
  + autograd (tests/test_softmax.py:53-57), ``F.cross_entropy`` / ``torch.logsumexp`` + autograd
  (tests/test_cross_entropy.py:51,64-66,288).
* ``linear_cross_entropy_func_ref`` cut out of ``quack/linear_cross_entropy.py`` the same way and
  run with autograd on CPU (fp32 upcast, as tests/test_linear_cross_entropy.py:33-35 does), and
  the closed form the reference's ``rms_final_reduce`` test compares with
  (tests/test_linear.py:793-803).
* ``torch.topk`` (largest, sorted) + ``torch.softmax`` over the k values + autograd, the ground
  truth of the reference's top-k test (tests/test_topk.py:40-80); needs no reference checkout:
  ``python tests/golden/make_golden.py --only topk``.
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


def load_linear_ce_ref(ref_root: Path):
    from typing import Literal, Optional

    src = (ref_root / "quack" / "linear_cross_entropy.py").read_text()
    ns = {"torch": torch, "Tensor": torch.Tensor, "F": F, "Optional": Optional, "Literal": Literal}
    for node in ast.parse(src).body:
        if isinstance(node, ast.FunctionDef) and node.name == "linear_cross_entropy_func_ref":
            exec(compile(ast.Module(body=[node], type_ignores=[]), "reference:linear_ce", "exec"), ns)
    return ns["linear_cross_entropy_func_ref"]


def gen_linear_ce(ref_root: Path) -> dict:
    fn = load_linear_ce_ref(ref_root)
    g = torch.Generator().manual_seed(4)
    cases = []
    for M, d, V, dt, red, ign in [(16, 64, 512, torch.bfloat16, "mean", False),
                                  (24, 32, 1000, torch.bfloat16, "sum", True),
                                  (8, 64, 640, torch.float32, "mean", True)]:
        x = (0.1 * torch.randn(M, d, generator=g)).to(dt)
        w = (torch.randn(V, d, generator=g) / d ** 0.5).to(dt)
        target = torch.randint(0, V, (M,), generator=g)
        ignore_index = V - 1 if ign else -100
        if ign:
            target[torch.rand(M, generator=g) < 0.3] = ignore_index
            target[1] = ignore_index
        xr, wr = x.float().clone().requires_grad_(), w.float().clone().requires_grad_()
        loss = fn(xr, wr, None, target, ignore_index=ignore_index, reduction=red)
        loss.backward()
        cases.append(dict(x=x, weight=w, target=target, ignore_index=ignore_index, reduction=red,
                          loss=loss.detach(), dx=xr.grad, dw=wr.grad))
    rms = []
    for M, N, dt in [(37, 1, torch.float32), (37, 16, torch.bfloat16), (5, 100, torch.float32)]:
        x = torch.randn(M, N, generator=g).abs().to(dt)
        scale, eps = 1.0 / 4096, 1e-6
        rms.append(dict(x=x, scale=scale, eps=eps,
                        rstd=torch.rsqrt(x.float().sum(dim=-1) * scale + eps)))
    return {"linear_cross_entropy": cases, "rms_final_reduce": rms}


def gen_topk() -> dict:
    g = torch.Generator().manual_seed(4)
    cases = []
    for M, N, k, dt, softmax in [
        (5, 64, 16, torch.float32, False), (3, 128, 32, torch.bfloat16, True),
        (4, 256, 16, torch.float16, False), (2, 1024, 32, torch.bfloat16, False),
        (3, 4096, 128, torch.bfloat16, True), (2, 4096, 64, torch.float32, True),
        (3, 2048, 8, torch.float32, False), (6, 32, 1, torch.float16, True),
    ]:
        x = torch.randn(M, N, generator=g).to(dt).requires_grad_()
        vals, idx = torch.topk(x, k, dim=-1, largest=True, sorted=True)
        out = torch.softmax(vals.float(), dim=-1).to(dt) if softmax else vals
        dvalues = torch.randn(M, k, generator=g).to(dt)
        (dx,) = torch.autograd.grad(out, x, dvalues)
        cases.append(dict(x=x.detach(), k=k, softmax=softmax, values=out.detach(), indices=idx.to(torch.int32),
                          dvalues=dvalues, dx=dx))
    return {"topk": cases}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None, help="regenerate one fixture file only (topk)")
    ap.add_argument("--reference", default=None, help="root of the reference project checkout")
    args = ap.parse_args()
    torch.manual_seed(0)
    torch.set_num_threads(1)  # fixed summation order in the generating run
    if args.only in (None, "topk"):
        torch.save(gen_topk(), HERE / "topk_golden.pt")
        print("topk_golden.pt", (HERE / "topk_golden.pt").stat().st_size, "bytes")
    if args.only == "topk":
        return
    if args.reference is None:
        ap.error("--reference is required for everything but --only topk")
    ref = load_reference_functions(Path(args.reference))
    torch.save({**gen_norm(ref), **gen_layernorm(ref)}, HERE / "norm_golden.pt")
    torch.save({**gen_softmax(), **gen_cross_entropy()}, HERE / "softmax_ce_golden.pt")
    torch.save(gen_linear_ce(Path(args.reference)), HERE / "linear_ce_golden.pt")
    for f in ("norm_golden.pt", "softmax_ce_golden.pt", "linear_ce_golden.pt"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
