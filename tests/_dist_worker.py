"""Worker of the multi-GPU test (one process per GPU, NCCL): row-sharded RMSNorm backward with the
dw / db all-reduce and vocabulary-sharded cross-entropy, each checked against the unsharded CPU
oracle on rank 0's copy of the global problem."""

import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import oracle  # noqa: E402
from quack_flydsl_b200 import sharded  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl")
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator().manual_seed(0)
    M, N = 1024, 8192
    x = torch.randn(M, N, generator=g).bfloat16()
    dout = torch.randn(M, N, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(N, generator=g)).bfloat16()
    rstd = oracle.rmsnorm_rstd_ref(x)
    b, e = sharded.row_shard(M, rank, world)
    dx, dw, db, _ = sharded.norm_bwd_row_sharded(x[b:e].to(dev), w.to(dev), dout[b:e].to(dev),
                                                 rstd[b:e].to(dev), has_bias=True)
    dx_ref, dw_ref, db_ref = oracle.rmsnorm_bwd_ref(x, w, dout, rstd, has_bias=True)
    tol = 2 * 2 ** -8
    ok = torch.allclose(dx.float().cpu(), dx_ref[b:e].bfloat16().float(), atol=tol * float(dx_ref.abs().max()), rtol=1e-2)
    ok &= torch.allclose(dw.float().cpu(), dw_ref.bfloat16().float(), atol=tol * float(dw_ref.abs().max()), rtol=1e-2)
    ok &= torch.allclose(db.float().cpu(), db_ref.bfloat16().float(), atol=tol * float(db_ref.abs().max()), rtol=1e-2)
    # every rank must hold bit-identical parameter gradients
    gathered = [torch.empty_like(dw) for _ in range(world)]
    dist.all_gather(gathered, dw)
    ok &= all(torch.equal(gathered[0], t) for t in gathered)

    # The fused column-sum + peer all-reduce kernel against the same sum through NCCL: LayerNorm
    # partials (two buffers), several steps in a row so that both parities and the step counter
    # are exercised; every rank must obtain the same bits.
    import importlib
    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    par = sharded.PeerAllReduce(dev, cap_cols=2 * N)
    gp = torch.Generator(device=dev).manual_seed(100 + rank)
    for step in range(5):
        P = 37 + step
        dwp = torch.randn(P, N, device=dev, generator=gp)
        dbp = torch.randn(P, N, device=dev, generator=gp)
        o32 = torch.empty(2, N, device=dev)
        o16 = torch.empty(2, N, device=dev, dtype=torch.bfloat16)
        par.reduce([dwp, dbp], outs=[o16[0], o16[1]], outs_f32=[o32[0], o32[1]])
        ref = torch.empty(2, N, device=dev)
        rn._norm_bwd_colsum(dwp, ref[0])
        rn._norm_bwd_colsum(dbp, ref[1])
        parts = [torch.empty_like(ref) for _ in range(world)]
        dist.all_gather(parts, ref)
        tot = parts[0].clone()
        for t in parts[1:]:
            tot += t  # rank order, like the kernel
        ok &= torch.equal(o32, tot)
        ok &= torch.equal(o16, tot.bfloat16())
    ok &= par.timeouts() == 0
    par.close()

    # The fused exchange + fold of the vocabulary-sharded row statistics against all-gather +
    # ce_combine: bit-identical loss and lse on every rank, several steps on one set of buffers.
    Ms = 3000
    pce = sharded.PeerAllReduce(dev, cap_cols=3 * Ms + 32)
    gc = torch.Generator(device=dev).manual_seed(7)
    tgt = torch.randint(0, 100, (Ms,), device=dev, generator=gc)
    tgt[::11] = -100
    for step in range(4):
        st = torch.randn(3, Ms, device=dev, generator=gp)
        st[1].abs_().add_(0.25)
        loss_f, lse_f = pce.ce_combine(st, tgt)
        loss_r, lse_r = sharded.ce_combine(sharded.gather_ce_stats(st), tgt)
        ok &= torch.equal(loss_f, loss_r) and torch.equal(lse_f, lse_r)
    ok &= pce.timeouts() == 0
    pce.close()

    Mc, Nc = 256, 128256
    logits = (2 * torch.randn(Mc, Nc, generator=g)).bfloat16()
    target = torch.randint(0, Nc, (Mc,), generator=g)
    target[::9] = -100
    cb, ce_ = sharded.vocab_shard(Nc, rank, world)
    xs = logits[:, cb:ce_].contiguous().to(dev).requires_grad_()
    loss = sharded.cross_entropy_vocab_parallel(xs, target.to(dev), cb, reduction="mean")
    loss.backward()
    loss_ref, lse_ref = oracle.cross_entropy_ref(logits, target)
    nvalid = int((target != -100).sum())
    ok &= torch.allclose(loss.detach().cpu(), loss_ref.sum() / nvalid, atol=0, rtol=1e-5)
    dx_ref = oracle.cross_entropy_bwd_ref(logits[:, cb:ce_].float(), target, torch.full((Mc,), 1.0 / nvalid),
                                          lse_ref, col_offset=cb)
    ok &= bool((oracle.bf16_ulp_diff(xs.grad, dx_ref.bfloat16()) <= 2).all())
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    if rank == 0:
        print("DIST_WORKER_PASS" if int(flag) == 1 else "DIST_WORKER_FAIL", flush=True)
    dist.destroy_process_group()
    sys.exit(0 if int(flag) == 1 else 1)


if __name__ == "__main__":
    main()
