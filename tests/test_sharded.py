"""Multi-rank paths.  CPU (gloo, world_size 2): the exchange logic of row-sharded norm backward
and vocabulary-sharded cross-entropy, with the oracle standing in for the local kernels.  GPU: the
shard kernels (statistics, combine, local backward) against the unsharded oracle, all shards
emulated on one device; and, when the box has >= 2 GPUs, the real NCCL path under torchrun."""

import importlib
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from _util import assert_close_to_oracle

sharded = importlib.import_module("quack_flydsl_b200.sharded")
ROOT = Path(__file__).resolve().parents[1]


def _gloo_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)  # same global problem on every rank
        M, N = 64, 1000
        x = torch.randn(M, N)
        dout = torch.randn(M, N)
        w = torch.randn(N)
        # --- row-sharded norm backward: local fp32 dw/db, one all-reduce, round afterwards ---
        b, e = sharded.row_shard(M, rank, world)
        rstd = oracle.rmsnorm_rstd_ref(x)
        _, dw_loc, db_loc = oracle.rmsnorm_bwd_ref(x[b:e], w, dout[b:e], rstd[b:e], has_bias=True)
        dw, db = sharded.allreduce_param_grads(dw_loc.float(), db_loc.float())
        _, dw_ref, db_ref = oracle.rmsnorm_bwd_ref(x, w, dout, rstd, has_bias=True)
        ok = torch.allclose(dw, dw_ref, atol=1e-4, rtol=1e-5) and torch.allclose(db, db_ref, atol=1e-4, rtol=1e-5)
        # dw only
        dw2, none = sharded.allreduce_param_grads(dw_loc.float(), None)
        ok = ok and none is None and torch.allclose(dw2, dw_ref, atol=1e-4, rtol=1e-5)
        # --- vocabulary-sharded cross-entropy: stats -> all-gather -> fold in rank order ---
        t = torch.randint(0, N, (M,))
        t[5] = -100
        cb, ce_ = sharded.vocab_shard(N, rank, world)
        stats = oracle.cross_entropy_shard_stats_ref(x[:, cb:ce_], t, cb)
        allstats = sharded.gather_ce_stats(stats)
        ok = ok and allstats.shape == (world, 3, M) and torch.equal(allstats[rank], stats)
        loss, lse = oracle.cross_entropy_combine_ref(allstats, t)
        loss_ref, lse_ref = oracle.cross_entropy_ref(x, t)
        ok = ok and torch.allclose(loss, loss_ref, atol=2e-6, rtol=1e-6) and torch.allclose(lse, lse_ref, atol=2e-6, rtol=1e-6)
        results[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


def test_exchange_logic_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = 29500 + os.getpid() % 2000
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert dict(results) == {0: True, 1: True}


def test_single_process_exchange_is_identity():
    dw, db = torch.randn(8), torch.randn(8)
    a, b = sharded.allreduce_param_grads(dw, db)
    assert torch.equal(a, dw) and torch.equal(b, db)
    st = torch.randn(3, 5)
    assert torch.equal(sharded.gather_ce_stats(st)[0], st)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [2, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_vocab_sharded_kernels_match_unsharded_oracle(G, dtype):
    M, N = 193, 128256 if dtype == torch.bfloat16 else 5000
    dev = "cuda"
    x = (2 * torch.randn(M, N, device=dev)).to(dtype)
    t = torch.randint(0, N, (M,), device=dev)
    t[torch.rand(M, device=dev) < 0.05] = -100
    w = torch.rand(N, device=dev) + 0.1
    spans = [sharded.vocab_shard(N, r, G) for r in range(G)]
    stats = torch.stack([sharded.ce_shard_stats(x[:, b:e], t, b) for b, e in spans])
    for g, (b, e) in enumerate(spans):
        ref = oracle.cross_entropy_shard_stats_ref(x[:, b:e].cpu(), t.cpu(), b)
        torch.testing.assert_close(stats[g].cpu(), ref, atol=1e-6, rtol=1e-5)
    loss, lse = sharded.ce_combine(stats, t, weight=w)
    loss_ref, lse_ref = oracle.cross_entropy_ref(x.cpu(), t.cpu(), weight=w.cpu())
    torch.testing.assert_close(lse.cpu(), lse_ref, atol=0, rtol=1e-5)
    torch.testing.assert_close(loss.cpu(), loss_ref, atol=1e-6, rtol=1e-5)
    assert (loss[t == -100] == 0).all()
    dloss = torch.randn(M, device=dev)
    dx = torch.cat([sharded.ce_shard_bwd(x[:, b:e], t, dloss, lse, b, weight=w) for b, e in spans], dim=1)
    dx_ref = oracle.cross_entropy_bwd_ref(x.cpu().float(), t.cpu(), dloss.cpu(), lse_ref, weight=w.cpu())
    if dtype == torch.bfloat16:
        assert_close_to_oracle(dx, dx_ref, dtype, atol=1e-2, rtol=1.6e-2, max_ulp=None, what="dx")
    else:
        torch.testing.assert_close(dx.cpu(), dx_ref, atol=5e-5, rtol=1e-4)


@pytest.mark.gpu
def test_row_sharded_norm_bwd_single_rank_matches_unsharded():
    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    M, N = 512, 4096
    x = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, device="cuda", dtype=torch.bfloat16)
    dout = torch.randn_like(x)
    rstd = torch.rsqrt(x.float().square().mean(-1) + 1e-6)
    dx, dw, db, _ = sharded.norm_bwd_row_sharded(x, w, dout, rstd, has_bias=True)
    dx2, dw2, db2, _ = rn.rmsnorm_bwd(x, w, dout, rstd, has_bias=True)
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2) and torch.equal(db, db2)


@pytest.mark.gpu
def test_peer_allreduce_single_rank_equals_column_sum():
    """With one rank the fused column-sum + all-reduce kernel must reproduce qb_colsum bit for bit
    (same summation order over P), for one and for two partial buffers, over several steps."""
    rn = importlib.import_module("quack_flydsl_b200.rmsnorm")
    dev = torch.device("cuda", 0)
    par = sharded.PeerAllReduce(dev, cap_cols=8192)
    try:
        for step, (P, N, n) in enumerate([(296, 4096, 2), (148, 8192, 1), (5, 1000, 2), (1, 32, 1), (296, 4096, 2)]):
            parts = [torch.randn(P, N, device=dev) for _ in range(n)]
            o32 = [torch.empty(N, device=dev) for _ in range(n)]
            o16 = [torch.empty(N, device=dev, dtype=torch.bfloat16) for _ in range(n)]
            par.reduce(parts, outs=o16, outs_f32=o32)
            for i in range(n):
                ref = torch.empty(N, device=dev)
                rn._norm_bwd_colsum(parts[i], ref)
                assert torch.equal(o32[i], ref), (step, i)
                assert torch.equal(o16[i], ref.bfloat16()), (step, i)
        with pytest.raises(ValueError, match="exceed the exchange buffer"):
            par.reduce([torch.randn(4, 8192, device=dev), torch.randn(4, 8192, device=dev)])
        assert par.timeouts() == 0
    finally:
        par.close()


@pytest.mark.gpu
def test_peer_ce_combine_single_rank_equals_ce_combine():
    """With one rank the fused exchange + fold must reproduce qb_ce_combine bit for bit (ignored
    rows, class weights, a row whose shard is all -inf), repeatedly on the same buffers."""
    dev = torch.device("cuda", 0)
    par = sharded.PeerAllReduce(dev, cap_cols=3 * 1000 + 8)
    try:
        for M in (1000, 1, 257):
            stats = torch.randn(3, M, device=dev)
            stats[1].abs_().add_(0.5)
            if M > 5:
                stats[0, 5] = float("-inf")
                stats[1, 5] = 0.0
            V = 50
            target = torch.randint(0, V, (M,), device=dev)
            target[::7] = -100
            w = torch.rand(V, device=dev) + 0.5
            for weight in (None, w):
                loss, lse = par.ce_combine(stats, target, weight)
                loss2, lse2 = sharded.ce_combine(stats[None], target, weight)
                assert torch.equal(loss, loss2) and torch.equal(lse.nan_to_num(), lse2.nan_to_num())
        with pytest.raises(ValueError, match="exceed the exchange buffer"):
            par.ce_combine(torch.randn(3, 2000, device=dev), torch.zeros(2000, device=dev, dtype=torch.long))
        assert par.timeouts() == 0
    finally:
        par.close()


@pytest.mark.gpu
def test_multi_gpu_nccl_paths():
    """Launches tests/_dist_worker.py under torchrun on 2 GPUs, as the reference does for its own
    distributed tests (tests/test_distributed_gemm.py:363-389)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs >= 2 GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29700 + os.getpid() % 200),
           str(ROOT / "tests" / "_dist_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(ROOT))
    assert res.returncode == 0 and "DIST_WORKER_PASS" in res.stdout, res.stdout[-3000:] + res.stderr[-3000:]
