"""Multi-GPU use of the row-reduction kernels: one process per GPU, torch.distributed (NCCL).

The reference has no multi-GPU path for these ops; rows are independent, so the forward kernels
and softmax / cross-entropy backward shard over rows with no communication at all.  Two steps need
an exchange:

* norm backward: every rank reduces dw / db over its own rows (fp32, deterministic two-stage
  reduction); one all-reduce(SUM) of the concatenated fp32 [dw | db] vector follows and the
  result is rounded to the parameter dtype afterwards, so every rank rounds the same sum;
* vocabulary-sharded cross-entropy: every rank holds a column slice of the logits and computes
  per-row (max, sum-exp, target logit); the (3, M) fp32 blocks are all-gathered and folded in rank
  order (the single-GPU analogue in the reference is the ``lse_partial`` mode,
  quack/cross_entropy.py:676-694); the backward is local given the global log-sum-exp.
"""

from __future__ import annotations

from ctypes import byref
from typing import Optional, Tuple

import torch
import torch.distributed as dist
from torch import Tensor

from quack_flydsl_b200 import _C


def row_shard(M: int, rank: int, world: int) -> Tuple[int, int]:
    """[begin, end) of the contiguous row block of ``rank`` when M rows are split over ``world``
    ranks (the first M % world ranks get one extra row)."""
    base, extra = divmod(M, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def vocab_shard(N: int, rank: int, world: int, multiple: int = 8) -> Tuple[int, int]:
    """[begin, end) of the column block of ``rank``; block starts are multiples of ``multiple``
    so that 16-bit rows stay 16-byte aligned."""
    per = -(-N // world)
    per = -(-per // multiple) * multiple
    begin = min(N, rank * per)
    return begin, min(N, begin + per)


def allreduce_param_grads(dw: Optional[Tensor], db: Optional[Tensor], group=None):
    """Sums fp32 parameter gradients over the ranks with ONE all-reduce of [dw | db].
    Returns fp32 tensors (views of the reduced buffer)."""
    parts = [t for t in (dw, db) if t is not None]
    if not parts:
        return dw, db
    for t in parts:
        assert t.dtype == torch.float32, "reduce in fp32, round afterwards"
    flat = torch.cat([t.reshape(-1) for t in parts]) if len(parts) > 1 else parts[0].reshape(-1).clone()
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out = []
    off = 0
    for t in parts:
        out.append(flat[off:off + t.numel()].view_as(t))
        off += t.numel()
    it = iter(out)
    return (next(it) if dw is not None else None), (next(it) if db is not None else None)


class PeerAllReduce:
    """Column sums of the norm backward's partial buffers added over the GPUs of one node by ONE
    kernel (``qb_colsum_allreduce``): stage 2 and the all-reduce of ``[dw | db]`` in a single
    launch, through plain stores into peer-mapped exchange buffers.  Every rank obtains
    bit-identical results.  Replaces ``_norm_bwd_colsum`` + ``dist.all_reduce`` (about 16 us of
    NCCL latency per step for a 32 KiB vector).

    Collective: construct it on every rank of ``group`` (one process per GPU, same node), call
    ``reduce`` on every rank the same number of times with the same shapes, and ``close`` it on
    every rank.  Calls must not overlap on one object (use one object per stream).
    """

    def __init__(self, device: torch.device, cap_cols: int = 32768, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > _C.QB_MAX_PEERS:
            raise ValueError(f"at most {_C.QB_MAX_PEERS} ranks")
        self.device = torch.device(device)
        self.cap_cols = -(-int(cap_cols) // 32) * 32
        self.seq = 0
        self.status = torch.zeros(1, device=self.device, dtype=torch.int32)
        lib = _C.lib()
        import ctypes
        local = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_C.QB_PEER_HANDLE_BYTES)
        self._local = None
        self._peers = [None] * self.world
        # A rank whose create or open fails still takes part in every collective of the set-up, so
        # that all ranks learn of the failure together and raise together (no rank is left waiting).
        error = None
        try:
            with torch.cuda.device(self.device):
                _C.check(lib.qb_peer_buffer_create(self.world, self.cap_cols, byref(local), handle),
                         "peer_buffer_create")
            self._local = local.value
            self._peers[self.rank] = self._local
        except Exception as exc:
            if self.world == 1:
                raise
            error = exc
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw if error is None else None, group=group)
            if error is None and all(h is not None for h in handles):
                try:
                    with torch.cuda.device(self.device):
                        for r in range(self.world):
                            if r == self.rank:
                                continue
                            peer = ctypes.c_void_p()
                            _C.check(lib.qb_peer_buffer_open(handles[r], byref(peer)), "peer_buffer_open")
                            self._peers[r] = peer.value
                except Exception as exc:
                    error = exc
            elif error is None:
                error = RuntimeError("a peer rank could not create its exchange buffer")
            # also the barrier: every buffer is mapped everywhere before the first store
            ok = torch.tensor([0 if error is not None else 1], device=self.device, dtype=torch.int32)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
            if int(ok) == 0:
                self._release()  # no kernel has run yet, and the all-reduce above was the barrier
                raise RuntimeError(f"PeerAllReduce set-up failed on at least one rank "
                                   f"(this rank: {error!r})")

    def reduce(self, partials, outs=None, outs_f32=None) -> None:
        """partials: one or two fp32 ``[P, cols]`` buffers of the same shape; outs / outs_f32:
        per buffer an output vector in the parameter dtype and / or in fp32 (entries may be None)."""
        partials = list(partials)
        n = len(partials)
        assert n in (1, 2)
        outs = list(outs) if outs is not None else [None] * n
        outs_f32 = list(outs_f32) if outs_f32 is not None else [None] * n
        p0 = partials[0]
        assert all(t.dtype == torch.float32 and t.is_contiguous() and t.shape == p0.shape for t in partials)
        cols = p0.numel() // p0.shape[0] if p0.shape[0] else 0
        self.seq += 1
        a = _C.ColsumAllreduceArgs()
        a.partial0 = p0.data_ptr()
        a.partial1 = partials[1].data_ptr() if n == 2 else None
        dt = None
        for i, (o, o32) in enumerate(zip(outs, outs_f32)):
            if o is not None:
                assert o.is_contiguous() and o.numel() == cols
                dt = o.dtype if dt is None else dt
                assert o.dtype == dt, "outputs share one dtype"
                setattr(a, f"out{i}", o.data_ptr())
            if o32 is not None:
                assert o32.dtype == torch.float32 and o32.is_contiguous() and o32.numel() == cols
                setattr(a, f"out{i}_f32", o32.data_ptr())
        for r in range(self.world):
            a.peers[r] = self._peers[r]
        a.status = self.status.data_ptr()
        a.P, a.cols, a.cap_cols = p0.shape[0], cols, self.cap_cols
        a.num_buffers = n
        a.out_dtype = _C.FLOAT_CODES[dt] if dt is not None else 0
        a.world, a.rank, a.seq = self.world, self.rank, self.seq
        _C.launch(_C.lib().qb_colsum_allreduce, a, p0, "colsum_allreduce")

    def ce_combine(self, stats: Tensor, target: Tensor, weight: Optional[Tensor] = None,
                   ignore_index: int = -100) -> Tuple[Tensor, Tensor]:
        """Vocabulary-sharded cross-entropy: exchanges this rank's (3, M) fp32 statistics with all
        ranks and folds them in rank order into (loss, lse), both fp32 (M,), in one kernel
        (``qb_ce_combine_exchange``) -- instead of ``gather_ce_stats`` + ``ce_combine``."""
        assert stats.dtype == torch.float32 and stats.dim() == 2 and stats.shape[0] == 3
        M = stats.shape[1]
        loss = torch.empty(M, device=stats.device, dtype=torch.float32)
        lse = torch.empty(M, device=stats.device, dtype=torch.float32)
        if M == 0:
            return loss, lse
        s_ = stats.contiguous()
        t_ = target.contiguous()
        w_ = weight.contiguous() if weight is not None else None
        self.seq += 1
        a = _C.CeCombineExchangeArgs()
        a.stats, a.target, a.weight = _C.ptr(s_), _C.ptr(t_), _C.ptr(w_)
        a.loss, a.lse = _C.ptr(loss), _C.ptr(lse)
        for r in range(self.world):
            a.peers[r] = self._peers[r]
        a.status = self.status.data_ptr()
        a.M, a.cap_cols = M, self.cap_cols
        a.ignore_index = int(ignore_index)
        a.num_classes = w_.numel() if w_ is not None else 0
        a.target_dtype = _C.INDEX_CODES[t_.dtype]
        a.weight_dtype = _C.float_code(w_)
        a.world, a.rank, a.seq = self.world, self.rank, self.seq
        _C.launch(_C.lib().qb_ce_combine_exchange, a, s_, "ce_combine_exchange")
        return loss, lse

    def timeouts(self) -> int:
        """Waits that gave up (0 in a healthy job); synchronises."""
        return int(self.status.item())

    def close(self) -> None:
        if self._local is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)  # nobody stores into a buffer that is being freed
        self._release()

    def _release(self) -> None:
        """Unmaps the peers' buffers and frees this rank's; no collective (the caller has made sure
        that no rank still stores into them)."""
        lib = _C.lib()
        with torch.cuda.device(self.device):
            for r, ptr in enumerate(self._peers):
                if r != self.rank and ptr is not None:
                    lib.qb_peer_buffer_close(ptr)
            if self._local is not None:
                lib.qb_peer_buffer_destroy(self._local)
        self._local = None
        self._peers = []


def gather_ce_stats(stats: Tensor, group=None) -> Tensor:
    """All-gathers the per-rank (3, M) fp32 blocks into (G, 3, M), in rank order."""
    assert stats.dtype == torch.float32 and stats.dim() == 2 and stats.shape[0] == 3
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    out = torch.empty((world,) + tuple(stats.shape), device=stats.device, dtype=stats.dtype)
    if world > 1:
        dist.all_gather_into_tensor(out.view(-1), stats.contiguous().view(-1), group=group)
    else:
        out[0].copy_(stats)
    return out


def norm_bwd_row_sharded(x, weight, dout, rstd, mean=None, dresidual_out=None, has_bias=False,
                         has_residual=False, weight_offset=0.0, group=None, peer=None):
    """Norm backward on this rank's rows followed by the dw / db all-reduce.
    Returns (dx, dw, db, dresidual) like ``rmsnorm_bwd`` (mean given => LayerNorm).
    ``peer``: a ``PeerAllReduce`` of the group; stage 2 and the all-reduce then run as one kernel
    instead of two column sums, a concatenation and an NCCL call."""
    from quack_flydsl_b200.rmsnorm import _finalize_partials, _rmsnorm_bwd
    from quack_flydsl_b200.rmsnorm_config import get_sm_count

    N = x.size(-1)
    dx = torch.empty_like(x)
    dresidual = None
    if dresidual_out is not None and dresidual_out.dtype != dx.dtype:
        dresidual = torch.empty_like(x, dtype=dresidual_out.dtype)
    P = get_sm_count(N, x.device, x.dtype)
    dw_partial = torch.empty(P, N, device=x.device, dtype=torch.float32) if weight is not None else None
    db_partial = torch.empty(P, N, device=x.device, dtype=torch.float32) if has_bias else None
    pdt = weight.dtype if weight is not None else x.dtype
    if peer is not None and x.numel() > 0 and (weight is not None or has_bias):
        _rmsnorm_bwd(x, weight, dout, rstd, dx, dw_partial, db_partial, dresidual_out, dresidual,
                     P, mean=mean, is_layernorm=mean is not None, weight_offset=weight_offset)
        parts = [t for t in (dw_partial, db_partial) if t is not None]
        outs = [torch.empty(N, device=x.device, dtype=pdt) for _ in parts]
        peer.reduce([t.view(P, -1) for t in parts], outs=outs)
        it = iter(outs)
        dw = next(it) if dw_partial is not None else None
        db = next(it) if db_partial is not None else None
        if has_residual and dresidual is None:
            dresidual = dx
        return dx, dw, db, dresidual
    if x.numel() > 0:
        _rmsnorm_bwd(x, weight, dout, rstd, dx, dw_partial, db_partial, dresidual_out, dresidual,
                     P, mean=mean, is_layernorm=mean is not None, weight_offset=weight_offset)
        dw32 = _finalize_partials(dw_partial, torch.float32) if weight is not None else None
        db32 = _finalize_partials(db_partial, torch.float32) if has_bias else None
    else:
        dw32 = torch.zeros(N, device=x.device) if weight is not None else None
        db32 = torch.zeros(N, device=x.device) if has_bias else None
    dw32, db32 = allreduce_param_grads(dw32, db32, group)
    dw = dw32.to(pdt) if dw32 is not None else None
    db = db32.to(pdt) if db32 is not None else None
    if has_residual and dresidual is None:
        dresidual = dx
    return dx, dw, db, dresidual


def ce_shard_stats(x_shard: Tensor, target: Tensor, col_offset: int, ignore_index: int = -100) -> Tensor:
    """(3, M) fp32: per-row max, sum exp(x - max) and target logit (0 unless this shard owns the
    target column) of a column slice of the logits whose first column is class ``col_offset``."""
    assert x_shard.dim() == 2 and target.dim() == 1
    _C.require_cuda(x_shard, "mX")
    M = x_shard.shape[0]
    stats = torch.empty(3, M, device=x_shard.device, dtype=torch.float32)
    if M == 0:
        return stats
    if x_shard.shape[1] == 0:
        stats[0].fill_(float("-inf"))
        stats[1:].zero_()
        return stats
    x_ = x_shard if x_shard.stride(-1) == 1 else x_shard.contiguous()
    t_ = target.contiguous()
    a = _C.CeFwdArgs()
    a.x, a.target = _C.ptr(x_), _C.ptr(t_)
    a.row_max, a.row_sumexp, a.row_tgt = stats[0].data_ptr(), stats[1].data_ptr(), stats[2].data_ptr()
    a.M, a.N = x_.shape
    a.x_row_stride = x_.stride(0)
    a.col_offset = int(col_offset)
    a.ignore_index = int(ignore_index)
    a.x_dtype = _C.float_code(x_)
    a.target_dtype = _C.INDEX_CODES[t_.dtype]
    a.cfg = _C.env_cfg("ce_fwd") or _C.make_cfg()
    with _C.device_of(x_):
        _C.check(_C.lib().qb_ce_fwd(byref(a), _C.stream_of(x_)), "ce_shard_stats")
    return stats


def ce_combine(stats_all: Tensor, target: Tensor, weight: Optional[Tensor] = None,
               ignore_index: int = -100) -> Tuple[Tensor, Tensor]:
    """Folds (G, 3, M) shard statistics in rank order into (loss, lse), both fp32 (M,)."""
    _C.require_cuda(stats_all, "stats")
    G, _, M = stats_all.shape
    loss = torch.empty(M, device=stats_all.device, dtype=torch.float32)
    lse = torch.empty(M, device=stats_all.device, dtype=torch.float32)
    if M == 0:
        return loss, lse
    s_ = stats_all.contiguous()
    t_ = target.contiguous()
    w_ = weight.contiguous() if weight is not None else None
    a = _C.CeCombineArgs()
    a.stats, a.target, a.weight = _C.ptr(s_), _C.ptr(t_), _C.ptr(w_)
    a.loss, a.lse = _C.ptr(loss), _C.ptr(lse)
    a.G, a.M = G, M
    a.ignore_index = int(ignore_index)
    a.num_classes = w_.numel() if w_ is not None else 0
    a.target_dtype = _C.INDEX_CODES[t_.dtype]
    a.weight_dtype = _C.float_code(w_)
    with _C.device_of(s_):
        _C.check(_C.lib().qb_ce_combine(byref(a), _C.stream_of(s_)), "ce_combine")
    return loss, lse


def ce_shard_bwd(x_shard, target, dloss, lse, col_offset, weight=None, ignore_index=-100,
                 inplace=False) -> Tensor:
    """Local gradient of a column slice: (exp(x - lse) - onehot_local) * dloss * w[target]."""
    _C.require_cuda(x_shard, "mX")
    x_ = x_shard if x_shard.stride(-1) == 1 else x_shard.contiguous()
    dx = x_ if inplace else torch.empty_like(x_)
    if x_.numel() == 0:
        return dx
    t_ = target.contiguous()
    dl = dloss if dloss.dtype == torch.float32 else dloss.float()
    w_ = weight.contiguous() if weight is not None else None
    a = _C.CeBwdArgs()
    a.x, a.target, a.dloss, a.lse = _C.ptr(x_), _C.ptr(t_), _C.ptr(dl), _C.ptr(lse.contiguous())
    a.weight, a.dx = _C.ptr(w_), _C.ptr(dx)
    a.M, a.N = x_.shape
    a.x_row_stride, a.dx_row_stride = x_.stride(0), dx.stride(0)
    a.dloss_stride = dl.stride(0)
    a.col_offset = int(col_offset)
    a.ignore_index = int(ignore_index)
    a.num_classes = w_.numel() if w_ is not None else 0
    a.x_dtype, a.dx_dtype = _C.float_code(x_), _C.float_code(dx)
    a.target_dtype = _C.INDEX_CODES[t_.dtype]
    a.weight_dtype = _C.float_code(w_)
    a.cfg = _C.env_cfg("ce_bwd") or _C.make_cfg()
    with _C.device_of(x_):
        _C.check(_C.lib().qb_ce_bwd(byref(a), _C.stream_of(x_)), "ce_shard_bwd")
    return dx


class VocabParallelCrossEntropy(torch.autograd.Function):
    """Per-row loss of logits whose vocabulary dimension is split over the ranks of ``group``."""

    @staticmethod
    def forward(ctx, x_shard, target, col_offset, weight, ignore_index, group, inplace_backward,
                peer=None):
        stats = ce_shard_stats(x_shard, target, col_offset, ignore_index)
        if peer is not None:
            loss, lse = peer.ce_combine(stats, target, weight, ignore_index)
        else:
            stats_all = gather_ce_stats(stats, group)
            loss, lse = ce_combine(stats_all, target, weight, ignore_index)
        ctx.save_for_backward(x_shard, target, lse, weight)
        ctx.col_offset, ctx.ignore_index, ctx.inplace = col_offset, ignore_index, inplace_backward
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x_shard, target, lse, weight = ctx.saved_tensors
        dx = ce_shard_bwd(x_shard, target, dloss, lse, ctx.col_offset, weight, ctx.ignore_index,
                          inplace=ctx.inplace)
        return dx, None, None, None, None, None, None, None


def cross_entropy_vocab_parallel(x_shard: Tensor, target: Tensor, col_offset: int,
                                 weight: Optional[Tensor] = None, ignore_index: int = -100,
                                 reduction: str = "mean", group=None,
                                 inplace_backward: bool = False, peer=None) -> Tensor:
    """Cross-entropy over vocabulary-sharded logits.  ``target`` holds global class ids and is
    replicated; ``col_offset`` is the global id of this rank's first column.  ``peer``: a
    ``PeerAllReduce`` of the group whose buffers hold 3 * M words; the exchange of the row
    statistics and their fold then run as one kernel instead of an all-gather + combine."""
    loss = VocabParallelCrossEntropy.apply(x_shard, target, col_offset, weight, ignore_index,
                                           group, inplace_backward, peer)
    if reduction == "none":
        return loss
    if reduction == "sum":
        return loss.sum()
    if reduction == "mean":
        if weight is not None:
            valid = target != ignore_index
            return loss.sum() / (weight[target.clamp(min=0)] * valid).sum()
        return loss.sum() / (target != ignore_index).sum().float()
    raise ValueError(
        f"Invalid reduction mode: {reduction}. Expected one of 'none', 'mean', or 'sum'"
    )
