"""Launch configuration of the RMSNorm / LayerNorm kernels (sm_100a only).

Mirrors the public surface of the reference's quack/rmsnorm_config.py:16-26,94-107,265-293:
the two frozen dataclasses, their ``from_analytical_heuristic`` factories, ``get_sm_count`` and
the explicit-config search spaces used by the tuned entry points.  The knobs that describe the
reference's shared-memory reload strategy (``reload_from``, ``delay_w_load``, ``reload_wdy``,
``reload_x``, ``use_tma``) are accepted for signature compatibility and ignored: the sm_100a
kernels keep rows in registers (forward) or in a cp.async ring (backward).
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import List, Optional

import torch


@dataclass(frozen=True)
class RmsNormFwdConfig:
    num_threads: int
    threads_per_row: int
    cluster_n: int
    reload_from: Optional[str] = None
    delay_w_load: bool = False

    @classmethod
    def from_analytical_heuristic(cls, N: int, dtype_width: int, arch_major: Optional[int] = None,
                                  is_layernorm: bool = False) -> "RmsNormFwdConfig":
        """The launch geometry of the C launcher's heuristic for an aligned row of N elements that
        is held as fp32 registers (fp32 input, or any input with a residual).  Packed 16-bit rows
        without a residual -- twice the elements per register -- are planned by the launcher with
        up to 16 chunks per thread and 256-thread CTAs from N = 6144, which this value does not
        describe; ``qb_last_kernel`` names the instantiation that actually ran."""
        vec = 128 // dtype_width
        k_target = 8
        # RMSNorm rows of 2 - 8 KB of 16-bit elements that fill a power-of-two tile exactly
        # (hidden sizes 1024, 2048, 4096): half the chunks per thread, twice the threads per row
        row_bytes = N * dtype_width // 8
        if not is_layernorm and vec == 8 and 2048 <= row_bytes <= 8192 and N % (vec * 4) == 0:
            tpr_c = N // (vec * 4)
            if tpr_c & (tpr_c - 1) == 0:
                k_target = 4
        threads, tpr, cluster_n = _plan(N, vec, pref_elems=16384 if vec == 8 else 8192,
                                        k_target=k_target, caps=(64, 32, 16), default_threads=128)
        return cls(num_threads=threads, threads_per_row=tpr, cluster_n=cluster_n)


@dataclass(frozen=True)
class RmsNormBwdConfig:
    num_threads: int
    threads_per_row: int
    cluster_n: int
    reload_wdy: Optional[str] = None
    reload_x: Optional[str] = None
    use_tma: bool = False
    smem_stages: int = 0  # cp.async ring depth; 0 = as deep as shared memory allows (<= 4)

    @classmethod
    def from_analytical_heuristic(cls, N: int, dtype_width: int, dout_width: Optional[int] = None,
                                  arch_major: Optional[int] = None, T_hint: int = 0,
                                  num_acc: int = 1) -> "RmsNormBwdConfig":
        vec = 128 // max(dtype_width, dout_width or dtype_width)
        wide = 16384 if vec == 8 else 8192
        threads, tpr, cluster_n = _plan(N, vec, pref_elems=wide if N <= 2 * wide else wide // 2,
                                        k_target=8, caps=(64 if vec == 8 else 32, 16, 8),
                                        default_threads=128)
        return cls(num_threads=threads, threads_per_row=tpr, cluster_n=cluster_n)


def _next_pow2(v: int) -> int:
    return 1 << max(0, (int(v) - 1).bit_length())


def _max_k(caps, threads: int, vec: int) -> int:
    cap = caps[2] if threads > 512 else (caps[1] if threads > 256 else caps[0])
    kmax = 16 if vec <= 4 else 8
    k = 1
    while k * 2 <= kmax and k * 2 * vec <= cap:
        k *= 2
    return k if k * vec <= cap else 0


def _plan(N: int, vec: int, pref_elems: int, k_target: int, caps, default_threads: int = 256):
    """Python restatement of the C launcher's geometry search (csrc/host_common.h: plan_rows)
    for the no-override case; used for reporting and for sizing the backward workspace."""
    while vec > 1 and N % vec:
        vec //= 2
    chunks = N // vec
    max_cap = max(t * _max_k(caps, t, vec) for t in (32, 64, 128, 256, 512, 1024))
    cluster_n = 1
    pref = min(pref_elems // vec, max_cap)
    while -(-chunks // cluster_n) > pref and cluster_n < 8:
        cluster_n *= 2
    if -(-chunks // cluster_n) > max_cap:
        cluster_n = 16
    while cluster_n > 1 and (cluster_n - 1) * -(-chunks // cluster_n) >= chunks:
        cluster_n //= 2
    cpc = -(-chunks // cluster_n)
    lo = 32 if cluster_n > 1 else 8
    want = min(1024, max(lo, _next_pow2(-(-cpc // k_target))))
    order = []
    t = want
    while t <= 1024:
        order.append(t)
        t *= 2
    t = want // 2
    while t >= lo:
        order.append(t)
        t //= 2
    tpr = 0
    for t in order:
        if -(-cpc // t) <= _max_k(caps, max(t, 32), vec):
            tpr = t
            break
    if tpr == 0:
        raise ValueError(f"a row of {N} elements does not fit (vector width {vec})")
    if cluster_n > 1:
        tpr = max(tpr, 32)
        return tpr, tpr, cluster_n
    K = _next_pow2(-(-cpc // tpr))
    threads = max(tpr, 32)
    while threads < default_threads and K <= _max_k(caps, threads * 2, vec):
        threads *= 2
    return threads, tpr, cluster_n


# What qb_norm_bwd_num_partials returns on B200 (148 SMs) by row length in units of 16-byte
# chunks: two 128-thread CTAs per SM, one 256-thread CTA per SM, clusters of 2 such CTAs, then the
# resident clusters of 8 / 16 CTAs of 128 threads and of 16 CTAs of 256 threads (a cluster has to
# fit into one GPC, which is why these are not 296 / cluster size).
_B200_PARTIALS_BY_CHUNKS = ((1024, 296), (2048, 148), (4096, 74), (8192, 32), (16384, 15))


def get_sm_count(N: int, device, dtype: Optional[torch.dtype] = None) -> int:
    """Number of partial-sum slices (persistent CTAs or clusters) the backward kernel uses by
    default, i.e. the first dimension of ``dw_partial`` (reference: quack/rmsnorm_config.py:265-293).

    Any positive value is functionally valid.  Eagerly the library is asked
    (``qb_norm_bwd_num_partials``: one persistent CTA -- two of 128 threads -- per SM, or as many
    clusters as are resident at once); inside ``torch.compile`` traces a pure-Python estimate of
    the same number is returned."""
    props = torch.cuda.get_device_properties(device)
    sms = props.multi_processor_count
    width = 32 if dtype == torch.float32 else 16
    if not torch.compiler.is_compiling():
        from quack_flydsl_b200 import _C

        code = _C.FLOAT_CODES[torch.float32 if width == 32 else torch.bfloat16]
        with torch.cuda.device(device):
            n = _C.lib().qb_norm_bwd_num_partials(int(N), code, 0, -1)
        if n > 0:
            return int(n)
    chunks = -(-int(N) * width // 128)
    per_148 = 7
    for limit, count in _B200_PARTIALS_BY_CHUNKS:
        if chunks <= limit:
            per_148 = count
            break
    return max(1, per_148 * sms // 148)


_CTA_THREAD_SIZE = (128, 256, 512)
_THREADS_PER_ROW = (32, 64, 128, 256, 512)
_CLUSTER_N = (1, 2, 4, 8)


def get_all_fwd_configs() -> List[RmsNormFwdConfig]:
    out = []
    for nt, tpr, cn in itertools.product(_CTA_THREAD_SIZE, _THREADS_PER_ROW, _CLUSTER_N):
        if tpr <= nt:
            out.append(RmsNormFwdConfig(nt, tpr, cn))
    return out


def get_all_bwd_configs() -> List[RmsNormBwdConfig]:
    out = []
    for nt, tpr, cn, st in itertools.product(_CTA_THREAD_SIZE, _THREADS_PER_ROW, _CLUSTER_N, (2, 3, 4)):
        if tpr <= nt:
            out.append(RmsNormBwdConfig(nt, tpr, cn, smem_stages=st))
    return out
