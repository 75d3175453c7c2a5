"""ctypes binding of libquack_b200.so (declared in include/quack_b200.h).

Plays the role of the TVM-FFI call boundary in the reference (the compiled functions invoked from
quack/rmsnorm.py:423, quack/softmax.py:207, quack/cross_entropy.py:364): tensors cross as raw
device pointers + sizes + strides, the stream is torch's current stream.  There is no fallback:
if the library is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, byref, c_char_p, c_float, c_int32, c_int64, c_void_p
from pathlib import Path
from typing import Optional

import torch

QB_F32, QB_F16, QB_BF16 = 0, 1, 2
QB_I32, QB_I64 = 0, 1
QB_OK, QB_ERR_INVALID, QB_ERR_UNSUPPORTED, QB_ERR_CUDA = 0, -1, -2, -3
QB_ABI_VERSION = 3

FLOAT_CODES = {torch.float32: QB_F32, torch.float16: QB_F16, torch.bfloat16: QB_BF16}
INDEX_CODES = {torch.int32: QB_I32, torch.int64: QB_I64}


class LaunchCfg(Structure):
    _fields_ = [
        ("num_threads", c_int32),
        ("threads_per_row", c_int32),
        ("cluster_n", c_int32),
        ("max_ctas", c_int32),
        ("stages", c_int32),
        ("flags", c_int32),
        ("ctas_per_sm", c_int32),
        ("reserved", c_int32),
    ]


class DeviceInfo(Structure):
    _fields_ = [
        ("device", c_int32),
        ("sm_count", c_int32),
        ("cc_major", c_int32),
        ("cc_minor", c_int32),
        ("max_smem_optin", c_int32),
        ("max_cluster", c_int32),
        ("reserved", c_int32 * 2),
    ]


class NormFwdArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("weight", c_void_p), ("bias", c_void_p), ("residual", c_void_p),
        ("out", c_void_p), ("residual_out", c_void_p), ("rstd", c_void_p), ("mean", c_void_p),
        ("M", c_int64), ("H", c_int64), ("N", c_int64),
        ("x_row_stride", c_int64), ("residual_row_stride", c_int64),
        ("out_row_stride", c_int64), ("residual_out_row_stride", c_int64),
        ("x_dtype", c_int32), ("weight_dtype", c_int32), ("bias_dtype", c_int32),
        ("residual_dtype", c_int32), ("out_dtype", c_int32), ("residual_out_dtype", c_int32),
        ("is_layernorm", c_int32), ("eps", c_float), ("weight_offset", c_float),
        ("pad0", c_int32), ("cfg", LaunchCfg),
    ]


class NormBwdArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("weight", c_void_p), ("dout", c_void_p), ("rstd", c_void_p),
        ("mean", c_void_p), ("dresidual_out", c_void_p), ("dx", c_void_p),
        ("dresidual", c_void_p), ("dw_partial", c_void_p), ("db_partial", c_void_p),
        ("M", c_int64), ("H", c_int64), ("N", c_int64),
        ("x_row_stride", c_int64), ("dout_row_stride", c_int64),
        ("dresidual_out_row_stride", c_int64), ("dx_row_stride", c_int64),
        ("dresidual_row_stride", c_int64),
        ("num_partials", c_int32), ("x_dtype", c_int32), ("weight_dtype", c_int32),
        ("dout_dtype", c_int32), ("dresidual_out_dtype", c_int32), ("dx_dtype", c_int32),
        ("dresidual_dtype", c_int32), ("is_layernorm", c_int32), ("weight_offset", c_float),
        ("pad0", c_int32), ("cfg", LaunchCfg),
    ]


class NormBwdStaticArgs(Structure):
    _fields_ = [("bwd", NormBwdArgs), ("dw", c_void_p), ("db", c_void_p),
                ("param_dtype", c_int32), ("pad0", c_int32)]


class RmsFinalReduceArgs(Structure):
    _fields_ = [("x", c_void_p), ("rstd", c_void_p), ("M", c_int64), ("N", c_int64),
                ("x_row_stride", c_int64), ("scale", c_float), ("eps", c_float),
                ("x_dtype", c_int32), ("pad0", c_int32)]


class ColsumArgs(Structure):
    _fields_ = [
        ("partial", c_void_p), ("out", c_void_p), ("out_f32", c_void_p),
        ("P", c_int64), ("cols", c_int64), ("out_dtype", c_int32), ("pad0", c_int32),
    ]


QB_MAX_PEERS = 8
QB_PEER_HANDLE_BYTES = 64


class ColsumAllreduceArgs(Structure):
    _fields_ = [
        ("partial0", c_void_p), ("partial1", c_void_p), ("out0", c_void_p), ("out1", c_void_p),
        ("out0_f32", c_void_p), ("out1_f32", c_void_p), ("peers", c_void_p * QB_MAX_PEERS),
        ("status", c_void_p), ("P", c_int64), ("cols", c_int64), ("cap_cols", c_int64),
        ("num_buffers", c_int32), ("out_dtype", c_int32), ("world", c_int32), ("rank", c_int32),
        ("seq", ctypes.c_uint32), ("pad0", c_int32),
    ]


class CeCombineExchangeArgs(Structure):
    _fields_ = [
        ("stats", c_void_p), ("target", c_void_p), ("weight", c_void_p), ("loss", c_void_p),
        ("lse", c_void_p), ("peers", c_void_p * QB_MAX_PEERS), ("status", c_void_p),
        ("M", c_int64), ("cap_cols", c_int64), ("ignore_index", c_int64), ("num_classes", c_int64),
        ("target_dtype", c_int32), ("weight_dtype", c_int32), ("world", c_int32), ("rank", c_int32),
        ("seq", ctypes.c_uint32), ("pad0", c_int32),
    ]


class SoftmaxFwdArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("out", c_void_p), ("M", c_int64), ("N", c_int64),
        ("x_row_stride", c_int64), ("out_row_stride", c_int64),
        ("x_dtype", c_int32), ("out_dtype", c_int32), ("cfg", LaunchCfg),
    ]


class SoftmaxBwdArgs(Structure):
    _fields_ = [
        ("dy", c_void_p), ("y", c_void_p), ("dx", c_void_p), ("M", c_int64), ("N", c_int64),
        ("dy_row_stride", c_int64), ("y_row_stride", c_int64), ("dx_row_stride", c_int64),
        ("dy_dtype", c_int32), ("y_dtype", c_int32), ("dx_dtype", c_int32), ("pad0", c_int32),
        ("cfg", LaunchCfg),
    ]


class CeFwdArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("target", c_void_p), ("target_logit", c_void_p), ("weight", c_void_p),
        ("loss", c_void_p), ("lse", c_void_p), ("dx", c_void_p),
        ("row_max", c_void_p), ("row_sumexp", c_void_p), ("row_tgt", c_void_p),
        ("M", c_int64), ("N", c_int64), ("x_row_stride", c_int64), ("dx_row_stride", c_int64),
        ("target_logit_row_stride", c_int64), ("col_offset", c_int64), ("ignore_index", c_int64),
        ("num_classes", c_int64),
        ("x_dtype", c_int32), ("target_dtype", c_int32), ("target_logit_dtype", c_int32),
        ("target_logit_ndim", c_int32), ("weight_dtype", c_int32), ("pad0", c_int32),
        ("cfg", LaunchCfg),
    ]


class CeBwdArgs(Structure):
    _fields_ = [
        ("x", c_void_p), ("target", c_void_p), ("dloss", c_void_p), ("lse", c_void_p),
        ("weight", c_void_p), ("dx", c_void_p),
        ("M", c_int64), ("N", c_int64), ("x_row_stride", c_int64), ("dx_row_stride", c_int64),
        ("dloss_stride", c_int64), ("col_offset", c_int64), ("ignore_index", c_int64),
        ("num_classes", c_int64),
        ("x_dtype", c_int32), ("dx_dtype", c_int32), ("target_dtype", c_int32),
        ("weight_dtype", c_int32), ("cfg", LaunchCfg),
    ]


class CeCombineArgs(Structure):
    _fields_ = [
        ("stats", c_void_p), ("target", c_void_p), ("weight", c_void_p),
        ("loss", c_void_p), ("lse", c_void_p),
        ("G", c_int64), ("M", c_int64), ("ignore_index", c_int64), ("num_classes", c_int64),
        ("target_dtype", c_int32), ("weight_dtype", c_int32),
    ]


class TopkFwdArgs(Structure):
    _fields_ = [("x", c_void_p), ("values", c_void_p), ("indices", c_void_p),
                ("M", c_int64), ("N", c_int64), ("k", c_int64), ("x_row_stride", c_int64),
                ("x_dtype", c_int32), ("softmax", c_int32)]


class TopkBwdArgs(Structure):
    _fields_ = [("dvalues", c_void_p), ("values", c_void_p), ("indices", c_void_p), ("dx", c_void_p),
                ("M", c_int64), ("N", c_int64), ("k", c_int64), ("dx_row_stride", c_int64),
                ("dvalues_dtype", c_int32), ("values_dtype", c_int32), ("dx_dtype", c_int32),
                ("softmax", c_int32)]


# code passed to qb_sizeof_args -> the Structure that must have that size
_SIZEOF_CODES = {
    0: LaunchCfg, 1: NormFwdArgs, 2: NormBwdArgs, 3: ColsumArgs, 4: SoftmaxFwdArgs,
    5: SoftmaxBwdArgs, 6: CeFwdArgs, 7: CeBwdArgs, 8: CeCombineArgs, 9: DeviceInfo,
    10: NormBwdStaticArgs, 11: RmsFinalReduceArgs, 12: TopkFwdArgs, 13: TopkBwdArgs,
    14: ColsumAllreduceArgs, 15: CeCombineExchangeArgs,
}

# every symbol include/quack_b200.h declares
EXPORTED_SYMBOLS = (
    "qb_norm_fwd", "qb_norm_bwd", "qb_norm_bwd_num_partials", "qb_colsum", "qb_softmax_fwd",
    "qb_softmax_bwd", "qb_ce_fwd", "qb_ce_bwd", "qb_ce_combine", "qb_query_device",
    "qb_last_error", "qb_abi_version", "qb_sizeof_args", "qb_norm_bwd_static",
    "qb_rms_final_reduce", "qb_ring_timeouts", "qb_last_kernel", "qb_topk_fwd", "qb_topk_bwd",
    "qb_colsum_allreduce", "qb_ce_combine_exchange", "qb_peer_buffer_bytes", "qb_peer_buffer_create", "qb_peer_buffer_open",
    "qb_peer_buffer_close", "qb_peer_buffer_destroy",
)

_LIB: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    """Location of the shared library (override with QUACK_B200_LIB for an experimental build)."""
    override = os.environ.get("QUACK_B200_LIB")
    if override:
        return Path(override)
    return Path(__file__).resolve().parent / "lib" / "libquack_b200.so"


def lib() -> ctypes.CDLL:
    """Loads (once) and returns the CUDA library; raises if it is missing or mismatched."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.exists():
        raise ImportError(
            f"{path} not found: the sm_100a kernels are not built. Run "
            "`python -m quack_flydsl_b200.build` (needs nvcc). There is no fallback path."
        )
    cdll = ctypes.CDLL(str(path))
    for name in EXPORTED_SYMBOLS:
        if not hasattr(cdll, name):
            raise ImportError(f"{path} does not export {name}")
    cdll.qb_last_error.restype = c_char_p
    cdll.qb_last_error.argtypes = []
    cdll.qb_abi_version.restype = ctypes.c_int
    cdll.qb_sizeof_args.restype = ctypes.c_int
    cdll.qb_sizeof_args.argtypes = [c_int32]
    if cdll.qb_abi_version() != QB_ABI_VERSION:
        raise ImportError(f"{path}: ABI version {cdll.qb_abi_version()} != {QB_ABI_VERSION}")
    for code, struct in _SIZEOF_CODES.items():
        want = cdll.qb_sizeof_args(code)
        if want != ctypes.sizeof(struct):
            raise ImportError(
                f"{path}: layout mismatch for {struct.__name__}: library {want} bytes, "
                f"binding {ctypes.sizeof(struct)} bytes"
            )
    for name, struct in (
        ("qb_norm_fwd", NormFwdArgs), ("qb_norm_bwd", NormBwdArgs), ("qb_colsum", ColsumArgs),
        ("qb_softmax_fwd", SoftmaxFwdArgs), ("qb_softmax_bwd", SoftmaxBwdArgs),
        ("qb_ce_fwd", CeFwdArgs), ("qb_ce_bwd", CeBwdArgs), ("qb_ce_combine", CeCombineArgs),
        ("qb_norm_bwd_static", NormBwdStaticArgs), ("qb_rms_final_reduce", RmsFinalReduceArgs),
        ("qb_topk_fwd", TopkFwdArgs), ("qb_topk_bwd", TopkBwdArgs),
        ("qb_colsum_allreduce", ColsumAllreduceArgs),
        ("qb_ce_combine_exchange", CeCombineExchangeArgs),
    ):
        fn = getattr(cdll, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [POINTER(struct), c_void_p]
    cdll.qb_norm_bwd_num_partials.restype = ctypes.c_int
    cdll.qb_norm_bwd_num_partials.argtypes = [c_int64, c_int32, c_int32, c_int32]
    cdll.qb_query_device.restype = ctypes.c_int
    cdll.qb_query_device.argtypes = [c_int32, POINTER(DeviceInfo)]
    cdll.qb_last_kernel.restype = c_char_p
    cdll.qb_last_kernel.argtypes = []
    cdll.qb_peer_buffer_bytes.restype = c_int64
    cdll.qb_peer_buffer_bytes.argtypes = [c_int32, c_int64]
    cdll.qb_peer_buffer_create.restype = ctypes.c_int
    cdll.qb_peer_buffer_create.argtypes = [c_int32, c_int64, POINTER(c_void_p), ctypes.c_char_p]
    cdll.qb_peer_buffer_open.restype = ctypes.c_int
    cdll.qb_peer_buffer_open.argtypes = [ctypes.c_char_p, POINTER(c_void_p)]
    cdll.qb_peer_buffer_close.restype = ctypes.c_int
    cdll.qb_peer_buffer_close.argtypes = [c_void_p]
    cdll.qb_peer_buffer_destroy.restype = ctypes.c_int
    cdll.qb_peer_buffer_destroy.argtypes = [c_void_p]
    cdll.qb_ring_timeouts.restype = ctypes.c_int
    cdll.qb_ring_timeouts.argtypes = [POINTER(ctypes.c_uint32)]
    _LIB = cdll
    return cdll


def last_error() -> str:
    return lib().qb_last_error().decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    """Turns a negative qb_status into the exception type the reference raises for that case."""
    if status == QB_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (QB_ERR_INVALID, QB_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def float_code(t: Optional[torch.Tensor]) -> int:
    return FLOAT_CODES[t.dtype] if t is not None else 0


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return t.data_ptr() if t is not None else None


def make_cfg(num_threads: int = 0, threads_per_row: int = 0, cluster_n: int = 0,
             max_ctas: int = 0, stages: int = 0, flags: int = 0, ctas_per_sm: int = 0) -> LaunchCfg:
    cfg = LaunchCfg()
    cfg.num_threads = int(num_threads)
    cfg.threads_per_row = int(threads_per_row)
    cfg.cluster_n = int(cluster_n)
    cfg.max_ctas = int(max_ctas)
    cfg.stages = int(stages)
    cfg.flags = int(flags)
    cfg.ctas_per_sm = int(ctas_per_sm)
    return cfg


def env_cfg(op: str) -> Optional[LaunchCfg]:
    """Launch override from
    QUACK_B200_CFG="op:threads:threads_per_row:cluster:max_ctas:stages:flags:ctas_per_sm;..."
    (used by tuning sweeps; 0 keeps the heuristic for a field)."""
    global _ENV_CFG_CACHE
    spec = os.environ.get("QUACK_B200_CFG")
    if not spec:
        return None
    if _ENV_CFG_CACHE[0] != spec:
        parsed = {}
        for item in spec.split(";"):
            parts = item.split(":")
            if parts and parts[0]:
                vals = [int(v) if v else 0 for v in parts[1:8]]
                vals += [0] * (7 - len(vals))
                parsed[parts[0]] = make_cfg(*vals)
        _ENV_CFG_CACHE = (spec, parsed)
    return _ENV_CFG_CACHE[1].get(op)


def require_cuda(t: torch.Tensor, name: str) -> None:
    # Same wording as the TVM-FFI check the reference relies on (tests/test_rmsnorm.py:364).
    if t.device.type != "cuda":
        raise ValueError(
            f"Mismatched Tensor on argument {name}: expected device_type=cuda, got {t.device.type}"
        )


def stream_of(t: torch.Tensor) -> int:
    return torch._C._cuda_getCurrentRawStream(t.get_device())


def launch(fn, args, t: torch.Tensor, what: str) -> None:
    """Calls ``fn(byref(args), stream)`` with ``t``'s device current and on torch's current stream
    of that device; raises on a negative status.  The lean form of
    ``with device_of(t): check(fn(byref(args), stream_of(t)), what)`` for the per-call hot path."""
    idx = t.get_device()
    cur = torch._C._cuda_getDevice()
    if cur == idx:
        rc = fn(byref(args), torch._C._cuda_getCurrentRawStream(idx))
    else:
        torch.cuda.set_device(idx)
        try:
            rc = fn(byref(args), torch._C._cuda_getCurrentRawStream(idx))
        finally:
            torch.cuda.set_device(cur)
    if rc != QB_OK:
        check(rc, what)


_ENV_CFG_CACHE = (None, {})


class device_of:
    """Makes the tensor's device current for the duration of a launch (no-op if it already is)."""

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def query_device(device: int = -1) -> DeviceInfo:
    info = DeviceInfo()
    check(lib().qb_query_device(device, byref(info)), "qb_query_device")
    return info


def norm_bwd_num_partials(N: int, x_dtype: torch.dtype, is_layernorm: bool, device) -> int:
    dev = torch.device(device)
    with torch.cuda.device(dev):
        n = lib().qb_norm_bwd_num_partials(int(N), FLOAT_CODES[x_dtype], int(is_layernorm),
                                           dev.index if dev.index is not None else -1)
    if n <= 0:
        check(n if n < 0 else QB_ERR_INVALID, "qb_norm_bwd_num_partials")
    return n


def ring_timeouts() -> int:
    """Waits of the shared-memory ring kernels that gave up on the current device since the library
    was loaded (0 in a healthy process).  Synchronises the device."""
    n = ctypes.c_uint32(0)
    check(lib().qb_ring_timeouts(byref(n)), "qb_ring_timeouts")
    return int(n.value)


def last_kernel() -> str:
    """Name (with template arguments) of the device kernel this thread's last call launched last."""
    return lib().qb_last_kernel().decode("utf-8", "replace")
