"""ctypes binding of the sm_100a library (``include/bms_b200.h``).

This is the only route to the kernels: there is no CPU fallback.  If the
library is missing or cannot be loaded, every call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading

from .build import LIBRARY

_lock = threading.Lock()
_lib = None

SUCCESS = 0
ERROR_INVALID_ARGUMENT = 1
ERROR_CUDA = 2
ERROR_UNSUPPORTED = 3

DTYPE_CODES = {"float32": 0, "bfloat16": 1, "float16": 2}


class Policy(ctypes.Structure):
    """``bms_policy``: kind 0 = DensityPolicy bands, kind 1 = linear."""

    _fields_ = [("kind", ctypes.c_int32), ("min_budget", ctypes.c_int32),
                ("max_budget", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("low_density", ctypes.c_double), ("high_density", ctypes.c_double)]


EXPORTS = (
    "bms_last_error", "bms_runtime_version", "bms_mask_count", "bms_masked_argmax",
    "bms_masked_reduce_batch", "bms_masked_sample", "bms_masked_sample_batch",
    "bms_mask_budget", "bms_expand_token_lists", "bms_expand_token_gaps", "bms_speculative_accept", "bms_verify_batch", "bms_set_launch_override", "bms_shard_granule_bytes",
    "bms_shard_partials", "bms_shard_partials_indexed", "bms_shard_merge", "bms_workspace_bytes",
    "bms_masked_reduce_batch_noalloc",
    "bms_exchange_bytes", "bms_exchange_create", "bms_exchange_open", "bms_exchange_close", "bms_exchange_destroy",
    "bms_shard_partials_exchange", "bms_shard_merge_exchange",
)


class IpcHandle(ctypes.Structure):
    """``bms_ipc_handle``: an exported exchange area (cudaIpcMemHandle_t)."""

    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


def _declare(lib) -> None:
    p, i32, i64, f64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_double
    lib.bms_last_error.argtypes = []
    lib.bms_last_error.restype = ctypes.c_char_p
    sig = {
        "bms_runtime_version": [p],
        "bms_mask_count": [p, i64, p, i32, p],
        "bms_masked_argmax": [p, i32, p, i64, p, p, i32, p],
        "bms_masked_reduce_batch": [p, i32, p, i64, i64, p, p, p, p, i64, i32, p],
        "bms_masked_reduce_batch_noalloc": [p, i32, p, i64, i64, p, p, p, i32, p],
        "bms_masked_sample": [p, i32, p, i64, f64, p, p, p, i32, p],
        "bms_masked_sample_batch": [p, i32, p, i64, i64, f64, p, p, p, p, p, i64, i32, p],
        "bms_mask_budget": [p, i64, i64, ctypes.POINTER(Policy), p, p, p, i32, p],
        "bms_expand_token_lists": [p, i64, p, i64, i64, p, p, i32, p],
        "bms_expand_token_gaps": [p, i64, p, i64, i64, p, p, i32, p],
        "bms_speculative_accept": [p, p, i32, p, i64, i64, i64, p, p, p, p, f64, p, p, p, p, p, p, i32, p],
        "bms_verify_batch": [p, i32, p, i64, i64, i64, p, p, ctypes.POINTER(Policy), p, p, p, p,
                             p, p, p, p, p, i64, p, i64, i32, p],
        "bms_set_launch_override": [i32, i32],
        "bms_shard_partials": [p, i32, p, i64, i64, i64, i64, f64, p, p, i64, i32, p],
        "bms_shard_partials_indexed": [p, i32, p, i64, p, i64, i64, i64, i64, f64, p, p, i64, i32, p],
        "bms_shard_merge": [p, i32, i32, i64, f64, p, p, i32, p, i64, i64, i64, p, i64, p, p, p, i32, p],
        "bms_exchange_create": [i32, i32, i64, ctypes.POINTER(p), ctypes.POINTER(IpcHandle)],
        "bms_exchange_open": [i32, ctypes.POINTER(IpcHandle), ctypes.POINTER(p)],
        "bms_exchange_close": [i32, p],
        "bms_exchange_destroy": [i32, p],
        "bms_shard_partials_exchange": [p, i32, p, i64, i64, i64, i64, p, i32, i32, i64, ctypes.c_uint32, i32, p],
        "bms_shard_merge_exchange": [p, i32, i32, i64, ctypes.c_uint32, i64, p, p, p, i32, p],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.bms_shard_granule_bytes.argtypes = [i32, i64]
    lib.bms_shard_granule_bytes.restype = i64
    lib.bms_workspace_bytes.argtypes = [i32]
    lib.bms_workspace_bytes.restype = i64
    lib.bms_exchange_bytes.argtypes = [i32, i64]
    lib.bms_exchange_bytes.restype = i64


def library():
    """Load ``_lib/libbms_b200.so`` once; raise if it was never built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIBRARY.exists():
                    raise RuntimeError(
                        f"CUDA library {LIBRARY} is missing; build it with "
                        "`python -m bitmask_speculation_b200.build` (no CPU fallback exists)")
                lib = ctypes.CDLL(str(LIBRARY))
                _declare(lib)
                _lib = lib
    return _lib


class NativeError(RuntimeError):
    """A contract violation or CUDA failure reported by the C ABI."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(rc: int) -> None:
    if rc != SUCCESS:
        msg = library().bms_last_error().decode(errors="replace")
        raise NativeError(rc, msg)


def set_launch_override(cluster: int = 0, clusters: int = 0) -> None:
    """Force the cluster size / cluster count of the selection kernels (tests only)."""
    check(library().bms_set_launch_override(cluster, clusters))
