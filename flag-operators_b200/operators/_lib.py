"""Loader for libflagops.so and the glue shared by the operator wrappers.

The library is built in-tree by ``flag-operators_b200/build.py`` into
``flag-operators_b200/lib/libflagops.so``.  A CUDA tensor handed to any
operator always runs through this library; if it cannot be loaded the call
raises instead of computing the result some other way.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get(
    "FLAGOPS_LIB", os.path.join(os.path.dirname(_HERE), "lib", "libflagops.so"))

# dtype codes (include/flagops.h: enum fo_dtype)
F32, F16, BF16, F64, I32, I64 = 0, 1, 2, 3, 4, 5
_DTYPE_CODE = {
    torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16,
    torch.float64: F64, torch.int32: I32, torch.int64: I64,
}
# status codes (enum fo_status)
_STATUS = {-1: "invalid argument", -2: "unsupported dtype", -3: "CUDA error",
           -4: "workspace too small", -5: "unsupported configuration"}

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> argtypes (every entry point returns int)
_SIGS = {
    "fo_rms_norm_fwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _f32,
                        _int, _int, _c_void_p],
    "fo_rms_norm_bwd_workspace_bytes": [_i64, _i64, _i64p],
    "fo_rms_norm_bwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64,
                        _i64, _int, _int, _c_void_p, _i64, _c_void_p],
    "fo_median_dim": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int, _c_void_p],
    "fo_median_all_workspace_bytes": [_i64, _i64p],
    "fo_median_all": [_c_void_p, _c_void_p, _i64, _int, _c_void_p, _i64, _c_void_p],
    "fo_scatter_reduce_workspace_bytes": [_i64, _int, _int, _int, _i64p],
    "fo_scatter_reduce_binned_bytes": [_i64, _i64, _int, _int, _i64p],
    "fo_scatter_reduce": [_c_void_p, _c_void_p, _c_void_p, _int, _i64p, _i64p, _i64p, _i64p,
                          _i64p, _int, _int, _int, _int, _int, _c_void_p, _i64, _c_void_p,
                          _c_void_p],
    "fo_scatter_reduce_noalloc": [_c_void_p, _c_void_p, _c_void_p, _int, _i64p, _i64p, _i64p,
                                  _i64p, _i64p, _int, _int, _int, _int, _int, _c_void_p,
                                  _c_void_p],
    "fo_ce_workspace_bytes": [_i64, _i64p],
    "fo_ce_fwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                  _i64, _i64, _i64, _i64, _f32, _int, _int, _c_void_p, _i64, _c_void_p],
    "fo_ce_bwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _int, _int, _c_void_p, _c_void_p,
                  _i64, _i64, _i64, _i64, _f32, _int, _int, _c_void_p],
    "fo_ce_scale_grad": [_c_void_p, _c_void_p, _int, _int, _i64, _i64, _i64, _int, _c_void_p],
    "fo_ce_shard_stats": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i64, _int,
                          _c_void_p],
    "fo_ce_shard_combine": [_c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                            _c_void_p, _i64, _i64, _i64, _f32, _int, _c_void_p],
    "fo_ce_shard_bwd": [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _int, _int, _c_void_p,
                        _c_void_p, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _int, _int,
                        _c_void_p],
    "fo_ce_count_valid": [_c_void_p, _i64, _i64, _c_void_p, _c_void_p],
    "fo_ce_shard_p2p_region_bytes": [_int, _i64, _i64p],
    "fo_ce_shard_p2p_fwd": [_c_void_p] * 7 + [_i64, _i64, _i64, _i64, _i64, _i64, _f32, _int,
                                              _int, _c_void_p, _int, _int, _i64, ctypes.c_uint32,
                                              _c_void_p],
    "fo_ce_p2p_timeouts": [_c_void_p],
    "fo_peer_export": [_c_void_p, _c_void_p, _i64p],
    "fo_peer_open": [_c_void_p, _i64, ctypes.POINTER(ctypes.c_void_p)],
    "fo_peer_close": [_c_void_p, _i64],
    "fo_peer_can_access": [_int, _int, ctypes.POINTER(ctypes.c_int)],
    "fo_ce_rows_fwd": [_c_void_p] * 7 + [_i64, _i64, _i64, _i64, _f32, _int, _int, _c_void_p],
    "fo_gdr_workspace_bytes": [_i64, _i64, _i64, _i64, _int, _i64p],
    "fo_gdr_fwd": [_c_void_p] * 8 + [_i64, _i64, _i64, _i64, _int, _int, _c_void_p, _i64,
                                     _c_void_p],
    "fo_gdr_fwd_stepwise": [_c_void_p] * 8 + [_i64, _i64, _i64, _i64, _int, _int, _c_void_p],
    "fo_gdr_timeouts": [_c_void_p],
    "fo_gdr_bwd_workspace_bytes": [_i64, _i64, _i64, _i64, _i64p],
    "fo_gdr_bwd": [_c_void_p] * 14 + [_i64, _i64, _i64, _i64, _int, _int, _c_void_p,
                                      _i64, _c_void_p],
    "fo_median_timeouts": [_c_void_p],
    "fo_tc05_selftest": [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _int, _int, _c_void_p],
}

_lock = threading.Lock()
_lib = None


class LibraryNotLoaded(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it on first use (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LibraryNotLoaded(
                f"libflagops.so not found at {LIB_PATH}; build it with "
                f"`python flag-operators_b200/build.py`")
        lib = ctypes.CDLL(LIB_PATH)
        lib.fo_last_error.restype = ctypes.c_char_p
        lib.fo_last_error.argtypes = []
        lib.fo_abi_version.restype = ctypes.c_int
        lib.fo_peer_handle_bytes.restype = ctypes.c_int
        lib.fo_peer_handle_bytes.argtypes = []
        for name, args in _SIGS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = ctypes.c_int
            fn.argtypes = args
        _lib = lib
        return lib


def declared_symbols() -> list[str]:
    return ["fo_last_error", "fo_abi_version", "fo_peer_handle_bytes", *_SIGS.keys()]


def call(name: str, *args) -> None:
    """Calls an entry point; a non-zero status raises RuntimeError with its message."""
    lib = load()
    fn = getattr(lib, name)
    rc = fn(*args)
    if rc != 0:
        msg = lib.fo_last_error().decode(errors="replace")
        kind = _STATUS.get(rc, f"status {rc}")
        if rc == -1:
            raise ValueError(f"{name}: {kind}: {msg}")
        raise RuntimeError(f"{name}: {kind}: {msg}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[t]
    except KeyError:
        raise TypeError(f"dtype {t} is not supported by flag-operators_b200") from None


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def i64_array(vals) -> ctypes.Array:
    arr = (ctypes.c_int64 * max(1, len(vals)))(*[int(v) for v in vals])
    return arr


def require_cuda(t: torch.Tensor, op: str) -> None:
    """The kernels run on CUDA tensors only; CPU tensors are rejected loudly."""
    if not t.is_cuda:
        raise RuntimeError(
            f"{op}: flag-operators_b200 computes on CUDA tensors only (got a {t.device} "
            f"tensor); move the inputs to a GPU")
    load()
