"""ctypes binding of ``libsparse_attn.so`` (C ABI in ``include/sparse_attn.h``).

The library is the product: there is no Python or CPU fallback.  If the
shared object is missing or cannot be loaded, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libsparse_attn.so"

SA_OK = 0
SA_ERR_INVALID_ARG = -1
SA_ERR_WORKSPACE = -2
SA_ERR_CUDA = -3
SA_ERR_UNSUPPORTED = -4

SA_VARIANT_AUTO = 0
SA_VARIANT_MMA = 1
SA_VARIANT_TCGEN05 = 2
SA_VARIANT_WS = 3
SA_VARIANT_WT = 4

SA_OPT_ROW_SCHEDULE = 1
SA_OPT_INDEXER_TC = 2
SA_OPT_SPIN_LIMIT = 3
SA_OPT_TEST_STALL = 4
SA_OPT_KV_POLICY = 5
SA_OPT_GATHER_ONLY = 6
SA_OPT_HEAD_GROUPS = 7

# every function the header declares, with its ctypes signature
_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)
_FWD_ARGS = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
             _I64P, _I64P, _I64P, _I64P, ctypes.c_float, _P, ctypes.c_size_t, _P]
SIGNATURES = {
    "sa_version": (ctypes.c_int, []),
    "sa_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "sa_last_cuda_error": (ctypes.c_int, []),
    "sa_variant_available": (ctypes.c_int, [ctypes.c_int]),
    "sa_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "sa_device_status_reset": (ctypes.c_int, []),
    "sa_set_option": (ctypes.c_int, [ctypes.c_int, _I64]),
    "sa_get_option": (_I64, [ctypes.c_int]),
    "sa_probe_gather": (ctypes.c_int, [_P, _I64, _P, _I64, _I64, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, _P, _P, _P]),
    "sa_index_faults": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]),
    "sa_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64, ctypes.c_int]),
    "sa_fwd": (ctypes.c_int, _FWD_ARGS),
    "sa_fwd_ex": (ctypes.c_int, _FWD_ARGS + [ctypes.c_int, ctypes.c_int]),
    "sa_fwd_noalloc": (ctypes.c_int, _FWD_ARGS[:16] + [_P, ctypes.c_int]),
    "sa_fwd_fp8": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                  _I64P, _I64P, _I64P, _I64P, _I64P, ctypes.c_float, _P,
                                  ctypes.c_size_t, _P, ctypes.c_int]),
    "sa_quantize_kv_fp8": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64P, _I64P, _I64P,
                                          _P]),
    "sa_bwd": (ctypes.c_int, [_P] * 10 + [_I64] * 6 + [_I64P] * 5 + [ctypes.c_float, _P]),
    "sa_bwd_ex": (ctypes.c_int, [_P] * 10 + [_I64] * 6 + [_I64P] * 5 + [ctypes.c_float, _P, _P]),
    "sa_dkv_zero_rows": (ctypes.c_int, [_P, _P] + [_I64] * 4 + [_I64P] * 2 + [_P]),
    "sa_dkv_cast_rows": (ctypes.c_int, [_P] * 3 + [_I64] * 4 + [_I64P] * 3 + [_P]),
    "sa_fwd_train": (ctypes.c_int, [_P] * 6 + [_I64] * 6 + [_I64P] * 4
                     + [ctypes.c_float, _P, ctypes.c_size_t, _P]),
    "sa_indexer_workspace_bytes": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "sa_indexer_topk": (ctypes.c_int, [_P] * 5 + [_I64] * 6 + [_I64P] * 5
                        + [_P, ctypes.c_size_t, _P]),
    # include/hc_sinkhorn.h
    "hcs_split_sinkhorn": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_float, _P]),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m sparse_attn.build` "
                    "(nvcc, sm_100a); sparse_attn has no fallback implementation")
            h = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def strerror(code: int) -> str:
    return lib().sa_strerror(code).decode()


def check(code: int) -> None:
    if code != SA_OK:
        msg = strerror(code)
        if code == SA_ERR_CUDA:
            msg += f" (cudaError {lib().sa_last_cuda_error()})"
        raise RuntimeError(f"sparse_attn: {msg} [status {code}]")


def device_status() -> int:
    """Error word of the tensor-core kernel on the current device (0 = healthy)."""
    v = ctypes.c_int(0)
    check(lib().sa_device_status(ctypes.byref(v)))
    return v.value


def device_status_reset() -> None:
    """Zero the error words that :func:`device_status` reads (current device)."""
    check(lib().sa_device_status_reset())


def set_option(option: int, value: int) -> int:
    """Set a process-wide library option (SA_OPT_*); returns the old value."""
    old = lib().sa_get_option(option)
    check(lib().sa_set_option(option, int(value)))
    return old


def index_faults(reset: bool = False) -> int:
    """Slots whose index was neither -1 nor in [0, kv_len), on the current
    device since the last reset (they were masked like -1)."""
    v = ctypes.c_uint64(0)
    check(lib().sa_index_faults(ctypes.byref(v), int(bool(reset))))
    return v.value


def i64_array(values) -> ctypes.Array:
    return (ctypes.c_int64 * len(values))(*values)
