"""ctypes binding of librepercep_b200.so (the C ABI in include/repercep_b200.h).

The library is loaded lazily on first use.  There is no fallback: if it is
missing or fails to load, every op raises, so a GPU run can never silently
take another code path.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librepercep_b200.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "repercep_b200.h"

RP_OK = 0
RP_SCALE_PER_BH = 0
RP_SCALE_PER_BLOCK128 = 1
RP_P_E4M3 = 0
RP_P_E4M3_HILO = 1
RP_DTYPE_BF16 = 0
RP_DTYPE_F16 = 1
RP_B_KN = 0
RP_B_NK = 1
RP_QUANT_PHASE_AMAX = 1
RP_QUANT_PHASE_APPLY = 2

STATUS_NAMES = {
    -1: "RP_ERR_INVALID",
    -2: "RP_ERR_UNSUPPORTED",
    -3: "RP_ERR_ALIGN",
    -4: "RP_ERR_ARCH",
    -5: "RP_ERR_CUDA",
    -6: "RP_ERR_WORKSPACE",
}

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_size_t = ctypes.c_size_t
_c_i64_p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/repercep_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "rp_abi_version": (_c_int, []),
    "rp_last_error": (ctypes.c_char_p, []),
    "rp_attn_rescale_tau": (_c_float, []),
    "rp_selftest_wait_timeout": (_c_int, [ctypes.c_longlong, _c_void_p]),
    "rp_device_status": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "rp_quant_workspace_bytes": (
        _c_int,
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size_t)],
    ),
    "rp_quant_fp8_e4m3": (
        _c_int,
        [
            _c_int,
            ctypes.POINTER(_c_void_p),
            _c_i64_p,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p),
            _c_void_p,
            _c_size_t,
            _c_void_p,
        ],
    ),
    "rp_quant_fp8_e4m3_ex": (
        _c_int,
        [
            _c_int,
            ctypes.POINTER(_c_void_p),
            _c_i64_p,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            ctypes.POINTER(_c_void_p),
            _c_int,
            ctypes.POINTER(_c_void_p),
            _c_void_p,
            _c_size_t,
            _c_void_p,
        ],
    ),
    "rp_quant_fp8_e4m3_noalloc": (
        _c_int,
        [
            _c_int,
            ctypes.POINTER(_c_void_p),
            _c_i64_p,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            ctypes.POINTER(_c_void_p),
            ctypes.POINTER(_c_void_p),
            _c_void_p,
        ],
    ),
    "rp_attn_fp8_fwd": (
        _c_int,
        [_c_void_p] * 6
        + [_c_int] * 6
        + [_c_float, _c_int, _c_int, _c_void_p, _c_i64_p, _c_void_p],
    ),
    "rp_attn_fp8_fwd_ex": (
        _c_int,
        [_c_void_p] * 6
        + [_c_int] * 7
        + [_c_float, _c_int, _c_int, _c_void_p, _c_i64_p, _c_int, _c_void_p],
    ),
    "rp_attn_fp8_fwd_chunked": (
        _c_int,
        [_c_void_p] * 6
        + [_c_int] * 7
        + [_c_float, _c_int, _c_void_p, _c_i64_p, _c_void_p],
    ),
    "rp_attn_fp8_prefix_decode": (
        _c_int,
        [_c_void_p] * 10
        + [_c_int] * 5
        + [_c_float, _c_int, _c_void_p, _c_i64_p, _c_void_p],
    ),
    "rp_fp8_gemm": (
        _c_int,
        [_c_void_p, _c_void_p, _c_void_p, _c_float, _c_float, _c_int, _c_int, _c_int, _c_void_p],
    ),
    "rp_fp8_gemm_ex": (
        _c_int,
        [
            _c_void_p,
            ctypes.c_int64,
            _c_void_p,
            ctypes.c_int64,
            _c_int,
            _c_void_p,
            ctypes.c_int64,
            _c_float,
            _c_void_p,
            ctypes.c_int64,
            _c_float,
            _c_void_p,
            _c_void_p,
            ctypes.c_int64,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_void_p,
        ],
    ),
    "rp_quant_fp8_rows": (
        _c_int,
        [_c_void_p, ctypes.c_int64, _c_int, _c_int, _c_int, _c_void_p, ctypes.c_int64, _c_void_p, _c_void_p],
    ),
    "rp_quant_fp8_e4m3_bh_phase": (
        _c_int,
        [
            _c_int,
            _c_int,
            _c_void_p,
            _c_void_p,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_void_p,
            _c_int,
            _c_void_p,
            _c_int,
            _c_void_p,
            _c_void_p,
        ],
    ),
    "rp_fp8_gemm_qkv_quant": (
        _c_int,
        [
            _c_void_p,
            ctypes.c_int64,
            _c_void_p,
            ctypes.c_int64,
            _c_void_p,
            ctypes.c_int64,
            _c_float,
            _c_void_p,
            ctypes.c_int64,
            _c_float,
            _c_void_p,
            _c_int,
            _c_int,
            _c_int,
            _c_int,
            _c_void_p,
            _c_void_p,
            _c_void_p,
            _c_void_p,
            _c_void_p,
            _c_void_p,
            _c_void_p,
        ],
    ),
}

ABI_VERSION = 4

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero rp_status."""

    def __init__(self, fn: str, code: int, message: str) -> None:
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(code, code)}: {message}")
        self.fn = fn
        self.code = code


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python -m repercep_runtime_b200.build` "
                "(the B200 path has no fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.rp_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"{LIB_PATH.name} ABI {lib.rp_abi_version()} != binding ABI {ABI_VERSION}"
            )
        _lib = lib
        return lib


def check(fn: str, rc: int) -> None:
    if rc != RP_OK:
        msg = load().rp_last_error().decode(errors="replace")
        raise NativeError(fn, rc, msg)


def i64_array(values) -> ctypes.Array:  # type: ignore[type-arg]
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * len(vals))(*vals)


def ptr_array(values) -> ctypes.Array:  # type: ignore[type-arg]
    vals = [int(v) for v in values]
    return (_c_void_p * len(vals))(*vals)


def rescale_tau() -> float:
    """Online-softmax rescale threshold (log2 units) of the attention kernels."""
    return float(load().rp_attn_rescale_tau())


def device_status(reset: bool = False) -> int:
    """Read the current device's pipeline status word (synchronises)."""
    lib = load()
    out = ctypes.c_int(0)
    check("rp_device_status", lib.rp_device_status(ctypes.byref(out), 1 if reset else 0))
    return int(out.value)
