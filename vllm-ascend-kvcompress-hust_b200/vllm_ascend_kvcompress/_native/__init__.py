"""ctypes binding of ``libkvc_b200.so`` (the C ABI declared in include/kvc.h).

The library is built in-tree by ``build_native.py`` for sm_100a.  There is no
fallback: if the library is missing or its ABI version differs, ``lib()``
raises, and every CUDA entry point of this package fails with it.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

ABI_VERSION = 1
LIB_NAME = "libkvc_b200.so"

KVC_OK = 0
STATUS = {0: "ok", -22: "EINVAL", -14: "ENULL", -71: "EALIGN", -95: "EUNSUPPORTED", -5: "ECUDA",
          -28: "ECAPACITY"}
CALIB_STATIC_SCRATCH_DOUBLES = 1 << 20
DEV_BLOCK_RANGE, DEV_TOKEN_RANGE, DEV_BUDGET, DEV_TIMEOUT = 1, 2, 4, 8
TENSOR_MAP_BYTES = 128
BF16, FP16 = 0, 1
AGG_MEAN, AGG_MAX = 0, 1
POLICY_GLOBAL, POLICY_V3 = 0, 1

_P = c_void_p
_SIGNATURES = {
    "kvc_abi_version": (c_int, []),
    "kvc_status_string": (ctypes.c_char_p, [c_int]),
    "kvc_coef_floats": (c_int64, [c_int, c_int, c_int, c_int]),
    "kvc_prepare_score_coefficients": (
        c_int, [_P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P, _P]),
    "kvc_score_paged_keys": (
        c_int, [_P, c_int, c_int, c_int64, c_int64, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, c_int,
                _P, c_int, c_int, _P, _P, _P, _P, _P]),
    "kvc_head_stats": (c_int, [_P, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, _P]),
    "kvc_tc_supported": (c_int, [c_int, c_int, c_int]),
    "kvc_encode_key_maps": (c_int, [_P, c_int, c_int, c_int64, c_int64, c_int, c_int, _P]),
    "kvc_fragment_words": (c_int64, [c_int, c_int]),
    "kvc_prepare_score_fragments": (
        c_int, [_P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int, _P, _P]),
    "kvc_score_paged_keys_tc": (
        c_int, [_P, c_int, c_int, c_int64, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, c_int, _P, _P, _P,
                _P, _P]),
    "kvc_normalize_aggregate": (c_int, [_P, c_int, c_int, c_int, _P, _P, _P, _P, c_int, c_int, _P, _P, _P]),
    "kvc_aggregate_rows": (c_int, [_P, c_int, c_int, _P, _P, c_int, c_int, _P, _P]),
    "kvc_select_keep": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P]),
    "kvc_compact": (
        c_int, [_P, _P, c_int, c_int64, c_int64, c_int64, _P, _P, _P, _P, _P, _P, c_int, c_int, _P, c_int, _P,
                _P, _P, _P]),
    "kvc_gather_slots": (c_int, [_P, c_int64, c_int, c_int64, c_int64, _P, c_int64, _P, _P, _P]),
    "kvc_scatter_slots": (c_int, [_P, c_int64, c_int, c_int64, c_int64, _P, c_int64, _P, _P, _P]),
    "kvc_calibration_workspace_doubles": (c_int64, [c_int64, c_int, c_int, c_int]),
    "kvc_calibration_accumulate": (
        c_int, [_P, c_int, c_int64, c_int64, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int64, _P]),
    "kvc_shift_positions": (c_int, [_P, _P, c_int, _P, c_int64, c_int64, _P, _P, _P]),
    "kvc_calibration_accumulate_noalloc": (
        c_int, [_P, c_int, c_int64, c_int64, c_int, c_int, c_int, _P, _P, _P, _P, _P]),
}

_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    override = os.environ.get("KVC_B200_LIBRARY")
    return Path(override) if override else Path(__file__).resolve().with_name(LIB_NAME)


def lib() -> ctypes.CDLL:
    """The loaded C ABI library (raises RuntimeError if absent or incompatible)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.is_file():
        raise RuntimeError(f"{LIB_NAME} is not built ({path}); run vllm-ascend-kvcompress-hust_b200/build_native.py")
    handle = ctypes.CDLL(str(path))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    got = handle.kvc_abi_version()
    if got != ABI_VERSION:
        raise RuntimeError(f"{LIB_NAME} ABI version {got} != expected {ABI_VERSION}")
    _lib = handle
    return handle


def exported_symbols() -> tuple[str, ...]:
    return tuple(_SIGNATURES)


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a non-zero C ABI status."""
    if status != KVC_OK:
        msg = lib().kvc_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {STATUS.get(status, status)} ({msg})")


def pointer_array(ptrs) -> ctypes.Array:
    """Host array of device pointers for the ``const void* const*`` arguments."""
    arr = (c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = int(p)
    return arr


__all__ = ["lib", "check", "pointer_array", "library_path", "exported_symbols", "c_float", "c_double", "c_int32"]
