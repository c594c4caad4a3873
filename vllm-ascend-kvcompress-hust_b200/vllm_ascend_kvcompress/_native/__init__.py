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
DEV_BLOCK_RANGE, DEV_TOKEN_RANGE, DEV_BUDGET, DEV_TIMEOUT, DEV_INDEX_RANGE = 1, 2, 4, 8, 16
TENSOR_MAP_BYTES = 128
IPC_HANDLE_BYTES = 64
TP_MAX_WORLD = 64
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
    "kvc_tc_partials_per_page": (c_int, []),
    "kvc_encode_key_maps": (c_int, [_P, c_int, c_int, c_int64, c_int64, c_int, c_int, _P]),
    "kvc_fragment_words": (c_int64, [c_int, c_int]),
    "kvc_prepare_score_fragments": (
        c_int, [_P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int, _P, _P]),
    "kvc_score_paged_keys_tc": (
        c_int, [_P, c_int, c_int, c_int64, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, c_int, _P, _P, _P,
                _P, _P]),
    "kvc_tc05_supported": (c_int, [c_int, c_int, c_int]),
    "kvc_prepare_score_fragments_tc05": (
        c_int, [_P, _P, c_int, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P, _P, _P, _P, _P, c_int, _P, _P]),
    "kvc_score_paged_keys_tc05": (
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
    "kvc_calibration_accumulate_post_rope": (
        c_int, [_P, c_int, c_int64, c_int64, c_int, c_int, c_int, c_int64, _P, _P, _P, _P, _P, _P, c_int64, _P]),
    "kvc_shift_positions": (c_int, [_P, _P, c_int, _P, c_int64, c_int64, _P, _P, _P]),
    "kvc_decode_offsets": (
        c_int, [_P, _P, c_int, c_int64, _P, c_int64, _P, _P, _P, c_int, c_int, _P, _P]),
    "kvc_expand_block_ids": (c_int, [_P, c_int64, c_int, _P, _P]),
    "kvc_stage_commit": (c_int, [_P, _P, c_int, c_int, _P, c_int, _P, _P, c_int, _P]),
    "kvc_calibration_accumulate_noalloc": (
        c_int, [_P, c_int, c_int64, c_int64, c_int, c_int, c_int, _P, _P, _P, _P, _P]),
    "kvc_tp_exchange_flag_words": (c_int, [c_int]),
    "kvc_tp_exchange_stamp_word": (c_int, [c_int]),
    "kvc_tp_exchange_inbox_floats": (c_int64, [c_int, c_int, c_int]),
    "kvc_tp_push_rows": (c_int, [_P, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P, _P, c_int, c_int, c_int32, _P]),
    "kvc_tp_exchange_max": (
        c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P, c_int, c_int, c_int32, _P, _P]),
    "kvc_ipc_export": (c_int, [c_int, _P, _P, _P]),
    "kvc_ipc_open": (c_int, [c_int, _P, _P]),
    "kvc_ipc_close": (c_int, [c_int, _P]),
    "kvc_can_access_peer": (c_int, [c_int, c_int]),
    "kvc_unrotate_queries": (c_int, [_P, c_int, c_int64, c_int64, c_int, c_int, c_int, c_int64, _P, _P]),
    "kvc_record_event": (c_int, [_P, _P]),
    "kvc_copy_async": (c_int, [_P, _P, c_int64, _P]),
    "kvc_triattention_step_size": (c_int64, []),
    "kvc_triattention_run": (c_int, [_P, c_int, _P, _P]),
}

SCORER_TENSOR, SCORER_FMA, SCORER_TCGEN05 = 0, 1, 2
STAGE_SCORE, STAGE_AGGREGATE, STAGE_SELECT, STAGE_COMPACT, STAGE_TABLES, STAGE_ALL = 1, 2, 4, 8, 16, 31
STAGE_EXCHANGE = 32
STEP_EVENTS = 8
STEP_EVENT_NAMES = ("prepare", "score", "head_stats", "normalize", "aggregate_rows", "select", "compact", "end")


class TriAttentionStep(ctypes.Structure):
    """``kvc_triattention_step`` (include/kvc.h), field for field."""

    _fields_ = [
        ("scorer", c_int32), ("kv_dtype", c_int32), ("score_layers", c_int32), ("kv_heads", c_int32),
        ("group", c_int32), ("head_dim", c_int32), ("rotary_dim", c_int32), ("n_off", c_int32),
        ("score_aggregation", c_int32), ("layer_aggregation", c_int32),
        ("budget", c_int32), ("prefix", c_int32), ("recent", c_int32), ("segments", c_int32), ("policy", c_int32),
        ("compact_layers", c_int32),
        ("num_blocks", c_int64), ("block_stride", c_int64), ("block_stride_bytes", c_int64), ("row_bytes", c_int64),
        ("key_maps", _P), ("score_k", _P), ("k_layers", _P), ("v_layers", _P),
        ("omega", _P), ("offsets", _P), ("q_real", _P), ("q_imag", _P), ("scale", _P), ("extra", _P),
        ("q_pass", _P), ("q_pass_t", _P),
        ("num_requests", c_int32), ("total_pages", c_int32),
        ("tokens", _P), ("page_off", _P), ("src_blocks", _P), ("src_block_off", _P), ("dst_blocks", _P),
        ("dst_block_off", _P), ("round_start", _P), ("semantic", _P), ("src_tables", _P), ("dst_tables", _P),
        ("score_coef", _P), ("raw", _P), ("partial", _P), ("mean", _P), ("var", _P), ("den", _P), ("rows", _P),
        ("agg", _P), ("keep", _P), ("staged_rows", _P), ("staged_row_stride", c_int32), ("staged_offsets", _P),
        ("error_flag", _P), ("cache_blocks_per_page", c_int32),
        ("error_host", _P), ("error_event", _P),
        ("peer_inbox", _P), ("peer_agg", _P), ("peer_flags", _P), ("world", c_int32), ("rank", c_int32),
        ("epoch", c_int32),
    ]

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
