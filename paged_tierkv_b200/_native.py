"""ctypes binding of ``lib/libtierkv_b200.so`` (declared in include/tierkv_b200.h).

The library is the only compute path: if it is missing, or no B200 is
present, calls raise instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

# status codes (include/tierkv_b200.h)
TKV_OK = 0
TKV_ERR_INVALID = 1
TKV_ERR_UNSUPPORTED = 2
TKV_ERR_WORKSPACE = 3
TKV_ERR_CUDA = 4
TKV_ERR_NO_DEVICE = 5
TKV_ERR_SCRATCH_LIMIT = 6
TKV_NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024

TKV_FORMAT_R = 0
TKV_FORMAT_S = 1
TKV_DTYPE_F16 = 0
TKV_DTYPE_BF16 = 1
TKV_DTYPE_F32 = 2

TKV_DEVERR_BAD_SLOT = 0x1
TKV_DEVERR_TIMEOUT = 0x2

EXPORTED_SYMBOLS = (
    "tkv_get_version",
    "tkv_status_string",
    "tkv_decode_plan",
    "tkv_decode_attention",
    "tkv_merge_partials",
    "tkv_block_scores",
    "tkv_quantize_rows_r",
    "tkv_demote_to_warm",
    "tkv_promote_to_hot",
    "tkv_read_device_errors",
    "tkv_decode_attention_noalloc",
    "tkv_noalloc_prepare",
    "tkv_noalloc_read_device_errors",
    "tkv_append_hot_tokens",
    "tkv_exchange_bytes",
    "tkv_exchange_alloc",
    "tkv_exchange_open",
    "tkv_exchange_close",
    "tkv_exchange_free",
    "tkv_decode_attention_exchange",
    "tkv_prefill_lse",
    "tkv_prefill_block_scores",
    "tkv_prefill_read_errors",
    "tkv_store_prefill_blocks",
)

TKV_EXCHANGE_MAX_RANKS = 8
TKV_IPC_HANDLE_BYTES = 64

TKV_APPEND_MAX_CELLS = 8


class TkvPools(ctypes.Structure):
    _fields_ = [
        ("hot_k", ctypes.c_void_p),
        ("hot_v", ctypes.c_void_p),
        ("warm_k", ctypes.c_void_p),
        ("warm_v", ctypes.c_void_p),
        ("k_scale", ctypes.c_void_p),
        ("k_zero", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
        ("v_zero", ctypes.c_void_p),
        ("hot_slots", ctypes.c_int64),
        ("warm_slots", ctypes.c_int64),
        ("kv_heads", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("format", ctypes.c_int32),
    ]


class TkvDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("query", ctypes.c_void_p),
        ("query_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_groups", ctypes.c_int32),
        ("max_blocks", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("block_states", ctypes.c_void_p),
        ("block_lengths", ctypes.c_void_p),
        ("table_stride", ctypes.c_int64),
        ("num_blocks_dev", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int32),
        ("scaling", ctypes.c_float),
        ("out", ctypes.c_void_p),
        ("out_lse", ctypes.c_void_p),
        ("score_sums", ctypes.c_void_p),
        ("num_splits", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class TkvTableCell(ctypes.Structure):
    _fields_ = [
        ("table", ctypes.c_void_p),
        ("index", ctypes.c_int64),
        ("value", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class TkvExchange(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("epoch", ctypes.c_uint32),
        ("rows_cap", ctypes.c_int32),
        ("units_cap", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("timeout_ns", ctypes.c_uint64),
        ("epoch_dev", ctypes.c_void_p),
        ("inbox", ctypes.c_void_p * 8),
    ]


_LIB = None


def library_path() -> str:
    """The in-tree build, or the file named by TIERKV_B200_LIBRARY."""
    return os.environ.get("TIERKV_B200_LIBRARY") or _build.lib_path()


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load the C-ABI library (once).  Raises RuntimeError if it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not os.path.exists(path):
        if build_if_missing:
            _build.build()
        else:
            raise RuntimeError(
                f"{path} is missing: build it with `python -m paged_tierkv_b200.build` "
                "(there is no fallback path)")
    lib = ctypes.CDLL(path)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    sigs = {
        "tkv_get_version": ([], i32),
        "tkv_status_string": ([i32], ctypes.c_char_p),
        "tkv_decode_plan": ([ctypes.POINTER(TkvPools), ctypes.POINTER(TkvDecodeArgs),
                             ctypes.POINTER(i32), ctypes.POINTER(ctypes.c_size_t)], i32),
        "tkv_decode_attention": ([ctypes.POINTER(TkvPools), ctypes.POINTER(TkvDecodeArgs), vp], i32),
        "tkv_merge_partials": ([vp, i64, vp, i64, i32, i32, i32, vp, i32, vp, vp], i32),
        "tkv_block_scores": ([vp, vp, i64, vp, i32, i32, i32, i32, vp, vp], i32),
        "tkv_quantize_rows_r": ([vp, i64, i32, vp, vp, vp, vp], i32),
        "tkv_demote_to_warm": ([ctypes.POINTER(TkvPools), vp, vp, vp, i32, i32, vp], i32),
        "tkv_promote_to_hot": ([ctypes.POINTER(TkvPools), vp, vp, vp, i32, vp], i32),
        "tkv_read_device_errors": ([vp, ctypes.POINTER(ctypes.c_uint32), vp], i32),
        "tkv_decode_attention_noalloc": ([ctypes.POINTER(TkvPools), ctypes.POINTER(TkvDecodeArgs),
                                          vp], i32),
        "tkv_noalloc_prepare": ([i32], i32),
        "tkv_noalloc_read_device_errors": ([ctypes.POINTER(ctypes.c_uint32), vp], i32),
        "tkv_append_hot_tokens": ([ctypes.POINTER(TkvPools), i32, i32, i32, vp, vp,
                                   ctypes.POINTER(TkvTableCell), i32, vp], i32),
        "tkv_exchange_bytes": ([i32, i32, i32, i32], ctypes.c_size_t),
        "tkv_exchange_alloc": ([ctypes.c_size_t, ctypes.POINTER(vp), vp], i32),
        "tkv_exchange_open": ([vp, ctypes.POINTER(vp)], i32),
        "tkv_exchange_close": ([vp], i32),
        "tkv_exchange_free": ([vp], i32),
        "tkv_decode_attention_exchange": ([ctypes.POINTER(TkvPools), ctypes.POINTER(TkvDecodeArgs),
                                           ctypes.POINTER(TkvExchange), vp], i32),
        "tkv_prefill_lse": ([vp, vp, i32, i32, i32, i32, i32, i32, ctypes.c_float, i32, vp, vp], i32),
        "tkv_prefill_block_scores": ([vp, vp, vp, i32, i32, i32, i32, i32, i32, ctypes.c_float, i32,
                                      i32, vp, vp, vp], i32),
        "tkv_prefill_read_errors": ([ctypes.POINTER(ctypes.c_uint32), vp], i32),
        "tkv_store_prefill_blocks": ([ctypes.POINTER(TkvPools), vp, vp, i32, vp, i32, vp], i32),
    }
    for name, (argtypes, restype) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _LIB = lib
    return lib


class TierKVError(RuntimeError):
    """A CUDA-side failure reported by the library."""


def check(status: int, what: str) -> None:
    """Map a tkv_status to the reference's exception types."""
    if status == TKV_OK:
        return
    msg = load().tkv_status_string(status).decode()
    if status in (TKV_ERR_INVALID, TKV_ERR_UNSUPPORTED, TKV_ERR_WORKSPACE, TKV_ERR_SCRATCH_LIMIT):
        raise ValueError(f"{what}: {msg}")
    raise TierKVError(f"{what}: {msg} (status {status})")
