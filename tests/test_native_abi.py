"""CPU checks of the C-ABI library: it loads, exports every declared symbol,
and its host-only entry points behave (no kernel is launched here)."""

import ctypes
import os
import re

import pytest

from paged_tierkv_b200 import _native as N
from paged_tierkv_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tierkv_b200.h")


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tkv_[a-z_0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    B.build()
    return N.load()


def test_header_lists_exactly_the_bound_symbols():
    assert _declared_functions() == sorted(N.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_functions():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_version_and_status_strings(lib):
    assert lib.tkv_get_version() == 1
    for code in range(6):
        assert lib.tkv_status_string(code).decode()
    assert lib.tkv_status_string(0) == b"ok"


def test_invalid_arguments_are_rejected_without_a_device(lib):
    # host-side validation runs before any device query
    pools = N.TkvPools()
    args = N.TkvDecodeArgs()
    splits = ctypes.c_int32()
    nbytes = ctypes.c_size_t()
    assert lib.tkv_decode_plan(None, None, None, None) == N.TKV_ERR_INVALID
    pools.head_dim = 96
    pools.block_size = 16
    assert lib.tkv_decode_plan(ctypes.byref(pools), ctypes.byref(args), ctypes.byref(splits),
                               ctypes.byref(nbytes)) == N.TKV_ERR_UNSUPPORTED
    assert lib.tkv_merge_partials(None, 0, None, 0, 1, 1, 128, None, 0, None, None) == N.TKV_ERR_INVALID
    assert lib.tkv_quantize_rows_r(None, 4, 128, None, None, None, None) == N.TKV_ERR_INVALID


def test_explicit_split_plan_needs_no_device(lib):
    """With num_splits given, planning is pure host arithmetic (workspace layout)."""
    pools = N.TkvPools(16, 16, 16, 16, 16, 16, 16, 16, 64, 64, 8, 16, 128, N.TKV_FORMAT_R)
    args = N.TkvDecodeArgs()
    args.batch, args.num_heads, args.num_kv_groups = 2, 32, 4
    args.max_blocks = args.num_blocks = 100
    args.table_stride = 100
    args.num_splits = 4
    splits = ctypes.c_int32()
    nbytes = ctypes.c_size_t()
    assert lib.tkv_decode_plan(ctypes.byref(pools), ctypes.byref(args), ctypes.byref(splits),
                               ctypes.byref(nbytes)) == N.TKV_OK
    assert splits.value == 4
    rows = 2 * 32
    assert nbytes.value >= rows * 4 * 128 * 4 + rows * 4 * 4
