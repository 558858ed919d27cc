"""The decode entry point that allocates nothing (``tkv_decode_attention_noalloc``).

Callers whose device memory is owned by someone else -- a serving runtime that
has given (nearly) all of HBM to its own pools, or a host that only binds this
C ABI and has no way to allocate device memory -- cannot provide the workspace
``tkv_decode_attention`` wants.  This entry point keeps that scratch in a fixed
device array inside the library.  The tests call it through the C ABI and check
it against the float64 oracle and against the workspace entry point, twice in a
row (the array keeps the previous call's contents), within the tolerance the
other decode tests use; check that an out-of-pool slot is reported through the
array's own error word; and check, in a fresh process under lazy module
loading, that ``tkv_noalloc_prepare`` commits the array up front so the call
itself takes no device memory.  They live in a file of their own so they are
collected after every other test, and they need nothing from earlier tests.
"""

import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import tierkv_oracle as orc  # noqa: E402
from tierkv_cases import make_case, oracle_decode, to_device  # noqa: E402

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)


def _args(d, case, out, scores, num_splits):
    from paged_tierkv_b200 import _native as N
    q = d["query"]
    b, hq, _ = q.shape
    t = d["block_table"]
    return N.TkvDecodeArgs(
        q.data_ptr(), N.TKV_DTYPE_F16, N.TKV_DTYPE_F16, b, hq, case["groups"], t.shape[1],
        t.data_ptr(), d["block_states"].data_ptr(), d["block_lengths"].data_ptr(), t.stride(0),
        d["num_blocks"].data_ptr(), t.shape[1], case["scaling"], out.data_ptr(), None,
        None if scores is None else scores.data_ptr(), num_splits, 0, None, 0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _read_errors():
    from paged_tierkv_b200 import _native as N
    bits = ctypes.c_uint32()
    status = N.load().tkv_noalloc_read_device_errors(ctypes.byref(bits), _stream())
    assert status == N.TKV_OK
    return int(bits.value)


@pytest.mark.parametrize("num_splits", [0, 1, 5])
def test_noalloc_matches_oracle_and_workspace_entry_point_twice(num_splits):
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops
    case = make_case(seed=77 + num_splits, batch=2, q_heads=32, kv_heads=8, head_dim=128,
                     num_blocks=70, max_blocks=72)
    ref_o, _, ref_s = oracle_decode(case)
    d = to_device(case)
    ws_out, ws_scores, _ = ops.decode_attention(
        d["query"], d["block_table"], d["block_states"], d["block_lengths"], d["pools"],
        d["num_blocks"], case["groups"], case["scaling"], return_scores=True,
        num_splits=num_splits)
    torch.cuda.synchronize()
    lib = N.load()
    pools = d["pools"].as_struct()
    assert lib.tkv_noalloc_prepare(-1) == N.TKV_OK
    _read_errors()  # start from a clear error word
    for _ in range(2):
        out = torch.full_like(ws_out, float("nan"))
        scores = torch.full_like(ws_scores, float("nan"))
        args = _args(d, case, out, scores, num_splits)
        status = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), _stream())
        assert status == N.TKV_OK, lib.tkv_status_string(status).decode()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        np.testing.assert_allclose(got, ref_o, atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(got, ws_out.float().cpu().numpy(), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(scores.cpu().numpy(), ref_s, atol=1e-4, rtol=1e-3)
        np.testing.assert_allclose(scores.cpu().numpy(), ws_scores.cpu().numpy(),
                                   atol=1e-4, rtol=1e-3)
    assert _read_errors() == 0


def test_noalloc_reports_an_out_of_pool_slot():
    """A HOT slot past the pool reads as zeros (like a COLD block with valid
    tokens) and sets TKV_DEVERR_BAD_SLOT in the array's sticky error word;
    reading the word clears it, and the next clean call leaves it clear."""
    from paged_tierkv_b200 import _native as N
    case = make_case(seed=19, batch=1, q_heads=8, kv_heads=2, head_dim=64, num_blocks=6,
                     states=[0, 1, 0, 0, 1, 0])
    ref_case = dict(case, block_states=case["block_states"].copy())
    ref_case["block_states"][0, 2] = orc.COLD_STATE
    ref_o, _, _ = oracle_decode(ref_case)
    bad = dict(case, block_table=case["block_table"].copy())
    bad["block_table"][0, 2] = case["hot_k"].shape[0] + 100
    lib = N.load()
    _read_errors()
    for c, expect in ((bad, N.TKV_DEVERR_BAD_SLOT), (case, 0)):
        d = to_device(c)
        out = torch.full((1, 8, 64), float("nan"), dtype=torch.float16, device="cuda")
        pools = d["pools"].as_struct()
        args = _args(d, c, out, None, 0)
        status = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), _stream())
        assert status == N.TKV_OK
        torch.cuda.synchronize()
        if expect:
            np.testing.assert_allclose(out.float().cpu().numpy(), ref_o, atol=ATOL, rtol=RTOL)
        assert _read_errors() & N.TKV_DEVERR_BAD_SLOT == expect
    assert _read_errors() == 0


def test_noalloc_rejects_calls_beyond_its_array():
    from paged_tierkv_b200 import _native as N
    case = make_case(seed=5, batch=2, q_heads=32, kv_heads=8, head_dim=128, num_blocks=8,
                     max_blocks=8)
    d = to_device(case)
    # score scratch alone: batch * heads * max_blocks * 4 bytes > 32 MiB
    wide = 140_000
    big = {k: torch.full((2, wide), v, dtype=torch.int32, device="cuda")
           for k, v in (("block_table", -1), ("block_states", 2), ("block_lengths", 0))}
    d.update(big)
    out = torch.empty((2, 32, 128), dtype=torch.float16, device="cuda")
    scores = torch.empty((1,), dtype=torch.float32, device="cuda")
    args = _args(d, case, out, scores, 0)
    lib = N.load()
    pools = d["pools"].as_struct()
    status = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), _stream())
    assert status == N.TKV_ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.tkv_status_string(status)


_LAZY_CHILD = textwrap.dedent("""
    import ctypes, json, sys
    import torch
    sys.path.insert(0, {root!r})
    sys.path.insert(0, {tests!r})
    from tierkv_cases import make_case, to_device
    from paged_tierkv_b200 import _native as N
    lib = N.load()
    case = make_case(seed=3, batch=2, q_heads=32, kv_heads=8, head_dim=128, num_blocks=40)
    d = to_device(case)
    out = torch.empty((2, 32, 128), dtype=torch.float16, device="cuda")
    q = d["query"]; t = d["block_table"]
    args = N.TkvDecodeArgs(q.data_ptr(), 0, 0, 2, 32, 4, t.shape[1], t.data_ptr(),
                           d["block_states"].data_ptr(), d["block_lengths"].data_ptr(), t.stride(0),
                           d["num_blocks"].data_ptr(), t.shape[1], case["scaling"], out.data_ptr(),
                           None, None, 3, 0, None, 0)
    pools = d["pools"].as_struct()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    st_prep = lib.tkv_noalloc_prepare(-1)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    st_call = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), stream)
    torch.cuda.synchronize()
    free2 = torch.cuda.mem_get_info()[0]
    print(json.dumps(dict(st_prep=st_prep, st_call=st_call, prepare_bytes=free0 - free1,
                          call_bytes=free1 - free2)))
""")


def test_noalloc_prepare_commits_the_array_under_lazy_loading():
    """Fresh process with CUDA_MODULE_LOADING=LAZY: the 32 MiB array is taken
    from the device when tkv_noalloc_prepare runs, not by the later call."""
    from paged_tierkv_b200 import _native as N
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    code = _LAZY_CHILD.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    import json
    r = json.loads(res.stdout.strip().splitlines()[-1])
    assert r["st_prep"] == N.TKV_OK and r["st_call"] == N.TKV_OK
    assert r["prepare_bytes"] >= N.TKV_NOALLOC_SCRATCH_BYTES
    assert r["call_bytes"] < N.TKV_NOALLOC_SCRATCH_BYTES
