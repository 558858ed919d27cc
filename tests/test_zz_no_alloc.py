"""The decode entry point that allocates nothing (``tkv_decode_attention_noalloc``).

Callers whose device memory is owned by someone else -- a serving runtime that
has given (nearly) all of HBM to its own pools, or a host that only binds this
C ABI and has no way to allocate device memory -- cannot provide the workspace
``tkv_decode_attention`` wants.  This entry point keeps that scratch in a fixed
device array inside the library.  The test calls it through the C ABI and
checks it against the workspace entry point, twice in a row (the array keeps
the previous call's contents), within the tolerance the other decode tests use.
It lives in its own file so it is collected after every other test, and it
needs nothing from earlier tests.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tierkv_cases import make_case, to_device  # noqa: E402

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


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


@pytest.mark.parametrize("num_splits", [0, 1, 5])
def test_noalloc_matches_workspace_entry_point_twice(num_splits):
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops
    case = make_case(seed=77 + num_splits, batch=2, q_heads=32, kv_heads=8, head_dim=128,
                     num_blocks=70, max_blocks=72)
    d = to_device(case)
    ref, ref_scores, _ = ops.decode_attention(
        d["query"], d["block_table"], d["block_states"], d["block_lengths"], d["pools"],
        d["num_blocks"], case["groups"], case["scaling"], return_scores=True,
        num_splits=num_splits)
    torch.cuda.synchronize()
    lib = N.load()
    pools = d["pools"].as_struct()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        scores = torch.full_like(ref_scores, float("nan"))
        args = _args(d, case, out, scores, num_splits)
        status = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), stream)
        assert status == N.TKV_OK, lib.tkv_status_string(status).decode()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(),
                                   atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(scores.cpu().numpy(), ref_scores.cpu().numpy(),
                                   atol=1e-4, rtol=1e-3)


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
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = lib.tkv_decode_attention_noalloc(ctypes.byref(pools), ctypes.byref(args), stream)
    assert status == N.TKV_ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.tkv_status_string(status)
