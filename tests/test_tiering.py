"""Batched storage sync (one policy tick) against the reference's own result.

Golden fixtures (tests/golden/make_tiering_golden.py) hold a compact pool's
complete state before and after the reference's ``sync_storage_states``
(tierkv_policy.py:1849-1867).  The CPU tests replay the bookkeeping and the
table cells; the GPU tests also move the data with the batched kernels and
compare every pool byte, stale rows of reused slots included.
"""

import glob
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from compact_pool_stub import CompactPoolStub  # noqa: E402
from paged_tierkv_b200 import tiering  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "tiering_*.npz")))
TABLES = ("block_states", "block_slot_indices", "block_lengths")


def _load(path):
    return dict(np.load(path))


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_bookkeeping_matches_reference(path):
    fx = _load(path)
    pool = CompactPoolStub(fx, "cpu")
    meta = pool.meta
    plan = tiering.plan_sync(pool, meta["layer"], meta["physical_indices"], meta["desired"])
    assert pool.bookkeeping() == meta["after"]
    # the recorded row and cells turn the "before" tables into the "after" tables
    for name, t in _apply_cells(fx, plan).items():
        np.testing.assert_array_equal(t, fx[f"after_{name}"], err_msg=name)


def _apply_cells(fx, plan):
    tables = {n: fx[f"before_{n}"].copy() for n in TABLES}
    if plan.state_row is not None:
        tables["block_states"][plan.layer, :len(plan.state_row)] = plan.state_row
    for name, cells in zip(TABLES, (plan.states, plan.slots, plan.lengths)):
        for (layer, logical), v in cells.items():
            tables[name][layer, logical] = v
    return tables


@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_transition_walk_equals_block_by_block_loop(path):
    """Walking only the transitions (the fast path) leaves the same
    bookkeeping and tables as the block-by-block loop."""
    fx = _load(path)
    fast = CompactPoolStub(fx, "cpu")
    slow = CompactPoolStub(fx, "cpu")
    meta = fast.meta
    plan_f = tiering.plan_sync(fast, meta["layer"], meta["physical_indices"], meta["desired"])
    assert plan_f.state_row is not None  # the fixtures take the fast path
    plan_s = tiering._plan_sync_loop(slow, tiering.SyncPlan(meta["layer"]), meta["layer"],
                                     meta["physical_indices"], meta["desired"])
    assert fast.bookkeeping() == slow.bookkeeping()
    assert plan_f.demotions == plan_s.demotions and plan_f.promotions == plan_s.promotions
    for name in TABLES:
        np.testing.assert_array_equal(_apply_cells(fx, plan_f)[name], _apply_cells(fx, plan_s)[name])


@pytest.mark.parametrize("kind", ["list", "int32", "uint8", "tensor", "float", "numpy_scalars"])
def test_plan_input_types_give_the_same_plan(kind):
    """plan_sync takes the block and state sequences the reference's loop
    would (lists, arrays, tensors, floats that int() truncates) and plans
    the same moves and cells for each."""
    path = FIXTURES[0]
    fx = _load(path)
    ref_pool = CompactPoolStub(fx, "cpu")
    meta = ref_pool.meta
    phys, want = list(meta["physical_indices"]), list(meta["desired"])
    ref = tiering.plan_sync(ref_pool, meta["layer"], phys, want)
    conv = {
        "list": lambda x: [int(v) for v in x],
        "int32": lambda x: np.asarray(x, dtype=np.int32),
        "uint8": lambda x: np.asarray(x, dtype=np.uint8) if max(x) < 256 else np.asarray(x),
        "tensor": lambda x: torch.tensor([int(v) for v in x], dtype=torch.int64),
        "float": lambda x: [float(v) + 0.25 for v in x],
        "numpy_scalars": lambda x: [np.int16(v) for v in x],
    }[kind]
    pool = CompactPoolStub(fx, "cpu")
    plan = tiering.plan_sync(pool, meta["layer"], conv(phys), conv(want))
    assert pool.bookkeeping() == ref_pool.bookkeeping()
    assert plan.demotions == ref.demotions and plan.promotions == ref.promotions
    np.testing.assert_array_equal(plan.state_row, ref.state_row)
    assert (plan.states, plan.slots, plan.lengths) == (ref.states, ref.slots, ref.lengths)


def test_fixtures_cover_slot_reuse_and_growth():
    """The scenarios exercise what the staging and growth paths are for."""
    staged_dem = staged_pro = grown = 0
    for path in FIXTURES:
        fx = _load(path)
        pool = CompactPoolStub(fx, "cpu")
        meta = pool.meta
        before = (pool.allocated_hot_slots, pool.allocated_warm_slots)
        plan = tiering.plan_sync(pool, meta["layer"], meta["physical_indices"], meta["desired"])
        d, p = plan.staged()
        staged_dem += len(d)
        staged_pro += len(p)
        grown += (pool.allocated_hot_slots, pool.allocated_warm_slots) != before
    assert staged_dem > 0 and staged_pro > 0 and grown > 0


def test_cold_to_hot_is_rejected_like_the_reference():
    fx = _load(os.path.join(GOLDEN, "tiering_swap.npz"))
    pool = CompactPoolStub(fx, "cpu")
    meta = pool.meta
    cold = [i for i, p in enumerate(meta["physical_indices"])
            if meta["before"]["physical_states"][str(p)] == tiering.COLD_STATE]
    desired = list(meta["desired"])
    desired[cold[0]] = tiering.HOT_STATE
    with pytest.raises(KeyError, match="cannot be promoted from COLD to HOT"):
        tiering.plan_sync(pool, meta["layer"], meta["physical_indices"], desired)


@pytest.mark.gpu
@pytest.mark.parametrize("path", FIXTURES, ids=lambda p: os.path.basename(p)[:-4])
def test_batched_sync_matches_reference_bytes(path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    fx = _load(path)
    pool = CompactPoolStub(fx, "cuda")
    meta = pool.meta
    plan = tiering.plan_sync(pool, meta["layer"], meta["physical_indices"], meta["desired"])
    stats = tiering.apply_sync(pool, plan)
    torch.cuda.synchronize()
    assert stats["demotions"] + stats["promotions"] > 0
    assert pool.bookkeeping() == meta["after"]
    got = {"hot_k": pool.hot_k_pool, "hot_v": pool.hot_v_pool, "warm_k": pool.warm_k_pool,
           "warm_v": pool.warm_v_pool, "k_scale": pool.k_scale, "k_zero": pool.k_zero,
           "v_scale": pool.v_scale, "v_zero": pool.v_zero, "block_states": pool.block_states,
           "block_slot_indices": pool.block_slot_indices, "block_lengths": pool.block_lengths,
           "physical_block_tables": pool.physical_block_tables}
    for name, t in got.items():
        want = fx[f"after_{name}"]
        have = t.cpu().numpy()
        assert have.shape == want.shape, name
        # compare bit patterns (signed zeros, NaN payloads)
        np.testing.assert_array_equal(have.view(np.uint8), want.view(np.uint8), err_msg=name)


@pytest.mark.gpu
def test_runtime_method_drop_in():
    """sync_storage_states bound to a runtime-like object, as the reference calls it."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import types
    fx = _load(FIXTURES[0])
    pool = CompactPoolStub(fx, "cuda")
    meta = pool.meta
    bm = types.SimpleNamespace(get_physical_indices=lambda s: list(meta["physical_indices"]),
                               get_states=lambda s: list(meta["desired"]))
    runtime = types.SimpleNamespace(block_manager=bm, kv_pool=pool)
    tiering.sync_storage_states(runtime, meta["layer"])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(pool.warm_k_pool.cpu().numpy(), fx["after_warm_k"])
    np.testing.assert_array_equal(pool.block_states.cpu().numpy(), fx["after_block_states"])


# ---------------------------------------------------------------------------
# decode-time append
# ---------------------------------------------------------------------------

def _append_runtime(fx, device):
    import types
    from compact_pool_stub import BlockManagerStub, LayerState
    pool = CompactPoolStub(fx, device)
    meta = pool.meta
    layers = {int(k): LayerState(*v) for k, v in meta["before_layers"].items()}
    rt = types.SimpleNamespace(layer_states=layers, block_manager=BlockManagerStub(meta["before_bm_free"]),
                               kv_pool=pool, block_size=meta["block_size"],
                               max_blocks_per_layer=meta["max_blocks_per_layer"])
    return rt, pool, meta


def _demote_open(rt, pool, layer):
    """The fixture's event: the layer's open block goes WARM (demote_to_warm +
    set_block_state), done with the batched tick's machinery."""
    p = rt.layer_states[layer].open_physical_idx
    plan = tiering.SyncPlan(layer)
    tiering._demote_to_warm(pool, plan, p)
    loc = pool.physical_locations[p]
    plan.states[(int(loc[0]), int(loc[1]))] = tiering.WARM_STATE
    return plan


def test_append_bookkeeping_matches_reference():
    fx = _load(os.path.join(GOLDEN, "append_decode.npz"))
    rt, pool, meta = _append_runtime(fx, "cpu")
    tables = {n: fx[f"before_{n}"].copy() for n in TABLES + ("physical_block_tables",)}

    def put(plan):
        for name, cells in zip(TABLES + ("physical_block_tables",),
                               (plan.states, plan.slots, plan.lengths, plan.physical)):
            for (layer, logical), v in cells.items():
                tables[name][layer, logical] = v

    for call in meta["calls"]:
        if "demote_open" in call:
            put(_demote_open(rt, pool, call["demote_open"]))
            continue
        i = call["index"]
        k = torch.from_numpy(fx[f"in_{i}_k"])
        v = torch.from_numpy(fx[f"in_{i}_v"])
        steps, new_block = tiering.plan_append(rt, call["layer"], k, v)
        assert new_block == call["new_block"], i
        for st in steps:
            put(st.plan)
    assert pool.bookkeeping() == meta["after"]
    assert {str(k): v.as_list() for k, v in rt.layer_states.items()} == meta["after_layers"]
    assert rt.block_manager.free == meta["after_bm_free"]
    for name, t in tables.items():
        np.testing.assert_array_equal(t, fx[f"after_{name}"], err_msg=name)


@pytest.mark.gpu
def test_fused_append_matches_reference_bytes():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    fx = _load(os.path.join(GOLDEN, "append_decode.npz"))
    rt, pool, meta = _append_runtime(fx, "cuda")
    launches = 0
    for call in meta["calls"]:
        if "demote_open" in call:
            tiering.apply_sync(pool, _demote_open(rt, pool, call["demote_open"]))
            continue
        i = call["index"]
        k = torch.from_numpy(fx[f"in_{i}_k"]).cuda()
        v = torch.from_numpy(fx[f"in_{i}_v"]).cuda()
        steps, new_block = tiering.plan_append(rt, call["layer"], k, v)
        launches += tiering.apply_append(pool, steps)
        assert new_block == call["new_block"], i
    torch.cuda.synchronize()
    assert launches == sum(1 for c in meta["calls"] if "index" in c) + 2  # + a second block, a promotion
    assert pool.bookkeeping() == meta["after"]
    got = {"hot_k": pool.hot_k_pool, "hot_v": pool.hot_v_pool, "warm_k": pool.warm_k_pool,
           "warm_v": pool.warm_v_pool, "k_scale": pool.k_scale, "k_zero": pool.k_zero,
           "v_scale": pool.v_scale, "v_zero": pool.v_zero, "block_states": pool.block_states,
           "block_slot_indices": pool.block_slot_indices, "block_lengths": pool.block_lengths,
           "physical_block_tables": pool.physical_block_tables}
    for name, t in got.items():
        want = fx[f"after_{name}"]
        have = t.cpu().numpy()
        assert have.shape == want.shape, name
        np.testing.assert_array_equal(have.view(np.uint8), want.view(np.uint8), err_msg=name)


@pytest.mark.gpu
def test_fused_append_rejects_bad_arguments():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import ctypes
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops
    pools = ops.TieredPools.allocate(4, 4, 2, 16, 64, "cuda")
    k = torch.zeros((2, 1, 64), dtype=torch.float16, device="cuda")
    ps = pools.as_struct()
    lib = N.load()
    stream = ops._stream(None)
    cells = (N.TkvTableCell * 1)()
    for slot, start, tokens in ((4, 0, 1), (-1, 0, 1), (0, 16, 1), (0, 15, 2), (0, 0, 0)):
        st = lib.tkv_append_hot_tokens(ctypes.byref(ps), slot, start, tokens, k.data_ptr(),
                                       k.data_ptr(), cells, 0, stream)
        assert st == N.TKV_ERR_INVALID, (slot, start, tokens)
    st = lib.tkv_append_hot_tokens(ctypes.byref(ps), 0, 0, 1, k.data_ptr(), k.data_ptr(), cells,
                                   N.TKV_APPEND_MAX_CELLS + 1, stream)
    assert st == N.TKV_ERR_INVALID
