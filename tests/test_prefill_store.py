"""Prefill with policy (append_prefill_with_policy, tierkv_policy.py:1722-1766)
against the reference's own result.

The fixture (tests/golden/make_tiering_golden.py, ``prefill_policy.npz``)
holds a compact pool's complete state before and after a series of prefills
made by the reference, with their inputs.  The CPU test replays the
bookkeeping (block manager, slots, dictionaries, table cells); the GPU tests
also store the data with the one-launch prefill store and compare every pool
byte, and check a head_dim 128 / block 32 layer against the oracle quantizer.
"""

import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from compact_pool_stub import (BlockManagerStub, CompactPoolStub, LayerState,  # noqa: E402
                               PrefillRuntimeStub)
from paged_tierkv_b200 import tiering  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TABLES = ("block_states", "block_slot_indices", "block_lengths", "physical_block_tables")
POOLS = ("hot_k", "hot_v", "warm_k", "warm_v", "k_scale", "k_zero", "v_scale", "v_zero")


def _fixture():
    return dict(np.load(os.path.join(GOLDEN, "prefill_policy.npz")))


def _runtime(fx, device):
    pool = CompactPoolStub(fx, device)
    meta = pool.meta
    bm = BlockManagerStub(meta["before_bm"]["free"])
    bm.tables = {int(k): [list(b) for b in v] for k, v in meta["before_bm"]["tables"].items()}
    layers = {int(k): LayerState(*v) for k, v in meta["before_layers"].items()}
    rt = PrefillRuntimeStub(pool, bm, layers, meta["block_size"], meta["max_blocks_per_layer"])
    return rt, pool, meta


def _call_inputs(fx, rt, call, device):
    rt.policy_mode, rt.hot_budget, rt.warm_budget = (call["policy_mode"], call["hot_budget"],
                                                     call["warm_budget"])
    i = call["index"]
    k = torch.from_numpy(fx[f"in_{i}_k"]).to(device)
    v = torch.from_numpy(fx[f"in_{i}_v"]).to(device)
    return k, v, torch.from_numpy(fx[f"in_{i}_scores"])


def _check_bookkeeping(rt, pool, meta):
    assert pool.bookkeeping() == meta["after"]
    assert {str(k): v.as_list() for k, v in rt.layer_states.items()} == meta["after_layers"]
    assert rt.block_manager.free == meta["after_bm"]["free"]
    assert {str(k): v for k, v in rt.block_manager.tables.items()} == meta["after_bm"]["tables"]


def test_fixture_covers_every_branch():
    meta = json.loads(str(_fixture()["meta"]))
    desired = [s for c in meta["calls"] for s in c["desired"]]
    assert {0, 1, 2} <= set(desired)
    assert any(c["tokens"] % meta["block_size"] for c in meta["calls"])      # a partial block
    assert any(len(c["desired"]) <= 2 for c in meta["calls"])                # all-HOT short layer
    assert meta["after"]["allocated_warm_slots"] > meta["before"]["allocated_warm_slots"]
    assert meta["after"]["allocated_hot_slots"] > meta["before"]["allocated_hot_slots"]


def test_prefill_bookkeeping_matches_reference():
    fx = _fixture()
    rt, pool, meta = _runtime(fx, "cpu")
    tables = {n: fx[f"before_{n}"].copy() for n in TABLES}
    for call in meta["calls"]:
        k, v, scores = _call_inputs(fx, rt, call, "cpu")
        assert rt._desired_prefill_states(len(scores), scores) == call["desired"]
        pp = tiering.plan_prefill(rt, call["layer"], k, v, scores)
        assert [e[0] for e in pp.entries] == [s for s in call["desired"] if s != 2]
        p = pp.plan
        for name, cells in zip(TABLES, (p.states, p.slots, p.lengths, p.physical)):
            for (layer, logical), val in cells.items():
                tables[name][layer, logical] = val
    _check_bookkeeping(rt, pool, meta)
    for name, t in tables.items():
        np.testing.assert_array_equal(t, fx[f"after_{name}"], err_msg=name)


def test_prefill_rejects_like_the_reference():
    fx = _fixture()
    rt, pool, meta = _runtime(fx, "cpu")
    k = torch.zeros((1, meta["kv_heads"], 20, meta["head_dim"]), dtype=torch.float16)
    with pytest.raises(ValueError):  # key and value lengths differ
        tiering.plan_prefill(rt, 1, k, k[:, :, :10], torch.zeros(2))
    with pytest.raises(RuntimeError):  # layer 0 already holds blocks
        tiering.plan_prefill(rt, 0, k, k, torch.zeros(2))
    long = torch.zeros((1, meta["kv_heads"], 16 * (meta["max_blocks_per_layer"] + 1), meta["head_dim"]),
                       dtype=torch.float16)
    with pytest.raises(RuntimeError):  # more blocks than the layer holds
        tiering.plan_prefill(rt, 1, long, long, torch.zeros(meta["max_blocks_per_layer"] + 1))


@pytest.mark.gpu
def test_prefill_store_matches_reference_bytes():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    fx = _fixture()
    rt, pool, meta = _runtime(fx, "cuda")
    for call in meta["calls"]:
        k, v, scores = _call_inputs(fx, rt, call, "cuda")
        tiering.append_prefill_with_policy(rt, call["layer"], k, v, scores)
    torch.cuda.synchronize()
    _check_bookkeeping(rt, pool, meta)
    got = dict(zip(POOLS, (pool.hot_k_pool, pool.hot_v_pool, pool.warm_k_pool, pool.warm_v_pool,
                           pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero)))
    got.update(zip(TABLES, (pool.block_states, pool.block_slot_indices, pool.block_lengths,
                            pool.physical_block_tables)))
    for name, t in got.items():
        want = fx[f"after_{name}"]
        have = t.cpu().numpy()
        assert have.shape == want.shape, name
        np.testing.assert_array_equal(have.view(np.uint8), want.view(np.uint8), err_msg=name)


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim,block_size", [(128, 32), (128, 16), (64, 32)])
def test_prefill_store_kernel_against_oracle(head_dim, block_size):
    """Direct C-ABI call: HOT entries copy rows and zero the tail, WARM entries
    quantize like the oracle and clear the tail; entries outside the pools or
    the input are skipped."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import ctypes
    import oracle.tierkv_oracle as orc
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(head_dim + block_size)
    kvh, tokens, hs, ws = 4, 5 * block_size - 3, 9, 7
    key = rng.standard_normal((kvh, tokens, head_dim)).astype(np.float16)
    val = (3 * rng.standard_normal((kvh, tokens, head_dim))).astype(np.float16)
    pools = ops.TieredPools.allocate(hs, ws, kvh, block_size, head_dim, "cuda")
    for t in (pools.hot_k, pools.hot_v, pools.warm_k, pools.warm_v):
        t.fill_(7)  # stale bytes the stores must overwrite
    entries = [(0, 3, 0, block_size), (1, 5, block_size, block_size), (0, 8, 2 * block_size, 5),
               (1, 0, 3 * block_size, block_size - 1), (0, 0, 4 * block_size, block_size - 3),
               (0, hs, 0, 4), (1, ws, 0, 4), (0, 1, tokens - 2, 4), (2, 2, 0, 4)]  # last 4 skipped
    dev = torch.tensor(entries, dtype=torch.int32, device="cuda")
    kd, vd = torch.from_numpy(key).cuda(), torch.from_numpy(val).cuda()
    ps = pools.as_struct()
    st = N.load().tkv_store_prefill_blocks(ctypes.byref(ps), kd.data_ptr(), vd.data_ptr(), tokens,
                                            dev.data_ptr(), len(entries), ops._stream(None))
    assert st == N.TKV_OK
    torch.cuda.synchronize()
    hk, hv = pools.hot_k.cpu().numpy(), pools.hot_v.cpu().numpy()
    wk, wv = pools.warm_k.cpu().numpy(), pools.warm_v.cpu().numpy()
    meta = [x.cpu().numpy().reshape(ws, kvh, block_size) for x in
            (pools.k_scale, pools.k_zero, pools.v_scale, pools.v_zero)]
    for state, slot, first, n in entries[:5]:
        for src, hot, warm, sc, zp in ((key, hk, wk, meta[0], meta[1]), (val, hv, wv, meta[2], meta[3])):
            rows = src[:, first:first + n, :]
            if state == 0:
                np.testing.assert_array_equal(hot[slot, :, :n], rows)
                assert not hot[slot, :, n:].view(np.uint16).any()
            else:
                codes, s, z = orc.quantize_rows_r(rows.reshape(-1, head_dim))
                np.testing.assert_array_equal(warm[slot, :, :n].reshape(-1, head_dim), codes)
                np.testing.assert_array_equal(sc[slot, :, :n].reshape(-1).view(np.uint16),
                                              np.asarray(s, np.float16).reshape(-1).view(np.uint16))
                np.testing.assert_array_equal(zp[slot, :, :n].reshape(-1).view(np.uint16),
                                              np.asarray(z, np.float16).reshape(-1).view(np.uint16))
                assert not warm[slot, :, n:].any()
                assert (sc[slot, :, n:] == 1).all() and (zp[slot, :, n:] == 0).all()
    # untouched slots keep their stale bytes (the skipped entries wrote nothing)
    assert (hk[1] == 7).all()
    assert (wk[2] == 7).all()
