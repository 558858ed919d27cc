"""One policy tick of the compact tiered pool, batched; fused decode append.

Drop-in for ``TieredKVRuntime.sync_storage_states`` (tierkv_policy.py:1849-1867)
over a ``CompactTieredKVTensorPool`` (tierkv_policy.py:701-1365).  The
reference walks the layer's blocks one by one; every HOT->WARM demotion
(``demote_to_warm``, 1042-1068) and WARM->HOT promotion (``promote_to_hot``,
1087-1115) runs its own handful of torch kernels, and every metadata update
(``_set_metadata``, 917-926; ``set_block_state``, 1037-1040) writes single
elements of the GPU block tables.  Here the tick is split in two:

* ``plan_sync`` replays the reference loop's bookkeeping exactly -- the same
  checks and errors, the same LIFO slot pops and pushes (growing the pool by
  the pool's own ``_alloc_*_slot`` when a free list runs dry), the same
  physical-block dictionaries and storage sets -- but only records the data
  moves and the table cells, in the reference's order;
* ``apply_sync`` performs all demotions in one launch of the demotion kernel,
  all promotions in one launch of the promotion kernel, and writes the table
  cells with one host->device copy.

Slot reuse inside one tick makes the reference's order matter: a demotion can
free a HOT slot that a later promotion fills (and a promotion a WARM slot that
a later demotion fills).  Such a move writes to a staging buffer first and is
copied into its slot after every move has read its source, so each slot ends
with exactly the bytes the sequential reference leaves there -- rows at or
beyond a block's length included, which the reference never touches.

The decode-time append (``append_to_layer``, tierkv_policy.py:1768-1816, with
``write_hot_tokens`` 934-967 and ``set_block_entry`` 1016-1035) is split the
same way: ``plan_append`` replays the bookkeeping (block-manager allocation,
slot allocation, dictionaries) and ``apply_append`` issues one fused launch
per block touched -- the new rows, the zeroed tail rows and every block-table
cell the reference writes one element at a time.

So is the prefill (``append_prefill_with_policy``, tierkv_policy.py:1722-1766,
whose per-block ``write_hot_tokens`` / ``write_warm_block`` /
``register_cold_block`` calls each run their own torch kernels):
``plan_prefill`` replays the loop's bookkeeping and ``apply_prefill`` stores
every block of the layer -- HOT rows copied, WARM rows quantized, tails
cleared -- in one launch and writes the table cells in one copy.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import ops

HOT_STATE = 0
WARM_STATE = 1
COLD_STATE = 2


@dataclass
class SyncPlan:
    """The data moves and table cells of one tick, in the reference's order."""

    layer: int
    demotions: list = field(default_factory=list)   # (hot slot, warm slot, length)
    promotions: list = field(default_factory=list)  # (warm slot, hot slot, length)
    states: dict = field(default_factory=dict)      # (layer, logical) -> state
    slots: dict = field(default_factory=dict)       # (layer, logical) -> slot
    lengths: dict = field(default_factory=dict)     # (layer, logical) -> length
    physical: dict = field(default_factory=dict)    # (layer, logical) -> physical block
    state_row: object = None  # block_states[layer, :len] written whole, before the cells

    def staged(self):
        """(demotions, promotions) whose destination another move of the tick
        reads: they go through staging."""
        read_hot = {h for h, _, _ in self.demotions}
        read_warm = {w for w, _, _ in self.promotions}
        dem = [i for i, (_, w, _) in enumerate(self.demotions) if w in read_warm]
        pro = [i for i, (_, h, _) in enumerate(self.promotions) if h in read_hot]
        return dem, pro


# ---------------------------------------------------------------------------
# bookkeeping (the reference's pool methods without their data movement)
# ---------------------------------------------------------------------------

def _metadata(pool, plan: SyncPlan, physical_idx: int, state: int, slot: int, length: int) -> None:
    """_set_metadata (tierkv_policy.py:917-926) with the table writes recorded."""
    pool.physical_states[physical_idx] = int(state)
    pool.physical_slots[physical_idx] = int(slot)
    pool.physical_lengths[physical_idx] = int(length)
    location = pool.physical_locations.get(physical_idx)
    if location is not None and pool.is_allocated():
        cell = (int(location[0]), int(location[1]))
        plan.states[cell] = int(state)
        plan.slots[cell] = int(slot)
        plan.lengths[cell] = int(length)


def _demote_to_warm(pool, plan: SyncPlan, physical_idx: int) -> None:
    """demote_to_warm (tierkv_policy.py:1042-1068)."""
    physical_idx = pool._check_physical_idx(physical_idx)
    state = pool.get_physical_state(physical_idx)
    if state == WARM_STATE:
        return
    if state == COLD_STATE:
        raise KeyError(f"Physical block {physical_idx} is not eligible for WARM demotion from COLD storage.")
    if state != HOT_STATE:
        raise KeyError(f"Physical block {physical_idx} is not present in HOT storage.")
    length = pool.get_block_length(physical_idx)
    hot_slot = int(pool.physical_slots[physical_idx])
    warm_slot = int(pool._alloc_warm_slot())
    plan.demotions.append((hot_slot, warm_slot, int(length)))
    pool._free_hot_slot(hot_slot)
    pool.hot_storage.discard(physical_idx)
    pool.warm_storage.add(physical_idx)
    pool.cold_storage.discard(physical_idx)
    _metadata(pool, plan, physical_idx, WARM_STATE, warm_slot, length)


def _demote_to_cold(pool, plan: SyncPlan, physical_idx: int) -> None:
    """demote_to_cold (tierkv_policy.py:1070-1085): frees the slot, moves nothing."""
    physical_idx = pool._check_physical_idx(physical_idx)
    state = pool.get_physical_state(physical_idx)
    if state == COLD_STATE:
        return
    if state == HOT_STATE:
        pool._free_hot_slot(pool.physical_slots.get(physical_idx, -1))
    elif state == WARM_STATE:
        pool._free_warm_slot(pool.physical_slots.get(physical_idx, -1))
    elif state is None:
        raise KeyError(f"Physical block {physical_idx} is not present in HOT or WARM storage.")
    length = pool.get_block_length(physical_idx)
    pool.hot_storage.discard(physical_idx)
    pool.warm_storage.discard(physical_idx)
    pool.cold_storage.add(physical_idx)
    _metadata(pool, plan, physical_idx, COLD_STATE, -1, length)


def _promote_to_hot(pool, plan: SyncPlan, physical_idx: int) -> None:
    """promote_to_hot (tierkv_policy.py:1087-1115)."""
    physical_idx = pool._check_physical_idx(physical_idx)
    state = pool.get_physical_state(physical_idx)
    if state == HOT_STATE:
        return
    if state == COLD_STATE:
        raise KeyError(f"Physical block {physical_idx} is not eligible for HOT promotion from COLD storage.")
    if state != WARM_STATE:
        raise KeyError(f"Physical block {physical_idx} is not present in WARM storage.")
    length = pool.get_block_length(physical_idx)
    warm_slot = int(pool.physical_slots[physical_idx])
    hot_slot = int(pool._alloc_hot_slot())
    plan.promotions.append((warm_slot, hot_slot, int(length)))
    pool._free_warm_slot(warm_slot)
    pool.hot_storage.add(physical_idx)
    pool.warm_storage.discard(physical_idx)
    pool.cold_storage.discard(physical_idx)
    _metadata(pool, plan, physical_idx, HOT_STATE, hot_slot, length)


def _int_array(values) -> np.ndarray:
    """int(x) for every x, as int64.  A 1-D integer sequence or array converts
    in one numpy call; anything else (floats, bools, tensors of other kinds)
    goes through int() one element at a time."""
    try:
        arr = np.asarray(values)
    except (TypeError, ValueError):
        arr = None
    if arr is not None and arr.ndim == 1 and arr.dtype.kind in "iu":
        return arr.astype(np.int64, copy=False)
    return np.asarray([int(x) for x in values], dtype=np.int64)


def plan_sync(pool, layer_idx: int, physical_indices, states) -> SyncPlan:
    """The loop of sync_storage_states (tierkv_policy.py:1849-1867), recording
    moves and table cells instead of performing them.  Updates the pool's
    bookkeeping (free lists, dictionaries, storage sets) in place, exactly as
    the reference does, and may grow its tensors through the pool's own slot
    allocators."""
    plan = SyncPlan(int(layer_idx))
    physical = _int_array(physical_indices).tolist()
    target = _int_array(states)
    if len(physical) != len(target):
        # zip() semantics of the reference loop
        n = min(len(physical), len(target))
        physical, target = physical[:n], target[:n]
    if not pool.is_allocated():
        return _plan_sync_loop(pool, plan, layer_idx, physical, target)
    # Blocks that keep their tier only rewrite their state cell with the same
    # value, so only the transitions are walked (in logical order, which is
    # all the slot allocators see); the state row is written whole.  A
    # transitioning block whose recorded location is not (layer, its logical
    # index) would make the order of cell writes observable: then the exact
    # per-block loop runs instead.
    get = pool.physical_states.get
    current = np.fromiter((-1 if (c := get(pidx)) is None else c for pidx in physical),
                          dtype=np.int64, count=len(physical))
    act = (((target == HOT_STATE) & ((current == WARM_STATE) | (current == COLD_STATE)))
           | ((target == COLD_STATE) & (current != COLD_STATE))
           | ((target == WARM_STATE) & ((current == HOT_STATE) | (current == COLD_STATE))))
    moving = np.nonzero(act)[0]
    for i in moving:
        loc = pool.physical_locations.get(physical[i])
        if loc is not None and (int(loc[0]), int(loc[1])) != (int(layer_idx), int(i)):
            return _plan_sync_loop(pool, plan, layer_idx, physical, target)
    for i in moving:
        _transition(pool, plan, physical[i], int(target[i]))
    plan.state_row = target.astype(np.int32)
    return plan


def _transition(pool, plan: SyncPlan, physical_idx: int, state: int) -> None:
    """One iteration of the reference loop without set_block_state."""
    current_state = pool.get_physical_state(physical_idx)
    if state == HOT_STATE:
        if current_state == WARM_STATE:
            _promote_to_hot(pool, plan, physical_idx)
        elif current_state == COLD_STATE:
            raise KeyError(f"Physical block {physical_idx} cannot be promoted from COLD to HOT.")
    elif state == COLD_STATE and current_state != COLD_STATE:
        _demote_to_cold(pool, plan, physical_idx)
    elif state == WARM_STATE:
        if current_state == HOT_STATE:
            _demote_to_warm(pool, plan, physical_idx)
        elif current_state == COLD_STATE:
            raise KeyError(f"Physical block {physical_idx} cannot be promoted from COLD to WARM.")


def _plan_sync_loop(pool, plan: SyncPlan, layer_idx: int, physical, target) -> SyncPlan:
    """The reference loop block by block, every cell write recorded in order."""
    for logical_idx, (physical_idx, state) in enumerate(zip(physical, target)):
        physical_idx = int(physical_idx)
        state = int(state)
        current_state = pool.get_physical_state(physical_idx)
        if state == HOT_STATE:
            if current_state == WARM_STATE:
                _promote_to_hot(pool, plan, physical_idx)
            elif current_state == COLD_STATE:
                raise KeyError(f"Physical block {physical_idx} cannot be promoted from COLD to HOT.")
        elif state == COLD_STATE and current_state != COLD_STATE:
            _demote_to_cold(pool, plan, physical_idx)
        elif state == WARM_STATE:
            if current_state == HOT_STATE:
                _demote_to_warm(pool, plan, physical_idx)
            elif current_state == COLD_STATE:
                raise KeyError(f"Physical block {physical_idx} cannot be promoted from COLD to WARM.")
        # set_block_state (tierkv_policy.py:1037-1040)
        if not pool.is_allocated():
            raise RuntimeError("CompactTieredKVTensorPool has not been allocated yet.")
        plan.states[(int(layer_idx), logical_idx)] = state
    return plan


# ---------------------------------------------------------------------------
# data movement and table writes
# ---------------------------------------------------------------------------

def _pools(pool) -> ops.TieredPools:
    return ops.TieredPools(pool.hot_k_pool, pool.hot_v_pool, pool.warm_k_pool, pool.warm_v_pool,
                           pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero)


def _rows(slots, lengths, kv_heads: int, block_size: int) -> np.ndarray:
    """Flat row indices (slot, head, t < length) of [slots, heads, bs, *] tensors."""
    slots = np.asarray(slots, dtype=np.int64)
    lengths = np.asarray(lengths, dtype=np.int64)
    h = np.arange(kv_heads, dtype=np.int64)
    t = np.arange(block_size, dtype=np.int64)
    rows = (slots[:, None, None] * kv_heads + h[None, :, None]) * block_size + t[None, None, :]
    return rows[np.broadcast_to(t[None, None, :] < lengths[:, None, None], rows.shape)]


def _to_device(parts, dev):
    """Several int64 host arrays in one pinned host->device copy."""
    host = torch.from_numpy(np.concatenate([np.asarray(x, dtype=np.int64) for x in parts]))
    buf = host.pin_memory().to(dev, non_blocking=True)
    out, off = [], 0
    for x in parts:
        out.append(buf[off:off + len(x)])
        off += len(x)
    return out


def apply_sync(pool, plan: SyncPlan, stream=None) -> dict:
    """Performs the plan's moves (one demotion and one promotion launch, plus
    staging copies for reused slots) and writes its table cells.  Returns
    counts of the moves, for tests and logs."""
    n_dem, n_pro = len(plan.demotions), len(plan.promotions)
    staged_dem, staged_pro = plan.staged()
    if n_dem or n_pro:
        if not pool.hot_k_pool.is_cuda:
            raise ValueError("TierKV storage sync requires CUDA pool tensors.")
        pools = _pools(pool)
        dev = pools.device
        kvh, bs, d = pools.kv_heads, pools.block_size, pools.head_dim
        sd, sp = set(staged_dem), set(staged_pro)
        direct_dem = [m for i, m in enumerate(plan.demotions) if i not in sd]
        direct_pro = [m for i, m in enumerate(plan.promotions) if i not in sp]
        sdm = [plan.demotions[i] for i in staged_dem]
        spm = [plan.promotions[i] for i in staged_pro]
        # every slot list and staging row index of the tick in one copy
        parts = []
        for moves in (direct_dem, direct_pro):
            for j in range(3):
                parts.append([m[j] for m in moves])
        for moves in (sdm, spm):
            parts.append([m[0] for m in moves])
            parts.append(list(range(len(moves))))
            parts.append([m[2] for m in moves])
            parts.append(_rows([m[1] for m in moves], [m[2] for m in moves], kvh, bs))
            parts.append(_rows(range(len(moves)), [m[2] for m in moves], kvh, bs))
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            dev_parts = _to_device(parts, dev)
        dd, dp = dev_parts[0:3], dev_parts[3:6]
        sdd, spp = dev_parts[6:11], dev_parts[11:16]
        i32 = lambda x: x.to(torch.int32)  # noqa: E731
        # phase 1: every move reads its source; direct moves write their slot
        # (no move of this tick reads it), staged moves write staging
        stage_w = stage_h = None
        if direct_dem:
            ops.demote_blocks_to_warm(pools, i32(dd[0]), i32(dd[1]), i32(dd[2]), stream=stream)
        if sdm:
            stage_w = ops.TieredPools.allocate(1, len(sdm), kvh, bs, d, dev)
            view = ops.TieredPools(pool.hot_k_pool, pool.hot_v_pool, stage_w.warm_k, stage_w.warm_v,
                                   stage_w.k_scale, stage_w.k_zero, stage_w.v_scale, stage_w.v_zero)
            ops.demote_blocks_to_warm(view, i32(sdd[0]), i32(sdd[1]), i32(sdd[2]), stream=stream)
        if direct_pro:
            ops.promote_blocks_to_hot(pools, i32(dp[0]), i32(dp[1]), i32(dp[2]), stream=stream)
        if spm:
            stage_h = ops.TieredPools.allocate(len(spm), 1, kvh, bs, d, dev)
            view = ops.TieredPools(stage_h.hot_k, stage_h.hot_v, pool.warm_k_pool, pool.warm_v_pool,
                                   pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero)
            ops.promote_blocks_to_hot(view, i32(spp[0]), i32(spp[1]), i32(spp[2]), stream=stream)
        # phase 2: staged results into their slots, rows below the length only
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            if sdm:
                dst, src = sdd[3], sdd[4]
                for real, st, width in ((pool.warm_k_pool, stage_w.warm_k, d),
                                        (pool.warm_v_pool, stage_w.warm_v, d),
                                        (pool.k_scale, stage_w.k_scale, 1), (pool.k_zero, stage_w.k_zero, 1),
                                        (pool.v_scale, stage_w.v_scale, 1), (pool.v_zero, stage_w.v_zero, 1)):
                    real.view(-1, width).index_copy_(0, dst, st.view(-1, width).index_select(0, src))
            if spm:
                dst, src = spp[3], spp[4]
                for real, st in ((pool.hot_k_pool, stage_h.hot_k), (pool.hot_v_pool, stage_h.hot_v)):
                    real.view(-1, d).index_copy_(0, dst, st.view(-1, d).index_select(0, src))
    _write_tables(pool, plan, stream)
    return {"demotions": n_dem, "promotions": n_pro, "staged_demotions": len(staged_dem),
            "staged_promotions": len(staged_pro)}


class _nullcontext:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


def _table_groups(pool, plan: SyncPlan):
    return [(pool.block_states, plan.states), (pool.block_slot_indices, plan.slots),
            (pool.block_lengths, plan.lengths), (pool.physical_block_tables, plan.physical)]


def _write_tables(pool, plan: SyncPlan, stream=None) -> None:
    """The recorded cells of block_states / block_slot_indices / block_lengths,
    last write winning as in the reference, in one host->device copy."""
    groups = [(t, cells) for t, cells in _table_groups(pool, plan) if cells]
    row = plan.state_row
    if not groups and row is None:
        return
    width = int(pool.block_states.shape[1])
    parts = [np.asarray(row, dtype=np.int64)] if row is not None else []
    for _, cells in groups:
        parts.append(np.fromiter((l * width + i for (l, i) in cells), dtype=np.int64, count=len(cells)))
        parts.append(np.fromiter(cells.values(), dtype=np.int64, count=len(cells)))
    dev = pool.block_states.device
    host = torch.from_numpy(np.concatenate(parts))
    if dev.type == "cuda":
        host = host.pin_memory()
    with torch.cuda.stream(stream) if stream is not None else _nullcontext():
        buf = host.to(dev, non_blocking=True)
        off = 0
        if row is not None:
            n = len(row)
            pool.block_states[plan.layer, :n].copy_(buf[:n])
            off = n
        for table, cells in groups:
            n = len(cells)
            idx, val = buf[off:off + n], buf[off + n:off + 2 * n]
            off += 2 * n
            table.view(-1).index_copy_(0, idx, val.to(table.dtype))


def sync_storage_states(self, seq_id: int) -> None:
    """Method-compatible replacement of TieredKVRuntime.sync_storage_states
    (tierkv_policy.py:1849-1867): ``TieredKVRuntime.sync_storage_states =
    paged_tierkv_b200.tiering.sync_storage_states``."""
    physical_indices = self.block_manager.get_physical_indices(seq_id)
    states = self.block_manager.get_states(seq_id)
    plan = plan_sync(self.kv_pool, seq_id, physical_indices, states)
    apply_sync(self.kv_pool, plan)


# ---------------------------------------------------------------------------
# decode-time append
# ---------------------------------------------------------------------------

@dataclass
class AppendStep:
    """One block's share of an append: rows [start, start + key.shape[-2]) of
    HOT slot `slot`, the table cells, and a promotion to run first (the open
    block was WARM)."""

    slot: int
    start: int
    key: torch.Tensor    # [1, kv_heads, take, head_dim] fp16, contiguous
    value: torch.Tensor
    plan: SyncPlan


def _write_hot_tokens(pool, plan: SyncPlan, physical_idx: int, start: int,
                      key_states: torch.Tensor, value_states: torch.Tensor):
    """write_hot_tokens (tierkv_policy.py:934-967) without its tensor work:
    returns (slot, key, value) after the reference's checks and bookkeeping."""
    physical_idx = pool._check_physical_idx(physical_idx)
    key_states, value_states = pool._coerce_kv(key_states, value_states)
    pool._ensure_metadata(key_states)
    start = int(start)
    tokens = int(key_states.shape[-2])
    if start < 0 or start + tokens > pool.block_size:
        raise ValueError("KV write exceeds the physical block capacity.")
    current_state = pool.get_physical_state(physical_idx)
    if current_state == COLD_STATE:
        raise KeyError(f"Physical block {physical_idx} is COLD and cannot be promoted.")
    if current_state == WARM_STATE:
        _promote_to_hot(pool, plan, physical_idx)
    slot_idx = pool.physical_slots.get(physical_idx)
    if slot_idx is None or current_state is None:
        slot_idx = pool._alloc_hot_slot()
    pool.hot_storage.add(physical_idx)
    pool.warm_storage.discard(physical_idx)
    pool.cold_storage.discard(physical_idx)
    _metadata(pool, plan, physical_idx, HOT_STATE, slot_idx, start + tokens)
    return int(slot_idx), key_states, value_states


def _set_block_entry(pool, plan: SyncPlan, layer_idx: int, logical_idx: int, physical_idx: int,
                     state: int) -> None:
    """set_block_entry (tierkv_policy.py:1016-1035) with the table writes recorded."""
    if not pool.is_allocated():
        raise RuntimeError("CompactTieredKVTensorPool has not been allocated yet.")
    layer_idx = int(layer_idx)
    logical_idx = int(logical_idx)
    physical_idx = pool._check_physical_idx(physical_idx)
    if layer_idx < 0 or layer_idx >= pool.num_layers:
        raise ValueError("layer_idx is out of range.")
    if logical_idx < 0 or logical_idx >= pool.max_blocks_per_layer:
        raise RuntimeError(
            f"Logical block {logical_idx} exceeds max_blocks_per_layer={pool.max_blocks_per_layer}.")
    pool.physical_locations[physical_idx] = (layer_idx, logical_idx)
    cell = (layer_idx, logical_idx)
    plan.physical[cell] = physical_idx
    plan.states[cell] = int(state)
    plan.slots[cell] = int(pool.physical_slots.get(physical_idx, -1))
    plan.lengths[cell] = int(pool.physical_lengths.get(physical_idx, 0))


def plan_append(self, seq_id: int, key_states: torch.Tensor, value_states: torch.Tensor):
    """The bookkeeping of append_to_layer (tierkv_policy.py:1768-1816) on a
    runtime (``layer_states``, ``block_manager``, ``kv_pool``, ``block_size``,
    ``max_blocks_per_layer``).  Returns (steps, allocated_new_block)."""
    if key_states.shape[-2] != value_states.shape[-2]:
        raise ValueError("Key and value states must have the same sequence length.")
    pool = self.kv_pool
    layer_state = self.layer_states[seq_id]
    offset = 0
    total_tokens = int(key_states.shape[-2])
    allocated_new_block = False
    steps = []
    while offset < total_tokens:
        new_logical_idx = None
        if layer_state.open_physical_idx is None:
            layer_state.open_physical_idx = self.block_manager.allocate_block(seq_id)
            layer_state.open_token_count = 0
            allocated_new_block = True
            new_logical_idx = layer_state.num_blocks
            if new_logical_idx >= self.max_blocks_per_layer:
                raise RuntimeError(
                    f"Layer {seq_id} exceeded max_blocks_per_layer={self.max_blocks_per_layer}.")
            pool._check_physical_idx(layer_state.open_physical_idx)
        physical_idx = layer_state.open_physical_idx
        plan = SyncPlan(int(seq_id))
        if pool.get_physical_state(physical_idx) == WARM_STATE:
            _promote_to_hot(pool, plan, physical_idx)
        remaining_capacity = self.block_size - layer_state.open_token_count
        take = min(remaining_capacity, total_tokens - offset)
        if offset == 0 and take == total_tokens:  # the whole input (one decode token)
            k_chunk, v_chunk = key_states.contiguous(), value_states.contiguous()
        else:
            k_chunk = key_states[:, :, offset:offset + take, :].contiguous()
            v_chunk = value_states[:, :, offset:offset + take, :].contiguous()
        start = layer_state.open_token_count
        slot, k_chunk, v_chunk = _write_hot_tokens(pool, plan, physical_idx, start, k_chunk, v_chunk)
        if new_logical_idx is not None:
            _set_block_entry(pool, plan, seq_id, new_logical_idx, physical_idx, HOT_STATE)
            layer_state.num_blocks += 1
        steps.append(AppendStep(slot, start, k_chunk, v_chunk, plan))
        layer_state.open_token_count += take
        offset += take
        if layer_state.open_token_count == self.block_size:
            layer_state.open_physical_idx = None
            layer_state.open_token_count = 0
    return steps, allocated_new_block


# HOT-only pool structs of recent appends, keyed by the pool tensors' pointers
# and shape (a decode loop appends to the same pools token after token)
_HOT_STRUCTS: dict = {}


def _hot_struct(pool):
    from . import _native as N
    hk, hv = pool.hot_k_pool, pool.hot_v_pool
    key = (hk.data_ptr(), hv.data_ptr(), tuple(hk.shape))
    st = _HOT_STRUCTS.get(key)
    if st is None:
        st = N.TkvPools(hk.data_ptr(), hv.data_ptr(), None, None, None, None, None, None,
                        int(hk.shape[0]), 0, int(hk.shape[1]), int(hk.shape[2]), int(hk.shape[3]),
                        ops.FORMAT_R)
        if len(_HOT_STRUCTS) >= 8:
            _HOT_STRUCTS.clear()
        _HOT_STRUCTS[key] = st
    return st


def apply_append(pool, steps, stream=None) -> int:
    """One fused launch per step (after its promotion, if any); returns the
    number of launches."""
    from . import _native as N
    import ctypes
    lib = N.load()
    launches = 0
    for step in steps:
        if step.plan.promotions:
            w, h, n = zip(*step.plan.promotions)
            ops.promote_blocks_to_hot(_pools(pool), list(w), list(h), list(n), stream=stream)
            launches += 1
        if not (step.key.is_cuda and pool.hot_k_pool.is_cuda):
            raise ValueError("TierKV decode append requires CUDA tensors.")
        key = step.key if step.key.data_ptr() % 16 == 0 else step.key.clone()
        value = step.value if step.value.data_ptr() % 16 == 0 else step.value.clone()
        cells = []
        for table, recorded in _table_groups(pool, step.plan):
            if recorded:
                width, base = int(table.shape[1]), table.data_ptr()
                cells.extend((base, layer * width + logical, int(v), 0)
                             for (layer, logical), v in recorded.items())
        if len(cells) > N.TKV_APPEND_MAX_CELLS:
            raise RuntimeError("append step records more table cells than one launch carries.")
        arr = (N.TkvTableCell * max(1, len(cells)))(*cells)
        ps = _hot_struct(pool)  # the append touches the HOT pool only
        N.check(lib.tkv_append_hot_tokens(ctypes.byref(ps), step.slot, step.start,
                                          int(key.shape[-2]), key.data_ptr(), value.data_ptr(),
                                          arr, len(cells), ops._stream(stream, key.device.index)),
                "tkv_append_hot_tokens")
        launches += 1
    return launches


def append_to_layer(self, seq_id: int, key_states: torch.Tensor, value_states: torch.Tensor) -> bool:
    """Method-compatible replacement of TieredKVRuntime.append_to_layer
    (tierkv_policy.py:1768-1816): ``TieredKVRuntime.append_to_layer =
    paged_tierkv_b200.tiering.append_to_layer``."""
    steps, allocated_new_block = plan_append(self, seq_id, key_states, value_states)
    apply_append(self.kv_pool, steps)
    return allocated_new_block


# ---------------------------------------------------------------------------
# prefill with policy
# ---------------------------------------------------------------------------

@dataclass
class PrefillPlan:
    """A prefilled layer: the bookkeeping's table cells (and promotions of
    blocks a stale WARM state left behind), and per written block one entry
    (state, slot, first token, length) in the reference's order."""

    plan: SyncPlan
    entries: list = field(default_factory=list)
    key: torch.Tensor | None = None    # [kv_heads, tokens, head_dim] fp16, contiguous
    value: torch.Tensor | None = None


def _prefill_kv(pool, key_states: torch.Tensor, value_states: torch.Tensor):
    """The checks of _coerce_kv (tierkv_policy.py:780-791) for the whole layer
    (every block's chunk has the layer's shape but for its token count), the
    fp16 conversion, and one contiguous copy at most."""
    if key_states.shape != value_states.shape:
        raise ValueError("Key and value tensors must have identical shape.")
    if key_states.ndim != 4 or key_states.shape[0] != 1:
        raise ValueError("KV tensors must have shape [1, kv_heads, tokens, head_dim].")
    if key_states.dtype != torch.float16:
        key_states = key_states.to(torch.float16)
    if value_states.dtype != torch.float16:
        value_states = value_states.to(torch.float16)
    return key_states.contiguous(), value_states.contiguous()


def _hot_block(pool, plan: SyncPlan, physical_idx: int, key, length: int,
               ensure: bool = True) -> int:
    """write_hot_tokens(physical_idx, 0, chunk) (tierkv_policy.py:934-967)
    without its tensor work; returns the slot.  ``ensure=False`` skips the
    geometry check of an input it has already passed."""
    physical_idx = pool._check_physical_idx(physical_idx)
    if ensure:
        pool._ensure_metadata(key)
    current_state = pool.get_physical_state(physical_idx)
    if current_state == COLD_STATE:
        raise KeyError(f"Physical block {physical_idx} is COLD and cannot be promoted.")
    if current_state == WARM_STATE:
        _promote_to_hot(pool, plan, physical_idx)
    slot_idx = pool.physical_slots.get(physical_idx)
    if slot_idx is None or current_state is None:
        slot_idx = pool._alloc_hot_slot()
    pool.hot_storage.add(physical_idx)
    pool.warm_storage.discard(physical_idx)
    pool.cold_storage.discard(physical_idx)
    _metadata(pool, plan, physical_idx, HOT_STATE, slot_idx, length)
    return int(slot_idx)


def _warm_block(pool, plan: SyncPlan, physical_idx: int, key, length: int,
                ensure: bool = True) -> int:
    """write_warm_block (tierkv_policy.py:969-1002) without its tensor work;
    returns the slot."""
    physical_idx = pool._check_physical_idx(physical_idx)
    if ensure:
        pool._ensure_metadata(key)
    current_state = pool.get_physical_state(physical_idx)
    if current_state == HOT_STATE:
        pool._free_hot_slot(pool.physical_slots.get(physical_idx, -1))
    elif current_state == WARM_STATE:
        pool._free_warm_slot(pool.physical_slots.get(physical_idx, -1))
    elif current_state == COLD_STATE:
        raise KeyError(f"Physical block {physical_idx} is COLD and cannot be promoted.")
    slot_idx = pool._alloc_warm_slot()
    pool.hot_storage.discard(physical_idx)
    pool.warm_storage.add(physical_idx)
    pool.cold_storage.discard(physical_idx)
    _metadata(pool, plan, physical_idx, WARM_STATE, slot_idx, length)
    return int(slot_idx)


def _cold_block(pool, plan: SyncPlan, physical_idx: int, length: int) -> None:
    """register_cold_block (tierkv_policy.py:1004-1014)."""
    physical_idx = pool._check_physical_idx(physical_idx)
    state = pool.get_physical_state(physical_idx)
    if state == HOT_STATE:
        pool._free_hot_slot(pool.physical_slots.get(physical_idx, -1))
    elif state == WARM_STATE:
        pool._free_warm_slot(pool.physical_slots.get(physical_idx, -1))
    pool.hot_storage.discard(physical_idx)
    pool.warm_storage.discard(physical_idx)
    pool.cold_storage.add(physical_idx)
    _metadata(pool, plan, physical_idx, COLD_STATE, -1, int(length))


def plan_prefill(self, seq_id: int, key_states: torch.Tensor, value_states: torch.Tensor,
                 block_scores: torch.Tensor, out: PrefillPlan | None = None) -> PrefillPlan:
    """The loop of append_prefill_with_policy (tierkv_policy.py:1722-1766) on a
    runtime (``layer_states``, ``block_manager``, ``kv_pool``, ``block_size``,
    ``max_blocks_per_layer``, ``_desired_prefill_states``): block-manager
    allocation and state updates, slot allocation (growing the pool through
    its own allocators), dictionaries, storage sets and table cells exactly as
    the reference leaves them, with the tensor work recorded in ``out``
    (filled in place, so a failure part-way leaves the part done)."""
    if key_states.shape[-2] != value_states.shape[-2]:
        raise ValueError("Key and value states must have the same sequence length.")
    pool = self.kv_pool
    layer_state = self.layer_states[seq_id]
    if layer_state.num_blocks != 0 or layer_state.open_physical_idx is not None:
        raise RuntimeError("append_prefill_with_policy expects an empty layer cache.")
    block_size = int(self.block_size)
    total_tokens = int(key_states.shape[-2])
    num_blocks = -(-total_tokens // block_size)
    if num_blocks > self.max_blocks_per_layer:
        raise RuntimeError(f"Layer {seq_id} exceeded max_blocks_per_layer={self.max_blocks_per_layer}.")
    desired_states = self._desired_prefill_states(num_blocks, block_scores)
    out = out if out is not None else PrefillPlan(SyncPlan(int(seq_id)))
    plan = out.plan
    allocate = self.block_manager.allocate_block
    update_state = self.block_manager.update_block_state
    add_entry = out.entries.append
    locations, slots_of, lengths_of = pool.physical_locations, pool.physical_slots, pool.physical_lengths
    cell_physical, cell_states, cell_slots, cell_lengths = (plan.physical, plan.states, plan.slots,
                                                            plan.lengths)
    layer = int(seq_id)
    key3 = None   # the layer's K as [1, kv_heads, tokens, head_dim] once checked
    checked = False  # the pool has accepted key3's geometry (_ensure_metadata)
    for logical_idx, desired_state in enumerate(desired_states):
        physical_idx = allocate(seq_id)
        if desired_state != HOT_STATE:
            update_state(seq_id, logical_idx, desired_state)
        start = logical_idx * block_size
        length = min(start + block_size, total_tokens) - start
        if desired_state in (HOT_STATE, WARM_STATE) or (desired_state == COLD_STATE
                                                         and not pool.is_allocated()):
            if out.key is None:  # the reference checks each chunk as it writes it
                pool._check_physical_idx(physical_idx)
                key, value = _prefill_kv(pool, key_states, value_states)
                out.key, out.value = key[0], value[0]
            if key3 is None:
                key3 = out.key[None]
        if desired_state == HOT_STATE:
            slot = _hot_block(pool, plan, physical_idx, key3, length, ensure=not checked)
            checked = True
            add_entry((HOT_STATE, slot, start, length))
        elif desired_state == WARM_STATE:
            slot = _warm_block(pool, plan, physical_idx, key3, length, ensure=not checked)
            checked = True
            add_entry((WARM_STATE, slot, start, length))
        elif desired_state == COLD_STATE:
            if not pool.is_allocated():
                slot = _hot_block(pool, plan, physical_idx, key3, length, ensure=not checked)
                checked = True
                add_entry((HOT_STATE, slot, start, length))
                _demote_to_cold(pool, plan, physical_idx)
            else:
                _cold_block(pool, plan, physical_idx, length)
        else:
            raise ValueError(f"Unsupported desired state: {desired_state}")
        # set_block_entry (tierkv_policy.py:1016-1035); the physical index has
        # passed its range check in the write above
        if not pool.is_allocated():
            raise RuntimeError("CompactTieredKVTensorPool has not been allocated yet.")
        if layer < 0 or layer >= pool.num_layers:
            raise ValueError("layer_idx is out of range.")
        if logical_idx >= pool.max_blocks_per_layer:
            raise RuntimeError(
                f"Logical block {logical_idx} exceeds max_blocks_per_layer={pool.max_blocks_per_layer}.")
        physical_idx = int(physical_idx)
        cell = (layer, logical_idx)
        locations[physical_idx] = cell
        cell_physical[cell] = physical_idx
        cell_states[cell] = int(desired_state)
        cell_slots[cell] = int(slots_of.get(physical_idx, -1))
        cell_lengths[cell] = int(lengths_of.get(physical_idx, 0))
    layer_state.num_blocks = num_blocks
    layer_state.open_physical_idx = None
    layer_state.open_token_count = 0
    return out


def _pools_struct(pool):
    """The pools as a tkv_pools struct; a pool not allocated yet is passed as
    null with 0 slots."""
    from . import _native as N
    hk, wk = pool.hot_k_pool, pool.warm_k_pool
    ref = hk if hk is not None else wk
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    return N.TkvPools(ptr(hk), ptr(pool.hot_v_pool), ptr(wk), ptr(pool.warm_v_pool),
                      ptr(pool.k_scale), ptr(pool.k_zero), ptr(pool.v_scale), ptr(pool.v_zero),
                      0 if hk is None else int(hk.shape[0]), 0 if wk is None else int(wk.shape[0]),
                      int(ref.shape[1]), int(ref.shape[2]), int(ref.shape[3]), ops.FORMAT_R)


def apply_prefill(pool, pplan: PrefillPlan, stream=None) -> int:
    """The recorded promotions (if any), every block's rows in one launch of
    the prefill store kernel, and the table cells in one host->device copy.
    Returns the number of store entries."""
    import ctypes
    from . import _native as N
    plan = pplan.plan
    if plan.promotions:
        w, h, n = zip(*plan.promotions)
        ops.promote_blocks_to_hot(_pools(pool), list(w), list(h), list(n), stream=stream)
    # a slot written twice keeps the last write (each write covers the whole
    # slot: rows below its length and the cleared rest)
    last = {}
    for e in pplan.entries:
        last[(e[0], e[1])] = e
    entries = list(last.values())
    if entries:
        key, value = pplan.key, pplan.value
        if not (key.is_cuda and pool.hot_k_pool is not None and pool.hot_k_pool.is_cuda):
            raise ValueError("TierKV prefill storage requires CUDA tensors.")
        host = torch.tensor(entries, dtype=torch.int32).pin_memory()
        with torch.cuda.stream(stream) if stream is not None else _nullcontext():
            dev = host.to(key.device, non_blocking=True)
        ps = _pools_struct(pool)
        N.check(N.load().tkv_store_prefill_blocks(ctypes.byref(ps), key.data_ptr(), value.data_ptr(),
                                                   int(key.shape[1]), dev.data_ptr(), len(entries),
                                                   ops._stream(stream)),
                "tkv_store_prefill_blocks")
        pplan._keep = (host, dev)  # the entry list lives as long as the plan
    _write_tables(pool, plan, stream)
    return len(entries)


def append_prefill_with_policy(self, seq_id: int, key_states: torch.Tensor,
                               value_states: torch.Tensor, block_scores: torch.Tensor) -> None:
    """Method-compatible replacement of TieredKVRuntime.append_prefill_with_policy
    (tierkv_policy.py:1722-1766): ``TieredKVRuntime.append_prefill_with_policy =
    paged_tierkv_b200.tiering.append_prefill_with_policy``.  If the reference
    loop would fail part-way, the blocks before the failure are stored as the
    reference stores them, then the error is raised."""
    pplan = PrefillPlan(SyncPlan(int(seq_id)))
    try:
        plan_prefill(self, seq_id, key_states, value_states, block_scores, out=pplan)
    finally:
        if pplan.entries or pplan.plan.promotions or pplan.plan.states:
            apply_prefill(self.kv_pool, pplan)
