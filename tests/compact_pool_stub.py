"""Loads the package's CompactPool from a golden fixture's "before" state.

Test infrastructure only.  The fixtures (tests/golden/make_tiering_golden.py)
are made by the reference's own ``CompactTieredKVTensorPool``, so their
"after" states pin both the ``compact_pool`` stand-in and the code under
test.
"""

from __future__ import annotations

import json

import numpy as np
import torch

from compact_pool import BlockAllocator, CompactPool, LayerState  # noqa: F401


def CompactPoolStub(fixture, device="cpu") -> CompactPool:
    meta = json.loads(str(fixture["meta"]))
    b = meta["before"]
    pool = CompactPool(num_layers=meta["num_layers"], block_size=meta["block_size"],
                       kv_heads=meta["kv_heads"], head_dim=meta["head_dim"],
                       max_blocks_per_layer=meta["max_blocks_per_layer"],
                       max_hot_slots=meta["max_hot_slots"], max_warm_slots=meta["max_warm_slots"],
                       hot_chunk_slots=meta["hot_chunk_slots"], warm_chunk_slots=meta["warm_chunk_slots"],
                       pool_blocks=meta["pool_blocks"], device=device)
    pool.meta = meta
    pool.hot_free_slots = list(b["hot_free_slots"])
    pool.warm_free_slots = list(b["warm_free_slots"])
    pool.physical_states = {int(k): v for k, v in b["physical_states"].items()}
    pool.physical_slots = {int(k): v for k, v in b["physical_slots"].items()}
    pool.physical_lengths = {int(k): v for k, v in b["physical_lengths"].items()}
    pool.physical_locations = {int(k): tuple(v) for k, v in b["physical_locations"].items()}
    pool.hot_storage = set(b["hot_storage"])
    pool.warm_storage = set(b["warm_storage"])
    pool.cold_storage = set(b["cold_storage"])
    pool.allocated_hot_slots = b["allocated_hot_slots"]
    pool.allocated_warm_slots = b["allocated_warm_slots"]
    t = lambda k: torch.from_numpy(np.ascontiguousarray(fixture[f"before_{k}"])).to(pool.device)  # noqa: E731
    pool.hot_k_pool, pool.hot_v_pool = t("hot_k"), t("hot_v")
    pool.warm_k_pool, pool.warm_v_pool = t("warm_k"), t("warm_v")
    pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero = t("k_scale"), t("k_zero"), t("v_scale"), t("v_zero")
    pool.block_states, pool.block_slot_indices = t("block_states"), t("block_slot_indices")
    pool.block_lengths, pool.physical_block_tables = t("block_lengths"), t("physical_block_tables")
    return pool


def BlockManagerStub(free) -> BlockAllocator:
    return BlockAllocator(free=free)


def desired_prefill_states(policy_mode, hot_budget, warm_budget, demoted_state, num_blocks,
                           block_scores):
    """TieredKVRuntime._desired_prefill_states (tierkv_policy.py:1695-1720): the
    first and last blocks stay HOT, the best-scored others fill the HOT budget,
    the next best the WARM budget (hot_warm_cold), the rest go to the demoted
    tier; layers of at most two blocks, or policy hot_only, stay all HOT."""
    num_blocks = int(num_blocks)
    if policy_mode == "hot_only" or num_blocks <= 2:
        return [0] * num_blocks
    if block_scores.ndim != 1 or len(block_scores) != num_blocks:
        raise ValueError("block_scores must be a 1D tensor matching prefill block count.")
    reserved = {0, num_blocks - 1}
    cands = sorted((i for i in range(num_blocks) if i not in reserved),
                   key=lambda i: float(block_scores[i]), reverse=True)
    extra = max(int(hot_budget) - len(reserved), 0)
    hot = set(cands[:extra])
    if policy_mode == "hot_warm_cold":
        warm = set(cands[extra:extra + max(int(warm_budget), 0)])
        return [0 if (i in reserved or i in hot) else (1 if i in warm else 2) for i in range(num_blocks)]
    return [0 if (i in reserved or i in hot) else int(demoted_state) for i in range(num_blocks)]


class PrefillRuntimeStub:
    """The attributes and the policy method of TieredKVRuntime that
    append_prefill_with_policy uses."""

    def __init__(self, pool, block_manager, layer_states, block_size, max_blocks_per_layer):
        self.kv_pool = pool
        self.block_manager = block_manager
        self.layer_states = layer_states
        self.block_size = block_size
        self.max_blocks_per_layer = max_blocks_per_layer
        self.policy_mode, self.hot_budget, self.warm_budget, self.demoted_state = "hot_warm", 2, 0, 1

    def _desired_prefill_states(self, num_blocks, block_scores):
        return desired_prefill_states(self.policy_mode, self.hot_budget, self.warm_budget,
                                      self.demoted_state, num_blocks, block_scores)
