"""Test stand-in for the reference's ``CompactTieredKVTensorPool``.

Test infrastructure only.  It carries the attributes and the slot-allocation
methods the batched storage sync uses, restated from tierkv_policy.py
(``_alloc_*_slot`` / ``_free_*_slot`` 897-915, ``_grow_hot_slots`` /
``_grow_warm_slots`` 857-895, ``get_physical_state`` / ``get_block_length``),
and is loaded from the "before" state of a golden fixture made by the
reference itself (tests/golden/make_tiering_golden.py), so the fixture's
"after" state pins both this stand-in and the code under test.
"""

from __future__ import annotations

import json

import numpy as np
import torch


class CompactPoolStub:
    def __init__(self, fixture, device="cpu"):
        meta = json.loads(str(fixture["meta"]))
        b = meta["before"]
        self.meta = meta
        self.device = torch.device(device)
        self.num_layers = meta["num_layers"]
        self.block_size = meta["block_size"]
        self.kv_heads = meta["kv_heads"]
        self.head_dim = meta["head_dim"]
        self.max_blocks_per_layer = meta["max_blocks_per_layer"]
        self.max_hot_slots = meta["max_hot_slots"]
        self.max_warm_slots = meta["max_warm_slots"]
        self.hot_chunk_slots = meta["hot_chunk_slots"]
        self.warm_chunk_slots = meta["warm_chunk_slots"]
        self.hot_free_slots = list(b["hot_free_slots"])
        self.warm_free_slots = list(b["warm_free_slots"])
        self.physical_states = {int(k): v for k, v in b["physical_states"].items()}
        self.physical_slots = {int(k): v for k, v in b["physical_slots"].items()}
        self.physical_lengths = {int(k): v for k, v in b["physical_lengths"].items()}
        self.physical_locations = {int(k): tuple(v) for k, v in b["physical_locations"].items()}
        self.hot_storage = set(b["hot_storage"])
        self.warm_storage = set(b["warm_storage"])
        self.cold_storage = set(b["cold_storage"])
        self.allocated_hot_slots = b["allocated_hot_slots"]
        self.allocated_warm_slots = b["allocated_warm_slots"]
        t = lambda k: torch.from_numpy(np.ascontiguousarray(fixture[f"before_{k}"])).to(self.device)  # noqa: E731
        self.hot_k_pool, self.hot_v_pool = t("hot_k"), t("hot_v")
        self.warm_k_pool, self.warm_v_pool = t("warm_k"), t("warm_v")
        self.k_scale, self.k_zero, self.v_scale, self.v_zero = t("k_scale"), t("k_zero"), t("v_scale"), t("v_zero")
        self.block_states, self.block_slot_indices = t("block_states"), t("block_slot_indices")
        self.block_lengths, self.physical_block_tables = t("block_lengths"), t("physical_block_tables")

    # -- the reference pool's interface used by the storage sync --
    def is_allocated(self) -> bool:
        return self.physical_block_tables is not None

    def _check_physical_idx(self, physical_idx):
        return int(physical_idx)

    def _coerce_kv(self, key_states, value_states):
        if key_states.shape != value_states.shape:
            raise ValueError("Key and value tensors must have identical shape.")
        if key_states.ndim != 4 or key_states.shape[0] != 1:
            raise ValueError("KV tensors must have shape [1, kv_heads, tokens, head_dim].")
        if key_states.shape[-2] > self.block_size:
            raise ValueError("A single stored block cannot exceed block_size tokens.")
        return (key_states.to(torch.float16).contiguous(), value_states.to(torch.float16).contiguous())

    def _ensure_metadata(self, key_states):
        if int(key_states.shape[1]) != self.kv_heads or int(key_states.shape[-1]) != self.head_dim:
            raise ValueError("KV tensor geometry changed after tensor-pool allocation.")

    def get_physical_state(self, physical_idx):
        return self.physical_states.get(int(physical_idx))

    def get_block_length(self, physical_idx) -> int:
        return int(self.physical_lengths.get(int(physical_idx), 0))

    def _new(self, capacity, dtype, fill=0):
        shape = (capacity, self.kv_heads, self.block_size, self.head_dim)
        return torch.full(shape, fill, dtype=dtype, device=self.device)

    def _meta(self, capacity, fill):
        return torch.full((capacity, self.kv_heads, self.block_size, 1), fill, dtype=torch.float16,
                          device=self.device)

    @staticmethod
    def _grow(old, new, old_capacity):
        if old is not None and old_capacity > 0:
            new[:old_capacity].copy_(old[:old_capacity])
        return new

    def _grow_hot_slots(self):
        if self.allocated_hot_slots >= self.max_hot_slots:
            raise RuntimeError("No HOT slots available in compact TierKV pool.")
        old = self.allocated_hot_slots
        new = min(self.max_hot_slots, old + max(1, self.hot_chunk_slots))
        self.hot_k_pool = self._grow(self.hot_k_pool, self._new(new, torch.float16), old)
        self.hot_v_pool = self._grow(self.hot_v_pool, self._new(new, torch.float16), old)
        self.hot_free_slots.extend(range(new - 1, old - 1, -1))
        self.allocated_hot_slots = new

    def _grow_warm_slots(self):
        if self.allocated_warm_slots >= self.max_warm_slots:
            raise RuntimeError("No WARM slots available in compact TierKV pool.")
        old = self.allocated_warm_slots
        new = min(self.max_warm_slots, old + max(1, self.warm_chunk_slots))
        self.warm_k_pool = self._grow(self.warm_k_pool, self._new(new, torch.uint8), old)
        self.warm_v_pool = self._grow(self.warm_v_pool, self._new(new, torch.uint8), old)
        self.k_scale = self._grow(self.k_scale, self._meta(new, 1), old)
        self.k_zero = self._grow(self.k_zero, self._meta(new, 0), old)
        self.v_scale = self._grow(self.v_scale, self._meta(new, 1), old)
        self.v_zero = self._grow(self.v_zero, self._meta(new, 0), old)
        self.warm_free_slots.extend(range(new - 1, old - 1, -1))
        self.allocated_warm_slots = new

    def _alloc_hot_slot(self) -> int:
        if not self.hot_free_slots:
            self._grow_hot_slots()
        return int(self.hot_free_slots.pop())

    def _alloc_warm_slot(self) -> int:
        if not self.warm_free_slots:
            self._grow_warm_slots()
        return int(self.warm_free_slots.pop())

    def _free_hot_slot(self, slot_idx) -> None:
        if int(slot_idx) >= 0:
            self.hot_free_slots.append(int(slot_idx))

    def _free_warm_slot(self, slot_idx) -> None:
        if int(slot_idx) >= 0:
            self.warm_free_slots.append(int(slot_idx))

    def bookkeeping(self) -> dict:
        """The state in the fixture's JSON form."""
        return {
            "hot_free_slots": list(self.hot_free_slots),
            "warm_free_slots": list(self.warm_free_slots),
            "physical_states": {str(k): v for k, v in self.physical_states.items()},
            "physical_slots": {str(k): v for k, v in self.physical_slots.items()},
            "physical_lengths": {str(k): v for k, v in self.physical_lengths.items()},
            "physical_locations": {str(k): list(v) for k, v in self.physical_locations.items()},
            "hot_storage": sorted(self.hot_storage),
            "warm_storage": sorted(self.warm_storage),
            "cold_storage": sorted(self.cold_storage),
            "allocated_hot_slots": self.allocated_hot_slots,
            "allocated_warm_slots": self.allocated_warm_slots,
        }


class LayerState:
    """LayerRuntimeState (tierkv_policy.py:1481-1484)."""

    def __init__(self, open_physical_idx=None, open_token_count=0, num_blocks=0):
        self.open_physical_idx = open_physical_idx
        self.open_token_count = open_token_count
        self.num_blocks = num_blocks

    def as_list(self):
        return [self.open_physical_idx, self.open_token_count, self.num_blocks]


class BlockManagerStub:
    """allocate_block of csrc/block_manager.cpp:36-50 (LIFO free list)."""

    def __init__(self, free):
        self.free = list(free)

    def allocate_block(self, seq_id):
        return self.free.pop()
