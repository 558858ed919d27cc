"""Test and benchmark stand-in for the reference's compact pool.

Not part of the product: the reference's ``CompactTieredKVTensorPool``
(tierkv_policy.py:701-1365) and its ``BlockManager`` (csrc/block_manager.cpp)
stay as they are and are what a runtime hands to ``paged_tierkv_b200.tiering``.
This class carries the same attributes and slot-allocation behaviour -- LIFO
free lists, growth by chunks of slots (``_alloc_*_slot`` / ``_free_*_slot``
897-915, ``_grow_*_slots`` 857-895), the per-physical-block dictionaries and
storage sets, the [num_layers, max_blocks_per_layer] int32 block tables -- so
the batched paths can be tested against the reference-made fixtures and
measured (``bench.py --config tick / append / prefill_store``) on the GPU box,
where the reference is not installed.  It holds no policy and moves no data
itself.
"""

from __future__ import annotations

import torch

HOT_STATE = 0
WARM_STATE = 1
COLD_STATE = 2


class CompactPool:
    def __init__(self, *, num_layers: int, block_size: int, kv_heads: int, head_dim: int,
                 max_blocks_per_layer: int, max_hot_slots: int, max_warm_slots: int,
                 hot_chunk_slots: int = 128, warm_chunk_slots: int = 128,
                 pool_blocks: int | None = None, device="cuda"):
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.num_layers = int(num_layers)
        self.block_size = int(block_size)
        self.kv_heads = int(kv_heads)
        self.head_dim = int(head_dim)
        self.max_blocks_per_layer = int(max_blocks_per_layer)
        self.pool_blocks = int(pool_blocks or self.num_layers * self.max_blocks_per_layer)
        self.max_hot_slots = int(max_hot_slots)
        self.max_warm_slots = int(max_warm_slots)
        self.hot_chunk_slots = int(hot_chunk_slots)
        self.warm_chunk_slots = int(warm_chunk_slots)
        self.hot_free_slots: list[int] = []
        self.warm_free_slots: list[int] = []
        self.physical_states: dict[int, int] = {}
        self.physical_slots: dict[int, int] = {}
        self.physical_lengths: dict[int, int] = {}
        self.physical_locations: dict[int, tuple[int, int]] = {}
        self.hot_storage: set[int] = set()
        self.warm_storage: set[int] = set()
        self.cold_storage: set[int] = set()
        self.allocated_hot_slots = 0
        self.allocated_warm_slots = 0
        self.hot_k_pool = self.hot_v_pool = None
        self.warm_k_pool = self.warm_v_pool = None
        self.k_scale = self.k_zero = self.v_scale = self.v_zero = None
        shape = (self.num_layers, self.max_blocks_per_layer)
        self.physical_block_tables = torch.full(shape, -1, dtype=torch.int32, device=self.device)
        self.block_slot_indices = torch.full(shape, -1, dtype=torch.int32, device=self.device)
        self.block_states = torch.full(shape, COLD_STATE, dtype=torch.int32, device=self.device)
        self.block_lengths = torch.zeros(shape, dtype=torch.int32, device=self.device)

    # -- queries ---------------------------------------------------------------
    def is_allocated(self) -> bool:
        return self.physical_block_tables is not None

    def _check_physical_idx(self, physical_idx) -> int:
        physical_idx = int(physical_idx)
        if physical_idx < 0 or physical_idx >= self.pool_blocks:
            raise RuntimeError(
                f"Physical block {physical_idx} is outside tensor-pool metadata capacity {self.pool_blocks}.")
        return physical_idx

    def get_physical_state(self, physical_idx):
        return self.physical_states.get(int(physical_idx))

    def get_block_length(self, physical_idx) -> int:
        return int(self.physical_lengths.get(int(physical_idx), 0))

    def get_layer_table(self, layer_idx: int):
        return self.block_slot_indices[int(layer_idx)], self.block_states[int(layer_idx)]

    def get_layer_lengths(self, layer_idx: int):
        return self.block_lengths[int(layer_idx)]

    # -- tensors ---------------------------------------------------------------
    def _coerce_kv(self, key_states, value_states):
        if key_states.shape != value_states.shape:
            raise ValueError("Key and value tensors must have identical shape.")
        if key_states.ndim != 4 or key_states.shape[0] != 1:
            raise ValueError("KV tensors must have shape [1, kv_heads, tokens, head_dim].")
        if key_states.shape[-2] > self.block_size:
            raise ValueError("A single stored block cannot exceed block_size tokens.")
        if key_states.dtype != torch.float16:
            key_states = key_states.to(torch.float16)
        if value_states.dtype != torch.float16:
            value_states = value_states.to(torch.float16)
        return key_states.contiguous(), value_states.contiguous()

    def _ensure_metadata(self, key_states) -> None:
        if (key_states.device != self.device or int(key_states.shape[1]) != self.kv_heads
                or int(key_states.shape[-1]) != self.head_dim):
            raise ValueError("KV tensor geometry changed after tensor-pool allocation.")

    def _kv(self, capacity, dtype):
        return torch.zeros((capacity, self.kv_heads, self.block_size, self.head_dim), dtype=dtype,
                           device=self.device)

    def _meta(self, capacity, fill):
        return torch.full((capacity, self.kv_heads, self.block_size, 1), fill, dtype=torch.float16,
                          device=self.device)

    @staticmethod
    def _grow(old, new, old_capacity):
        if old is not None and old_capacity > 0:
            new[:old_capacity].copy_(old[:old_capacity])
        return new

    def _grow_hot_slots(self) -> None:
        if self.allocated_hot_slots >= self.max_hot_slots:
            raise RuntimeError("No HOT slots available in compact TierKV pool.")
        old = self.allocated_hot_slots
        new = min(self.max_hot_slots, old + max(1, self.hot_chunk_slots))
        self.hot_k_pool = self._grow(self.hot_k_pool, self._kv(new, torch.float16), old)
        self.hot_v_pool = self._grow(self.hot_v_pool, self._kv(new, torch.float16), old)
        self.hot_free_slots.extend(range(new - 1, old - 1, -1))
        self.allocated_hot_slots = new

    def _grow_warm_slots(self) -> None:
        if self.allocated_warm_slots >= self.max_warm_slots:
            raise RuntimeError("No WARM slots available in compact TierKV pool.")
        old = self.allocated_warm_slots
        new = min(self.max_warm_slots, old + max(1, self.warm_chunk_slots))
        self.warm_k_pool = self._grow(self.warm_k_pool, self._kv(new, torch.uint8), old)
        self.warm_v_pool = self._grow(self.warm_v_pool, self._kv(new, torch.uint8), old)
        self.k_scale = self._grow(self.k_scale, self._meta(new, 1), old)
        self.k_zero = self._grow(self.k_zero, self._meta(new, 0), old)
        self.v_scale = self._grow(self.v_scale, self._meta(new, 1), old)
        self.v_zero = self._grow(self.v_zero, self._meta(new, 0), old)
        self.warm_free_slots.extend(range(new - 1, old - 1, -1))
        self.allocated_warm_slots = new

    # -- slots -----------------------------------------------------------------
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
        """The slot bookkeeping as plain lists and dictionaries (string keys)."""
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


class BlockAllocator:
    """The reference's BlockManager (csrc/block_manager.cpp:36-105): LIFO
    allocation over a free list initialised N-1, ..., 0, and per sequence the
    list of (physical block, state) its blocks were allocated with (HOT) and
    later set to (update_block_state)."""

    def __init__(self, total_blocks: int | None = None, free=None):
        self.free = list(free) if free is not None else list(range(int(total_blocks) - 1, -1, -1))
        self.tables: dict = {}  # seq_id -> [[physical, state], ...]

    def allocate_block(self, seq_id) -> int:
        if not self.free:
            raise RuntimeError("No free physical blocks available.")
        physical = self.free.pop()
        self.tables.setdefault(seq_id, []).append([physical, 0])
        return physical

    def update_block_state(self, seq_id, logical_id: int, state: int) -> None:
        blocks = self.tables.get(seq_id)
        if blocks is None:
            raise RuntimeError("Sequence not found for state update.")
        if logical_id < 0 or logical_id >= len(blocks):
            raise RuntimeError("Logical block ID out of range.")
        if int(state) not in (0, 1, 2):
            raise RuntimeError("Invalid block state.")
        blocks[logical_id][1] = int(state)

    def get_physical_indices(self, seq_id) -> list:
        return [b[0] for b in self.tables.get(seq_id, [])]

    def get_states(self, seq_id) -> list:
        return [b[1] for b in self.tables.get(seq_id, [])]
