"""Golden fixtures for the batched storage sync, made by the reference itself.

Usage (only where a checkout of xiaoMartintin/Paged_TierKV is available):

    python tests/golden/make_tiering_golden.py --reference <path-to-Paged_TierKV>

For each scenario it builds a ``CompactTieredKVTensorPool``
(tierkv_policy.py:701-1365) on the CPU through the reference's own
``write_hot_tokens`` / ``set_block_entry`` / ``demote_to_warm`` /
``demote_to_cold``, records the pool's complete state, then runs the
reference's ``TieredKVRuntime.sync_storage_states`` (tierkv_policy.py:1849-1867,
called unbound with a stand-in block manager that returns the scenario's
physical indices and desired states) and records the complete state again.
A state is the slot bookkeeping (free lists, per-physical state / slot /
length / location, storage sets, allocated capacities), the layer tables and
every pool tensor, so the fixture pins slot numbering (LIFO reuse, growth by
chunks) and every stored byte, stale rows of reused slots included.

Scenarios (seeded): LIFO reuse in both directions within one sync (a
demotion frees a HOT slot a later promotion takes, and the reverse), pool
growth during the sync, partial blocks, HOT->COLD and WARM->COLD, no-ops.

``append_decode.npz`` records the decode-time append the same way: a
two-layer pool filled through the reference's ``TieredKVRuntime.append_to_layer``
(tierkv_policy.py:1768-1816, called unbound on a stand-in runtime whose
block manager allocates physical blocks like csrc/block_manager.cpp:36-50,
LIFO from a free list initialised N-1..0), its state, then a recorded
sequence of multi-token and one-token appends on both layers (block
boundaries, pool growth, an open block demoted to WARM and appended to again,
which promotes it) with their inputs, return values and the state after.

``prefill_policy.npz`` records ``TieredKVRuntime.append_prefill_with_policy``
(tierkv_policy.py:1722-1766, called unbound on a stand-in runtime with the
reference's own ``_desired_prefill_states``, 1695-1720): a pool with a
prefilled layer, its state, then prefills of further layers under the three
policy modes (partial last block, one- and two-block layers, WARM pool
growth) with their inputs and scores, the desired states, and the state after.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

HOT, WARM, COLD = 0, 1, 2


def _state(pool):
    book = {
        "hot_free_slots": [int(x) for x in pool.hot_free_slots],
        "warm_free_slots": [int(x) for x in pool.warm_free_slots],
        "physical_states": {str(k): int(v) for k, v in pool.physical_states.items()},
        "physical_slots": {str(k): int(v) for k, v in pool.physical_slots.items()},
        "physical_lengths": {str(k): int(v) for k, v in pool.physical_lengths.items()},
        "physical_locations": {str(k): [int(v[0]), int(v[1])] for k, v in pool.physical_locations.items()},
        "hot_storage": sorted(int(x) for x in pool.hot_storage),
        "warm_storage": sorted(int(x) for x in pool.warm_storage),
        "cold_storage": sorted(int(x) for x in pool.cold_storage),
        "allocated_hot_slots": int(pool.allocated_hot_slots),
        "allocated_warm_slots": int(pool.allocated_warm_slots),
    }
    arrays = {
        "hot_k": pool.hot_k_pool, "hot_v": pool.hot_v_pool, "warm_k": pool.warm_k_pool,
        "warm_v": pool.warm_v_pool, "k_scale": pool.k_scale, "k_zero": pool.k_zero,
        "v_scale": pool.v_scale, "v_zero": pool.v_zero,
        "block_states": pool.block_states, "block_slot_indices": pool.block_slot_indices,
        "block_lengths": pool.block_lengths, "physical_block_tables": pool.physical_block_tables,
    }
    return book, {k: v.detach().cpu().numpy().copy() for k, v in arrays.items()}


def build(tp, torch, *, seed, n_blocks, kv_heads, head_dim, block_size, chunk, partial_every,
          initial_warm, initial_cold, desired_fn):
    rng = np.random.default_rng(seed)
    gen = torch.Generator().manual_seed(seed)
    pool = tp.CompactTieredKVTensorPool(num_layers=1, block_size=block_size,
                                        max_seq_len=block_size * n_blocks, pool_blocks=n_blocks + 8,
                                        pool_chunk_blocks=chunk)
    physical = rng.permutation(n_blocks + 8)[:n_blocks].tolist()  # physical ids != logical ids
    for logical, p in enumerate(physical):
        length = block_size if (partial_every == 0 or logical % partial_every) else int(rng.integers(1, block_size))
        k = torch.randn((1, kv_heads, length, head_dim), generator=gen).to(torch.float16)
        v = torch.randn((1, kv_heads, length, head_dim), generator=gen).to(torch.float16)
        pool.write_hot_tokens(p, 0, k, v)
        pool.set_block_entry(0, logical, p, HOT)
    # initial tiering in a shuffled order, so the free lists are not sorted
    order = rng.permutation(n_blocks).tolist()
    states = [HOT] * n_blocks
    for logical in order:
        if logical in initial_warm:
            pool.demote_to_warm(physical[logical])
            pool.set_block_state(0, logical, WARM)
            states[logical] = WARM
        elif logical in initial_cold:
            pool.demote_to_cold(physical[logical])
            pool.set_block_state(0, logical, COLD)
            states[logical] = COLD
    before_book, before = _state(pool)
    desired = desired_fn(states, rng)
    bm = types.SimpleNamespace(get_physical_indices=lambda seq_id: list(physical),
                               get_states=lambda seq_id: list(desired))
    runtime = types.SimpleNamespace(block_manager=bm, kv_pool=pool)
    tp.TieredKVRuntime.sync_storage_states(runtime, 0)
    after_book, after = _state(pool)
    meta = {
        "seed": seed, "kv_heads": kv_heads, "head_dim": head_dim, "block_size": block_size,
        "num_layers": 1, "max_blocks_per_layer": int(pool.max_blocks_per_layer),
        "pool_blocks": int(pool.pool_blocks),
        "max_hot_slots": int(pool.max_hot_slots), "max_warm_slots": int(pool.max_warm_slots),
        "hot_chunk_slots": int(pool.hot_chunk_slots), "warm_chunk_slots": int(pool.warm_chunk_slots),
        "layer": 0, "physical_indices": [int(x) for x in physical], "desired": [int(x) for x in desired],
        "before": before_book, "after": after_book,
    }
    out = {"meta": np.array(json.dumps(meta))}
    out.update({f"before_{k}": v for k, v in before.items()})
    out.update({f"after_{k}": v for k, v in after.items()})
    return out


def _swap(states, rng):
    """Swap tiers: some HOT become WARM (and COLD), some WARM become HOT (and COLD)."""
    out = list(states)
    for i, s in enumerate(states):
        r = rng.random()
        if s == HOT:
            out[i] = WARM if r < 0.45 else (COLD if r < 0.55 else HOT)
        elif s == WARM:
            out[i] = HOT if r < 0.45 else (COLD if r < 0.6 else WARM)
    return out


def _demote_many(states, rng):
    """Most HOT blocks go WARM: the WARM pool has to grow during the sync."""
    return [WARM if (s == HOT and rng.random() < 0.8) else s for s in states]


def _alternate(states, rng):
    """Alternating demotion / promotion in logical order (chains of slot reuse)."""
    out = list(states)
    for i, s in enumerate(states):
        if s == HOT and i % 2 == 0:
            out[i] = WARM
        elif s == WARM and i % 2 == 1:
            out[i] = HOT
    return out


SCENARIOS = {
    "tiering_swap": dict(seed=101, n_blocks=24, kv_heads=2, head_dim=64, block_size=16, chunk=4,
                         partial_every=5, initial_warm=set(range(3, 20, 2)),
                         initial_cold={4, 10, 16}, desired_fn=_swap),
    "tiering_grow": dict(seed=202, n_blocks=20, kv_heads=1, head_dim=128, block_size=16, chunk=3,
                         partial_every=4, initial_warm={1, 2}, initial_cold={7},
                         desired_fn=_demote_many),
    "tiering_alternate": dict(seed=303, n_blocks=18, kv_heads=1, head_dim=64, block_size=32, chunk=5,
                              partial_every=6, initial_warm=set(range(1, 18, 2)), initial_cold=set(),
                              desired_fn=_alternate),
}


class _BlockManager:
    """csrc/block_manager.cpp:36-50: LIFO over [N-1, ..., 0]."""

    def __init__(self, n):
        self.free = list(range(n - 1, -1, -1))

    def allocate_block(self, seq_id):
        return self.free.pop()


def _layer_states(rt):
    return {str(k): [v.open_physical_idx, int(v.open_token_count), int(v.num_blocks)]
            for k, v in rt.layer_states.items()}


def build_append(tp, torch, *, seed=404, kv_heads=2, head_dim=64, block_size=16, layers=2):
    gen = torch.Generator().manual_seed(seed)
    max_blocks = 10
    pool = tp.CompactTieredKVTensorPool(num_layers=layers, block_size=block_size,
                                        max_seq_len=block_size * max_blocks,
                                        pool_blocks=layers * max_blocks, pool_chunk_blocks=3)
    bm = _BlockManager(layers * max_blocks)
    rt = types.SimpleNamespace(layer_states={i: tp.LayerRuntimeState() for i in range(layers)},
                               block_manager=bm, kv_pool=pool, block_size=block_size,
                               max_blocks_per_layer=max_blocks)

    def kv(tokens):
        k = torch.randn((1, kv_heads, tokens, head_dim), generator=gen).to(torch.float16)
        v = torch.randn((1, kv_heads, tokens, head_dim), generator=gen).to(torch.float16)
        return k, v

    # set-up: a 21-token and a 3-token prompt, then a few decode tokens
    for layer, n in ((0, 21), (1, 3), (0, 1), (1, 1)):
        tp.TieredKVRuntime.append_to_layer(rt, layer, *kv(n))
    # layer 0's first (full) block goes WARM, so both pools exist
    first = next(p for p, loc in pool.physical_locations.items() if tuple(loc) == (0, 0))
    pool.demote_to_warm(first)
    pool.set_block_state(0, 0, WARM)
    before_book, before = _state(pool)
    before_layers = _layer_states(rt)
    before_bm = list(bm.free)
    calls, inputs = [], {}
    plan = [(0, 1)] * 3 + [(1, 1)] * 4 + [(1, 14), (0, 1), (1, 1)] + [(0, 1), (1, 1)] * 12
    for i, (layer, n) in enumerate(plan):
        if i == 5:
            # the open block of layer 0 goes WARM; the next append promotes it
            open_p = rt.layer_states[0].open_physical_idx
            pool.demote_to_warm(open_p)
            loc = pool.physical_locations[open_p]
            pool.set_block_state(loc[0], loc[1], WARM)
            calls.append({"demote_open": 0})
        k, v = kv(n)
        inputs[f"in_{i}_k"], inputs[f"in_{i}_v"] = k.numpy(), v.numpy()
        new_block = tp.TieredKVRuntime.append_to_layer(rt, layer, k, v)
        calls.append({"layer": layer, "tokens": n, "index": i, "new_block": bool(new_block)})
    after_book, after = _state(pool)
    meta = {
        "seed": seed, "kv_heads": kv_heads, "head_dim": head_dim, "block_size": block_size,
        "num_layers": layers, "max_blocks_per_layer": max_blocks, "pool_blocks": int(pool.pool_blocks),
        "max_hot_slots": int(pool.max_hot_slots), "max_warm_slots": int(pool.max_warm_slots),
        "hot_chunk_slots": int(pool.hot_chunk_slots), "warm_chunk_slots": int(pool.warm_chunk_slots),
        "before": before_book, "after": after_book, "before_layers": before_layers,
        "after_layers": _layer_states(rt), "before_bm_free": before_bm, "after_bm_free": list(bm.free),
        "calls": calls,
    }
    out = {"meta": np.array(json.dumps(meta))}
    out.update({f"before_{k}": v for k, v in before.items()})
    out.update({f"after_{k}": v for k, v in after.items()})
    out.update(inputs)
    return out


class _PrefillBlockManager(_BlockManager):
    """csrc/block_manager.cpp:36-77: LIFO allocation, per-sequence (physical,
    state) lists, update_block_state."""

    def __init__(self, n):
        super().__init__(n)
        self.tables = {}

    def allocate_block(self, seq_id):
        p = super().allocate_block(seq_id)
        self.tables.setdefault(seq_id, []).append([p, HOT])
        return p

    def update_block_state(self, seq_id, logical_id, state):
        self.tables[seq_id][logical_id][1] = int(state)


# (layer, tokens, policy_mode, hot_budget, warm_budget) of the recorded calls
PREFILL_CALLS = [
    (1, 150, "hot_warm_cold", 4, 3),   # 10 blocks, the last partial: HOT / WARM / COLD
    (2, 37, "hot_warm", 2, 0),         # 3 blocks: the middle one demoted to WARM
    (3, 20, "hot_warm_cold", 4, 3),    # 2 blocks: all HOT whatever the scores
    (4, 64, "hot_warm_cold", 3, 0),    # 4 blocks: one extra HOT, one COLD
    (5, 200, "hot_warm", 3, 0),        # 13 blocks: the WARM pool grows several times
]


def build_prefill(tp, torch, *, seed=505, kv_heads=2, head_dim=64, block_size=16, layers=6):
    """append_prefill_with_policy (tierkv_policy.py:1722-1766) called unbound on a
    stand-in runtime: state before, the recorded calls with their inputs and
    the desired states they produced, state after."""
    import types as _types
    gen = torch.Generator().manual_seed(seed)
    max_blocks = 16
    pool = tp.CompactTieredKVTensorPool(num_layers=layers, block_size=block_size,
                                        max_seq_len=block_size * max_blocks,
                                        pool_blocks=layers * max_blocks, pool_chunk_blocks=2)
    bm = _PrefillBlockManager(layers * max_blocks)
    rt = _types.SimpleNamespace(layer_states={i: tp.LayerRuntimeState() for i in range(layers)},
                                block_manager=bm, kv_pool=pool, block_size=block_size,
                                max_blocks_per_layer=max_blocks, policy_mode="hot_warm",
                                hot_budget=2, warm_budget=0, demoted_state=WARM)
    rt._desired_prefill_states = _types.MethodType(tp.TieredKVRuntime._desired_prefill_states, rt)

    def kv(tokens):
        k = torch.randn((1, kv_heads, tokens, head_dim), generator=gen).to(torch.float16)
        v = torch.randn((1, kv_heads, tokens, head_dim), generator=gen).to(torch.float16)
        return k, v

    # set-up: layer 0 prefilled with one WARM block, so both pools exist
    k, v = kv(40)
    tp.TieredKVRuntime.append_prefill_with_policy(rt, 0, k, v, torch.tensor([0.9, 0.1, 0.5]))
    before_book, before = _state(pool)
    before_layers = _layer_states(rt)
    before_bm = {"free": list(bm.free), "tables": {str(k2): v2 for k2, v2 in bm.tables.items()}}
    calls, inputs = [], {}
    for i, (layer, tokens, mode, hot, warm) in enumerate(PREFILL_CALLS):
        rt.policy_mode, rt.hot_budget, rt.warm_budget = mode, hot, warm
        nb = -(-tokens // block_size)
        scores = torch.rand(nb, generator=gen)
        k, v = kv(tokens)
        inputs[f"in_{i}_k"], inputs[f"in_{i}_v"] = k.numpy(), v.numpy()
        inputs[f"in_{i}_scores"] = scores.numpy()
        desired = rt._desired_prefill_states(nb, scores)
        tp.TieredKVRuntime.append_prefill_with_policy(rt, layer, k, v, scores)
        calls.append({"layer": layer, "tokens": tokens, "policy_mode": mode, "hot_budget": hot,
                      "warm_budget": warm, "index": i, "desired": [int(x) for x in desired]})
    after_book, after = _state(pool)
    meta = {
        "seed": seed, "kv_heads": kv_heads, "head_dim": head_dim, "block_size": block_size,
        "num_layers": layers, "max_blocks_per_layer": max_blocks, "pool_blocks": int(pool.pool_blocks),
        "max_hot_slots": int(pool.max_hot_slots), "max_warm_slots": int(pool.max_warm_slots),
        "hot_chunk_slots": int(pool.hot_chunk_slots), "warm_chunk_slots": int(pool.warm_chunk_slots),
        "before": before_book, "after": after_book, "before_layers": before_layers,
        "after_layers": _layer_states(rt), "before_bm": before_bm,
        "after_bm": {"free": list(bm.free), "tables": {str(k2): v2 for k2, v2 in bm.tables.items()}},
        "calls": calls,
    }
    out = {"meta": np.array(json.dumps(meta))}
    out.update({f"before_{k2}": v2 for k2, v2 in before.items()})
    out.update({f"after_{k2}": v2 for k2, v2 in after.items()})
    out.update(inputs)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a Paged_TierKV checkout (read-only)")
    args = ap.parse_args(argv)
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    import tierkv_policy as tp  # noqa: E402  (the reference)
    for name, kw in SCENARIOS.items():
        out = build(tp, torch, **kw)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **out)
        meta = json.loads(str(out["meta"]))
        print(name, os.path.getsize(path), "bytes; desired", meta["desired"])
    out = build_append(tp, torch)
    path = os.path.join(HERE, "append_decode.npz")
    np.savez_compressed(path, **out)
    print("append_decode", os.path.getsize(path), "bytes")
    out = build_prefill(tp, torch)
    path = os.path.join(HERE, "prefill_policy.npz")
    np.savez_compressed(path, **out)
    print("prefill_policy", os.path.getsize(path), "bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
