"""Seeded tiered-cache cases for the parity tests (host numpy + upload helpers).

A case holds one shared pool for all sequences (HOT and WARM slots drawn
from shuffled permutations, COLD slot -1), per-sequence tables, and a query.
WARM blocks are quantized by the oracle (Format R: tierkv_policy.py:21-36;
Format S: symmetric absmax per (block, kv head)).
"""

from __future__ import annotations

import numpy as np

from oracle import tierkv_oracle as orc


def make_case(seed: int, *, batch=1, q_heads=8, kv_heads=4, head_dim=64, block_size=16,
              num_blocks=8, max_blocks=None, probs=(0.4, 0.4, 0.2), states=None, lengths=None,
              fmt="R", nb_per_seq=None, value_scale=1.0, spare_slots=3):
    rng = np.random.default_rng(seed)
    max_blocks = max_blocks or num_blocks + 3
    nbs = np.full(batch, num_blocks, np.int32) if nb_per_seq is None else np.asarray(nb_per_seq, np.int32)
    st = np.full((batch, max_blocks), orc.COLD_STATE, np.int32)
    ln = np.zeros((batch, max_blocks), np.int32)
    for s in range(batch):
        n = int(nbs[s])
        if states is not None:
            st[s, :n] = np.asarray(states, np.int32)[:n]
        else:
            st[s, :n] = rng.choice(3, size=n, p=probs)
        if lengths is not None:
            ln[s, :n] = np.asarray(lengths, np.int32)[:n]
        else:
            ln[s, :n] = block_size
            # a few partial blocks in the middle
            for b in range(n):
                if rng.random() < 0.15:
                    ln[s, b] = int(rng.integers(0, block_size + 1))
    n_hot = int(sum((st[s, :nbs[s]] == 0).sum() for s in range(batch)))
    n_warm = int(sum((st[s, :nbs[s]] == 1).sum() for s in range(batch)))
    hot_slots = n_hot + spare_slots
    warm_slots = n_warm + spare_slots
    hot_perm = rng.permutation(hot_slots)
    warm_perm = rng.permutation(warm_slots)
    table = np.full((batch, max_blocks), -1, np.int32)
    hk = (rng.standard_normal((hot_slots, kv_heads, block_size, head_dim)) * value_scale).astype(np.float16)
    hv = (rng.standard_normal((hot_slots, kv_heads, block_size, head_dim)) * value_scale).astype(np.float16)
    src_k = (rng.standard_normal((warm_slots, kv_heads, block_size, head_dim)) * value_scale).astype(np.float16)
    src_v = (rng.standard_normal((warm_slots, kv_heads, block_size, head_dim)) * value_scale).astype(np.float16)
    ih = iw = 0
    for s in range(batch):
        for b in range(int(nbs[s])):
            if st[s, b] == 0:
                table[s, b] = hot_perm[ih]
                ih += 1
            elif st[s, b] == 1:
                table[s, b] = warm_perm[iw]
                iw += 1
    if fmt == "R":
        wk, ks, kz = orc.quantize_rows_r(src_k)
        wv, vs, vz = orc.quantize_rows_r(src_v)
        ks, kz, vs, vz = (a[..., 0] for a in (ks, kz, vs, vz))
    else:
        wk = np.zeros(src_k.shape, np.int8)
        wv = np.zeros(src_v.shape, np.int8)
        ks = np.ones((warm_slots, kv_heads), np.float32)
        vs = np.ones((warm_slots, kv_heads), np.float32)
        for sl in range(warm_slots):
            for h in range(kv_heads):
                wk[sl, h], ks[sl, h] = orc.quantize_block_s(src_k[sl, h], block_size)
                wv[sl, h], vs[sl, h] = orc.quantize_block_s(src_v[sl, h], block_size)
        kz = vz = None
    query = rng.standard_normal((batch, q_heads, head_dim)).astype(np.float16)
    return dict(query=query, block_table=table, block_states=st, block_lengths=ln,
                num_blocks=nbs, hot_k=hk, hot_v=hv, warm_k=wk, warm_v=wv, k_scale=ks,
                k_zero=kz, v_scale=vs, v_zero=vz, groups=q_heads // kv_heads,
                scaling=float(head_dim ** -0.5), fmt=fmt, max_blocks=max_blocks)


def oracle_decode(case, dtype=np.float64):
    return orc.decode_attention(
        case["query"], case["block_table"], case["block_states"], case["block_lengths"],
        case["num_blocks"], case["hot_k"], case["hot_v"], case["warm_k"], case["warm_v"],
        case["k_scale"], case["k_zero"], case["v_scale"], case["v_zero"], case["groups"],
        case["scaling"], fmt=case["fmt"], dtype=dtype)


def to_device(case, device="cuda"):
    import torch
    from paged_tierkv_b200.ops import FORMAT_R, FORMAT_S, TieredPools

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)

    pools = TieredPools(t(case["hot_k"]), t(case["hot_v"]), t(case["warm_k"]), t(case["warm_v"]),
                        t(case["k_scale"]), t(case["k_zero"]), t(case["v_scale"]), t(case["v_zero"]),
                        FORMAT_R if case["fmt"] == "R" else FORMAT_S)
    return dict(pools=pools, query=t(case["query"]), block_table=t(case["block_table"]),
                block_states=t(case["block_states"]), block_lengths=t(case["block_lengths"]),
                num_blocks=t(case["num_blocks"]))
