"""Seeded inputs of benchmark configuration 1 (the parity configuration).

Batch 4, 32 query heads, 8 KV heads, head_dim 128, 2048 tokens per sequence,
block size 16 (128 blocks).  Per sequence: HOT = block 0 (sink) + the last 31
blocks; WARM = 64 blocks drawn by a seeded permutation of the middle blocks
1..96; COLD = the remaining 32 (evicted: slot -1, no data).  K, V and the
query are fp16 N(0, 1).  All sequences share one HOT pool (slots
``s * 32 + i`` in logical order) and one WARM pool (slots ``s * 64 + j``).
WARM data is returned as the fp16 source rows (``warm_src_k/v``) that the
caller quantizes (reference quantizer, oracle or the demotion kernel).
"""

from __future__ import annotations

import hashlib

import numpy as np

BATCH, Q_HEADS, KV_HEADS, HEAD_DIM, BLOCK, NUM_BLOCKS = 4, 32, 8, 128, 16, 128
HOT_PER_SEQ, WARM_PER_SEQ = 32, 64


def c1_inputs(seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    table = np.full((BATCH, NUM_BLOCKS), -1, np.int32)
    states = np.full((BATCH, NUM_BLOCKS), 2, np.int32)
    lengths = np.full((BATCH, NUM_BLOCKS), BLOCK, np.int32)
    for s in range(BATCH):
        hot = [0] + list(range(NUM_BLOCKS - 31, NUM_BLOCKS))
        middle = np.arange(1, NUM_BLOCKS - 31)
        warm = sorted(int(b) for b in rng.permutation(middle)[:WARM_PER_SEQ])
        for i, b in enumerate(hot):
            table[s, b] = s * HOT_PER_SEQ + i
            states[s, b] = 0
        for j, b in enumerate(warm):
            table[s, b] = s * WARM_PER_SEQ + j
            states[s, b] = 1
    shape_h = (BATCH * HOT_PER_SEQ, KV_HEADS, BLOCK, HEAD_DIM)
    shape_w = (BATCH * WARM_PER_SEQ, KV_HEADS, BLOCK, HEAD_DIM)
    hot_k = rng.standard_normal(shape_h, dtype=np.float32).astype(np.float16)
    hot_v = rng.standard_normal(shape_h, dtype=np.float32).astype(np.float16)
    warm_src_k = rng.standard_normal(shape_w, dtype=np.float32).astype(np.float16)
    warm_src_v = rng.standard_normal(shape_w, dtype=np.float32).astype(np.float16)
    query = rng.standard_normal((BATCH, Q_HEADS, HEAD_DIM), dtype=np.float32).astype(np.float16)
    return dict(batch=BATCH, q_heads=Q_HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM,
                block_size=BLOCK, num_blocks=NUM_BLOCKS, scaling=float(HEAD_DIM ** -0.5),
                block_table=table, block_states=states, block_lengths=lengths,
                hot_k=hot_k, hot_v=hot_v, warm_src_k=warm_src_k, warm_src_v=warm_src_v,
                query=query)


def digest(inp: dict) -> str:
    h = hashlib.sha256()
    for key in ("block_table", "block_states", "block_lengths", "hot_k", "hot_v",
                "warm_src_k", "warm_src_v", "query"):
        h.update(np.ascontiguousarray(inp[key]).tobytes())
    return h.hexdigest()
