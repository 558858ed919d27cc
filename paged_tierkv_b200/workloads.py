"""Seeded synthetic tiered-cache workloads built on the device.

Stands in for the benchmark configurations (random-init shapes, N(0, 1) K/V
and queries; no dataset is involved).  Per sequence of ``N`` blocks: HOT =
block 0 (sink) + the most recent ``n_hot - 1`` blocks; WARM = ``n_warm``
blocks of the middle drawn by a seeded permutation; COLD = the rest (slot
-1, no data).  All sequences share one HOT and one WARM pool whose slots are
handed out in a seeded random order, as a paged allocator would.  WARM
blocks are produced by the demotion kernel from fp16 N(0, 1) staging data.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import ops, sharding


def tier_counts(num_blocks: int, hot_frac: float, warm_frac: float | None = None):
    """(n_hot, n_warm, n_cold).  Without ``warm_frac`` the non-HOT blocks split
    2:1 WARM:COLD (benchmark configuration 5)."""
    n_hot = min(num_blocks, max(1, int(round(hot_frac * num_blocks))))
    rest = num_blocks - n_hot
    if warm_frac is None:
        n_warm = int(round(rest * 2.0 / 3.0))
    else:
        n_warm = min(rest, int(round(warm_frac * num_blocks)))
    return n_hot, n_warm, rest - n_warm


@dataclass
class Workload:
    pools: ops.TieredPools
    query: torch.Tensor
    block_table: torch.Tensor
    block_states: torch.Tensor
    block_lengths: torch.Tensor
    num_blocks: int
    groups: int
    scaling: float
    n_hot: int
    n_warm: int
    n_cold: int
    info: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.query.shape[0])

    def algorithmic_bytes(self) -> int:
        """HBM bytes one decode call must move (tierkv_policy.py:1261-1263 accounting):
        HOT 4*D B and WARM 2*D + 8 B (Format R) per token and kv head, COLD 0,
        plus 12 B of table entries per block and the query/output rows."""
        p = self.pools
        d, bs, hkv = p.head_dim, p.block_size, p.kv_heads
        warm_meta = 8 * bs if p.fmt == ops.FORMAT_R else 8
        per_seq_head = self.n_hot * bs * 4 * d + self.n_warm * (bs * 2 * d + warm_meta)
        tables = 12 * self.num_blocks
        qo = 2 * self.query.shape[1] * d * 2
        return self.batch * (hkv * per_seq_head + tables + qo)


def assign_tiers(batch: int, num_blocks: int, n_hot: int, n_warm: int, seed: int) -> torch.Tensor:
    """States [batch, num_blocks]: HOT = block 0 + the last n_hot - 1 blocks,
    WARM = n_warm middle blocks chosen by a seeded permutation, COLD = rest."""
    cpu = torch.Generator().manual_seed(seed)
    states = torch.full((batch, num_blocks), ops.COLD_STATE, dtype=torch.int32)
    for s in range(batch):
        hot_blocks = torch.cat([torch.zeros(1, dtype=torch.long),
                                torch.arange(num_blocks - (n_hot - 1), num_blocks, dtype=torch.long)]) \
            if n_hot > 1 else torch.zeros(1, dtype=torch.long)
        middle = torch.arange(1, num_blocks - (n_hot - 1), dtype=torch.long)
        warm_blocks = middle[torch.randperm(middle.numel(), generator=cpu)[:n_warm]]
        states[s, hot_blocks] = ops.HOT_STATE
        states[s, warm_blocks] = ops.WARM_STATE
    return states


def materialize(states: torch.Tensor, lengths: torch.Tensor, *, q_heads: int, kv_heads: int,
                head_dim: int, block_size: int, seed: int = 0, device="cuda",
                fmt: int = ops.FORMAT_R, chunk_blocks: int = 2048) -> Workload:
    """Pools, tables and a query for the given per-sequence tier states.

    Slots are handed out in a seeded random order; HOT data is fp16 N(0, 1)
    and WARM blocks are demoted on the device from fp16 N(0, 1) staging data."""
    device = torch.device(device)
    batch, nb = states.shape
    cpu = torch.Generator().manual_seed(seed)
    is_hot = states == ops.HOT_STATE
    is_warm = states == ops.WARM_STATE
    n_hot_all = int(is_hot.sum())
    n_warm_all = int(is_warm.sum())
    table = torch.full((batch, nb), -1, dtype=torch.int32)
    table[is_hot] = torch.randperm(max(1, n_hot_all), generator=cpu)[:n_hot_all].to(torch.int32)
    table[is_warm] = torch.randperm(max(1, n_warm_all), generator=cpu)[:n_warm_all].to(torch.int32)
    hot_slots = max(1, n_hot_all)
    warm_slots = max(1, n_warm_all)
    pools = ops.TieredPools.allocate(hot_slots, warm_slots, kv_heads, block_size, head_dim,
                                     device, fmt=fmt)
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    for start in range(0, hot_slots, chunk_blocks):
        n = min(chunk_blocks, hot_slots - start)
        pools.hot_k[start:start + n].normal_(generator=gen)
        pools.hot_v[start:start + n].normal_(generator=gen)
    if n_warm_all > 0:
        cb = min(chunk_blocks, warm_slots)
        shape = (cb, kv_heads, block_size, head_dim)
        stage_k = torch.empty(shape, dtype=torch.float16, device=device)
        stage_v = torch.empty(shape, dtype=torch.float16, device=device)
        for start in range(0, warm_slots, cb):
            n = min(cb, warm_slots - start)
            stage_k.normal_(generator=gen)
            stage_v.normal_(generator=gen)
            staging = ops.TieredPools(stage_k, stage_v, pools.warm_k, pools.warm_v, pools.k_scale,
                                      pools.k_zero, pools.v_scale, pools.v_zero, fmt)
            src = torch.arange(n, dtype=torch.int32, device=device)
            ops.demote_blocks_to_warm(staging, src, src + start,
                                      torch.full((n,), block_size, dtype=torch.int32, device=device))
        del stage_k, stage_v
    query = torch.randn((batch, q_heads, head_dim), generator=gen, device=device,
                        dtype=torch.float32).to(torch.float16)
    per_seq = lambda m: int(m.sum()) // max(1, batch)  # noqa: E731
    return Workload(pools=pools, query=query, block_table=table.to(device),
                    block_states=states.to(device), block_lengths=lengths.to(device),
                    num_blocks=nb, groups=q_heads // kv_heads, scaling=head_dim ** -0.5,
                    n_hot=per_seq(is_hot), n_warm=per_seq(is_warm),
                    n_cold=nb - per_seq(is_hot) - per_seq(is_warm))


def make_workload(*, batch: int, q_heads: int, kv_heads: int, head_dim: int, block_size: int,
                  ctx_tokens: int, hot_frac: float, warm_frac: float | None = None, seed: int = 0,
                  device="cuda", fmt: int = ops.FORMAT_R, chunk_blocks: int = 2048) -> Workload:
    """Benchmark workload: ``batch`` sequences of ``ctx_tokens`` with the tier mix
    of :func:`tier_counts`."""
    nb = math.ceil(ctx_tokens / block_size)
    n_hot, n_warm, n_cold = tier_counts(nb, hot_frac, warm_frac)
    states = assign_tiers(batch, nb, n_hot, n_warm, seed)
    lengths = torch.full((batch, nb), block_size, dtype=torch.int32)
    lengths[:, nb - 1] = ctx_tokens - (nb - 1) * block_size
    wl = materialize(states, lengths, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                     block_size=block_size, seed=seed, device=device, fmt=fmt,
                     chunk_blocks=chunk_blocks)
    wl.info = dict(batch=batch, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                   block_size=block_size, ctx_tokens=ctx_tokens, hot_frac=hot_frac,
                   blocks_per_seq=nb, hot_blocks=n_hot, warm_blocks=n_warm, cold_blocks=n_cold,
                   seed=seed, warm_format="R" if fmt == ops.FORMAT_R else "S")
    return wl


# Configuration 4's partition: the sharding module's time-balanced ranges.
balanced_block_ranges = sharding.balanced_block_ranges
WARM_TIME_PER_BYTE = sharding.WARM_TIME_PER_BYTE


def decode(wl: Workload, **kw):
    """One decode call of the workload through the public API."""
    return ops.decode_attention(wl.query, wl.block_table, wl.block_states, wl.block_lengths,
                                wl.pools, wl.num_blocks, wl.groups, wl.scaling, **kw)
