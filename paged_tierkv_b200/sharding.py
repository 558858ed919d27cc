"""Multi-GPU partitioning of the tiered decode path (one process per GPU).

The reference runs on one GPU; these are the two ways the path is spread over
the GPUs of one node:

* data parallel: each rank owns whole sequences (``dp_slice``).  Sequences
  are independent, so there is no collective on the data path.
* context parallel: one long context is split into contiguous logical-block
  ranges (``block_range``); rank r keeps the KV blocks of its range in its
  own pools.  Each rank runs the decode kernel on its range and produces a
  normalised partial (o fp32, LSE); one all-gather of the packed
  [o | LSE] buffer (NCCL over NVLink) and the LSE-merge kernel give every rank
  the full-context output (``ContextShardedDecode``).  ``P2PContextDecode``
  does the same inside the decode launch: partials are stored into every
  rank's inbox over CUDA IPC peer memory as 64-bit words tagged with the
  call's epoch, and merged by the same kernel once every word it needs
  carries that epoch.  Block scores need no second exchange:
  p_global = p_local * exp(lse_local - lse_global).

COLD blocks stay exact under sharding: each rank adds the analytic
``n * exp(0 - m)`` term of the COLD tokens in its own range.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable

import torch

from . import ops


def dp_slice(batch: int, rank: int, world: int) -> slice:
    """Contiguous share of ``batch`` sequences for ``rank`` (sizes differ by <= 1)."""
    base, extra = divmod(int(batch), int(world))
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def block_range(num_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous logical-block range [start, end) of ``rank``; the sink block
    is on rank 0 and the most recent blocks on the last rank."""
    per = -(-int(num_blocks) // int(world)) if num_blocks > 0 else 0
    start = min(rank * per, num_blocks)
    return start, min(start + per, num_blocks)


# Time per HBM byte of a WARM tile relative to a HOT tile: the decode
# kernel's marginal rates measured on B200 over configuration-5 mixes (7.19
# TB/s all-HOT, 6.04 TB/s WARM-heavy).
WARM_TIME_PER_BYTE = 7.19 / 6.04


def balanced_block_ranges(states: torch.Tensor, world: int, block_size: int, head_dim: int):
    """Contiguous block ranges [start, end), one per rank, whose estimated
    decode times are as equal as possible across ``world`` ranks, for the
    block states of one sequence's layer (``states``: [num_blocks] or
    [1, num_blocks]; the first row is used): HBM bytes per token (HOT 4*D, WARM
    2*D + 8, COLD only its table entry) with WARM bytes weighted by
    ``WARM_TIME_PER_BYTE``, since the consumers make WARM tiles slower per
    byte than HOT ones.  (Measured on configuration 4 at 2 GPUs: balancing
    bytes left the WARM-only rank 13 % slower than the rank with the recent
    HOT window, and the exchange waits for the slower one.)  The LSE merge
    does not depend on where the boundaries fall."""
    st = states.reshape(-1, states.shape[-1])[0].tolist()
    cost = [block_size * (4 * head_dim if s == ops.HOT_STATE else
                          (2 * head_dim + 8) * WARM_TIME_PER_BYTE if s == ops.WARM_STATE else 0)
            + 12 for s in st]
    total = float(sum(cost))
    bounds, acc, r = [0], 0.0, 1
    for i, c in enumerate(cost):
        acc += c
        while r < world and acc >= total * r / world:
            bounds.append(i + 1)
            r += 1
    while len(bounds) < world + 1:
        bounds.append(len(st))
    bounds[-1] = len(st)
    return [(bounds[k], bounds[k + 1]) for k in range(world)]


@dataclass
class ShardResult:
    out: torch.Tensor                   # [batch, num_heads, head_dim]
    lse: torch.Tensor                   # [batch, num_heads] global natural-log LSE
    score_sums: torch.Tensor | None     # [batch, num_heads, local_blocks] global mass


def _local_cuda(query, table, states, lengths, pools, num_blocks, groups, scaling, o_out, lse_out,
                return_scores):
    _, scores, _ = ops.decode_attention(query, table, states, lengths, pools, num_blocks, groups,
                                        scaling, out=o_out, out_dtype=torch.float32,
                                        return_lse=lse_out, return_scores=return_scores)
    return scores


def _merge_cuda(part_o, part_lse, out_dtype):
    return ops.merge_partials(part_o, part_lse, out_dtype=out_dtype, return_lse=True)


class ContextShardedDecode:
    """Decode of context-sharded sequences over a process group.

    ``local_fn(query, table, states, lengths, pools, num_blocks, groups,
    scaling, o_out, lse_out, return_scores) -> score_sums or None`` fills the
    rank's normalised partial; ``merge_fn(part_o [P,R,D], part_lse [P,R],
    out_dtype) -> (out [R,D], lse [R])`` merges gathered partials.  The
    defaults are the sm_100a kernels; tests substitute CPU stand-ins to check
    the partitioning and exchange logic over gloo.
    """

    def __init__(self, group=None, local_fn: Callable | None = None,
                 merge_fn: Callable | None = None):
        self.group = group
        self.local_fn = local_fn or _local_cuda
        self.merge_fn = merge_fn or _merge_cuda
        self._bufs: dict = {}
        # device errors of the local decode launches (an out-of-pool slot),
        # reported one call behind without synchronizing
        self.watch = ops.DeviceErrorWatch(what="context-sharded decode")

    def check(self) -> None:
        """Raise ``ops.TierKVDeviceError`` for device errors recorded by any
        call so far (waits for the outstanding error-word copies)."""
        self.watch.check()

    def _buffers(self, rows: int, d: int, world: int, device):
        key = (rows, d, world, str(device))
        b = self._bufs.get(key)
        if b is None:
            n = rows * (d + 1)
            b = (torch.empty(n, dtype=torch.float32, device=device),
                 torch.empty(world * n, dtype=torch.float32, device=device))
            self._bufs[key] = b
        return b

    def __call__(self, query: torch.Tensor, block_table: torch.Tensor, block_states: torch.Tensor,
                 block_lengths: torch.Tensor, pools, num_blocks, num_key_value_groups: int,
                 scaling: float, *, out_dtype=torch.float16, return_scores: bool = False) -> ShardResult:
        """``query`` [B, Hq, D]; the tables hold only this rank's block range
        ([B, local_T]) and ``num_blocks`` counts the valid local blocks."""
        import torch.distributed as dist
        world = dist.get_world_size(self.group)
        b, hq, d = query.shape
        rows = b * hq
        watched = query.is_cuda and self.local_fn is _local_cuda
        if watched:
            self.watch.poll()
        local, gathered = self._buffers(rows, d, world, query.device)
        o_local = local[:rows * d].view(b, hq, d)
        lse_local = local[rows * d:].view(b, hq)
        scores = self.local_fn(query, block_table, block_states, block_lengths, pools, num_blocks,
                               num_key_value_groups, scaling, o_local, lse_local, return_scores)
        if watched:
            self.watch.record(ops.workspace_error_word(query.device.index))
        if world > 1:
            dist.all_gather_into_tensor(gathered, local, group=self.group)
            parts = gathered.view(world, rows * (d + 1))
        else:
            parts = local.view(1, rows * (d + 1))
        out, lse = self.merge_fn(parts[:, :rows * d].view(world, rows, d), parts[:, rows * d:],
                                 out_dtype)
        lse = lse.view(b, hq)
        if scores is not None:
            w = torch.exp(lse_local - lse)
            w = torch.where(torch.isfinite(lse_local), w, torch.zeros_like(w))
            scores = scores * w.unsqueeze(-1)
        return ShardResult(out=out.view(b, hq, d), lse=lse, score_sums=scores)


# ---------------------------------------------------------------------------
# exchange over peer memory (one launch per rank instead of all-gather + merge)
# ---------------------------------------------------------------------------

class PeerExchange:
    """This rank's inbox and the other ranks' inboxes mapped into this process
    (CUDA IPC over NVLink; no multicast), for ``tkv_decode_attention_exchange``.

    Capacities (``rows_cap`` = batch * num_heads, ``units_cap`` = batch *
    kv_heads, ``head_dim``) fix the inbox layout and must be equal on every
    rank.  ``next()`` returns the exchange descriptor of the next call; every
    rank must make the same sequence of calls.  ``close()`` unmaps the peers'
    inboxes after a barrier and frees this rank's.
    """

    def __init__(self, group=None, *, rows_cap: int, units_cap: int, head_dim: int,
                 timeout_ns: int = 0, inboxes=None, rank: int | None = None,
                 device_epoch: bool = False):
        from . import _native as N
        self._N = N
        lib = N.load()
        self.group = group
        self.rows_cap, self.units_cap, self.head_dim = int(rows_cap), int(units_cap), int(head_dim)
        self.timeout_ns = int(timeout_ns)
        self.epoch = 0
        self._own = None
        self._mapped = []
        # device_epoch: the epoch lives in device memory and every launch
        # advances it, so CUDA graph replays see a new epoch every call
        self.epoch_device = torch.device("cuda", torch.cuda.current_device())
        self.epoch_t = (torch.ones(1, dtype=torch.int32, device=self.epoch_device)
                        if device_epoch else None)
        if inboxes is not None:
            # caller-provided inbox addresses (e.g. several inboxes in one process)
            self.world = len(inboxes)
            self.rank = int(rank or 0)
            self.inbox = [int(x) for x in inboxes]
            return
        import torch.distributed as dist
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > N.TKV_EXCHANGE_MAX_RANKS:
            raise ValueError(f"at most {N.TKV_EXCHANGE_MAX_RANKS} ranks share a context")
        nbytes = lib.tkv_exchange_bytes(self.world, self.rows_cap, self.units_cap, self.head_dim)
        if nbytes == 0:
            raise ValueError("invalid exchange capacities")
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * N.TKV_IPC_HANDLE_BYTES)()
        N.check(lib.tkv_exchange_alloc(nbytes, ctypes.byref(ptr), handle), "tkv_exchange_alloc")
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.inbox = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.inbox.append(self._own)
                continue
            buf = (ctypes.c_uint8 * N.TKV_IPC_HANDLE_BYTES).from_buffer_copy(h)
            m = ctypes.c_void_p()
            N.check(lib.tkv_exchange_open(buf, ctypes.byref(m)), "tkv_exchange_open")
            self._mapped.append(m.value)
            self.inbox.append(m.value)
        dist.barrier(group=group)

    def next(self):
        """The descriptor of the next call (epochs run 1, 2, ...; never 0)."""
        x = self._N.TkvExchange()
        if self.epoch_t is not None:
            x.epoch_dev = self.epoch_t.data_ptr()
        else:
            self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
            x.epoch = self.epoch
        x.world, x.rank = self.world, self.rank
        x.rows_cap, x.units_cap, x.timeout_ns = self.rows_cap, self.units_cap, self.timeout_ns
        for q, ptr in enumerate(self.inbox):
            x.inbox[q] = ptr
        return x

    def resync(self) -> None:
        """Bring the ranks' epochs back into step after a timed-out exchange.

        Collective: every rank of the group calls it, between calls, once any
        rank has raised a timeout (the application agrees on that, e.g. with
        its own all-reduce of an error flag).  Waits for this rank's GPU work,
        meets the other ranks, and moves every rank to one epoch beyond the
        largest epoch any rank has used, so no word in any inbox (all of them
        stamped with older epochs) can satisfy the next call's wait before its
        peer has published for it."""
        torch.cuda.synchronize()
        if self.epoch_t is not None:
            cur = int(self.epoch_t.item())
        else:
            cur = int(self.epoch)
        nxt = cur + 2
        if self._own is not None:  # a process group: agree on the largest epoch
            import torch.distributed as dist
            t = torch.tensor([nxt], dtype=torch.int64, device=self.epoch_device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            nxt = int(t.item())
        nxt &= 0xFFFFFFFF
        if nxt == 0:
            nxt = 1
        if self.epoch_t is not None:
            self.epoch_t.fill_(nxt)
        else:
            self.epoch = nxt - 1  # next() hands out nxt
        if self._own is not None:
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier(group=self.group)

    def close(self) -> None:
        lib = self._N.load()
        if self._own is not None:
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            for m in self._mapped:
                lib.tkv_exchange_close(m)
            self._mapped = []
            dist.barrier(group=self.group)
            lib.tkv_exchange_free(self._own)
            self._own = None


class P2PContextDecode:
    """Context-sharded decode whose exchange and merge run inside the decode
    launch (``tkv_decode_attention_exchange``): one kernel per rank per call,
    no collective.  Returns the same ShardResult as ContextShardedDecode, with
    scores normalised over the whole contexts."""

    def __init__(self, exchange: PeerExchange):
        self.exchange = exchange
        # device errors of the launches (a peer that did not publish within
        # the exchange's timeout, an out-of-pool slot), reported one call
        # behind without synchronizing
        self.watch = ops.DeviceErrorWatch(what="exchange decode")

    def check(self) -> None:
        """Raise ``ops.TierKVDeviceError`` for device errors recorded by any
        eager call so far (waits for the outstanding error-word copies).
        Calls replayed from a CUDA graph are not watched: after replays, read
        the stream's error word with ``ops.read_device_errors``."""
        self.watch.check()

    def __call__(self, query: torch.Tensor, block_table: torch.Tensor, block_states: torch.Tensor,
                 block_lengths: torch.Tensor, pools, num_blocks, num_key_value_groups: int,
                 scaling: float, *, out_dtype=torch.float16, return_scores: bool = False,
                 out: torch.Tensor | None = None) -> ShardResult:
        """Raises ``ops.TierKVDeviceError`` before launching when an earlier
        call's launch recorded a device error; after a timeout every rank must
        call ``exchange.resync()`` before the next call."""
        self.watch.poll()
        o, scores, lse = ops.decode_attention(query, block_table, block_states, block_lengths, pools,
                                              num_blocks, num_key_value_groups, scaling,
                                              return_scores=return_scores, return_lse=True,
                                              out=out, out_dtype=out_dtype,
                                              exchange=self.exchange.next())
        self.watch.record(ops.workspace_error_word(query.device.index))
        return ShardResult(o, lse, scores)
