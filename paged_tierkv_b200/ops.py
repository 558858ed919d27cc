"""Tensor-level front end of the sm_100a tiered decode path.

PyTorch supplies device memory and the current stream; every computation is
one call into the C-ABI library (``_native``).  Shapes follow the reference's
pool layout (tierkv_policy.py:129-135, 835-841) with an added batch axis on
the per-sequence tables and the query.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N

HOT_STATE = 0
WARM_STATE = 1
COLD_STATE = 2

FORMAT_R = N.TKV_FORMAT_R
FORMAT_S = N.TKV_FORMAT_S

_DTYPE = {torch.float16: N.TKV_DTYPE_F16, torch.bfloat16: N.TKV_DTYPE_BF16,
          torch.float32: N.TKV_DTYPE_F32}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# torch's raw current-stream accessor (what its own kernel launchers use);
# building a torch.cuda.Stream object per call costs microseconds
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(stream, device_index: int | None = None) -> ctypes.c_void_p:
    if stream is None:
        if _RAW_STREAM is not None:
            idx = torch.cuda.current_device() if device_index is None else device_index
            return ctypes.c_void_p(_RAW_STREAM(idx))
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


@dataclass
class TieredPools:
    """The eight pool tensors of one layer (or one shared pool of a batch).

    Format R (the reference layout): warm_k/warm_v uint8 and fp16 meta
    [warm_slots, kv_heads, block_size] (a trailing 1 is accepted).
    Format S: warm_k/warm_v int8 and fp32 k_scale/v_scale [warm_slots, kv_heads];
    k_zero/v_zero are unused (None).
    """

    hot_k: torch.Tensor
    hot_v: torch.Tensor
    warm_k: torch.Tensor
    warm_v: torch.Tensor
    k_scale: torch.Tensor
    k_zero: torch.Tensor | None
    v_scale: torch.Tensor
    v_zero: torch.Tensor | None
    fmt: int = FORMAT_R

    @property
    def kv_heads(self) -> int:
        return int(self.hot_k.shape[1])

    @property
    def block_size(self) -> int:
        return int(self.hot_k.shape[2])

    @property
    def head_dim(self) -> int:
        return int(self.hot_k.shape[3])

    @property
    def hot_slots(self) -> int:
        return int(self.hot_k.shape[0])

    @property
    def warm_slots(self) -> int:
        return int(self.warm_k.shape[0])

    @property
    def device(self) -> torch.device:
        return self.hot_k.device

    @classmethod
    def allocate(cls, hot_slots: int, warm_slots: int, kv_heads: int, block_size: int,
                 head_dim: int, device, fmt: int = FORMAT_R) -> "TieredPools":
        """Zero pools with the reference's initial meta values (scale 1, zero 0)."""
        kv = (hot_slots, kv_heads, block_size, head_dim)
        wk = (warm_slots, kv_heads, block_size, head_dim)
        hot_k = torch.zeros(kv, dtype=torch.float16, device=device)
        hot_v = torch.zeros(kv, dtype=torch.float16, device=device)
        if fmt == FORMAT_R:
            meta = (warm_slots, kv_heads, block_size, 1)
            return cls(hot_k, hot_v,
                       torch.zeros(wk, dtype=torch.uint8, device=device),
                       torch.zeros(wk, dtype=torch.uint8, device=device),
                       torch.ones(meta, dtype=torch.float16, device=device),
                       torch.zeros(meta, dtype=torch.float16, device=device),
                       torch.ones(meta, dtype=torch.float16, device=device),
                       torch.zeros(meta, dtype=torch.float16, device=device), FORMAT_R)
        meta = (warm_slots, kv_heads)
        return cls(hot_k, hot_v,
                   torch.zeros(wk, dtype=torch.int8, device=device),
                   torch.zeros(wk, dtype=torch.int8, device=device),
                   torch.ones(meta, dtype=torch.float32, device=device), None,
                   torch.ones(meta, dtype=torch.float32, device=device), None, FORMAT_S)

    def _key(self):
        return tuple(id(getattr(self, n)) for n in ("hot_k", "hot_v", "warm_k", "warm_v", "k_scale",
                                                    "k_zero", "v_scale", "v_zero")) + (self.fmt,)

    def validate(self) -> None:
        """Shape/dtype/layout checks; repeated calls on the same tensors are free."""
        key = self._key()
        if getattr(self, "_validated", None) == key:
            return
        self._validate()
        object.__setattr__(self, "_validated", key)

    def _validate(self) -> None:
        hk = self.hot_k
        if hk.ndim != 4:
            raise ValueError("hot pools must have shape [slots, kv_heads, block_size, head_dim].")
        if not hk.is_cuda:
            raise ValueError("TierKV pools must be CUDA tensors.")
        for name in ("hot_k", "hot_v"):
            t = getattr(self, name)
            if t.shape != hk.shape or t.dtype != torch.float16 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous fp16 tensor shaped like hot_k.")
        wdt = torch.uint8 if self.fmt == FORMAT_R else torch.int8
        for name in ("warm_k", "warm_v"):
            t = getattr(self, name)
            if (t.ndim != 4 or tuple(t.shape[1:]) != tuple(hk.shape[1:]) or t.dtype != wdt
                    or not t.is_contiguous() or t.shape[0] != self.warm_k.shape[0]):
                raise ValueError(f"{name} must be a contiguous {wdt} tensor "
                                 "[warm_slots, kv_heads, block_size, head_dim].")
        n_meta = self.warm_slots * self.kv_heads * (self.block_size if self.fmt == FORMAT_R else 1)
        names = ("k_scale", "k_zero", "v_scale", "v_zero") if self.fmt == FORMAT_R else ("k_scale", "v_scale")
        mdt = torch.float16 if self.fmt == FORMAT_R else torch.float32
        for name in names:
            t = getattr(self, name)
            if t is None or t.dtype != mdt or t.numel() != n_meta or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous {mdt} tensor with {n_meta} elements.")

    def struct(self) -> N.TkvPools:
        """validate() and as_struct() for repeated calls: the struct is rebuilt
        only when a tensor object or its data pointer changes."""
        key = self._key() + tuple(t.data_ptr() if t is not None else 0 for t in (
            self.hot_k, self.hot_v, self.warm_k, self.warm_v, self.k_scale, self.k_zero,
            self.v_scale, self.v_zero))
        cached = getattr(self, "_struct_cache", None)
        if cached is not None and cached[0] == key:
            return cached[1]
        self.validate()
        st = self.as_struct()
        object.__setattr__(self, "_struct_cache", (key, st))
        return st

    def as_struct(self) -> N.TkvPools:
        return N.TkvPools(
            _ptr(self.hot_k), _ptr(self.hot_v), _ptr(self.warm_k), _ptr(self.warm_v),
            _ptr(self.k_scale), _ptr(self.k_zero), _ptr(self.v_scale), _ptr(self.v_zero),
            self.hot_slots, self.warm_slots, self.kv_heads, self.block_size, self.head_dim,
            int(self.fmt))


# ---------------------------------------------------------------------------
# workspace: one zero-filled buffer per (device, stream), grown on demand
# ---------------------------------------------------------------------------
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def workspace_for(device: torch.device, stream_handle: int, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), stream_handle)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _as_table(t: torch.Tensor, batch: int, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        raise ValueError(f"{name} must be int32.")
    if t.ndim == 1:
        t = t.unsqueeze(0)
    if t.ndim != 2 or t.shape[0] != batch:
        raise ValueError(f"{name} must have shape [batch, max_blocks].")
    if t.stride(1) != 1 or (batch > 1 and t.stride(0) < t.shape[1]):
        t = t.contiguous()
    return t


def _row_stride(t: torch.Tensor) -> int:
    """Row stride of a [batch, max_blocks] table; a single row may carry any stride."""
    return int(t.stride(0)) if t.shape[0] > 1 else int(t.shape[1])


def decode_attention(query: torch.Tensor, block_table: torch.Tensor, block_states: torch.Tensor,
                     block_lengths: torch.Tensor, pools: TieredPools, num_blocks,
                     num_key_value_groups: int, scaling: float, *, return_scores: bool = False,
                     return_lse: bool = False, out: torch.Tensor | None = None,
                     out_dtype: torch.dtype | None = None, num_splits: int = 0,
                     chunk_blocks: int = 0, exchange=None, stream=None):
    """Tiered paged decode attention over a batch of sequences.

    query [B, Hq, D] or [B, Hq, 1, D]; tables [B, T] (or [T] for B = 1) int32;
    num_blocks: int (all sequences) or an int32 CUDA tensor [B].
    num_splits / chunk_blocks (8, 16 or 32): CTAs per (sequence, kv head) and
    blocks per claimed work chunk; 0 lets the planner choose.
    exchange: a ``_native.TkvExchange`` (see ``sharding.PeerExchange``): this
    rank holds one block range of every sequence; the partials of all ranks
    are exchanged over peer memory and merged inside the same launch, and the
    returned output, LSE and scores are those of the whole contexts.
    Returns (out [B, Hq, D], score_sums [B, Hq, T] or None, lse [B, Hq] or None).
    """
    if query.ndim == 4:
        if query.shape[2] != 1:
            raise ValueError("decode attention takes one query token per sequence.")
        query = query[:, :, 0, :]
    if query.ndim != 3:
        raise ValueError("query must have shape [batch, num_heads, head_dim].")
    if not query.is_cuda:
        raise ValueError("TierKV decode requires CUDA tensors.")
    if query.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("TierKV decode supports fp16/bf16 query tensors only.")
    query = query.contiguous()
    if query.data_ptr() % 16:  # the kernel reads the query in 16-byte vectors
        query = query.clone()
    pstruct = pools.struct()
    batch, num_heads, head_dim = query.shape
    if head_dim != pools.head_dim:
        raise ValueError("query head_dim does not match the pools.")
    table = _as_table(block_table, batch, "block_table")
    states = _as_table(block_states, batch, "block_states")
    lengths = _as_table(block_lengths, batch, "block_lengths")
    row_stride = _row_stride(table)
    if not (row_stride == _row_stride(states) == _row_stride(lengths)):
        table, states, lengths = table.contiguous(), states.contiguous(), lengths.contiguous()
        row_stride = _row_stride(table)
    max_blocks = int(table.shape[1])
    nb_dev = None
    if isinstance(num_blocks, torch.Tensor):
        nb_dev = num_blocks.to(device=query.device, dtype=torch.int32).contiguous()
        nb_uniform = max_blocks
    else:
        nb_uniform = int(num_blocks)
    odt = out_dtype or query.dtype
    if out is None:
        out = torch.empty((batch, num_heads, head_dim), dtype=odt, device=query.device)
    elif out.dtype != odt or tuple(out.shape[-3:]) != (batch, num_heads, head_dim) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [batch, num_heads, head_dim] tensor.")
    scores = (torch.empty((batch, num_heads, max_blocks), dtype=torch.float32, device=query.device)
              if return_scores else None)
    if isinstance(return_lse, torch.Tensor):
        lse = return_lse  # caller-provided [batch, num_heads] fp32 destination
        if lse.dtype != torch.float32 or lse.numel() != batch * num_heads or not lse.is_contiguous():
            raise ValueError("the LSE destination must be a contiguous fp32 [batch, num_heads] tensor.")
    else:
        lse = (torch.empty((batch, num_heads), dtype=torch.float32, device=query.device)
               if return_lse else None)
    lib = N.load()
    dev_index = query.device.index
    st = _stream(stream, dev_index)
    args = N.TkvDecodeArgs(
        _ptr(query), _DTYPE[query.dtype], _DTYPE[odt], batch, num_heads, int(num_key_value_groups),
        max_blocks, _ptr(table), _ptr(states), _ptr(lengths), row_stride, _ptr(nb_dev),
        nb_uniform, float(scaling), _ptr(out), _ptr(lse), _ptr(scores), int(num_splits),
        int(chunk_blocks), None, 0)
    # The stream's workspace usually fits already; the plan (and a larger
    # workspace) is only needed when the library reports that it does not.
    ws = _WORKSPACES.get((dev_index, st.value or 0))
    for attempt in range(2):
        if ws is None or attempt:
            splits = ctypes.c_int32()
            nbytes = ctypes.c_size_t()
            N.check(lib.tkv_decode_plan(ctypes.byref(pstruct), ctypes.byref(args),
                                        ctypes.byref(splits), ctypes.byref(nbytes)), "tkv_decode_plan")
            ws = workspace_for(query.device, st.value or 0, nbytes.value)
        args.workspace = ws.data_ptr()
        args.workspace_bytes = ws.numel()
        if exchange is not None:
            status = lib.tkv_decode_attention_exchange(ctypes.byref(pstruct), ctypes.byref(args),
                                                       ctypes.byref(exchange), st)
            what = "tkv_decode_attention_exchange"
        else:
            status = lib.tkv_decode_attention(ctypes.byref(pstruct), ctypes.byref(args), st)
            what = "tkv_decode_attention"
        if status != N.TKV_ERR_WORKSPACE or attempt:
            break
    N.check(status, what)
    return out, scores, lse


def plan_splits(pools: TieredPools, batch: int, num_heads: int, num_key_value_groups: int,
                num_blocks: int, max_blocks: int, query_dtype=torch.float16) -> int:
    """The split count the automatic planner picks for a launch of this shape."""
    lib = N.load()
    pstruct = pools.as_struct()
    args = N.TkvDecodeArgs(None, _DTYPE[query_dtype], _DTYPE[query_dtype], batch, num_heads,
                           num_key_value_groups, max_blocks, None, None, None, max_blocks, None,
                           num_blocks, 1.0, None, None, None, 0, 0, None, 0)
    splits = ctypes.c_int32()
    nbytes = ctypes.c_size_t()
    N.check(lib.tkv_decode_plan(ctypes.byref(pstruct), ctypes.byref(args), ctypes.byref(splits),
                                ctypes.byref(nbytes)), "tkv_decode_plan")
    return int(splits.value)


def workspace_error_word(device_index: int | None = None, stream=None) -> torch.Tensor:
    """The device error word (int32 [1]) of the workspace that decode calls on
    ``stream`` (default: the current stream) of ``device_index`` use."""
    dev = torch.cuda.current_device() if device_index is None else int(device_index)
    st = _stream(stream, dev)
    ws = workspace_for(torch.device("cuda", dev), st.value or 0, 1 << 16)
    return ws[:4].view(torch.int32)


class TierKVDeviceError(N.TierKVError):
    """Error bits (TKV_DEVERR_*) that a decode launch recorded on the device:
    ``bits & TKV_DEVERR_BAD_SLOT`` -- a HOT/WARM table entry outside its pool
    (read as zeros); ``bits & TKV_DEVERR_TIMEOUT`` -- a bounded wait gave up
    (a peer that never published its partials, or a stalled pipeline), so the
    output of that call is not valid."""

    def __init__(self, bits: int, call: int, what: str = "decode"):
        self.bits = int(bits)
        self.call = int(call)
        names = [n for b, n in ((N.TKV_DEVERR_BAD_SLOT, "out-of-pool slot"),
                                (N.TKV_DEVERR_TIMEOUT, "bounded wait timed out")) if self.bits & b]
        super().__init__(f"{what} call {self.call} recorded device error 0x{self.bits:x} "
                         f"({', '.join(names) or 'unknown'})")


class DeviceErrorWatch:
    """Reports the device error bits of decode calls without synchronizing.

    ``record(word)`` enqueues, on the current stream, a 4-byte copy of the
    call's error word into pinned host memory and an event behind it (every
    ``period``-th call; none while a CUDA graph is being captured).
    ``poll()`` reads the copies whose events have completed, never waiting,
    and raises :class:`TierKVDeviceError` for the first one that holds error
    bits; it then clears the error word on the device (the bits are sticky
    there) and drops the copies made before.  Polling before each call thus
    reports an error one call (or a few, while the GPU runs behind) after the
    call that recorded it.  ``check()`` waits for every outstanding copy, so
    it reports everything recorded so far; call it after the last call.
    While a CUDA graph is being captured nothing is recorded or polled, so
    calls replayed from a graph are not watched: after replays, read the
    word itself (``read_device_errors``)."""

    def __init__(self, depth: int = 8, period: int = 1, what: str = "decode"):
        self.depth = int(depth)
        self.period = max(1, int(period))
        self.what = what
        self._host = None
        self._slots: list = []      # (event, slot index, call number, error word)
        self._next_slot = 0
        self.calls = 0

    def record(self, word: torch.Tensor) -> None:
        self.calls += 1
        if self.calls % self.period or torch.cuda.is_current_stream_capturing():
            return
        if self._host is None:
            self._host = torch.zeros(self.depth, dtype=torch.int32).pin_memory()
        if len(self._slots) >= self.depth:   # the GPU is `depth` recorded calls behind
            self._slots[0][0].synchronize()
            self.poll()
            if len(self._slots) >= self.depth:
                self._slots.pop(0)
        slot = self._next_slot
        self._next_slot = (slot + 1) % self.depth
        self._host[slot:slot + 1].copy_(word, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._slots.append((ev, slot, self.calls, word))

    def poll(self) -> None:
        if not self._slots or torch.cuda.is_current_stream_capturing():
            return  # event queries are not permitted while a graph is captured
        while self._slots and self._slots[0][0].query():
            _, slot, call, word = self._slots.pop(0)
            bits = int(self._host[slot])
            if bits:
                word.zero_()
                self._slots.clear()
                raise TierKVDeviceError(bits, call, self.what)

    def check(self) -> None:
        if self._slots and not torch.cuda.is_current_stream_capturing():
            self._slots[-1][0].synchronize()
        self.poll()


def read_device_errors(device=None, stream=None) -> int:
    """Read and clear the device error bits of the current stream's workspace."""
    st = _stream(stream)
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    ws = workspace_for(dev, st.value or 0, 1 << 16)
    bits = ctypes.c_uint32()
    N.check(N.load().tkv_read_device_errors(ws.data_ptr(), ctypes.byref(bits), st),
            "tkv_read_device_errors")
    return int(bits.value)


def read_prefill_errors(stream=None) -> int:
    """Read and clear the error bits the prefill kernels of the current device recorded."""
    st = _stream(stream)
    bits = ctypes.c_uint32()
    N.check(N.load().tkv_prefill_read_errors(ctypes.byref(bits), st), "tkv_prefill_read_errors")
    return int(bits.value)


def merge_partials(part_o: torch.Tensor, part_lse: torch.Tensor, *, out_dtype=torch.float16,
                   return_lse: bool = False, out: torch.Tensor | None = None, stream=None):
    """LSE merge: part_o [P, R, D] fp32, part_lse [P, R] fp32 -> out [R, D] (+ lse [R]).

    The part axis may be strided (e.g. views into one all-gathered buffer);
    rows and head_dim must be contiguous within a part."""
    if part_o.ndim != 3 or part_lse.shape != part_o.shape[:2]:
        raise ValueError("part_o must be [parts, rows, head_dim] and part_lse [parts, rows].")
    if part_o.dtype != torch.float32 or part_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32.")
    parts, rows, d = part_o.shape
    if part_o.stride(2) != 1 or part_o.stride(1) != d:
        part_o = part_o.contiguous()
    if part_lse.stride(1) != 1:
        part_lse = part_lse.contiguous()
    if out is None:
        out = torch.empty((rows, d), dtype=out_dtype, device=part_o.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=part_o.device) if return_lse else None
    N.check(N.load().tkv_merge_partials(part_o.data_ptr(), part_o.stride(0), part_lse.data_ptr(),
                                        part_lse.stride(0), parts, rows, d, out.data_ptr(),
                                        _DTYPE[out.dtype], _ptr(lse), _stream(stream)),
            "tkv_merge_partials")
    return (out, lse) if return_lse else out


def block_scores(score_sums: torch.Tensor, block_lengths: torch.Tensor, num_blocks, *, stream=None):
    """mean over heads of score_sums / clamp(length, 1) for b < num_blocks (tierkv_policy.py:1905-1912).

    score_sums [B, Hq, T] (or [Hq, T]); block_lengths [B, T] (or [T]).  Returns
    [B, T] (or [T]) with zeros beyond num_blocks."""
    squeeze = score_sums.ndim == 2
    if squeeze:
        score_sums = score_sums.unsqueeze(0)
    b, hq, t = score_sums.shape
    lengths = _as_table(block_lengths, b, "block_lengths")
    score_sums = score_sums.contiguous()
    out = torch.empty((b, t), dtype=torch.float32, device=score_sums.device)
    nb_dev = None
    if isinstance(num_blocks, torch.Tensor):
        nb_dev = num_blocks.to(device=score_sums.device, dtype=torch.int32).contiguous()
        nb = t
    else:
        nb = int(num_blocks)
    N.check(N.load().tkv_block_scores(score_sums.data_ptr(), lengths.data_ptr(), _row_stride(lengths),
                                      _ptr(nb_dev), nb, b, hq, t, out.data_ptr(), _stream(stream)),
            "tkv_block_scores")
    return out[0] if squeeze else out


def quantize_fp16_to_int8(tensor: torch.Tensor, *, stream=None):
    """Drop-in for tierkv_policy.quantize_fp16_to_int8 (tierkv_policy.py:21-36) on CUDA tensors.

    Returns (codes uint8 like tensor, scale fp16 [..., 1], zero_point fp16 [..., 1]),
    bit-exact with the reference."""
    if not tensor.is_cuda:
        raise ValueError("quantize_fp16_to_int8 on this path requires a CUDA tensor.")
    if tensor.dtype != torch.float16:
        tensor = tensor.to(torch.float16)
    x = tensor.contiguous()
    d = int(x.shape[-1])
    rows = x.numel() // d if d else 0
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scale = torch.empty(x.shape[:-1] + (1,), dtype=torch.float16, device=x.device)
    zero = torch.empty(x.shape[:-1] + (1,), dtype=torch.float16, device=x.device)
    N.check(N.load().tkv_quantize_rows_r(x.data_ptr(), rows, d, codes.data_ptr(), scale.data_ptr(),
                                         zero.data_ptr(), _stream(stream)), "tkv_quantize_rows_r")
    return codes, scale, zero


def _slot_list(x, device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(x), dtype=torch.int32, device=device)


def demote_blocks_to_warm(pools: TieredPools, src_hot_slots, dst_warm_slots, lengths, *,
                          clear_tail: bool = False, stream=None) -> None:
    """Batched HOT->WARM demotion (tierkv_policy.py:1042-1068; clear_tail -> 329-361)."""
    pools.validate()
    dev = pools.device
    src = _slot_list(src_hot_slots, dev)
    dst = _slot_list(dst_warm_slots, dev)
    ln = _slot_list(lengths, dev)
    if not (src.numel() == dst.numel() == ln.numel()):
        raise ValueError("slot lists and lengths must have the same length.")
    ps = pools.as_struct()
    N.check(N.load().tkv_demote_to_warm(ctypes.byref(ps), src.data_ptr(), dst.data_ptr(),
                                        ln.data_ptr(), int(src.numel()), int(bool(clear_tail)),
                                        _stream(stream)), "tkv_demote_to_warm")


def promote_blocks_to_hot(pools: TieredPools, src_warm_slots, dst_hot_slots, lengths, *,
                          stream=None) -> None:
    """Batched WARM->HOT promotion, Format R (tierkv_policy.py:1087-1115 / 375-402)."""
    pools.validate()
    dev = pools.device
    src = _slot_list(src_warm_slots, dev)
    dst = _slot_list(dst_hot_slots, dev)
    ln = _slot_list(lengths, dev)
    if not (src.numel() == dst.numel() == ln.numel()):
        raise ValueError("slot lists and lengths must have the same length.")
    ps = pools.as_struct()
    N.check(N.load().tkv_promote_to_hot(ctypes.byref(ps), src.data_ptr(), dst.data_ptr(),
                                        ln.data_ptr(), int(src.numel()), _stream(stream)),
            "tkv_promote_to_hot")


# ---------------------------------------------------------------------------
# prefill block scores
# ---------------------------------------------------------------------------

def _prefill_shapes(query: torch.Tensor, key: torch.Tensor):
    if query.ndim != 4 or key.ndim != 4:
        raise ValueError("query / key must have shape [batch, heads, tokens, head_dim].")
    if query.dtype != torch.float16 or key.dtype != torch.float16:
        raise ValueError("prefill block scores take fp16 query / key states.")
    if not (query.is_cuda and key.is_cuda):
        raise ValueError("prefill block scores require CUDA tensors.")
    b, hq, tq, d = query.shape
    if key.shape[0] != b or key.shape[3] != d or hq % key.shape[1] != 0:
        raise ValueError("query / key shapes do not match.")
    return b, hq, int(key.shape[1]), tq, int(key.shape[2]), d


def _aligned16(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def prefill_lse(query: torch.Tensor, key: torch.Tensor, scaling: float, *, causal: bool = True,
                stream=None) -> torch.Tensor:
    """Natural-log LSE [B, Hq, Tq] fp32 of softmax(Q K^T * scaling [+ causal mask])."""
    b, hq, hkv, tq, tk, d = _prefill_shapes(query, key)
    q, k = _aligned16(query), _aligned16(key)
    lse = torch.empty((b, hq, tq), dtype=torch.float32, device=query.device)
    N.check(N.load().tkv_prefill_lse(q.data_ptr(), k.data_ptr(), b, hq, hkv, tq, tk, d,
                                     float(scaling), int(bool(causal)), lse.data_ptr(),
                                     _stream(stream)), "tkv_prefill_lse")
    return lse


def prefill_block_scores(query: torch.Tensor, key: torch.Tensor, scaling: float, block_size: int,
                         *, lse: torch.Tensor | None = None, causal: bool = True,
                         return_token_mass: bool = False, stream=None):
    """Exact prefill block scores without attention weights: the mean over
    (batch, heads, queries) of the softmax mass each key receives, averaged
    per block of ``block_size`` keys (the reference's compute_block_scores on
    the eager weights, tierkv_policy.py:1378-1388).  ``lse`` [B, Hq, Tq] fp32
    (natural log) from the caller's flash attention skips the LSE pass."""
    b, hq, hkv, tq, tk, d = _prefill_shapes(query, key)
    q, k = _aligned16(query), _aligned16(key)
    if lse is None:
        lse = prefill_lse(q, k, scaling, causal=causal, stream=stream)
    lse = lse.to(device=query.device, dtype=torch.float32).contiguous()
    if tuple(lse.shape) != (b, hq, tq):
        raise ValueError("lse must have shape [batch, num_heads, query_tokens].")
    nb = (tk + int(block_size) - 1) // int(block_size)
    mass = torch.empty(tk, dtype=torch.float32, device=query.device)
    scores = torch.empty(nb, dtype=torch.float32, device=query.device)
    N.check(N.load().tkv_prefill_block_scores(q.data_ptr(), k.data_ptr(), lse.data_ptr(), b, hq, hkv,
                                              tq, tk, d, float(scaling), int(bool(causal)),
                                              int(block_size), mass.data_ptr(), scores.data_ptr(),
                                              _stream(stream)), "tkv_prefill_block_scores")
    return (scores, mass) if return_token_mass else scores
