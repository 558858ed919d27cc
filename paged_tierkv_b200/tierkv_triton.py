"""Drop-in replacement of the reference module ``tierkv_triton``.

``tierkv_decode_attention`` keeps the signature, argument meaning, return
contract and validation errors of tierkv_triton.py:272-465 in
xiaoMartintin/Paged_TierKV, but runs the sm_100a C-ABI kernels instead of
Triton.  Install it for the reference's model integration
(modeling_llama.py:61-67 does ``from tierkv_triton import
tierkv_decode_attention``) with::

    import sys, paged_tierkv_b200.tierkv_triton as shim
    sys.modules["tierkv_triton"] = shim

There is no fallback: if the library is missing the call raises RuntimeError,
exactly where the reference raises when Triton is unavailable
(tierkv_triton.py:267-269).
"""

from __future__ import annotations

import torch

from . import _native
from .ops import FORMAT_R, DeviceErrorWatch, TieredPools, decode_attention, workspace_error_word


def _require_backend():
    try:
        _native.load()
    except Exception as exc:  # the library is the only compute path
        raise RuntimeError(
            "The sm_100a TierKV library is not available. Build it with "
            "`python -m paged_tierkv_b200.build` or use TIERKV_ATTENTION_BACKEND=eager.") from exc


# The pool sets of the last two calls.  A runtime passes the same pool tensors
# layer after layer, so their checks and their C struct are reused; the
# bound keeps pools the runtime has replaced (grown) from staying alive.  Only
# sets of contiguous tensors are kept: the cached entry then holds the caller's
# own tensor objects, so their ids cannot be reused while it lives, and a
# non-contiguous pool, which is copied on every call, is never served from a
# stale copy.  The key holds each tensor's address, shape and strides, so a
# tensor changed in place (resize_ / set_ that keep its address) is checked
# and described anew.
_POOLS_CACHE: list = []

# Device errors of the kernel (a HOT/WARM table entry outside its pool, read
# as zeros -- undefined behaviour in the reference's kernel) are raised as
# ops.TierKVDeviceError without synchronizing: every ERROR_CHECK_PERIOD-th
# call copies the error word to pinned memory behind the launch, and a later
# call raises once that copy has landed.  check_device_errors() waits for it.
ERROR_CHECK_PERIOD = 16
_WATCH = DeviceErrorWatch(period=ERROR_CHECK_PERIOD, what="tierkv_decode_attention")


def check_device_errors() -> None:
    """Raise ops.TierKVDeviceError for device errors recorded so far by the
    calls this module has checked (waits for the outstanding copies)."""
    _WATCH.check()


def _pools_of(tensors) -> TieredPools:
    key = tuple((id(t), t.data_ptr(), t.shape, t.stride()) if t is not None else None
                for t in tensors)
    for k, pools in _POOLS_CACHE:
        if k == key:
            return pools
    hk, hv, wk, wv, ks, kz, vs, vz = tensors
    pools = TieredPools(hk.contiguous(), hv.contiguous(), wk.contiguous(), wv.contiguous(),
                        ks.contiguous(), kz.contiguous(), vs.contiguous(),
                        kz.new_empty(0) if vz is None else vz.contiguous(), FORMAT_R)
    held = (pools.hot_k, pools.hot_v, pools.warm_k, pools.warm_v, pools.k_scale, pools.k_zero,
            pools.v_scale, pools.v_zero)
    if all(a is b for a, b in zip(held, tensors) if b is not None):
        _POOLS_CACHE.insert(0, (key, pools))
        del _POOLS_CACHE[2:]
    return pools


def tierkv_decode_attention(
    query_states: torch.Tensor,
    block_table: torch.Tensor,
    block_states: torch.Tensor,
    block_lengths: torch.Tensor,
    hot_k_pool: torch.Tensor,
    hot_v_pool: torch.Tensor,
    warm_k_pool: torch.Tensor,
    warm_v_pool: torch.Tensor,
    k_scale: torch.Tensor,
    k_zero: torch.Tensor,
    v_scale: torch.Tensor,
    v_zero: torch.Tensor,
    num_blocks: int,
    num_key_value_groups: int,
    scaling: float,
    return_scores: bool = False,
):
    """Tiered decode attention for one sequence (batch 1, query_len 1).

    Returns ``(out, None)`` or ``(out, score_sums)`` where out is
    ``[1, 1, num_heads, head_dim]`` in the query dtype and score_sums is
    ``[num_heads, block_table.shape[0]]`` fp32 (zero beyond num_blocks).
    """
    _require_backend()
    if query_states.ndim != 4:
        raise ValueError("query_states must have shape [batch, num_heads, query_len, head_dim].")
    if query_states.shape[0] != 1:
        raise ValueError("TierKV decode supports batch size 1 only.")
    if query_states.shape[-2] != 1:
        raise ValueError("TierKV decode supports query_len == 1 only.")
    if not query_states.is_cuda:
        raise ValueError("TierKV decode requires CUDA tensors.")
    if query_states.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("TierKV decode supports fp16/bf16 query tensors only.")
    if int(num_blocks) <= 0:
        raise ValueError("num_blocks must be positive.")
    if int(num_blocks) > block_table.shape[0]:
        raise ValueError("num_blocks exceeds the provided block table length.")

    pools = _pools_of((hot_k_pool, hot_v_pool, warm_k_pool, warm_v_pool, k_scale, k_zero, v_scale,
                       v_zero))
    _, num_heads, _, head_dim = query_states.shape
    _WATCH.poll()
    out, scores, _ = decode_attention(
        query_states, block_table.reshape(1, -1), block_states.reshape(1, -1),
        block_lengths.reshape(1, -1), pools, int(num_blocks), int(num_key_value_groups),
        float(scaling), return_scores=bool(return_scores))
    if (_WATCH.calls + 1) % _WATCH.period == 0:
        _WATCH.record(workspace_error_word(query_states.device.index))
    else:
        _WATCH.calls += 1
    out = out.view(1, 1, num_heads, head_dim)
    if return_scores:
        return out, scores[0]
    return out, None
