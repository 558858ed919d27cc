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
from .ops import FORMAT_R, TieredPools, decode_attention


def _require_backend():
    try:
        _native.load()
    except Exception as exc:  # the library is the only compute path
        raise RuntimeError(
            "The sm_100a TierKV library is not available. Build it with "
            "`python -m paged_tierkv_b200.build` or use TIERKV_ATTENTION_BACKEND=eager.") from exc


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

    pools = TieredPools(hot_k_pool.contiguous(), hot_v_pool.contiguous(), warm_k_pool.contiguous(),
                        warm_v_pool.contiguous(), k_scale.contiguous(), k_zero.contiguous(),
                        v_scale.contiguous(), k_zero.new_empty(0) if v_zero is None else v_zero.contiguous(),
                        FORMAT_R)
    _, num_heads, _, head_dim = query_states.shape
    out, scores, _ = decode_attention(
        query_states, block_table.reshape(1, -1), block_states.reshape(1, -1),
        block_lengths.reshape(1, -1), pools, int(num_blocks), int(num_key_value_groups),
        float(scaling), return_scores=bool(return_scores))
    out = out.view(1, 1, num_heads, head_dim)
    if return_scores:
        return out, scores[0]
    return out, None
