"""Prefill block scoring for the reference's model code.

``compute_prefill_block_scores`` (modeling_llama.py:281-302) has two paths:
with eager attention it scores blocks from the materialised weights
(``TierKVPolicyEngine.compute_block_scores``, tierkv_policy.py:1378-1388);
with SDPA / flash prefill the weights do not exist and it falls back to a
sink + recency proxy.  The replacement below keeps the same signature and the
same eager path, and -- given the layer's query / key states -- computes the
exact eager scores on the GPU without the weights (``ops.prefill_block_scores``),
so the SDPA / flash model scores its blocks as the eager model does.
"""

from __future__ import annotations

import torch

from . import ops


def compute_prefill_block_scores(policy_engine, attn_weights, seq_len: int, block_size: int,
                                 device, *, query_states: torch.Tensor | None = None,
                                 key_states: torch.Tensor | None = None,
                                 scaling: float | None = None,
                                 lse: torch.Tensor | None = None) -> torch.Tensor:
    if attn_weights is not None:
        return policy_engine.compute_block_scores(attn_weights)
    if query_states is not None and key_states is not None and scaling is not None:
        return ops.prefill_block_scores(query_states, key_states, scaling, block_size, lse=lse)
    # the reference's proxy when nothing else is known (modeling_llama.py:291-302)
    num_blocks = (int(seq_len) + int(block_size) - 1) // int(block_size)
    if num_blocks <= 0:
        return torch.empty(0, device=device, dtype=torch.float32)
    scores = torch.arange(num_blocks, device=device, dtype=torch.float32)
    if num_blocks > 1:
        scores = scores / float(num_blocks - 1)
    scores[0] = 1.0
    scores[-1] = 1.0
    return scores
