"""B200-native (sm_100a) tiered paged decode attention.

A from-scratch implementation of the decode hot path of Paged-TierKV
(HOT fp16 / WARM 8-bit / COLD evicted KV blocks) behind the reference's own
Python surface:

* ``paged_tierkv_b200.tierkv_triton.tierkv_decode_attention`` -- drop-in for
  the reference's ``tierkv_triton.tierkv_decode_attention``;
* ``paged_tierkv_b200.ops`` -- batched tensor API (decode, LSE merge, block
  scores, HOT<->WARM conversion);
* ``paged_tierkv_b200.sharding`` -- data-parallel batches and block-range
  sharded long contexts over several GPUs.

All computation goes through the C-ABI library ``lib/libtierkv_b200.so``
(include/tierkv_b200.h); there is no CPU or Triton fallback.
"""

from . import _native  # noqa: F401
from .ops import (  # noqa: F401
    COLD_STATE,
    FORMAT_R,
    FORMAT_S,
    HOT_STATE,
    WARM_STATE,
    TieredPools,
    block_scores,
    decode_attention,
    demote_blocks_to_warm,
    merge_partials,
    promote_blocks_to_hot,
    quantize_fp16_to_int8,
)

__all__ = [
    "COLD_STATE", "FORMAT_R", "FORMAT_S", "HOT_STATE", "WARM_STATE", "TieredPools",
    "block_scores", "decode_attention", "demote_blocks_to_warm", "merge_partials",
    "promote_blocks_to_hot", "quantize_fp16_to_int8",
]
