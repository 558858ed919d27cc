"""Generate golden fixtures by running the reference's own CPU code.

Usage (only where a checkout of xiaoMartintin/Paged_TierKV is available):

    python tests/golden/make_golden.py --reference <path-to-Paged_TierKV>

It imports the reference modules read-only (``tierkv_policy``,
``tierkv_triton``) and records, as ``.npz`` files next to this script:

* ``quant_r.npz``   -- ``quantize_fp16_to_int8`` / ``dequantize_int8_to_fp16``
  (tierkv_policy.py:21-44) on seeded N(0,1) tensors and crafted edge rows.
* ``decode_*.npz``  -- pools built with the reference's own pool classes
  (``TieredKVTensorPool`` dense layout, tierkv_policy.py:55-698, and
  ``CompactTieredKVTensorPool``, tierkv_policy.py:701-1365) through
  ``write_hot_tokens`` / ``demote_to_warm`` / ``demote_to_cold``, the
  resulting tables, and the output of ``_eager_reference_decode``
  (tierkv_triton.py:708-820).  Each file also lists the demotions that were
  performed (hot slot, warm slot, length); the reference never clears a freed
  HOT slot, so the HOT pool still holds each demoted block's fp16 source and
  the demotion kernel can be checked against the reference.
* ``c1_out.npz``    -- benchmark configuration 1 (B=4, 32 q / 8 kv heads,
  D=128, 2048 tokens, block 16; 32 HOT / 64 WARM / 32 COLD blocks per
  sequence) with inputs from ``tests/golden/c1_inputs.py`` and WARM blocks
  quantized by the reference quantizer; only the output and an input digest
  are stored.

The fixtures are small (about 1.3 MB in total) and committed; the GPU box
never needs the reference checkout.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(path: str):
    sys.path.insert(0, os.path.abspath(path))
    import torch  # noqa: F401
    import tierkv_policy as tp
    import tierkv_triton as tt
    return tp, tt


def make_quant(tp):
    import torch
    rng = np.random.default_rng(1234)
    x_randn = rng.standard_normal((1, 32, 16, 128)).astype(np.float16)
    rows = [
        np.zeros(128),
        np.full(128, 1.5),
        np.eye(1, 128, 37)[0] * 3.0,
        1.0 + np.linspace(0.0, 0.05, 128),
        -2.0 - np.linspace(0.0, 0.02, 128),
        np.linspace(-60000.0, 60000.0, 128),
        np.linspace(-3e-6, 5e-6, 128),
        100.0 + np.linspace(0.0, 0.0625, 128),
        rng.standard_normal(128) * 1e-3,
        rng.standard_normal(128) * 100.0,
        np.abs(rng.standard_normal(128)) + 0.5,
        -np.abs(rng.standard_normal(128)) - 7.0,
        np.round(rng.standard_normal(128) * 4.0) / 4.0,
    ]
    x_edge = np.stack(rows).astype(np.float16)
    x_d64 = rng.standard_normal((1, 4, 16, 64)).astype(np.float16)
    x_d16 = rng.standard_normal((1, 2, 9, 16)).astype(np.float16)
    out = {}
    for name, x in (("randn", x_randn), ("edge", x_edge), ("d64", x_d64), ("d16", x_d16)):
        q, s, z = tp.quantize_fp16_to_int8(torch.from_numpy(x))
        deq = tp.dequantize_int8_to_fp16(q, s, z)
        out[f"{name}_x"] = x
        out[f"{name}_codes"] = q.numpy()
        out[f"{name}_scale"] = s.numpy()
        out[f"{name}_zero"] = z.numpy()
        out[f"{name}_deq"] = deq.numpy()
    np.savez_compressed(os.path.join(HERE, "quant_r.npz"), **out)


def _pool_arrays(pool):
    names = ["hot_k_pool", "hot_v_pool", "warm_k_pool", "warm_v_pool",
             "k_scale", "k_zero", "v_scale", "v_zero"]
    return {n: getattr(pool, n).numpy().copy() for n in names}


def _run_case(tp, tt, name, *, layout, kv_heads, q_heads, head_dim, lengths, states, seed,
              block_size=16):
    """Build one pool through the reference's pool API and record everything."""
    import torch
    torch.manual_seed(seed)
    rng = np.random.default_rng(seed)
    nb = len(lengths)
    max_blocks = nb + 3
    if layout == "dense":
        pool = tp.TieredKVTensorPool(num_layers=1, block_size=block_size,
                                     max_seq_len=max_blocks * block_size,
                                     max_blocks_per_layer=max_blocks,
                                     pool_blocks=max_blocks + 2, pool_chunk_blocks=4)
    else:
        pool = tp.CompactTieredKVTensorPool(num_layers=1, block_size=block_size,
                                            max_seq_len=max_blocks * block_size,
                                            max_blocks_per_layer=max_blocks,
                                            pool_blocks=max_blocks + 2, pool_chunk_blocks=4,
                                            hot_chunk_slots=3, warm_chunk_slots=2)
    # physical ids deliberately differ from logical ids (LIFO allocation in the
    # reference BlockManager hands out 0, 1, 2, ... ; use a shuffled order).
    phys = [int(p) for p in rng.permutation(max_blocks + 2)[:nb]]
    for logical, (p, n) in enumerate(zip(phys, lengths)):
        k = torch.from_numpy(rng.standard_normal((1, kv_heads, n, head_dim)).astype(np.float16))
        v = torch.from_numpy(rng.standard_normal((1, kv_heads, n, head_dim)).astype(np.float16))
        pool.write_hot_tokens(p, 0, k, v)
        pool.set_block_entry(0, logical, p, tp.HOT_STATE)
    demotions = []
    for logical, (p, st) in enumerate(zip(phys, states)):
        if st == tp.WARM_STATE:
            src = pool.physical_slots[p] if layout == "compact" else p
            pool.demote_to_warm(p)
            dst = pool.physical_slots[p] if layout == "compact" else p
            demotions.append((src, dst, pool.get_block_length(p)))
        elif st == tp.COLD_STATE:
            pool.demote_to_cold(p)
        pool.set_block_state(0, logical, st)
    if layout == "compact":
        table, bstates = pool.get_layer_table(0)
        blens = pool.get_layer_lengths(0)
    else:
        table, bstates = pool.get_layer_table(0)
        blens = pool.get_layer_lengths(0)
    scaling = head_dim ** -0.5
    groups = q_heads // kv_heads
    query = torch.from_numpy(rng.standard_normal((1, q_heads, 1, head_dim)).astype(np.float16))
    out = tt._eager_reference_decode(query, table, bstates, blens,
                                     pool.hot_k_pool, pool.hot_v_pool,
                                     pool.warm_k_pool, pool.warm_v_pool,
                                     pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero,
                                     num_blocks=nb, num_key_value_groups=groups, scaling=scaling)
    rec = dict(_pool_arrays(pool))
    rec.update(
        block_table=table.numpy().copy(), block_states=bstates.numpy().copy(),
        block_lengths=blens.numpy().copy(), num_blocks=np.int32(nb),
        groups=np.int32(groups), scaling=np.float32(scaling),
        query=query.numpy()[0, :, 0, :].copy(), out=out.numpy()[0, 0].copy(),
        demotions=np.array(demotions, dtype=np.int32).reshape(-1, 3),
        clear_tail=np.int32(1 if layout == "dense" else 0),
    )
    np.savez_compressed(os.path.join(HERE, f"decode_{name}.npz"), **rec)


def make_decode(tp, tt):
    H, W, C = tp.HOT_STATE, tp.WARM_STATE, tp.COLD_STATE
    # geometry of tierkv_triton.py:823-1101 (kv 4, q 8, D 64, block 16)
    _run_case(tp, tt, "pres_mixed", layout="dense", kv_heads=4, q_heads=8, head_dim=64,
              lengths=[16] * 5, states=[H, W, C, H, W], seed=21)
    _run_case(tp, tt, "pres_split", layout="dense", kv_heads=4, q_heads=8, head_dim=64,
              lengths=[16] * 8, states=[H, W, H, H, W, H, H, W], seed=22)
    # geometry of main.py:452-634 (kv 2, q 4, D 16), 41 tokens -> [16, 16, 9]
    _run_case(tp, tt, "main_mixed", layout="dense", kv_heads=2, q_heads=4, head_dim=16,
              lengths=[16, 16, 9], states=[H, W, C], seed=23)
    # compact pool, partial blocks in the middle, Llama-3-8B head geometry
    _run_case(tp, tt, "compact_partial", layout="compact", kv_heads=8, q_heads=32, head_dim=128,
              lengths=[16, 5, 16, 9, 16, 3, 16], states=[H, W, C, W, W, H, H], seed=24)
    # dense pool with partial WARM blocks (tail rows cleared) and MHA (g = 1)
    _run_case(tp, tt, "dense_partial_mha", layout="dense", kv_heads=4, q_heads=4, head_dim=128,
              lengths=[16, 7, 16, 12, 1], states=[H, W, W, C, W], seed=25)
    # GQA group 8 at head_dim 64 (TinyLlama-like geometry), all WARM
    _run_case(tp, tt, "compact_g8_warm", layout="compact", kv_heads=4, q_heads=32, head_dim=64,
              lengths=[16, 16, 16, 11], states=[W, W, W, W], seed=26)


def make_c1(tp, tt):
    import torch
    sys.path.insert(0, HERE)
    from c1_inputs import c1_inputs, digest
    inp = c1_inputs(seed=0)
    hot_k, hot_v = inp["hot_k"], inp["hot_v"]
    # Quantize the WARM source blocks with the reference quantizer.
    wk = torch.from_numpy(inp["warm_src_k"])
    wv = torch.from_numpy(inp["warm_src_v"])
    qk, sk, zk = tp.quantize_fp16_to_int8(wk)
    qv, sv, zv = tp.quantize_fp16_to_int8(wv)
    groups = inp["q_heads"] // inp["kv_heads"]
    # _eager_reference_decode reads hot_k_pool[slot] before looking at the
    # block state (tierkv_triton.py:759), so the HOT pool must have at least
    # as many slots as the WARM pool; pad it with zero slots for this call.
    pad = max(0, qk.shape[0] - hot_k.shape[0])
    hot_k = np.concatenate([hot_k, np.zeros((pad,) + hot_k.shape[1:], np.float16)])
    hot_v = np.concatenate([hot_v, np.zeros((pad,) + hot_v.shape[1:], np.float16)])
    outs = []
    for s in range(inp["batch"]):
        q = torch.from_numpy(inp["query"][s][None, :, None, :])
        out = tt._eager_reference_decode(
            q, torch.from_numpy(inp["block_table"][s]), torch.from_numpy(inp["block_states"][s]),
            torch.from_numpy(inp["block_lengths"][s]),
            torch.from_numpy(hot_k), torch.from_numpy(hot_v), qk, qv, sk, zk, sv, zv,
            num_blocks=inp["num_blocks"], num_key_value_groups=groups, scaling=inp["scaling"])
        outs.append(out.numpy()[0, 0])
    np.savez_compressed(os.path.join(HERE, "c1_out.npz"), out=np.stack(outs),
                        input_digest=np.frombuffer(digest(inp).encode(), dtype=np.uint8),
                        warm_codes_digest=np.frombuffer(
                            hashlib.sha256(qk.numpy().tobytes() + qv.numpy().tobytes()
                                           + sk.numpy().tobytes() + zk.numpy().tobytes()
                                           + sv.numpy().tobytes() + zv.numpy().tobytes()
                                           ).hexdigest().encode(), dtype=np.uint8))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of xiaoMartintin/Paged_TierKV")
    args = ap.parse_args()
    tp, tt = _load_reference(args.reference)
    make_quant(tp)
    make_decode(tp, tt)
    make_c1(tp, tt)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
