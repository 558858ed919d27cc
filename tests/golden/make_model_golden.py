"""Decode calls of the reference's own model code, recorded for the drop-in.

Usage (only where a checkout of xiaoMartintin/Paged_TierKV is available; CPU):

    python tests/golden/make_model_golden.py --reference <path-to-Paged_TierKV>

Benchmark configuration 2's model -- a random-init TinyLlama-1.1B-shaped
decoder (22 layers, hidden 2048, 32 q / 4 kv heads, head_dim 64, SwiGLU 5632,
vocab 32000, RoPE theta 10000, fp16) -- runs on the CPU through the
reference's patched ``modeling_llama.py`` (loaded as
``transformers.models.llama.modeling_llama``, as main.py:139-165 does) with its
``TieredKVRuntime`` (tierkv_policy.py:1503-1912; compact pools, the
reference's C++ ``BlockManager`` built from csrc/block_manager.cpp into a
temporary directory), ``policy_mode="hot_warm_cold"``, policy interval 64,
the eager prefill with policy and a greedy decode (the loop of
tierkv_eval.py:287-300).  On the CPU the model takes its eager decode branch
(modeling_llama.py:469-501); at each recorded (decode step, layer) the script
captures what the GPU branch (modeling_llama.py:426-455) would hand
``tierkv_decode_attention`` at that moment:

* ``runtime.get_layer_table(layer)`` (tierkv_policy.py:1869-1872, which also
  creates the 1-slot placeholder pools of tierkv_policy.py:814-826 when a pool
  is still unallocated): the full ``[num_layers, max_blocks_per_layer]`` int32
  tables whose row the call receives, and ``num_blocks``;
* the runtime's pool tensors' shapes, and the contents of every HOT / WARM
  slot the layer's table references (the other slots are never read);
* the post-RoPE ``query_states`` [1, 32, 1, 64] and ``return_scores`` as the
  GPU branch computes it (``should_collect_decode_scores``);
* the model's own attention output for that call (eager: dequantized K/V,
  COLD tokens as zeros, fp16 matmuls, fp32 softmax; ``attn_output`` before
  the reshape of modeling_llama.py:503), and the output of the reference's
  fp32 oracle of the Triton kernel, ``tierkv_triton._eager_reference_decode``
  (tierkv_triton.py:708-820), on the same tensors.

Recorded calls: layers 0, 11 and 21 at decode steps 1, 63, 64 (the first
policy tick: the call sees the tiers from before the tick) and 65 / 70 (after
it), the first calls after a growth of a pool during decode (at most
``max_growth`` per run), and a second run with a 2-block prompt whose WARM
pool is still the 1-slot placeholder.
The prompts are block-aligned (a partial last prefill block trips a known
policy issue of the reference).  Prompt ids are seeded uniform-random tokens;
nothing here comes from a dataset.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "model_c2_calls.npz")

LAYERS = (0, 11, 21)
STEPS = (1, 63, 64, 65, 70)


def load_reference(path: str):
    sys.path.insert(0, path)
    import torch  # noqa: F401
    import tierkv_policy as tp
    import tierkv_triton as tt
    name = "transformers.models.llama.modeling_llama"
    spec = importlib.util.spec_from_file_location(name, os.path.join(path, "modeling_llama.py"))
    ml = importlib.util.module_from_spec(spec)
    sys.modules[name] = ml
    spec.loader.exec_module(ml)
    from torch.utils.cpp_extension import load
    build = tempfile.mkdtemp(prefix="tierkv_block_manager_")
    bm = load(name="tierkv_block_manager_ref",
              sources=[os.path.join(path, "csrc", "block_manager.cpp")],
              build_directory=build, verbose=False)
    return tp, tt, ml, bm


def build_model(ml, seed: int):
    import torch
    cfg = ml.LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                         num_hidden_layers=22, num_attention_heads=32, num_key_value_heads=4,
                         head_dim=64, max_position_embeddings=2048, rms_norm_eps=1e-5,
                         rope_theta=10000.0)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = ml.LlamaForCausalLM(cfg).to(torch.float16).eval()
    return model, cfg


class Recorder:
    """Hooks on the runtime and the modeling module that capture one decode
    call of a layer: the tables and pools when the eager branch reconstructs
    the layer (after the step's KV append), then the query and the output
    when the eager attention runs."""

    def __init__(self, tp, tt, ml, runtime, scenario: str, want, max_growth: int):
        self.tp, self.tt, self.ml, self.rt = tp, tt, ml, runtime
        self.scenario = scenario
        self.want = want
        self.max_growth = max_growth
        self.calls = []
        self.pending = None
        self.collect = {}
        self.last_caps = None
        self.growth_pending = False
        rt = runtime
        orig_rl = rt.reconstruct_layer
        orig_collect = rt.should_collect_decode_scores

        def collect_hook(seq_id, run_policy):
            v = orig_collect(seq_id, run_policy)
            self.collect[int(seq_id)] = (bool(v), bool(run_policy))
            return v

        def rl_hook(seq_id, allow_decode_reconstruct=False):
            if rt.current_query_length == 1:
                self._maybe_snapshot(int(seq_id))
            return orig_rl(seq_id, allow_decode_reconstruct=allow_decode_reconstruct)

        rt.reconstruct_layer = rl_hook
        rt.should_collect_decode_scores = collect_hook
        orig_attn = ml.eager_attention_forward

        def attn_hook(module, query, key, value, attention_mask, scaling, dropout=0.0, **kw):
            out, w = orig_attn(module, query, key, value, attention_mask, scaling, dropout, **kw)
            p = self.pending
            if p is not None and query.shape[-2] == 1 and module.layer_idx == p["layer"]:
                self._finish(p, query, out, module)
                self.pending = None
            return out, w

        ml.eager_attention_forward = attn_hook
        self._restore = (ml, orig_attn)

    def close(self):
        ml, orig = self._restore
        ml.eager_attention_forward = orig

    def _caps(self):
        pool = self.rt.kv_pool
        return (0 if pool.hot_k_pool is None else int(pool.hot_k_pool.shape[0]),
                0 if pool.warm_k_pool is None else int(pool.warm_k_pool.shape[0]))

    def _maybe_snapshot(self, layer: int):
        # the GPU branch fetches the layer's table on every decode call, which
        # creates the placeholder pools; do the same on every call
        self.rt.get_layer_table(layer)
        step = int(self.rt.decode_step)
        caps = self._caps()
        if self.last_caps is not None and caps != self.last_caps:
            self.growth_pending = True
        self.last_caps = caps
        reason = None
        if (step, layer) in self.want:
            reason = "step"
        elif self.growth_pending and self.max_growth > 0:
            reason = "after_growth"
            self.max_growth -= 1
        if reason is None:
            return
        self.growth_pending = False
        import torch
        rt, pool = self.rt, self.rt.kv_pool
        bt, bst, bln, nb = rt.get_layer_table(layer)  # creates placeholders like the GPU path
        nb = int(nb)
        st = bst[:nb].numpy()
        tb = bt[:nb].numpy()
        hot_ids = np.unique(tb[st == self.tp.HOT_STATE]).astype(np.int64)
        warm_ids = np.unique(tb[st == self.tp.WARM_STATE]).astype(np.int64)
        sel = lambda t, ids: t[torch.from_numpy(ids)].numpy().copy()  # noqa: E731
        collect, run_policy = self.collect.get(layer, (False, False))
        self.pending = dict(
            scenario=self.scenario, reason=reason, step=step, layer=layer, num_blocks=nb,
            return_scores=collect, policy_tick=run_policy,
            row_offset=int(bt.storage_offset()),
            hot_shape=list(pool.hot_k_pool.shape), warm_shape=list(pool.warm_k_pool.shape),
            meta_shape=list(pool.k_scale.shape),
            arrays=dict(
                table2d=pool.block_slot_indices.numpy().copy(),
                states2d=pool.block_states.numpy().copy(),
                lengths2d=pool.block_lengths.numpy().copy(),
                hot_ids=hot_ids, warm_ids=warm_ids,
                hot_k=sel(pool.hot_k_pool, hot_ids), hot_v=sel(pool.hot_v_pool, hot_ids),
                warm_k=sel(pool.warm_k_pool, warm_ids), warm_v=sel(pool.warm_v_pool, warm_ids),
                k_scale=sel(pool.k_scale, warm_ids), k_zero=sel(pool.k_zero, warm_ids),
                v_scale=sel(pool.v_scale, warm_ids), v_zero=sel(pool.v_zero, warm_ids)),
            tensors=(bt, bst, bln, pool.hot_k_pool, pool.hot_v_pool, pool.warm_k_pool,
                     pool.warm_v_pool, pool.k_scale, pool.k_zero, pool.v_scale, pool.v_zero))

    def _finish(self, p, query, out, module):
        import torch
        bt, bst, bln, hk, hv, wk, wv, ks, kz, vs, vz = p.pop("tensors")
        # the reference's oracle reads hot_k_pool[slot] before it looks at the
        # state (tierkv_triton.py:758-759), so WARM slot ids must also be valid
        # HOT indices: pad the HOT pools (zeros) for this call only
        need = max(int(hk.shape[0]), int(wk.shape[0]))
        if need > hk.shape[0]:
            pad = torch.zeros((need - hk.shape[0],) + tuple(hk.shape[1:]), dtype=hk.dtype)
            hk, hv = torch.cat([hk, pad]), torch.cat([hv, pad])
        ref = self.tt._eager_reference_decode(
            query, bt, bst, bln, hk, hv, wk, wv, ks, kz, vs, vz,
            num_blocks=p["num_blocks"], num_key_value_groups=module.num_key_value_groups,
            scaling=module.scaling)
        p["groups"] = int(module.num_key_value_groups)
        p["scaling"] = float(module.scaling)
        a = p["arrays"]
        a["query"] = query.numpy().copy()                 # [1, Hq, 1, D] fp16
        a["model_out"] = out.numpy().copy()               # [1, 1, Hq, D] fp16 (eager branch)
        a["ref_out"] = ref.numpy().copy()                 # [1, 1, Hq, D] (reference oracle)
        self.calls.append(p)


def run_scenario(tp, tt, ml, bm, model, cfg, *, name, prompt_len, decode_steps, hot_budget,
                 warm_budget, seed, want, max_growth):
    import torch
    max_seq = prompt_len + decode_steps + 16
    max_blocks = -(-max_seq // 16)
    cache = tp.initialize_global_tierkv(
        block_manager=bm.BlockManager(total_blocks=cfg.num_hidden_layers * max_blocks),
        num_layers=cfg.num_hidden_layers, block_size=16, hot_budget=hot_budget,
        max_seq_len=max_seq, attention_backend="eager", policy_interval=64,
        policy_mode="hot_warm_cold", warm_budget=warm_budget)
    rt = cache.runtime
    rt.demoted_state = tp.WARM_STATE
    rt.cold_block_policy = "zero"
    rt.tiered_layer_indices = set(range(cfg.num_hidden_layers))
    rec = Recorder(tp, tt, ml, rt, name, want, max_growth)
    gen = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=gen)
    mask = torch.ones((1, prompt_len + decode_steps), dtype=torch.long)
    try:
        with torch.no_grad():
            out = model(input_ids=ids, attention_mask=mask[:, :prompt_len], past_key_values=cache,
                        use_cache=True, logits_to_keep=1)
            rec.last_caps = rec._caps()
            for step in range(decode_steps):
                nxt = torch.argmax(out.logits[:, -1, :], dim=-1, keepdim=True)
                out = model(input_ids=nxt, attention_mask=mask[:, :prompt_len + step + 1],
                            past_key_values=cache, use_cache=True, logits_to_keep=1)
    finally:
        rec.close()
    tp.reset_global_tierkv()
    return rec.calls


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=OUT)
    args = ap.parse_args()
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    tp, tt, ml, bm = load_reference(os.path.abspath(args.reference))
    model, cfg = build_model(ml, seed=2)
    want = {(s, layer) for s in STEPS for layer in LAYERS}
    calls = run_scenario(tp, tt, ml, bm, model, cfg, name="prompt256", prompt_len=256,
                         decode_steps=70, hot_budget=4, warm_budget=8, seed=3, want=want,
                         max_growth=2)
    calls += run_scenario(tp, tt, ml, bm, model, cfg, name="prompt32", prompt_len=32,
                          decode_steps=2, hot_budget=4, warm_budget=8, seed=4,
                          want={(1, 0), (2, 21)}, max_growth=1)
    arrays, meta = {}, []
    for i, c in enumerate(calls):
        for k, v in c.pop("arrays").items():
            arrays[f"c{i}_{k}"] = v
        meta.append(c)
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(args.out, **arrays)
    for c in meta:
        print(c["scenario"], c["reason"], "step", c["step"], "layer", c["layer"], "nb",
              c["num_blocks"], "hot", c["hot_shape"][0], "warm", c["warm_shape"][0],
              "scores", c["return_scores"], "tick", c["policy_tick"])
    for i, c in enumerate(meta):
        a, b = arrays[f"c{i}_model_out"].astype(np.float32), arrays[f"c{i}_ref_out"].astype(np.float32)
        print(i, "max |model - ref_oracle|", float(np.abs(a - b).max()))
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
