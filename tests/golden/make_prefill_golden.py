"""Golden prefill block scores made by the reference itself.

Usage (only where a checkout of xiaoMartintin/Paged_TierKV is available):

    python tests/golden/make_prefill_golden.py --reference <path-to-Paged_TierKV>

For seeded fp16 query / key states it runs the reference's eager attention
(``eager_attention_forward``, modeling_llama.py:225-245, with a causal mask
built the way the model masks a prefill) and
``TierKVPolicyEngine.compute_block_scores`` (tierkv_policy.py:1378-1388) on
the resulting weights -- the exact scores the reference computes when the
attention weights exist -- and stores inputs and scores in
``prefill_scores.npz``.  CPU only.
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [  # (name, batch, q_heads, kv_heads, tokens, head_dim, block_size, seed)
    ("g4_d64_t100", 1, 8, 2, 100, 64, 16, 1),
    ("g1_d64_t77", 2, 4, 4, 77, 64, 16, 2),
    ("g8_d128_t160_bs32", 1, 8, 1, 160, 128, 32, 3),
]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args(argv)
    sys.path.insert(0, os.path.abspath(args.reference))
    import importlib.util
    import torch
    import transformers.models.llama  # noqa: F401  (the package its relative imports name)
    import tierkv_policy as tp  # noqa: E402  (the reference)
    # the reference's modeling_llama.py lives inside transformers' llama
    # package (relative imports): load the file under that package, read-only
    spec = importlib.util.spec_from_file_location(
        "transformers.models.llama.modeling_llama_tierkv_ref",
        os.path.join(os.path.abspath(args.reference), "modeling_llama.py"))
    ml = importlib.util.module_from_spec(spec)
    ml.__package__ = "transformers.models.llama"
    sys.modules[spec.name] = ml
    spec.loader.exec_module(ml)
    out = {}
    for name, b, hq, hkv, t, d, bs, seed in CASES:
        gen = torch.Generator().manual_seed(seed)
        q = torch.randn((b, hq, t, d), generator=gen).to(torch.float16)
        k = torch.randn((b, hkv, t, d), generator=gen).to(torch.float16)
        v = torch.randn((b, hkv, t, d), generator=gen).to(torch.float16)
        scaling = d ** -0.5
        mask = torch.full((t, t), torch.finfo(torch.float16).min, dtype=torch.float16).triu(1)
        module = types.SimpleNamespace(num_key_value_groups=hq // hkv, training=False)
        _, weights = ml.eager_attention_forward(module, q, k, v, mask[None, None], scaling)
        scores = tp.TierKVPolicyEngine(bs, None).compute_block_scores(weights)
        out[f"{name}_q"] = q.numpy()
        out[f"{name}_k"] = k.numpy()
        out[f"{name}_scores"] = scores.float().numpy()
        out[f"{name}_meta"] = np.array([b, hq, hkv, t, d, bs], np.int64)
        out[f"{name}_scaling"] = np.array([scaling], np.float64)
        print(name, scores.shape, scores.dtype)
    path = os.path.join(HERE, "prefill_scores.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
