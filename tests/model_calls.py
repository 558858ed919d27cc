"""Loader for ``tests/golden/model_c2_calls.npz``: decode calls recorded from
the reference's own model code and runtime (tests/golden/make_model_golden.py).

Each call carries the runtime's full ``[num_layers, max_blocks]`` tables (the
call receives row ``layer``), its pool shapes, the contents of the HOT / WARM
slots the layer references, the query, ``num_blocks``, ``return_scores`` and
two outputs: the model's own eager attention output and the reference's fp32
oracle (``_eager_reference_decode``) on the same tensors.
"""

from __future__ import annotations

import json
import os

import numpy as np

from oracle import tierkv_oracle as orc

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "model_c2_calls.npz")


def load():
    data = np.load(PATH)
    meta = json.loads(str(data["meta"]))
    calls = []
    for i, m in enumerate(meta):
        c = dict(m)
        prefix = f"c{i}_"
        for k in data.files:
            if k.startswith(prefix):
                c[k[len(prefix):]] = data[k]
        calls.append(c)
    return calls


def host_pools(c, fill_unused=0.0):
    """Full-size host pools of the call's shapes: referenced slots hold the
    recorded contents, the others ``fill_unused`` (fp16 pools and meta) or
    code 0xFF (WARM codes)."""
    hot = np.full(c["hot_shape"], fill_unused, np.float16)
    hk, hv = hot.copy(), hot.copy()
    hk[c["hot_ids"]] = c["hot_k"]
    hv[c["hot_ids"]] = c["hot_v"]
    wk = np.full(c["warm_shape"], 0xFF, np.uint8)
    wv = wk.copy()
    wk[c["warm_ids"]] = c["warm_k"]
    wv[c["warm_ids"]] = c["warm_v"]
    meta = np.full(c["meta_shape"], fill_unused, np.float16)
    ks, kz, vs, vz = meta.copy(), meta.copy(), meta.copy(), meta.copy()
    for arr, key in ((ks, "k_scale"), (kz, "k_zero"), (vs, "v_scale"), (vz, "v_zero")):
        arr[c["warm_ids"]] = c[key]
    return hk, hv, wk, wv, ks, kz, vs, vz


def oracle(c, dtype=np.float64):
    """The float64 oracle on the call's inputs: (out [Hq, D], lse [Hq],
    score_sums [Hq, max_blocks])."""
    hk, hv, wk, wv, ks, kz, vs, vz = host_pools(c)
    layer = c["layer"]
    row = lambda k: c[k][layer:layer + 1]  # noqa: E731
    q = c["query"][:, :, 0, :]
    o, lse, sc = orc.decode_attention(q, row("table2d"), row("states2d"), row("lengths2d"),
                                      np.array([c["num_blocks"]], np.int32), hk, hv, wk, wv,
                                      ks[..., 0], kz[..., 0], vs[..., 0], vz[..., 0], c["groups"],
                                      c["scaling"], dtype=dtype)
    return o[0], lse[0], sc[0]
