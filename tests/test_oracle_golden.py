"""The CPU oracle against golden vectors produced by the reference's own code.

Bit-exact for the Format R quantizer (codes, scales, zero points, dequantized
values); fp32 round-off for attention (the reference oracle is fp32 too).
"""

import glob
import os

import numpy as np
import pytest

from oracle import tierkv_oracle as orc
from c1_inputs import c1_inputs, digest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint16)


@pytest.mark.parametrize("name", ["randn", "edge", "d64", "d16"])
def test_quantizer_matches_reference(name):
    g = np.load(os.path.join(GOLDEN, "quant_r.npz"))
    codes, scale, zp = orc.quantize_rows_r(g[f"{name}_x"])
    np.testing.assert_array_equal(codes, g[f"{name}_codes"])
    np.testing.assert_array_equal(_bits(scale), _bits(g[f"{name}_scale"]))
    np.testing.assert_array_equal(_bits(zp), _bits(g[f"{name}_zero"]))
    deq = orc.dequantize_rows_r(codes, scale, zp)
    np.testing.assert_array_equal(_bits(deq), _bits(g[f"{name}_deq"]))


DECODE_CASES = sorted(os.path.basename(p)[7:-4] for p in glob.glob(os.path.join(GOLDEN, "decode_*.npz")))


@pytest.mark.parametrize("case", DECODE_CASES)
def test_decode_matches_reference(case):
    g = np.load(os.path.join(GOLDEN, f"decode_{case}.npz"))
    out, lse, scores = orc.decode_attention(
        g["query"][None], g["block_table"][None], g["block_states"][None], g["block_lengths"][None],
        int(g["num_blocks"]), g["hot_k_pool"], g["hot_v_pool"], g["warm_k_pool"], g["warm_v_pool"],
        g["k_scale"], g["k_zero"], g["v_scale"], g["v_zero"], int(g["groups"]), float(g["scaling"]),
        dtype=np.float32)
    ref = g["out"].astype(np.float32)
    # the reference casts its fp32 result to fp16; compare within one fp16 ulp
    np.testing.assert_allclose(out[0].astype(np.float16).astype(np.float32), ref, atol=1e-3, rtol=1e-3)
    nb = int(g["num_blocks"])
    np.testing.assert_allclose(scores[0, :, :nb].sum(-1), 1.0, atol=1e-5)
    assert np.all(scores[0, :, nb:] == 0)


@pytest.mark.parametrize("case", DECODE_CASES)
def test_demotion_matches_reference(case):
    """Re-run the recorded demotions with the oracle on the HOT pool contents."""
    g = np.load(os.path.join(GOLDEN, f"decode_{case}.npz"))
    dem = g["demotions"]
    if dem.shape[0] == 0:
        pytest.skip("no WARM blocks in this case")
    wk = np.zeros_like(g["warm_k_pool"])
    wv = np.zeros_like(g["warm_v_pool"])
    ks = np.ones_like(g["k_scale"]); kz = np.zeros_like(g["k_zero"])
    vs = np.ones_like(g["v_scale"]); vz = np.zeros_like(g["v_zero"])
    orc.demote_blocks_r(g["hot_k_pool"], g["hot_v_pool"], wk, wv, ks, kz, vs, vz,
                        dem[:, 0], dem[:, 1], dem[:, 2], clear_tail=bool(g["clear_tail"]))
    for d in dem[:, 1]:
        np.testing.assert_array_equal(wk[d], g["warm_k_pool"][d])
        np.testing.assert_array_equal(wv[d], g["warm_v_pool"][d])
        for ours, ref in ((ks, "k_scale"), (kz, "k_zero"), (vs, "v_scale"), (vz, "v_zero")):
            np.testing.assert_array_equal(_bits(ours[d]), _bits(g[ref][d]))


def test_c1_matches_reference():
    g = np.load(os.path.join(GOLDEN, "c1_out.npz"))
    inp = c1_inputs(seed=0)
    assert digest(inp).encode() == g["input_digest"].tobytes(), "c1 input generator drifted"
    qk, sk, zk = orc.quantize_rows_r(inp["warm_src_k"])
    qv, sv, zv = orc.quantize_rows_r(inp["warm_src_v"])
    out, _, _ = orc.decode_attention(
        inp["query"], inp["block_table"], inp["block_states"], inp["block_lengths"],
        inp["num_blocks"], inp["hot_k"], inp["hot_v"], qk, qv, sk, zk, sv, zv,
        inp["q_heads"] // inp["kv_heads"], inp["scaling"], dtype=np.float32)
    np.testing.assert_allclose(out.astype(np.float16).astype(np.float32), g["out"].astype(np.float32),
                               atol=1e-3, rtol=1e-3)
