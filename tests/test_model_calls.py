"""The drop-in under the reference's own model code and runtime (configuration 2).

``tests/golden/model_c2_calls.npz`` holds decode calls recorded from the
reference's TinyLlama-shaped model (22 layers, 32 q / 4 kv heads, head_dim
64) running under its ``TieredKVRuntime`` (hot_warm_cold policy, interval
64): what modeling_llama.py:426-455 hands ``tierkv_decode_attention`` --
row ``layer`` of the runtime's [num_layers, max_blocks] tables
(get_layer_table, tierkv_policy.py:1869-1872), the runtime's whole pool
tensors (grown between calls; the 1-slot WARM placeholder of
tierkv_policy.py:814-826 before any WARM block exists), the query,
``num_blocks`` and ``return_scores`` (True on the policy tick) -- with the
model's own attention output and the reference oracle's.

CPU: the float64 oracle reproduces the reference's recorded outputs.
GPU: every recorded call goes through the shim (``sys.modules["tierkv_triton"]``
stand-in) with pools of the runtime's shapes whose unreferenced slots hold NaN
(so a read of a wrong slot shows), in recording order with the pools updated
in place and replaced on growth, as the runtime does.  Tolerances:

* against the float64 oracle and the reference's fp32 oracle
  (``_eager_reference_decode``, stored rounded to fp16): 2e-3 abs / 1e-2 rel,
  the north star's bound;
* against the model's own eager branch output: 3e-3 abs / 1e-2 rel -- that
  branch multiplies fp16-rounded attention weights with fp16 values, which
  the recorder measured at up to 9.8e-4 from the fp32 oracle on these calls;
* score sums (tick calls): 1e-4 abs / 1e-3 rel of the oracle's, and the block
  scores the runtime derives from them (block_scores_from_probability_sums,
  tierkv_policy.py:1905-1912) through ``ops.block_scores``.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import model_calls  # noqa: E402
from oracle import tierkv_oracle as orc  # noqa: E402

CALLS = model_calls.load()
ATOL, RTOL = 2e-3, 1e-2


def test_fixture_covers_the_runtime_cases():
    reasons = {c["reason"] for c in CALLS}
    assert {"step", "after_growth"} <= reasons
    assert any(c["return_scores"] and c["policy_tick"] for c in CALLS)
    assert any(c["warm_shape"][0] == 1 for c in CALLS)      # WARM placeholder
    assert any(c["hot_shape"] != CALLS[0]["hot_shape"] for c in CALLS)  # grown pools
    ticks = [c for c in CALLS if c["policy_tick"]]
    after = [c for c in CALLS if c["scenario"] == "prompt256" and c["step"] > 64]
    cold = lambda c: int((c["states2d"][c["layer"], :c["num_blocks"]] == 2).sum())  # noqa: E731
    assert max(cold(c) for c in after) > max(cold(c) for c in ticks)  # the tick evicted blocks


@pytest.mark.parametrize("i", range(len(CALLS)))
def test_oracle_reproduces_the_reference_outputs(i):
    c = CALLS[i]
    out, _, scores = model_calls.oracle(c)
    ref = c["ref_out"][0, 0].astype(np.float64)
    np.testing.assert_allclose(out, ref, atol=1e-3, rtol=1e-3)   # ref is fp16-rounded
    np.testing.assert_allclose(out, c["model_out"][0, 0].astype(np.float64), atol=3e-3, rtol=RTOL)
    nb = c["num_blocks"]
    np.testing.assert_allclose(scores[:, :nb].sum(-1), 1.0, atol=1e-9)


def _device_pools(c, dev):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            for a in model_calls.host_pools(c, fill_unused=np.nan)]


@pytest.mark.gpu
def test_recorded_model_calls_through_the_shim():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import _native, ops
    from paged_tierkv_b200 import tierkv_triton as shim
    _native.load(build_if_missing=True)
    dev = "cuda"
    pools = None
    shim.check_device_errors()
    ops.read_device_errors()
    for i, c in enumerate(CALLS):
        host = model_calls.host_pools(c, fill_unused=np.nan)
        if pools is None or any(tuple(p.shape) != h.shape for p, h in zip(pools, host)):
            pools = [torch.from_numpy(np.ascontiguousarray(h)).to(dev) for h in host]  # growth
        else:
            for p, h in zip(pools, host):  # the runtime writes its pools in place
                p.copy_(torch.from_numpy(np.ascontiguousarray(h)))
        tables = [torch.from_numpy(c[k]).to(dev) for k in ("table2d", "states2d", "lengths2d")]
        layer = c["layer"]
        q = torch.from_numpy(c["query"]).to(dev)
        out, scores = shim.tierkv_decode_attention(
            q, tables[0][layer], tables[1][layer], tables[2][layer], *pools,
            num_blocks=c["num_blocks"], num_key_value_groups=c["groups"], scaling=c["scaling"],
            return_scores=c["return_scores"])
        torch.cuda.synchronize()
        hq, d = q.shape[1], q.shape[3]
        assert tuple(out.shape) == (1, 1, hq, d) and out.dtype == q.dtype and out.is_contiguous()
        assert out.reshape(1, 1, -1).shape == (1, 1, hq * d)  # modeling_llama.py:503
        got = out[0, 0].float().cpu().numpy()
        ref_o, _, ref_s = model_calls.oracle(c)
        msg = f"call {i}: {c['scenario']} step {c['step']} layer {layer}"
        np.testing.assert_allclose(got, ref_o, atol=ATOL, rtol=RTOL, err_msg=msg)
        np.testing.assert_allclose(got, c["ref_out"][0, 0].astype(np.float32), atol=ATOL, rtol=RTOL,
                                   err_msg=msg)
        np.testing.assert_allclose(got, c["model_out"][0, 0].astype(np.float32), atol=3e-3,
                                   rtol=RTOL, err_msg=msg)
        if c["return_scores"]:
            maxb = c["table2d"].shape[1]
            assert tuple(scores.shape) == (hq, maxb)
            s = scores.cpu().numpy()
            np.testing.assert_allclose(s, ref_s, atol=1e-4, rtol=1e-3, err_msg=msg)
            nb = c["num_blocks"]
            lengths = tables[2][layer]
            got_b = ops.block_scores(scores, lengths, nb)
            ref_b = orc.block_scores_from_probability_sums(s, c["lengths2d"][layer], nb)
            np.testing.assert_allclose(got_b.cpu().numpy()[:nb], ref_b, atol=1e-7, rtol=1e-5,
                                       err_msg=msg)
        else:
            assert scores is None
    shim.check_device_errors()
    assert ops.read_device_errors() == 0
