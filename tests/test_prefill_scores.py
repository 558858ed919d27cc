"""Prefill block scores without attention weights.

The oracle (float64 eager restatement) is pinned to scores the reference
itself computed from its eager weights (tests/golden/make_prefill_golden.py);
the GPU passes are checked against both, at the fixture sizes and at larger
ones (tiles with ragged ends, GQA groups, a query block after a prefix)."""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import tierkv_oracle as orc  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "prefill_scores.npz")
CASES = ("g4_d64_t100", "g1_d64_t77", "g8_d128_t160_bs32")


def _case(name):
    f = np.load(GOLDEN)
    b, hq, hkv, t, d, bs = (int(x) for x in f[f"{name}_meta"])
    return f[f"{name}_q"], f[f"{name}_k"], float(f[f"{name}_scaling"][0]), bs, f[f"{name}_scores"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_scores(name):
    q, k, scaling, bs, ref = _case(name)
    got = orc.prefill_block_scores(q, k, scaling, bs)
    # the reference rounds the weights and their means to fp16
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=1e-6)


def test_proxy_path_is_the_reference_proxy():
    from paged_tierkv_b200 import prefill
    s = prefill.compute_prefill_block_scores(None, None, 70, 16, "cpu")
    assert s.tolist() == [1.0, 0.25, 0.5, 0.75, 1.0]


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_gpu_scores_match_reference_and_oracle(name):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import ops
    q, k, scaling, bs, ref = _case(name)
    qd, kd = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
    got = ops.prefill_block_scores(qd, kd, scaling, bs).cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=3e-3, atol=1e-6)
    np.testing.assert_allclose(got, orc.prefill_block_scores(q, k, scaling, bs), rtol=1e-3, atol=1e-7)
    lse = ops.prefill_lse(qd, kd, scaling).cpu().numpy()
    np.testing.assert_allclose(lse, orc.prefill_lse(q, k, scaling), atol=2e-3, rtol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("b,hq,hkv,tq,tk,d,bs,causal", [
    (1, 32, 8, 300, 300, 128, 16, True),    # ragged tiles, group 4
    (2, 8, 1, 129, 129, 64, 32, True),      # group 8
    (1, 16, 16, 70, 200, 128, 16, True),    # a query block after a 130-token prefix
    (1, 16, 2, 640, 640, 64, 16, True),     # 40 items per key tile: two column-pass parts
    (1, 8, 2, 700, 700, 128, 16, True),     # more key tiles than pipeline stages
    (2, 4, 2, 90, 333, 128, 32, False),     # bidirectional, ragged
])
def test_gpu_scores_at_larger_sizes(b, hq, hkv, tq, tk, d, bs, causal):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(b * 1000 + tq)
    q = rng.standard_normal((b, hq, tq, d)).astype(np.float16)
    k = rng.standard_normal((b, hkv, tk, d)).astype(np.float16)
    scaling = d ** -0.5
    qd, kd = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
    ops.read_prefill_errors()  # clear
    lse_gpu = ops.prefill_lse(qd, kd, scaling, causal=causal)
    lse_ref = orc.prefill_lse(q, k, scaling, causal=causal)
    np.testing.assert_allclose(lse_gpu.cpu().numpy(), lse_ref, rtol=1e-5, atol=2e-4)
    scores, mass = ops.prefill_block_scores(qd, kd, scaling, bs, causal=causal,
                                            return_token_mass=True)
    np.testing.assert_allclose(scores.cpu().numpy(),
                               orc.prefill_block_scores(q, k, scaling, bs, causal=causal),
                               rtol=1e-3, atol=1e-7)
    # every query row's mass sums to one
    np.testing.assert_allclose(mass.sum().item(), b * hq * tq, rtol=1e-4)
    # an LSE supplied by the caller (here the oracle's) gives the same scores
    lse = torch.from_numpy(lse_ref.astype(np.float32)).cuda()
    again = ops.prefill_block_scores(qd, kd, scaling, bs, lse=lse, causal=causal)
    np.testing.assert_allclose(again.cpu().numpy(), scores.cpu().numpy(), rtol=1e-4, atol=1e-8)
    assert ops.read_prefill_errors() == 0


@pytest.mark.gpu
def test_prefill_scores_reject_bad_inputs():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import ops
    q = torch.zeros((1, 4, 8, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        ops.prefill_block_scores(q.float(), q, 0.125, 16)
    with pytest.raises(ValueError):
        ops.prefill_block_scores(q, torch.zeros((1, 3, 8, 64), dtype=torch.float16, device="cuda"), 0.125, 16)
    with pytest.raises(ValueError):  # the scale must be positive
        ops.prefill_block_scores(q, q, -0.125, 16)
    with pytest.raises(ValueError):  # causal with fewer keys than queries
        ops.prefill_block_scores(q, torch.zeros((1, 4, 4, 64), dtype=torch.float16, device="cuda"), 0.125, 16)
