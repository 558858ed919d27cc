"""Decode attention at the benchmark's full sizes (GPU).

Configuration 5 (32 sequences x 32768 tokens, 32 q / 8 kv heads, head_dim 128;
block 16 at 25 % HOT / 50 % WARM / 25 % COLD with Format R for fp16 and bf16
queries and with Format S; the rest of its sweep -- hot fractions 1.0, 0.5,
0.1 at block 16 and all four at block 32, the non-HOT blocks split 2:1
WARM:COLD), configuration 3's attention shape (64 sequences x 8192 tokens,
20 % / 60 % / 20 %) and configuration 4 (one 131072-token context,
10 % / 60 % / 30 %), built as ``bench.py`` builds them,
decoded through the public API and checked three ways:

* against the float64 oracle on sampled sequences (the oracle finishes one
  full-context sequence in about a second): LSE within 1e-3 abs / 1e-4 rel and
  per-block score mass within 1e-4 abs / 1e-3 rel (the tolerances of the
  small-case parity tests); the output within 2e-3 abs / 1e-2 rel and, because
  a long context averages V down to a few thousandths, also within 1 % of the
  output's own scale (its largest magnitude);
* size-independent properties over every sequence: each query head's block
  score mass sums to 1, and the result does not depend on how the context is
  split over CTAs (1, 2, 8 splits and the planned count agree within 1 % of
  the output scale: the split merge is exact math, so only rounding differs);
* the kernel reports no device error.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import tierkv_oracle as orc  # noqa: E402
from paged_tierkv_b200 import ops  # noqa: E402

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
SCALE_FRAC = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)


def _host_sequence(wl, s):
    """Host copies of sequence s: its table row with slots renumbered into
    compact host pools holding only the slots it uses."""
    table = wl.block_table[s].cpu().numpy()
    states = wl.block_states[s].cpu().numpy()
    lengths = wl.block_lengths[s].cpu().numpy()
    remap = table.copy()
    picks = {}
    for state in (0, 1):
        ids = np.unique(table[states == state])
        picks[state] = torch.from_numpy(ids.astype(np.int64)).to(wl.query.device)
        lut = {int(x): i for i, x in enumerate(ids)}
        sel = np.nonzero(states == state)[0]
        remap[sel] = [lut[int(x)] for x in table[sel]]
    p = wl.pools
    g = lambda t, i: None if t is None else t.index_select(0, picks[i]).cpu().numpy()  # noqa: E731
    return dict(query=wl.query[s:s + 1].float().cpu().numpy(), table=remap[None], states=states[None],
                lengths=lengths[None], hot_k=g(p.hot_k, 0), hot_v=g(p.hot_v, 0),
                warm_k=g(p.warm_k, 1), warm_v=g(p.warm_v, 1), k_scale=g(p.k_scale, 1),
                k_zero=g(p.k_zero, 1), v_scale=g(p.v_scale, 1), v_zero=g(p.v_zero, 1))


def _oracle(wl, s):
    h = _host_sequence(wl, s)
    return orc.decode_attention(h["query"], h["table"], h["states"], h["lengths"], wl.num_blocks,
                                h["hot_k"], h["hot_v"], h["warm_k"], h["warm_v"], h["k_scale"],
                                h["k_zero"], h["v_scale"], h["v_zero"], wl.groups, wl.scaling,
                                fmt="R" if wl.pools.fmt == ops.FORMAT_R else "S",
                                dtype=np.float64)


def _decode(wl, **kw):
    from paged_tierkv_b200 import ops, workloads
    out, scores, lse = workloads.decode(wl, return_scores=True, return_lse=True, **kw)
    torch.cuda.synchronize()
    assert ops.read_device_errors() == 0
    return out, scores, lse


def _check(wl, sampled):
    out, scores, lse = _decode(wl)
    nb = wl.num_blocks
    mass = scores[:, :, :nb].double().sum(-1)
    torch.testing.assert_close(mass, torch.ones_like(mass), atol=1e-4, rtol=0)
    for s in sampled:
        ref_o, ref_lse, ref_sc = _oracle(wl, s)
        got = out[s].float().cpu().numpy()
        np.testing.assert_allclose(got, ref_o[0], atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(got, ref_o[0], atol=SCALE_FRAC * np.abs(ref_o[0]).max(), rtol=0)
        np.testing.assert_allclose(lse[s].cpu().numpy(), ref_lse[0], atol=1e-3, rtol=1e-4)
        np.testing.assert_allclose(scores[s, :, :nb].cpu().numpy(), ref_sc[0, :, :nb], atol=1e-4,
                                   rtol=1e-3)
    scale = float(out.float().abs().max())
    for splits in (1, 2, 8):
        other, _, _ = _decode(wl, num_splits=splits)
        torch.testing.assert_close(other.float(), out.float(), atol=SCALE_FRAC * scale, rtol=0)


@pytest.mark.parametrize("fmt,qdtype", [("R", torch.float16), ("S", torch.float16),
                                         ("R", torch.bfloat16)])
def test_configuration_5_full_size(fmt, qdtype):
    from paged_tierkv_b200 import workloads
    wl = workloads.make_workload(batch=32, q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                                 ctx_tokens=32768, hot_frac=0.25, seed=0, device="cuda",
                                 fmt=ops.FORMAT_R if fmt == "R" else ops.FORMAT_S)
    assert (wl.n_hot, wl.n_warm, wl.n_cold) == (512, 1024, 512)
    wl.query = wl.query.to(qdtype)
    _check(wl, sampled=(0, 31))


@pytest.mark.parametrize("block_size,hot_frac", [(16, 1.0), (16, 0.5), (16, 0.1), (32, 1.0),
                                                 (32, 0.5), (32, 0.25), (32, 0.1)])
def test_configuration_5_sweep_full_size(block_size, hot_frac):
    from paged_tierkv_b200 import workloads
    wl = workloads.make_workload(batch=32, q_heads=32, kv_heads=8, head_dim=128,
                                 block_size=block_size, ctx_tokens=32768, hot_frac=hot_frac,
                                 seed=int(hot_frac * 100) + block_size, device="cuda")
    nb = 32768 // block_size
    assert (wl.n_hot, wl.n_warm, wl.n_cold) == workloads.tier_counts(nb, hot_frac)
    _check(wl, sampled=(5,))


def test_configuration_3_attention_full_size():
    from paged_tierkv_b200 import workloads
    wl = workloads.make_workload(batch=64, q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                                 ctx_tokens=8192, hot_frac=0.2, warm_frac=0.6, seed=33,
                                 device="cuda")
    assert (wl.n_hot, wl.n_warm, wl.n_cold) == (102, 307, 103)
    _check(wl, sampled=(0, 63))


def test_configuration_4_full_context():
    from paged_tierkv_b200 import workloads
    wl = workloads.make_workload(batch=1, q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                                 ctx_tokens=131072, hot_frac=0.10, warm_frac=0.60, seed=5,
                                 device="cuda")
    assert wl.num_blocks == 8192
    _check(wl, sampled=(0,))
