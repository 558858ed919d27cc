"""bench.py's host-side pieces (no GPU): the reference arm builds its inputs on
the host, imports nothing of the package, and reports the same workload
``config`` as our arm, whose tier layout and byte count it reproduces."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from paged_tierkv_b200 import ops, workloads  # noqa: E402


@pytest.mark.parametrize("nb", [1, 2, 7, 128, 2048])
@pytest.mark.parametrize("hot,warm", [(1.0, None), (0.5, None), (0.25, None), (0.1, None),
                                      (0.2, 0.6), (0.1, 0.6)])
def test_host_tier_counts_match_workloads(nb, hot, warm):
    assert bench.host_tier_counts(nb, hot, warm) == workloads.tier_counts(nb, hot, warm)


@pytest.mark.parametrize("seed", [0, 1234, 99])
@pytest.mark.parametrize("nb,hot", [(2048, 0.25), (2048, 0.1), (128, 0.5), (3, 1.0)])
def test_host_states_match_workloads(seed, nb, hot):
    n_hot, n_warm, _ = workloads.tier_counts(nb, hot)
    ref = workloads.assign_tiers(2, nb, n_hot, n_warm, seed)[0].numpy()
    np.testing.assert_array_equal(bench.host_first_states(nb, n_hot, n_warm, seed), ref)


@pytest.mark.parametrize("bs", [16, 32])
def test_host_bytes_match_workload_accounting(bs):
    batch, nb = 3, 40
    n_hot, n_warm, n_cold = workloads.tier_counts(nb, 0.25)
    pools = ops.TieredPools.allocate(1, 1, 8, bs, 128, "cpu")
    wl = workloads.Workload(pools=pools, query=torch.zeros(batch, 32, 128, dtype=torch.float16),
                            block_table=None, block_states=None, block_lengths=None,
                            num_blocks=nb, groups=4, scaling=1.0, n_hot=n_hot, n_warm=n_warm,
                            n_cold=n_cold)
    assert bench.host_bytes_per_step(batch, nb, n_hot, n_warm, bs, 128, 8, 32) == \
        wl.algorithmic_bytes()


def test_reference_arm_runs_on_the_host_with_our_config():
    code = (
        "import runpy, sys\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--steps', '2', '--warmup', '1',"
        " '--batch', '4', '--ctx', '4096']\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        f"runpy.run_path({os.path.join(ROOT, 'bench.py')!r}, run_name='__main__')\n"
        "import torch\n"
        "print('IMPORTED', any(m.startswith('paged_tierkv_b200') for m in sys.modules),"
        " torch.cuda.is_initialized(), file=sys.stderr)\n")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert "IMPORTED False False" in res.stderr
    assert line["impl"] == "reference" and line["value"] > 0
    args = bench.argparse.Namespace(batch=4, ctx=4096, hot_frac=0.25, warm_frac=None,
                                    block_size=16)
    assert line["config"] == bench.bench_config(args, 1)
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_balanced_block_ranges_cover_the_context_with_equal_estimated_time(world):
    """Configuration 4's partition: contiguous ranges that cover every block
    once, each rank's estimated decode time within one block of the mean
    (WARM bytes weighted by the kernel's measured time per byte)."""
    nb, bs, d = 8192, 16, 128
    n_hot, n_warm, _ = workloads.tier_counts(nb, 0.10, 0.60)
    states = workloads.assign_tiers(1, nb, n_hot, n_warm, seed=5000)
    ranges = workloads.balanced_block_ranges(states, world, bs, d)
    assert len(ranges) == world and ranges[0][0] == 0 and ranges[-1][1] == nb
    assert all(ranges[k][1] == ranges[k + 1][0] for k in range(world - 1))
    st = states.reshape(-1)[:nb].tolist()

    def cost(s):
        if s == ops.HOT_STATE:
            return bs * 4 * d + 12
        if s == ops.WARM_STATE:
            return bs * (2 * d + 8) * workloads.WARM_TIME_PER_BYTE + 12
        return 12
    per = [sum(cost(s) for s in st[a:b]) for a, b in ranges]
    mean = sum(per) / world
    assert max(abs(c - mean) for c in per) <= cost(ops.HOT_STATE) + 1e-6
    if world > 1:  # the HOT window at the end: the last rank holds fewer blocks
        sizes = [b - a for a, b in ranges]
        assert sizes[-1] < sizes[0]
