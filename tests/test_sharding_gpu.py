"""Context-sharded decode on 2, 4 and 8 GPUs (each world size skipped with
fewer GPUs): each rank runs the sm_100a kernel on its block range; the packed
partials are all-gathered over NCCL and merged by the LSE-merge kernel, or
exchanged over CUDA IPC peer memory inside the decode launch; the result must
match the unsharded oracle on every rank."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import torch.distributed as dist
    from tierkv_cases import make_case, to_device
    from paged_tierkv_b200 import _native, sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        _native.load(build_if_missing=True)
        case = make_case(seed=41, batch=3, q_heads=32, kv_heads=8, head_dim=128, num_blocks=57,
                         max_blocks=57)
        start, end = sharding.block_range(57, rank, world)
        sl = slice(start, end)
        local = dict(case, block_table=np.ascontiguousarray(case["block_table"][:, sl]),
                     block_states=np.ascontiguousarray(case["block_states"][:, sl]),
                     block_lengths=np.ascontiguousarray(case["block_lengths"][:, sl]))
        d = to_device(local, device=f"cuda:{rank}")
        res = sharding.ContextShardedDecode()(d["query"], d["block_table"], d["block_states"],
                                              d["block_lengths"], d["pools"], end - start,
                                              case["groups"], case["scaling"], return_scores=True)
        torch.cuda.synchronize()
        q.put((rank, start, end, res.out.float().cpu().numpy(), res.score_sums.cpu().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_context_sharded_decode_nccl(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    from oracle import tierkv_oracle as orc
    from tierkv_cases import make_case
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    case = make_case(seed=41, batch=3, q_heads=32, kv_heads=8, head_dim=128, num_blocks=57,
                     max_blocks=57)
    ref, _, ref_scores = orc.decode_attention(
        case["query"], case["block_table"], case["block_states"], case["block_lengths"], 57,
        case["hot_k"], case["hot_v"], case["warm_k"], case["warm_v"], case["k_scale"],
        case["k_zero"], case["v_scale"], case["v_zero"], case["groups"], case["scaling"],
        dtype=np.float64)
    for rank, start, end, out, scores in results:
        np.testing.assert_allclose(out, ref, atol=2e-3, rtol=1e-2)
        np.testing.assert_allclose(scores, ref_scores[:, :, start:end], atol=1e-4, rtol=1e-3)


def _worker_p2p(rank, world, port, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import torch.distributed as dist
    from tierkv_cases import make_case, to_device
    from paged_tierkv_b200 import _native, ops, sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ex = None
    try:
        _native.load(build_if_missing=True)
        case = make_case(seed=43, batch=3, q_heads=32, kv_heads=8, head_dim=128, num_blocks=57,
                         max_blocks=57)
        start, end = sharding.block_range(57, rank, world)
        sl = slice(start, end)
        local = dict(case, block_table=np.ascontiguousarray(case["block_table"][:, sl]),
                     block_states=np.ascontiguousarray(case["block_states"][:, sl]),
                     block_lengths=np.ascontiguousarray(case["block_lengths"][:, sl]))
        d = to_device(local, device=f"cuda:{rank}")
        ex = sharding.PeerExchange(rows_cap=3 * 32, units_cap=3 * 8, head_dim=128,
                                   timeout_ns=2_000_000_000)
        dec = sharding.P2PContextDecode(ex)
        outs = []
        for _ in range(3):  # both inbox parities, back to back
            res = dec(d["query"], d["block_table"], d["block_states"], d["block_lengths"], d["pools"],
                      end - start, case["groups"], case["scaling"], return_scores=True)
            outs.append((res.out.float().cpu().numpy(), res.score_sums.cpu().numpy()))
        torch.cuda.synchronize()
        q.put((rank, start, end, outs, ops.read_device_errors()))
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_context_sharded_decode_peer_exchange(world):
    """One process per GPU: the exchange of partials over CUDA IPC peer memory
    inside the decode launch (no collective on the data path)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    from oracle import tierkv_oracle as orc  # noqa: F401
    from tierkv_cases import make_case, oracle_decode
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_p2p, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    case = make_case(seed=43, batch=3, q_heads=32, kv_heads=8, head_dim=128, num_blocks=57,
                     max_blocks=57)
    ref, _, ref_scores = oracle_decode(case)
    for rank, start, end, outs, err in sorted(results, key=lambda r: r[0]):
        assert err == 0
        for out, scores in outs:
            np.testing.assert_allclose(out, ref, atol=2e-3, rtol=1e-2)
            np.testing.assert_allclose(scores, ref_scores[:, :, start:end], atol=1e-4, rtol=1e-3)
