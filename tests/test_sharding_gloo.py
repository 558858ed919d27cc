"""World-size-2 gloo checks of the multi-GPU partitioning logic on CPU.

The local partial and the merge are the CPU oracle here (the CUDA kernels are
checked against the same oracle in the GPU tests); what runs for real is the
block-range partition, the packed all-gather and the score rescaling of
``paged_tierkv_b200.sharding``."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from paged_tierkv_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_dp_slices_cover_the_batch():
    for batch in (1, 7, 32, 33):
        for world in (1, 2, 3, 8):
            idx = []
            for r in range(world):
                idx += list(range(batch))[sharding.dp_slice(batch, r, world)]
            assert idx == list(range(batch))


def test_block_ranges_are_contiguous_and_complete():
    for nb in (0, 1, 5, 128, 8192):
        for world in (1, 2, 4, 8):
            rs = [sharding.block_range(nb, r, world) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == nb
            for (a, b), (c, _) in zip(rs, rs[1:]):
                assert b == c and a <= b


def _oracle_local(query, table, states, lengths, pools, num_blocks, groups, scaling, o_out, lse_out,
                  return_scores):
    from oracle import tierkv_oracle as orc
    out, lse, scores = orc.decode_attention(
        query.numpy(), table.numpy(), states.numpy(), lengths.numpy(), num_blocks,
        pools["hot_k"], pools["hot_v"], pools["warm_k"], pools["warm_v"], pools["k_scale"],
        pools["k_zero"], pools["v_scale"], pools["v_zero"], groups, scaling, dtype=np.float64)
    o_out.copy_(torch.from_numpy(out))
    lse_out.copy_(torch.from_numpy(lse))
    return torch.from_numpy(scores) if return_scores else None


def _oracle_merge(part_o, part_lse, out_dtype):
    from oracle import tierkv_oracle as orc
    o, lse = orc.merge_partials(part_o.numpy(), part_lse.numpy())
    return torch.from_numpy(o).to(torch.float32), torch.from_numpy(lse).to(torch.float32)


def _worker(rank, world, port, result_q, partition="count"):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from tierkv_cases import make_case
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_case(seed=31, batch=2, q_heads=8, kv_heads=2, head_dim=64, num_blocks=23,
                         max_blocks=23)
        nb = int(case["num_blocks"][0])
        if partition == "time":
            start, end = sharding.balanced_block_ranges(
                torch.from_numpy(case["block_states"]), world, case["hot_k"].shape[2],
                case["hot_k"].shape[3])[rank]
        else:
            start, end = sharding.block_range(nb, rank, world)
        sl = slice(start, end)
        pools = {k: case[k] for k in ("hot_k", "hot_v", "warm_k", "warm_v", "k_scale", "k_zero",
                                      "v_scale", "v_zero")}
        dec = sharding.ContextShardedDecode(local_fn=_oracle_local, merge_fn=_oracle_merge)
        res = dec(torch.from_numpy(case["query"]),
                  torch.from_numpy(np.ascontiguousarray(case["block_table"][:, sl])),
                  torch.from_numpy(np.ascontiguousarray(case["block_states"][:, sl])),
                  torch.from_numpy(np.ascontiguousarray(case["block_lengths"][:, sl])),
                  pools, end - start, case["groups"], case["scaling"], out_dtype=torch.float32,
                  return_scores=True)
        result_q.put((rank, start, end, res.out.numpy(), res.lse.numpy(), res.score_sums.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("partition", ["count", "time"])
@pytest.mark.parametrize("world", [2, 4])
def test_context_sharded_decode_over_ranks(world, partition):
    from oracle import tierkv_oracle as orc
    from tierkv_cases import make_case
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, partition))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    case = make_case(seed=31, batch=2, q_heads=8, kv_heads=2, head_dim=64, num_blocks=23,
                     max_blocks=23)
    ref, ref_lse, ref_scores = orc.decode_attention(
        case["query"], case["block_table"], case["block_states"], case["block_lengths"], 23,
        case["hot_k"], case["hot_v"], case["warm_k"], case["warm_v"], case["k_scale"],
        case["k_zero"], case["v_scale"], case["v_zero"], case["groups"], case["scaling"],
        dtype=np.float64)
    for rank, start, end, out, lse, scores in results:
        np.testing.assert_allclose(out, ref, atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(lse, ref_lse, atol=1e-5, rtol=1e-6)
        np.testing.assert_allclose(scores, ref_scores[:, :, start:end], atol=1e-6, rtol=1e-5)


def test_a_rank_that_fails_is_seen_by_the_others():
    """A rank raising before the exchange must not hang its peer: the peer's
    collective ends with an error once the group times out."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "raised"
    assert got[0].startswith("error")


def _failing_worker(rank, world, port, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            result_q.put((1, "raised"))
            raise SystemExit(0)  # leaves between steps, before the collective
        buf = torch.zeros(4)
        out = torch.zeros(8)
        try:
            dist.all_gather_into_tensor(out, buf)
            result_q.put((0, "no error"))
        except Exception as exc:  # gloo timeout / peer closed
            result_q.put((0, f"error: {type(exc).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
