"""Context-sharded decode with the peer-memory exchange, on one GPU.

No launch here waits for another launch: with one rank the kernel exchanges
with itself; the two-rank case has the other rank's partials written into the
inbox by the host beforehand as epoch-tagged words (what the peer's kernel
would have stored), so the launch finds them published; the timeout case
waits on words nothing writes and must come back with TKV_DEVERR_TIMEOUT.  The real
two-process exchange over CUDA IPC is in test_sharding_gpu.py.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tierkv_cases import make_case, oracle_decode, to_device  # noqa: E402

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)


def _inbox(world, rows, units, d):
    from paged_tierkv_b200 import _native as N
    n = N.load().tkv_exchange_bytes(world, rows, units, d)
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def _words(box, world, rows, d):
    """The inbox as its two regions of 64-bit words: o [2][rows][world][d] and
    lse [2][rows][world] (epoch parity); a word is epoch << 32 | fp32 bits."""
    o_bytes = 2 * rows * world * d * 8
    o = box[:o_bytes].view(torch.int64).view(2, rows, world, d)
    lse = box[o_bytes:o_bytes + 2 * rows * world * 8].view(torch.int64).view(2, rows, world)
    return o, lse


def _tag(values, epoch):
    bits = values.contiguous().float().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (int(epoch) << 32)


def _publish(box, world, rows, d, sender, epoch, o, lse):
    """What rank `sender`'s launch of call `epoch` stores into this inbox."""
    ow, lw = _words(box, world, rows, d)
    ow[epoch & 1, :, sender, :] = _tag(o.view(rows, d), epoch)
    lw[epoch & 1, :, sender] = _tag(lse.view(rows), epoch)


def _run(d, case, **kw):
    from paged_tierkv_b200 import ops
    return ops.decode_attention(d["query"], d["block_table"], d["block_states"], d["block_lengths"],
                                d["pools"], d["num_blocks"], case["groups"], case["scaling"], **kw)


@pytest.mark.parametrize("splits", [1, 5])
def test_one_rank_exchange_equals_plain_decode(splits):
    from paged_tierkv_b200 import sharding
    case = make_case(seed=60 + splits, batch=2, q_heads=32, kv_heads=8, head_dim=128, num_blocks=45)
    d = to_device(case)
    ref, ref_s, ref_l = _run(d, case, num_splits=splits, return_scores=True, return_lse=True)
    rows, units = 2 * 32, 2 * 8
    box = _inbox(1, rows, units, 128)
    ex = sharding.PeerExchange(rows_cap=rows, units_cap=units, head_dim=128,
                               inboxes=[box.data_ptr()], rank=0)
    for _ in range(3):  # epochs 1, 2, 3: both parities
        out, s, lse = _run(d, case, num_splits=splits, return_scores=True, return_lse=True,
                           exchange=ex.next())
        torch.cuda.synchronize()
        if splits == 1:  # one partial: the exchange merge is exact
            assert torch.equal(out, ref)
            assert torch.equal(lse, ref_l)
            assert torch.equal(s, ref_s)
        else:  # dynamic chunk claiming varies the partials from run to run
            torch.testing.assert_close(out.float(), ref.float(), atol=2e-4, rtol=2e-3)
            torch.testing.assert_close(lse, ref_l, atol=1e-5, rtol=1e-5)
            torch.testing.assert_close(s, ref_s, atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("world", [2, 8])
@pytest.mark.parametrize("splits", [1, 4])
def test_ranks_with_the_peers_already_published(splits, world):
    """Rank 0 of `world` ranks runs; the other ranks' partials of its calls are
    computed from their block ranges and written into rank 0's inbox by the
    host beforehand."""
    from paged_tierkv_b200 import ops, sharding
    nb = 70
    case = make_case(seed=80 + splits + world, batch=2, q_heads=32, kv_heads=8, head_dim=128,
                     num_blocks=nb, max_blocks=nb)
    ref, _, ref_scores = oracle_decode(case)
    cuts = [0, 33, nb] if world == 2 else [0, 9, 17, 26, 35, 44, 52, 61, nb]
    shards = []
    for r in range(world):
        sl = slice(cuts[r], cuts[r + 1])
        sh = dict(case, block_table=np.ascontiguousarray(case["block_table"][:, sl]),
                  block_states=np.ascontiguousarray(case["block_states"][:, sl]),
                  block_lengths=np.ascontiguousarray(case["block_lengths"][:, sl]))
        dd = to_device(sh)
        dd["num_blocks"] = cuts[r + 1] - cuts[r]
        shards.append((sh, dd))
    rows, units, D = 2 * 32, 2 * 8, 128
    boxes = [_inbox(world, rows, units, D) for _ in range(world)]
    ex = sharding.PeerExchange(rows_cap=rows, units_cap=units, head_dim=D,
                               inboxes=[b.data_ptr() for b in boxes], rank=0)
    for call in range(3):
        x = ex.next()
        par = x.epoch & 1
        # what ranks 1.. would have stored into rank 0's inbox
        for r in range(1, world):
            dr = shards[r][1]
            o_r = torch.empty((2, 32, D), dtype=torch.float32, device="cuda")
            _, _, l_r = ops.decode_attention(dr["query"], dr["block_table"], dr["block_states"],
                                             dr["block_lengths"], dr["pools"], dr["num_blocks"],
                                             case["groups"], case["scaling"], out=o_r,
                                             out_dtype=torch.float32, return_lse=True,
                                             num_splits=splits)
            _publish(boxes[0], world, rows, D, r, x.epoch, o_r, l_r)
        torch.cuda.synchronize()
        d0 = shards[0][1]
        out, scores, lse = _run(d0, shards[0][0], num_splits=splits, return_scores=True,
                                return_lse=True, exchange=x)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
        # rank 0's scores are normalised over the whole contexts
        np.testing.assert_allclose(scores.cpu().numpy(), ref_scores[:, :, :cuts[1]], atol=1e-4,
                                   rtol=1e-3)
        # rank 0 published its partial to every rank (itself included), every
        # word tagged with the epoch
        for r in range(world):
            ow, lw = _words(boxes[r], world, rows, D)
            assert ((ow[par, :, 0, :] >> 32) == x.epoch).all()
            assert ((lw[par, :, 0] >> 32) == x.epoch).all()
        assert ops.read_device_errors() == 0


def test_peer_that_never_publishes_times_out():
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops, sharding
    case = make_case(seed=90, batch=1, q_heads=8, kv_heads=2, head_dim=64, num_blocks=6)
    d = to_device(case)
    rows, units = 8, 2
    box0, box1 = _inbox(2, rows, units, 64), _inbox(2, rows, units, 64)
    ex = sharding.PeerExchange(rows_cap=rows, units_cap=units, head_dim=64,
                               inboxes=[box0.data_ptr(), box1.data_ptr()], rank=0,
                               timeout_ns=20_000_000)
    ops.read_device_errors()  # clear
    _run(d, case, exchange=ex.next())
    torch.cuda.synchronize()
    assert ops.read_device_errors() & N.TKV_DEVERR_TIMEOUT


def test_timeout_raises_from_the_sharding_api_and_resync_recovers():
    """A peer that never publishes: the call comes back (bounded wait), the
    next call raises TierKVDeviceError with the timeout bit before it
    launches, and after resync() the exchange works again with the peer's
    partials published for the new epoch."""
    from paged_tierkv_b200 import _native as N
    from paged_tierkv_b200 import ops, sharding
    nb, cut, D = 40, 17, 128
    case = make_case(seed=93, batch=1, q_heads=32, kv_heads=8, head_dim=D, num_blocks=nb,
                     max_blocks=nb)
    ref, _, _ = oracle_decode(case)
    shards = []
    for sl in (slice(0, cut), slice(cut, nb)):
        shards.append(dict(case, block_table=np.ascontiguousarray(case["block_table"][:, sl]),
                           block_states=np.ascontiguousarray(case["block_states"][:, sl]),
                           block_lengths=np.ascontiguousarray(case["block_lengths"][:, sl])))
    d0, d1 = to_device(shards[0]), to_device(shards[1])
    rows, units, world = 32, 8, 2
    box0, box1 = _inbox(world, rows, units, D), _inbox(world, rows, units, D)
    ex = sharding.PeerExchange(rows_cap=rows, units_cap=units, head_dim=D,
                               inboxes=[box0.data_ptr(), box1.data_ptr()], rank=0,
                               timeout_ns=20_000_000)
    dec = sharding.P2PContextDecode(ex)
    ops.read_device_errors()  # clear
    args = lambda dd: (dd["query"], dd["block_table"], dd["block_states"],  # noqa: E731
                       dd["block_lengths"], dd["pools"], cut, case["groups"], case["scaling"])
    dec(*args(d0))  # nothing publishes rank 1's partials: the wait runs out
    with pytest.raises(ops.TierKVDeviceError) as err:
        dec.check()
    assert err.value.bits & N.TKV_DEVERR_TIMEOUT and err.value.call == 1
    dec.check()  # reported once; the device word was cleared
    ex.resync()
    x_epoch = ex.epoch + 1  # the epoch the next call uses
    assert x_epoch >= 3
    o1 = torch.empty((1, 32, D), dtype=torch.float32, device="cuda")
    from paged_tierkv_b200 import ops as o
    _, _, l1 = o.decode_attention(d1["query"], d1["block_table"], d1["block_states"],
                                  d1["block_lengths"], d1["pools"], nb - cut, case["groups"],
                                  case["scaling"], out=o1, out_dtype=torch.float32, return_lse=True)
    _publish(box0, world, rows, D, 1, x_epoch, o1, l1)
    torch.cuda.synchronize()
    res = dec(*args(d0))
    dec.check()
    np.testing.assert_allclose(res.out.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_exchange_argument_checks():
    from paged_tierkv_b200 import sharding
    case = make_case(seed=91, batch=2, q_heads=8, kv_heads=2, head_dim=64, num_blocks=6)
    d = to_device(case)
    box = _inbox(1, 16, 4, 64)
    small = sharding.PeerExchange(rows_cap=8, units_cap=2, head_dim=64, inboxes=[box.data_ptr()], rank=0)
    with pytest.raises(ValueError):  # batch 2 x 8 heads > rows_cap 8
        _run(d, case, exchange=small.next())
    x = sharding.PeerExchange(rows_cap=16, units_cap=4, head_dim=64, inboxes=[box.data_ptr()],
                              rank=0).next()
    x.epoch = 0
    with pytest.raises(ValueError):
        _run(d, case, exchange=x)


def test_device_epoch_under_graph_replay():
    """The epoch in device memory advances in stream order, so replays of a
    captured call each use a new epoch (and alternate the inbox parity)."""
    from paged_tierkv_b200 import sharding
    case = make_case(seed=95, batch=1, q_heads=32, kv_heads=8, head_dim=128, num_blocks=40)
    d = to_device(case)
    ref, _, ref_l = _run(d, case, num_splits=1, return_lse=True)
    rows, units = 32, 8
    box = _inbox(1, rows, units, 128)
    ex = sharding.PeerExchange(rows_cap=rows, units_cap=units, head_dim=128,
                               inboxes=[box.data_ptr()], rank=0, device_epoch=True)
    dec = sharding.P2PContextDecode(ex)
    out = torch.empty_like(ref)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        dec(d["query"], d["block_table"], d["block_states"], d["block_lengths"], d["pools"],
            d["num_blocks"], case["groups"], case["scaling"], out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        dec(d["query"], d["block_table"], d["block_states"], d["block_lengths"], d["pools"],
            d["num_blocks"], case["groups"], case["scaling"], out=out)
    torch.cuda.synchronize()
    for i in range(4):
        with torch.cuda.stream(side):
            out.zero_()
            g.replay()
        torch.cuda.synchronize()
        # the planner may split the blocks: equal up to the merge's rounding
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-4, rtol=2e-3)
    # the warm-up call, the capture (not run) and four replays: epoch 1 + 1 + 4
    assert int(ex.epoch_t.item()) == 6
    # the last replay (epoch 5, odd parity) stamped every word it wrote
    ow, lw = _words(box, 1, rows, 128)
    assert ((ow[1] >> 32) == 5).all() and ((lw[1] >> 32) == 5).all()
    assert ((ow[0] >> 32) == 4).all()
