"""GPU bit-exactness of the HOT<->WARM conversion kernels.

Codes, scales and zero points must equal the reference's (tierkv_policy.py:21-44)
bit for bit; fp16 values are compared as raw bits.  The one exception is the
sign of a zero point whose row minimum is a zero and whose row holds zeros of
both signs: torch's reduction then returns whichever zero its reduction order
meets first (on the CPU, ``amin`` and ``min`` of the same row already disagree),
so those rows compare by value.  Rows whose zeros all carry one sign are
compared bit for bit against torch run by CUDA on the same GPU."""

import glob
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import tierkv_oracle as orc  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from paged_tierkv_b200 import _native
    _native.load(build_if_missing=True)


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16)


def _zero_bits(a):
    b = _bits(a).copy()
    b[b == 0x8000] = 0
    return b


@pytest.mark.parametrize("name", ["randn", "edge", "d64", "d16"])
def test_quantize_matches_reference_golden(name):
    from paged_tierkv_b200 import ops
    g = np.load(os.path.join(GOLDEN, "quant_r.npz"))
    x = torch.from_numpy(g[f"{name}_x"]).cuda()
    codes, scale, zero = ops.quantize_fp16_to_int8(x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), g[f"{name}_codes"])
    np.testing.assert_array_equal(_bits(scale.cpu().numpy()), _bits(g[f"{name}_scale"]))
    np.testing.assert_array_equal(_zero_bits(zero.cpu().numpy()), _zero_bits(g[f"{name}_zero"]))


@pytest.mark.parametrize("dim", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("sigma", [1e-3, 1.0, 300.0])
def test_quantize_random_rows_match_oracle(dim, sigma):
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(dim + int(sigma * 10))
    x = (rng.standard_normal((4099, dim)) * sigma + rng.standard_normal((4099, 1)) * sigma * 0.5)
    x = x.astype(np.float16)
    codes, scale, zero = ops.quantize_fp16_to_int8(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    rc, rs, rz = orc.quantize_rows_r(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(_bits(scale.cpu().numpy()), _bits(rs))
    np.testing.assert_array_equal(_zero_bits(zero.cpu().numpy()), _zero_bits(rz))


def test_quantize_matches_torch_cuda_reference_ops():
    """The reference quantizer's exact torch ops, evaluated by CUDA torch on this GPU."""
    from paged_tierkv_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((64, 8, 16, 128), generator=g, device="cuda", dtype=torch.float16)
    x[0, 0, 0] = 0.0
    x[1, 0, 0] = 2.5
    mn = x.amin(dim=-1, keepdim=True)
    mx = x.amax(dim=-1, keepdim=True)
    sc = (mx - mn) / 255.0
    sc = torch.where(sc == 0, torch.ones_like(sc), sc.to(torch.float16)).to(torch.float16)
    zp = (-torch.round(mn / sc)).to(torch.float16)
    q = torch.clamp(torch.round(x / sc) + zp, 0, 255).to(torch.uint8)
    codes, scale, zero = ops.quantize_fp16_to_int8(x)
    torch.cuda.synchronize()
    assert torch.equal(codes, q)
    assert torch.equal(scale.view(torch.int16), sc.view(torch.int16))
    assert torch.equal(zero.view(torch.int16), zp.view(torch.int16))


def _torch_quantize(x):
    mn = x.amin(dim=-1, keepdim=True)
    mx = x.amax(dim=-1, keepdim=True)
    sc = (mx - mn) / 255.0
    sc = torch.where(sc == 0, torch.ones_like(sc), sc.to(torch.float16)).to(torch.float16)
    zp = (-torch.round(mn / sc)).to(torch.float16)
    q = torch.clamp(torch.round(x / sc) + zp, 0, 255).to(torch.uint8)
    return q, sc, zp


@pytest.mark.parametrize("dim", [64, 128])
def test_zero_point_sign_of_zero_minima_matches_torch_cuda(dim):
    """Rows whose minimum is exactly zero: all +0, all -0, positives with +0
    minima, positives with -0 minima (zero point -0 resp. +0, bit for bit);
    rows mixing +0 and -0 minima match by value."""
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(dim)
    rows = []
    kinds = []
    for kind in ("pos", "neg", "pos_min", "neg_min", "mixed"):
        for _ in range(64):
            r = np.abs(rng.standard_normal(dim)).astype(np.float16) + np.float16(0.01)
            if kind == "pos":
                r[:] = np.float16(0.0)
            elif kind == "neg":
                r[:] = np.float16(-0.0)
            else:
                idx = rng.choice(dim, size=int(rng.integers(1, 6)), replace=False)
                if kind == "pos_min":
                    r[idx] = np.float16(0.0)
                elif kind == "neg_min":
                    r[idx] = np.float16(-0.0)
                else:
                    r[idx] = np.float16(0.0)
                    r[rng.choice(np.setdiff1d(np.arange(dim), idx), size=2, replace=False)] = \
                        np.float16(-0.0)
            rows.append(r)
            kinds.append(kind)
    x = torch.from_numpy(np.stack(rows)).cuda()
    q, sc, zp = _torch_quantize(x)
    codes, scale, zero = ops.quantize_fp16_to_int8(x)
    torch.cuda.synchronize()
    assert torch.equal(codes, q)
    assert torch.equal(scale.view(torch.int16), sc.view(torch.int16))
    single = torch.tensor([k != "mixed" for k in kinds], device="cuda")
    zb, tb = zero.view(torch.int16)[:, 0], zp.view(torch.int16)[:, 0]
    assert torch.equal(zb[single], tb[single])
    assert torch.equal(zero[~single], zp[~single])  # by value: +0 == -0
    # the oracle agrees on the single-sign rows, bit for bit
    rc, rs, rz = orc.quantize_rows_r(x.cpu().numpy())
    keep = single.cpu().numpy()
    np.testing.assert_array_equal(_bits(zero.cpu().numpy())[keep], _bits(rz)[keep])


DECODE_CASES = sorted(os.path.basename(p)[7:-4] for p in glob.glob(os.path.join(GOLDEN, "decode_*.npz")))


@pytest.mark.parametrize("case_name", DECODE_CASES)
def test_demotion_matches_reference_pools(case_name):
    """Replay the reference's demotions (compact: tail untouched; dense: tail cleared)."""
    from paged_tierkv_b200 import ops
    g = np.load(os.path.join(GOLDEN, f"decode_{case_name}.npz"))
    dem = g["demotions"]
    if dem.shape[0] == 0:
        pytest.skip("no WARM blocks")
    if g["hot_k_pool"].shape[-1] not in (64, 128):
        pytest.skip("demotion kernel is built for head_dim 64 and 128")
    c = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    # start from sentinel-filled WARM pools so untouched tail rows are visible
    wk = torch.full_like(c(g["warm_k_pool"]), 77)
    wv = torch.full_like(c(g["warm_v_pool"]), 78)
    ks = torch.full_like(c(g["k_scale"]), 3.0)
    kz = torch.full_like(c(g["k_zero"]), 5.0)
    vs = torch.full_like(c(g["v_scale"]), 3.0)
    vz = torch.full_like(c(g["v_zero"]), 5.0)
    pools = ops.TieredPools(c(g["hot_k_pool"]), c(g["hot_v_pool"]), wk, wv, ks, kz, vs, vz)
    clear = bool(g["clear_tail"])
    ops.demote_blocks_to_warm(pools, dem[:, 0], dem[:, 1], dem[:, 2], clear_tail=clear)
    torch.cuda.synchronize()
    bs = g["hot_k_pool"].shape[2]
    for _, dst, n in dem:
        rows = slice(0, bs) if clear else slice(0, int(n))
        np.testing.assert_array_equal(wk[dst, :, rows].cpu().numpy(), g["warm_k_pool"][dst, :, rows])
        np.testing.assert_array_equal(wv[dst, :, rows].cpu().numpy(), g["warm_v_pool"][dst, :, rows])
        for ours, ref in ((ks, "k_scale"), (kz, "k_zero"), (vs, "v_scale"), (vz, "v_zero")):
            np.testing.assert_array_equal(_zero_bits(ours[dst, :, rows].cpu().numpy()),
                                          _zero_bits(g[ref][dst, :, rows]))
        if not clear and int(n) < bs:
            assert (wk[dst, :, int(n):] == 77).all()  # compact pool leaves the tail alone
            assert (ks[dst, :, int(n):] == 3.0).all()


@pytest.mark.parametrize("head_dim", [64, 128])
def test_promotion_matches_dequantize(head_dim):
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(head_dim)
    slots, kvh, bs = 9, 4, 16
    src = rng.standard_normal((slots, kvh, bs, head_dim)).astype(np.float16)
    codes, sc, zp = orc.quantize_rows_r(src)
    deq = orc.dequantize_rows_r(codes, sc, zp)
    c = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    hot = torch.full((slots, kvh, bs, head_dim), 7.0, dtype=torch.float16, device="cuda")
    pools = ops.TieredPools(hot, hot.clone(), c(codes), c(codes), c(sc), c(zp), c(sc), c(zp))
    lengths = [16, 5, 0, 16]
    src_slots, dst_slots = [2, 4, 6, 8], [0, 1, 3, 5]
    ops.promote_blocks_to_hot(pools, src_slots, dst_slots, lengths)
    torch.cuda.synchronize()
    hk = pools.hot_k.cpu().numpy()
    for s, d, n in zip(src_slots, dst_slots, lengths):
        np.testing.assert_array_equal(_bits(hk[d, :, :n]), _bits(deq[s, :, :n]))
        assert (hk[d, :, n:] == 7.0).all()


def test_format_s_demotion_matches_oracle():
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(4)
    slots, kvh, bs, d = 6, 4, 16, 128
    hot = rng.standard_normal((slots, kvh, bs, d)).astype(np.float16)
    pools = ops.TieredPools.allocate(slots, slots, kvh, bs, d, "cuda", fmt=ops.FORMAT_S)
    pools.hot_k.copy_(torch.from_numpy(hot))
    pools.hot_v.copy_(torch.from_numpy(hot[::-1].copy()))
    src, dst, lens = [0, 1, 2], [5, 3, 4], [16, 9, 1]
    ops.demote_blocks_to_warm(pools, src, dst, lens)
    torch.cuda.synchronize()
    for s, t, n in zip(src, dst, lens):
        for h in range(kvh):
            rc, rs = orc.quantize_block_s(hot[s, h], n)
            np.testing.assert_array_equal(pools.warm_k[t, h].cpu().numpy(), rc)
            assert pools.k_scale[t, h].item() == rs


def test_merge_partials_matches_oracle():
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(8)
    parts, rows, d = 5, 37, 128
    po = rng.standard_normal((parts, rows, d)).astype(np.float32)
    pl = (rng.standard_normal((parts, rows)) * 3).astype(np.float32)
    pl[1, :5] = -np.inf
    pl[:, 7] = -np.inf
    ref_o, ref_l = orc.merge_partials(po, pl)
    out, lse = ops.merge_partials(torch.from_numpy(po).cuda(), torch.from_numpy(pl).cuda(),
                                  out_dtype=torch.float32, return_lse=True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), ref_o, atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_l, atol=1e-5, rtol=1e-6)
    # strided part axis: one packed buffer per part, as after an all-gather
    packed = np.concatenate([po.reshape(parts, -1), pl], axis=1)
    pk = torch.from_numpy(packed).cuda()
    o2 = ops.merge_partials(pk[:, :rows * d].view(parts, rows, d), pk[:, rows * d:],
                            out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(o2.cpu().numpy(), ref_o, atol=1e-5, rtol=1e-5)


def test_block_scores_match_oracle():
    from paged_tierkv_b200 import ops
    rng = np.random.default_rng(2)
    hq, t, nb = 32, 50, 43
    s = rng.random((hq, t)).astype(np.float32)
    lens = rng.integers(0, 17, size=t).astype(np.int32)
    ref = orc.block_scores_from_probability_sums(s, lens, nb)
    got = ops.block_scores(torch.from_numpy(s).cuda(), torch.from_numpy(lens).cuda(), nb)
    torch.cuda.synchronize()
    g = got.cpu().numpy()
    np.testing.assert_allclose(g[:nb], ref, rtol=1e-6, atol=1e-7)
    assert np.all(g[nb:] == 0)
