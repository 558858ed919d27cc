"""The drop-in's pool-set cache (paged_tierkv_b200/tierkv_triton.py): repeated
calls with the same contiguous pool tensors reuse one TieredPools; a set with
a non-contiguous tensor is copied on every call and never cached, so an
in-place update of the caller's pool is always seen.  Host logic only."""

import torch

from paged_tierkv_b200 import tierkv_triton as T


def _pool_set(slots=4, warm=3, hkv=2, bs=16, d=64, strided_hot=False):
    if strided_hot:
        hk = torch.zeros(slots, hkv, bs, 2 * d, dtype=torch.float16)[..., ::2]
    else:
        hk = torch.zeros(slots, hkv, bs, d, dtype=torch.float16)
    hv = torch.zeros(slots, hkv, bs, d, dtype=torch.float16)
    wk = torch.zeros(warm, hkv, bs, d, dtype=torch.uint8)
    wv = torch.zeros(warm, hkv, bs, d, dtype=torch.uint8)
    meta = [torch.ones(warm, hkv, bs, dtype=torch.float16) for _ in range(4)]
    return (hk, hv, wk, wv, *meta)


def test_contiguous_set_is_reused():
    T._POOLS_CACHE.clear()
    ts = _pool_set()
    a = T._pools_of(ts)
    b = T._pools_of(ts)
    assert a is b
    assert a.hot_k is ts[0] and a.v_zero is ts[7]


def test_non_contiguous_set_is_copied_every_call():
    T._POOLS_CACHE.clear()
    ts = _pool_set(strided_hot=True)
    assert not ts[0].is_contiguous()
    a = T._pools_of(ts)
    assert T._POOLS_CACHE == []
    ts[0].fill_(3.0)  # the caller updates its strided pool in place
    b = T._pools_of(ts)
    assert a is not b
    assert bool((b.hot_k == 3.0).all())


def test_cache_holds_two_sets():
    T._POOLS_CACHE.clear()
    s1, s2, s3 = _pool_set(), _pool_set(), _pool_set()
    p1 = T._pools_of(s1)
    p2 = T._pools_of(s2)
    assert T._pools_of(s1) is p1 and T._pools_of(s2) is p2
    T._pools_of(s3)
    assert len(T._POOLS_CACHE) == 2
    assert T._pools_of(s1) is not p1  # the oldest set was dropped
