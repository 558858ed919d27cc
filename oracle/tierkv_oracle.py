"""CPU oracle for the tiered paged decode-attention path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped path (``paged_tierkv_b200``)
never routes through it and fails loudly when its CUDA library is missing.

It restates, in numpy, the reference algorithms of xiaoMartintin/Paged_TierKV
(file:line references are into that project):

* ``quantize_rows_r``     -- tierkv_policy.py:21-36  (``quantize_fp16_to_int8``)
* ``dequantize_rows_r``   -- tierkv_policy.py:39-44  (``dequantize_int8_to_fp16``)
* ``decode_attention``    -- tierkv_triton.py:708-820 (``_eager_reference_decode``)
                             plus the score pass of tierkv_triton.py:121-145
* ``merge_partials``      -- tierkv_triton.py:231-264 (split-KV LSE reduce)
* ``block_scores_from_probability_sums`` -- tierkv_policy.py:1905-1912
* ``demote_blocks_r``     -- tierkv_policy.py:1042-1068 (compact pool, tail rows
                             left untouched) and 329-361 (dense pool, tail rows
                             cleared to code 0 / scale 1 / zero 0)

Format S (int8, symmetric absmax per (block, kv head)) has no reference
implementation; ``quantize_block_s`` restates the wording of the benchmark
configuration ("symmetric absmax scale per block per KV head", round half to
even as torch.round).  Its parity is unpinned by any reference test.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own CPU code
(quantizer, pools, ``_eager_reference_decode``) and stores its outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
them (bit-exact for codes/scales/zero points, fp32 round-off for attention).

Arithmetic conventions follow PyTorch's fp16 semantics: every fp16 tensor op
is evaluated in fp32 and rounded to nearest-even fp16 ("opmath"), and
``torch.round`` is round-half-to-even (``np.rint``).
"""

from __future__ import annotations

import numpy as np

HOT_STATE = 0
WARM_STATE = 1
COLD_STATE = 2

_F16 = np.float16
_F32 = np.float32


def _h(x) -> np.ndarray:
    """Round an fp32 array to fp16 (round to nearest even), like torch's opmath."""
    return np.asarray(x, dtype=_F32).astype(_F16)


# ---------------------------------------------------------------------------
# Format R quantizer (the reference's WARM layout)
# ---------------------------------------------------------------------------

def quantize_rows_r(x: np.ndarray):
    """Per-row asymmetric uint8 quantization over the last axis.

    Restates tierkv_policy.py:21-36 with per-op fp16 rounding:
      mn, mx  = amin/amax over the row (exact)
      scale   = h(h(mx - mn) / 255);  scale == 0 -> 1
      zp      = h(-rint(h(mn / scale)))
      code    = uint8(clamp(h(rint(h(x / scale)) + zp), 0, 255))
    NaN codes (only reachable for NaN/overflowing rows) convert to 0, which is
    what the reference's CUDA cast produces.
    Returns (codes uint8, scale fp16 [..., 1], zero_point fp16 [..., 1]).
    """
    x = np.asarray(x)
    if x.dtype != _F16:
        x = x.astype(_F16)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        mn = x.min(axis=-1, keepdims=True)
        mx = x.max(axis=-1, keepdims=True)
        diff = _h(mx.astype(_F32) - mn.astype(_F32))
        scale = _h(diff.astype(_F32) / _F32(255.0))
        scale = np.where(scale == 0, _F16(1.0), scale).astype(_F16)
        zp = _h(-np.rint(_h(mn.astype(_F32) / scale.astype(_F32)).astype(_F32)))
        t = _h(x.astype(_F32) / scale.astype(_F32))
        s = _h(np.rint(t.astype(_F32)) + zp.astype(_F32))
        c = np.where(np.isnan(s), np.nan, np.minimum(np.maximum(s, _F16(0)), _F16(255)))
        codes = np.where(np.isnan(c), 0, c).astype(_F32).astype(np.uint8)
    return codes, scale, zp


def dequantize_rows_r(codes: np.ndarray, scale: np.ndarray, zp: np.ndarray) -> np.ndarray:
    """tierkv_policy.py:39-44: h(h(h(code) - zp) * scale)."""
    q = np.asarray(codes).astype(_F16)
    t = _h(q.astype(_F32) - np.asarray(zp, _F16).astype(_F32))
    return _h(t.astype(_F32) * np.asarray(scale, _F16).astype(_F32))


# ---------------------------------------------------------------------------
# Format S quantizer (benchmark wording; no reference implementation)
# ---------------------------------------------------------------------------

def quantize_block_s(x: np.ndarray, length: int):
    """Symmetric int8 over one block of one KV head: x [block_size, D] fp16.

    s = absmax(rows < length) / 127 in fp32 (IEEE division); s == 0 -> 1;
    code = clamp(rint(x / s), -127, 127) for rows < length, 0 for tail rows.
    Returns (codes int8 [block_size, D], scale fp32 scalar).
    """
    x = np.asarray(x, dtype=_F16)
    n = int(max(0, min(int(length), x.shape[0])))
    codes = np.zeros(x.shape, dtype=np.int8)
    if n == 0:
        return codes, _F32(1.0)
    xv = x[:n].astype(_F32)
    amax = _F32(np.max(np.abs(xv)))
    s = _F32(amax / _F32(127.0))
    if s == 0:
        s = _F32(1.0)
    q = np.rint(xv / s)
    codes[:n] = np.clip(q, -127, 127).astype(np.int8)
    return codes, s


# ---------------------------------------------------------------------------
# Demotion into pools (compact / dense semantics)
# ---------------------------------------------------------------------------

def demote_blocks_r(hot_k, hot_v, warm_k, warm_v, k_scale, k_zero, v_scale, v_zero,
                    src_slots, dst_slots, lengths, clear_tail: bool) -> None:
    """In-place HOT->WARM demotion of whole blocks (all KV heads), Format R.

    compact pool (tierkv_policy.py:1042-1068): rows t >= length of the WARM
    slot keep whatever they held.  dense pool (tierkv_policy.py:329-361):
    those rows are cleared (code 0, scale 1, zero 0).  Meta arrays may be
    [slots, kv_heads, block_size] or [..., 1].
    """
    bs = hot_k.shape[2]
    for src, dst, n in zip(src_slots, dst_slots, lengths):
        n = int(n)
        for kind, (hp, wp, sp, zp_) in enumerate(((hot_k, warm_k, k_scale, k_zero),
                                                  (hot_v, warm_v, v_scale, v_zero))):
            rows = hp[int(src), :, :n, :]
            codes, sc, z = quantize_rows_r(rows)
            wp[int(dst), :, :n, :] = codes
            sp.reshape(sp.shape[0], sp.shape[1], bs)[int(dst), :, :n] = sc[..., 0]
            zp_.reshape(zp_.shape[0], zp_.shape[1], bs)[int(dst), :, :n] = z[..., 0]
            if clear_tail and n < bs:
                wp[int(dst), :, n:, :] = 0
                sp.reshape(sp.shape[0], sp.shape[1], bs)[int(dst), :, n:] = 1
                zp_.reshape(zp_.shape[0], zp_.shape[1], bs)[int(dst), :, n:] = 0


# ---------------------------------------------------------------------------
# Decode attention (the eager oracle path) and its score pass
# ---------------------------------------------------------------------------

def _gather_kv(slots, states, hot_k, hot_v, warm_k, warm_v, k_scale, k_zero,
               v_scale, v_zero, fmt: str, dtype):
    """Reconstruct K/V for a list of logical blocks: [nb, kv_heads, bs, D].

    HOT: pool values; WARM: dequantized in ``dtype`` (the reference oracle
    dequantizes in fp32: tierkv_triton.py:760-769); COLD (or any state other
    than HOT/WARM): zeros (tierkv_triton.py:770-777)."""
    nb = len(slots)
    _, hkv, bs, d = hot_k.shape
    k = np.zeros((nb, hkv, bs, d), dtype)
    v = np.zeros((nb, hkv, bs, d), dtype)
    hot = states == HOT_STATE
    warm = states == WARM_STATE
    if hot.any():
        hs = slots[hot]
        k[hot] = hot_k[hs].astype(dtype)
        v[hot] = hot_v[hs].astype(dtype)
    if warm.any():
        ws = slots[warm]
        if fmt == "R":
            def meta(a):
                return a.reshape(a.shape[0], a.shape[1], bs)[ws].astype(dtype)[..., None]
            k[warm] = (warm_k[ws].astype(dtype) - meta(k_zero)) * meta(k_scale)
            v[warm] = (warm_v[ws].astype(dtype) - meta(v_zero)) * meta(v_scale)
        elif fmt == "S":
            ks = np.asarray(k_scale).reshape(-1, hkv)[ws].astype(dtype)[:, :, None, None]
            vs = np.asarray(v_scale).reshape(-1, hkv)[ws].astype(dtype)[:, :, None, None]
            k[warm] = warm_k[ws].astype(dtype) * ks
            v[warm] = warm_v[ws].astype(dtype) * vs
        else:
            raise ValueError(f"unknown warm format {fmt!r}")
    return k, v


def decode_attention(query, block_table, block_states, block_lengths, num_blocks,
                     hot_k, hot_v, warm_k, warm_v, k_scale, k_zero, v_scale, v_zero,
                     num_key_value_groups: int, scaling: float, fmt: str = "R",
                     dtype=np.float32, max_blocks: int | None = None):
    """Tiered paged decode attention for a batch of sequences.

    query [B, Hq, D]; tables [B, T] int32 (T = max blocks per layer);
    num_blocks int or [B].  Semantics of tierkv_triton.py:708-820: tokens
    t >= block_lengths[b] are masked; COLD tokens that are valid keep logit 0
    and value 0; a row with no valid token yields output 0 (nan_to_num).
    Returns (out [B, Hq, D] dtype, lse [B, Hq] natural log, score_sums
    [B, Hq, T]) where score_sums[h, b] is the softmax mass of block b
    (tierkv_triton.py:121-145; zero for b >= num_blocks).
    """
    query = np.asarray(query)
    bsz, hq, d = query.shape
    table = np.asarray(block_table).reshape(bsz, -1)
    states_all = np.asarray(block_states).reshape(bsz, -1)
    lengths_all = np.asarray(block_lengths).reshape(bsz, -1)
    t_max = table.shape[1] if max_blocks is None else int(max_blocks)
    bs = hot_k.shape[2]
    g = int(num_key_value_groups)
    hkv = hq // g
    nbs = np.broadcast_to(np.asarray(num_blocks), (bsz,))
    out = np.zeros((bsz, hq, d), dtype)
    lse = np.full((bsz, hq), -np.inf, dtype)
    scores = np.zeros((bsz, hq, t_max), dtype)
    for s in range(bsz):
        nb = int(nbs[s])
        if nb <= 0:
            continue
        slots = table[s, :nb].astype(np.int64)
        states = states_all[s, :nb]
        lens = np.clip(lengths_all[s, :nb], 0, bs)
        k, v = _gather_kv(slots, states, hot_k, hot_v, warm_k, warm_v,
                          k_scale, k_zero, v_scale, v_zero, fmt, dtype)
        # [hkv, nb*bs, d]
        kf = k.transpose(1, 0, 2, 3).reshape(hkv, nb * bs, d)
        vf = v.transpose(1, 0, 2, 3).reshape(hkv, nb * bs, d)
        valid = (np.arange(bs)[None, :] < lens[:, None]).reshape(-1)
        q = query[s].astype(dtype).reshape(hkv, g, d)
        logits = np.matmul(q, kf.transpose(0, 2, 1)) * dtype(scaling)  # [hkv, g, T]
        logits = np.where(valid[None, None, :], logits, -np.inf)
        with np.errstate(invalid="ignore", divide="ignore"):
            m = logits.max(axis=-1, keepdims=True)
            e = np.exp(logits - m)
            ssum = e.sum(axis=-1, keepdims=True)
            p = np.nan_to_num(e / ssum, nan=0.0)
            lse_s = (m + np.log(ssum))[..., 0]
        out[s] = np.matmul(p, vf).reshape(hq, d)
        lse[s] = np.where(np.isfinite(lse_s), lse_s, -np.inf).reshape(hq)
        scores[s, :, :nb] = p.reshape(hq, nb, bs).sum(axis=-1)
    return out, lse, scores


def merge_partials(part_o, part_lse):
    """LSE merge of P partial results (tierkv_triton.py:231-264).

    part_o [P, R, D] (each partial normalised), part_lse [P, R] natural log;
    empty partials carry lse = -inf.  Returns (o [R, D], lse [R]); a row whose
    partials are all empty gives o = 0, lse = -inf."""
    part_o = np.asarray(part_o, np.float64)
    part_lse = np.asarray(part_lse, np.float64)
    with np.errstate(invalid="ignore", divide="ignore"):
        m = part_lse.max(axis=0)
        msafe = np.where(np.isfinite(m), m, 0.0)
        w = np.exp(part_lse - msafe[None, :])
        w = np.where(np.isfinite(part_lse), w, 0.0)
        wsum = w.sum(axis=0)
        o = np.einsum("pr,prd->rd", w, part_o)
        o = np.where(wsum[:, None] > 0, o / np.where(wsum > 0, wsum, 1.0)[:, None], 0.0)
        lse = np.where(wsum > 0, msafe + np.log(np.where(wsum > 0, wsum, 1.0)), -np.inf)
    return o, lse


def block_scores_from_probability_sums(score_sums, block_lengths, num_blocks: int):
    """tierkv_policy.py:1905-1912: mean over heads / clamp(length, 1)."""
    nb = int(num_blocks)
    if nb == 0:
        return np.zeros((0,), np.float32)
    s = np.asarray(score_sums, np.float32)[:, :nb].mean(axis=0)
    lens = np.maximum(np.asarray(block_lengths)[:nb], 1).astype(np.float32)
    return (s / lens).astype(np.float32)



# ---------------------------------------------------------------------------
# Prefill block scores (modeling_llama.py:281-289 with tierkv_policy.py:1378-1388)
# ---------------------------------------------------------------------------

def prefill_lse(query, key, scaling: float, causal: bool = True):
    """LSE (natural log) per query row of the scaled, causally masked logits.
    query [B, Hq, Tq, D], key [B, Hkv, Tk, D]; key j is visible to query i iff
    j <= i + (Tk - Tq).  Float64."""
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    b, hq, tq, _ = q.shape
    g = hq // k.shape[1]
    k = np.repeat(k, g, axis=1)                      # repeat_kv (modeling_llama.py:213-222)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scaling
    if causal:
        tk = k.shape[2]
        mask = np.arange(tk)[None, :] > (np.arange(tq)[:, None] + (tk - tq))
        s = np.where(mask[None, None], -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    return (m + np.log(np.exp(s - m).sum(axis=-1, keepdims=True)))[..., 0]


def prefill_block_scores(query, key, scaling: float, block_size: int, causal: bool = True):
    """The reference's prefill scores on the eager weights, in float64:
    weights = softmax(Q K^T * scaling + causal mask) (modeling_llama.py:225-245),
    mean over (batch, heads, queries) per key, then the mean of each
    block_size chunk of keys, the last one partial (tierkv_policy.py:1378-1388).
    (The reference rounds the weights and the means to fp16.)"""
    q = np.asarray(query, np.float64)
    k = np.asarray(key, np.float64)
    lse = prefill_lse(q, k, scaling, causal)
    g = q.shape[1] // k.shape[1]
    kk = np.repeat(k, g, axis=1)
    s = np.einsum("bhqd,bhkd->bhqk", q, kk) * scaling
    tq, tk = q.shape[2], k.shape[2]
    w = np.exp(s - lse[..., None])
    if causal:
        mask = np.arange(tk)[None, :] > (np.arange(tq)[:, None] + (tk - tq))
        w = np.where(mask[None, None], 0.0, w)
    token = w.mean(axis=(0, 1, 2))
    return np.array([token[i:i + block_size].mean() for i in range(0, tk, block_size)])
