// tkv_prefill.cu -- prefill block scores without materialising attention weights.
//
// The reference scores a prefilled layer's blocks from the eager attention
// weights: softmax(Q K^T * scaling + causal mask) over keys, averaged over
// (batch, heads, queries) per key, then per block of block_size keys
// (TierKVPolicyEngine.compute_block_scores, tierkv_policy.py:1378-1388, called
// from modeling_llama.py:281-289); with SDPA / flash prefill it falls back to
// a sink + recency proxy (modeling_llama.py:291-302) because the weights never
// exist.  Here the exact scores come from two tensor-core passes over Q K^T:
//   LSE pass        per query row: LSE of the scaled, causally masked logits
//                   (skipped when the caller's flash attention returns it);
//   column pass     per key: sum over the group's query heads and every query
//                   row of exp(s * scaling - LSE_q) -- the attention mass each
//                   key receives -- accumulated per key;
//   block_mean_kernel  token mass / (batch * heads * queries), then the mean
//                   over each block's keys.
//
// Both passes are one warp-specialised tcgen05 kernel.  A CTA keeps 128 rows
// resident in shared memory as the MMA's A operand (M = 128): query rows for
// the LSE pass, key rows for the column pass.  Warp 8 streams 128-row tiles of
// the other operand (key tiles, or the (head, query tile) pairs that can see
// the keys) through a ring of shared-memory stages by TMA; one thread of warp 9
// issues tcgen05.mma (fp16 in, fp32 accumulate, N = 128) into one of two
// 128-column TMEM accumulators; warps 0-7 read the accumulator with tcgen05.ld,
// one thread per TMEM lane (resident row) and column half, so the softmax
// statistics need no cross-thread reduction until the two halves of a row
// merge at the end.  Exponentials run in the log2 domain on the MUFU unit
// (a share of the LSE pass's on the FMA pipe), which bounds the kernel: one
// exp per logit, while the MMA of a tile takes half the time its 128 x 128
// exps do.
//
// Every mbarrier wait is bounded (TKV_DEVERR_TIMEOUT in the prefill error
// word); in-flight copies and MMAs are waited for before the CTA frees its
// TMEM and exits.
#include <cuda_fp16.h>
#include <math.h>

#include "tierkv_b200.h"
#include "tkv_internal.h"
#include "tkv_ptx.cuh"

namespace tkv {

// Error bits (TKV_DEVERR_*) of the prefill kernels of this device.
__device__ uint32_t g_tkv_prefill_err;

constexpr float kLog2eP = 1.4426950408889634f;
constexpr int kTileRows = 128;       // M of every MMA and the rows (N) of every streamed tile
// The epilogue is WG warpgroups: warp w < 4 WG reads TMEM lanes 32 (w % 4) ..
// (its lane quarter) in the accumulator columns [128 / WG * (w / 4), + 128 /
// WG) of its warpgroup; warp 4 WG is the TMA producer, warp 4 WG + 1 the MMA
// issuer, warp 4 WG + 2 (column pass) stages the query LSEs of each item.
// Warpgroups per pass are a build-time choice; two measured best on B200 for
// both passes (four repeat the per-item overhead in more warps).
#ifndef TKV_PF_WG_LSE
#define TKV_PF_WG_LSE 2
#endif
#ifndef TKV_PF_WG_COLS
#define TKV_PF_WG_COLS 2
#endif
template <int WG>
struct PfWarps {
  static_assert(WG == 1 || WG == 2 || WG == 4, "warpgroups");
  static constexpr int kEpiThreads = 128 * WG;
  static constexpr int kProdWarp = 4 * WG;
  static constexpr int kMmaWarp = 4 * WG + 1;
  static constexpr int kLseWarp = 4 * WG + 2;
  static constexpr int kThreads = kEpiThreads + 96;
  static constexpr int kCols = kTileRows / WG;   // accumulator columns per warpgroup
  static constexpr int kChunks = kCols / 32;     // 32-column TMEM loads per item
};
constexpr uint32_t kTmemCols = 256;  // two fp32 accumulators of 128 columns
constexpr uint32_t kIdesc = umma_idesc_f16_f32(128, 128);

template <int D, int WG>
struct PfLayout {
  static constexpr int kTile = kTileRows * D * 2;  // [D/64][128 rows][64] fp16, 128B-swizzled
  static constexpr int kStages = D == 128 ? 2 : 4;
  static constexpr int kBarOff = kTile * (1 + kStages);
  // full[S], empty[S], resident, tfull[2], tempty[2], done, lfull[4], lempty[4]
  static constexpr int kNumBars = 2 * kStages + 14;
  static constexpr int kLseOff = kBarOff + kNumBars * 8;
  // column pass: a ring of 4 items' 128 query LSEs (2 KB); LSE pass: the
  // other warpgroups' (max, sum) per row, [WG - 1][128][2] (<= 3 KB)
  static constexpr int kTaddrOff = kLseOff + 4096;
  static constexpr int kBytes = kTaddrOff + 16 + 1024;  // + slack to align the base to 1024
};

// The CTA's share of a pass: the resident tile (map row, map head) and n
// streamed tiles.
struct PfWork {
  int n;          // streamed tiles
  int res_row, res_head;
  int b, kvh;
  int q0;         // LSE pass: first query row of the resident tile
  int k0;         // column pass: first key of the resident tile
  int qt_first, per_head, i0;  // column pass: item i -> (head hh, query tile)
};

// LSE pass: CTA = (batch, head, 128-query tile); item i = key tile i.  The
// grid runs the query tiles that see the most keys first.
__device__ __forceinline__ PfWork lse_work(const PrefillParams& p) {
  PfWork w{};
  const int nqt = (p.tq + kTileRows - 1) / kTileRows;
  const int bh_count = p.batch * p.num_heads;
  const int idx = blockIdx.x;
  const int qt = p.causal ? nqt - 1 - idx / bh_count : idx / bh_count;
  const int bh = idx % bh_count;
  w.b = bh / p.num_heads;
  w.kvh = (bh % p.num_heads) / p.groups;
  w.q0 = qt * kTileRows;
  w.res_row = w.q0;
  w.res_head = bh;
  const int last_key = p.causal ? min(p.tk, w.q0 + kTileRows + p.q_offset) : p.tk;
  w.n = (last_key + kTileRows - 1) / kTileRows;
  return w;
}

// Column pass: CTA = (batch, kv head, 128-key tile, part); the key tile's
// items are the (query head of the group, 128-query tile) pairs that can see
// its keys, cut into parts of p.part_items.  Key tiles with the most items run
// first.
__device__ __forceinline__ PfWork cols_work(const PrefillParams& p) {
  PfWork w{};
  const int kvb = p.batch * p.kv_heads;
  const int idx = blockIdx.x;
  const int kt = idx / (p.parts * kvb);
  const int rem = idx % (p.parts * kvb);
  const int part = rem / kvb;
  const int bk = rem % kvb;
  w.b = bk / p.kv_heads;
  w.kvh = bk % p.kv_heads;
  w.k0 = kt * kTileRows;
  w.res_row = w.k0;
  w.res_head = bk;
  const int nqt = (p.tq + kTileRows - 1) / kTileRows;
  w.qt_first = p.causal ? max(0, w.k0 - p.q_offset) / kTileRows : 0;
  w.per_head = max(0, nqt - w.qt_first);
  const int total = p.groups * w.per_head;
  w.i0 = part * p.part_items;
  w.n = max(0, min(total - w.i0, p.part_items));
  return w;
}

// Walks a column-pass CTA's items in order without a division per item:
// (query head of the group, query tile), query tiles innermost.
struct ItemIter {
  int hh, qt;
  __device__ __forceinline__ void start(const PfWork& w, int i) {
    hh = (w.i0 + i) / w.per_head;
    qt = w.qt_first + (w.i0 + i) % w.per_head;
  }
  __device__ __forceinline__ void next(const PfWork& w) {
    if (++qt == w.qt_first + w.per_head) {
      qt = w.qt_first;
      ++hh;
    }
  }
};

__device__ __forceinline__ void tmem_wait_ld_into(uint32_t (&v)[32]) {
  // the wait "rewrites" the registers, so no use of them moves above it
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]),
                 "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
                 "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                 "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

// Logits per 32 whose exp2 runs on the FMA pipe (ex2_fma) instead of MUFU.
// MUFU retires 16 exp2 per SM clock and is the busiest pipe of both passes
// while the FMA and ALU pipes idle, so a share of the exps moves over (the
// shares measured best on B200: 4 / 32 in the LSE pass, 2 / 32 in the column
// pass, whose epilogue spends more issue slots per logit).
constexpr int kLseFmaExps = 4;
constexpr int kColsFmaExps = 2;

// Logit j of a 32-chunk takes the FMA-pipe exp2 when kFma of 32 do (every
// (32 / kFma)-th logit).
template <int kFma>
__device__ __forceinline__ float ex2_mix(float x, int j) {
  constexpr int kStride = 32 / (kFma > 0 ? kFma : 1);
  static_assert(kFma == 0 || (kFma <= 16 && kStride * kFma == 32), "exps per 32");
  if (kFma > 0 && j % kStride == kStride - 1) return ex2_fma(x);
  return ex2(x);
}

// Column pass, 32 logits of one key row: sum += exp2(s c - LSE2_j); with kMask
// only the columns j with j + rel >= 0 (those whose query sees the key).
template <bool kMask>
__device__ __forceinline__ void cols_chunk(const uint32_t (&v)[32], const float* l, float c,
                                           int rel, float (&sum)[4]) {
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const float4 l4 = *reinterpret_cast<const float4*>(l + j);
    float x0 = fmaf(__uint_as_float(v[j]), c, -l4.x);
    float x1 = fmaf(__uint_as_float(v[j + 1]), c, -l4.y);
    float x2 = fmaf(__uint_as_float(v[j + 2]), c, -l4.z);
    float x3 = fmaf(__uint_as_float(v[j + 3]), c, -l4.w);
    if (kMask) {
      x0 = j + rel >= 0 ? x0 : -INFINITY;
      x1 = j + 1 + rel >= 0 ? x1 : -INFINITY;
      x2 = j + 2 + rel >= 0 ? x2 : -INFINITY;
      x3 = j + 3 + rel >= 0 ? x3 : -INFINITY;
    }
    sum[0] += ex2_mix<kColsFmaExps>(x0, j);
    sum[1] += ex2_mix<kColsFmaExps>(x1, j + 1);
    sum[2] += ex2_mix<kColsFmaExps>(x2, j + 2);
    sum[3] += ex2_mix<kColsFmaExps>(x3, j + 3);
  }
}

// LSE pass, 32 logits of one query row, online in the log2 domain: m is the
// running max of s c, l the sum of exp2(s c - m).  With kMask only columns
// j < jmax count.  The max is taken on the raw logits (c > 0), so each logit
// costs one FFMA ahead of its exp2.
template <bool kMask>
__device__ __forceinline__ void lse_chunk(uint32_t (&v)[32], float c, int jmax, float& m,
                                          float& l) {
  float cm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (kMask && j >= jmax) v[j] = __float_as_uint(-INFINITY);
    cm = fmaxf(cm, __uint_as_float(v[j]));
  }
  const float mn = fmaxf(m, cm * c);
  if (mn == -INFINITY) return;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    s0 += ex2_mix<kLseFmaExps>(fmaf(__uint_as_float(v[j]), c, -mn), j);
    s1 += ex2_mix<kLseFmaExps>(fmaf(__uint_as_float(v[j + 1]), c, -mn), j + 1);
    s2 += ex2_mix<kLseFmaExps>(fmaf(__uint_as_float(v[j + 2]), c, -mn), j + 2);
    s3 += ex2_mix<kLseFmaExps>(fmaf(__uint_as_float(v[j + 3]), c, -mn), j + 3);
  }
  l = l * ex2(m - mn) + ((s0 + s1) + (s2 + s3));
  m = mn;
}

template <int D, bool kCols, int WG>
__global__ void __launch_bounds__(PfWarps<WG>::kThreads, 2)
    umma_pass_kernel(const __grid_constant__ PrefillParams p,
                     const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k) {
  using L = PfLayout<D, WG>;
  using Wp = PfWarps<WG>;
  constexpr int S = L::kStages;
  constexpr int kEpiThreads = Wp::kEpiThreads;
  constexpr int kProdWarp = Wp::kProdWarp;
  constexpr int kMmaWarp = Wp::kMmaWarp;
  constexpr int kWgCols = Wp::kCols;
  extern __shared__ uint8_t pf_raw[];
  const uint32_t raw = smem_u32(pf_raw);
  uint8_t* smem = pf_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* res_full = bars + 2 * S;
  uint64_t* tfull = res_full + 1;
  uint64_t* tempty = res_full + 3;
  uint64_t* done = res_full + 5;
  uint64_t* lfull = done + 1;   // column pass: LSE ring slot written
  uint64_t* lempty = done + 5;  // column pass: LSE ring slot read by every epilogue warp
  float* lse_s = reinterpret_cast<float*>(smem + L::kLseOff);
  uint32_t* taddr_s = reinterpret_cast<uint32_t*>(smem + L::kTaddrOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const PfWork w = kCols ? cols_work(p) : lse_work(p);
  if (w.n <= 0) return;  // CTA-uniform: an empty part of a short key tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(res_full, 1);
    mbar_init(tfull, 1);
    mbar_init(tfull + 1, 1);
    mbar_init(tempty, kEpiThreads);
    mbar_init(tempty + 1, kEpiThreads);
    mbar_init(done, 1);
    for (int k = 0; k < 4; ++k) {
      mbar_init(lfull + k, 32);
      mbar_init(lempty + k, kEpiThreads / 32);
    }
    fence_mbar_init();
  }
  if (warp == kProdWarp) tmem_alloc(taddr_s, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *taddr_s;

  if (warp == kProdWarp) {
    // ---- TMA producer
    if (lane == 0) {
      const CUtensorMap* rmap = kCols ? &tm_k : &tm_q;
      const CUtensorMap* smap = kCols ? &tm_q : &tm_k;
      prefetch_tensormap(rmap);
      prefetch_tensormap(smap);
      mbar_arrive_expect_tx(res_full, L::kTile);
      tma_load_4d(smem, rmap, 0, w.res_row, 0, w.res_head, res_full);
      bool ok = true;
      int issued = 0;
      ItemIter it;
      if (kCols) it.start(w, 0);
      for (int i = 0; i < w.n; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(empty + s, ((i / S) - 1) & 1)) {
          ok = false;
          break;
        }
        int row, head;
        if (kCols) {
          row = it.qt * kTileRows;
          head = w.b * p.num_heads + w.kvh * p.groups + it.hh;
          it.next(w);
        } else {
          row = i * kTileRows;
          head = w.b * p.kv_heads + w.kvh;
        }
        mbar_arrive_expect_tx(full + s, L::kTile);
        tma_load_4d(smem + L::kTile * (1 + s), smap, 0, row, 0, head, full + s);
        issued = i + 1;
      }
      // no copy may still be landing in shared memory when the CTA exits
      ok = mbar_wait(res_full, 0) && ok;
      for (int i = max(0, issued - S); i < issued; ++i) ok = mbar_wait(full + i % S, (i / S) & 1) && ok;
      if (!ok) atomicOr(p.err, TKV_DEVERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == Wp::kLseWarp) {
    // ---- column pass: the query LSEs of item i (log2 domain, +inf past the
    // last query row) into ring slot i % 4, up to four items ahead
    if (kCols) {
      ItemIter it;
      it.start(w, 0);
      const int hbase = w.kvh * p.groups;
      bool ok = true;
      for (int i = 0; i < w.n; ++i) {
        const int slot = i & 3;
        if (i >= 4 && ok && !mbar_wait(lempty + slot, ((i >> 2) - 1) & 1)) ok = false;
        __syncwarp();
        const int q0 = it.qt * kTileRows;
        const float* src = p.lse + ((size_t)w.b * p.num_heads + hbase + it.hh) * p.tq;
#pragma unroll
        for (int k = 0; k < kTileRows / 32; ++k) {
          const int q = q0 + 32 * k + lane;
          lse_s[slot * kTileRows + 32 * k + lane] = q < p.tq ? __ldg(src + q) * kLog2eP : INFINITY;
        }
        mbar_arrive(lfull + slot);
        it.next(w);
      }
      if (!ok && lane == 0) atomicOr(p.err, TKV_DEVERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer: S^T tile (kCols) or S tile = resident (A) x streamed (B)^T
    if (lane == 0) {
      bool ok = mbar_wait(res_full, 0);
      const uint32_t a_base = smem_u32(smem);
      for (int i = 0; ok && i < w.n; ++i) {
        const int s = i % S, acc = i & 1;
        if (!mbar_wait(full + s, (i / S) & 1) ||
            (i >= 2 && !mbar_wait(tempty + acc, ((i >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t b_base = smem_u32(smem + L::kTile * (1 + s));
        const uint32_t d = tmem + (uint32_t)(acc * kTileRows);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          // 64-element K chunks are 128 rows x 128 bytes apart; K steps of 16 are 32 bytes
          const uint32_t off = (uint32_t)((ks >> 2) * kTileRows * 128 + (ks & 3) * 32);
          umma_f16(d, umma_desc_k_sw128(a_base + off), umma_desc_k_sw128(b_base + off), kIdesc,
                   ks > 0 ? 1u : 0u);
        }
        umma_commit(empty + s);
        umma_commit(tfull + acc);
      }
      umma_commit(done);  // every MMA issued above has completed once this phase does
      ok = mbar_wait(done, 0) && ok;
      if (!ok) atomicOr(p.err, TKV_DEVERR_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---- epilogue: thread t owns resident row t % 128 (its TMEM lane) in
    // the accumulator columns [cb, cb + kWgCols) of its warpgroup
    const int t = threadIdx.x;
    const int row = t & (kTileRows - 1);
    const int wg = t >> 7;
    const int cb = wg * kWgCols;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    const float c = p.scaling * kLog2eP;
    bool ok = true;
    if (kCols) {
      const int key = w.k0 + row;
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      ItemIter cur;
      cur.start(w, 0);
      for (int i = 0; i < w.n; ++i) {
        const int slot = i & 3;
        // after a timeout the loop keeps its shape (no waits), so whole warps
        // run tcgen05.ld and every thread meets the final barriers
        if (ok && !mbar_wait(lfull + slot, (i >> 2) & 1)) ok = false;
        const float* ls = lse_s + slot * kTileRows + cb;
        const int q0 = cur.qt * kTileRows;
        cur.next(w);
        const int acc = i & 1;
        if (ok && !mbar_wait(tfull + acc, (i >> 1) & 1)) ok = false;
        __syncwarp();
        tc_fence_after();
        // causal: query column j sees this row's key iff j >= key - q_offset - q0
        const bool diag = p.causal && q0 + p.q_offset < w.k0 + kTileRows - 1;
#pragma unroll
        for (int c2 = 0; c2 < Wp::kChunks; ++c2) {
          uint32_t v[32];
          const int col0 = cb + 32 * c2;
          tmem_ld32(lane_base + (uint32_t)(acc * kTileRows + col0), v);
          tmem_wait_ld_into(v);
          if (c2 == Wp::kChunks - 1) {
            tc_fence_before();
            mbar_arrive(tempty + acc);
          }
          if (diag) cols_chunk<true>(v, ls + 32 * c2, c, col0 - (key - p.q_offset - q0), sum);
          else cols_chunk<false>(v, ls + 32 * c2, c, 0, sum);
        }
        __syncwarp();  // the warp's reads of the ring slot are done
        if (lane == 0) mbar_arrive(lempty + slot);
      }
      if (ok && key < p.tk) atomicAdd(p.token_mass + key, (sum[0] + sum[1]) + (sum[2] + sum[3]));
    } else {
      const int q = w.q0 + row;
      const int qpos = q + p.q_offset;
      float m = -INFINITY, l = 0.f;  // running max (scaled, log2 domain) and sum of this half
      for (int i = 0; i < w.n; ++i) {
        const int acc = i & 1;
        if (ok && !mbar_wait(tfull + acc, (i >> 1) & 1)) ok = false;
        __syncwarp();
        tc_fence_after();
        const int k0 = i * kTileRows;
        // CTA-uniform: does any key of the tile fall outside some row's view?
        const bool edge =
            k0 + kTileRows > p.tk || (p.causal && k0 + kTileRows - 1 > w.q0 + p.q_offset);
        const int jmax = (p.causal ? min(p.tk, qpos + 1) : p.tk) - k0;  // columns j < jmax count
#pragma unroll
        for (int c2 = 0; c2 < Wp::kChunks; ++c2) {
          uint32_t v[32];
          const int col0 = cb + 32 * c2;
          tmem_ld32(lane_base + (uint32_t)(acc * kTileRows + col0), v);
          tmem_wait_ld_into(v);
          if (c2 == Wp::kChunks - 1) {
            tc_fence_before();
            mbar_arrive(tempty + acc);
          }
          if (edge) lse_chunk<true>(v, c, jmax - col0, m, l);
          else lse_chunk<false>(v, c, 0, m, l);
        }
      }
      // merge the warpgroups' shares of each row
      float* mrg = lse_s;  // [WG - 1][128][2]
      if (wg != 0) {
        mrg[((wg - 1) * kTileRows + row) * 2] = m;
        mrg[((wg - 1) * kTileRows + row) * 2 + 1] = l;
      }
      if (WG > 1) named_barrier(1, kEpiThreads);
      if (wg == 0 && ok && q < p.tq) {
        float mm = m;
#pragma unroll
        for (int o = 1; o < WG; ++o) mm = fmaxf(mm, mrg[((o - 1) * kTileRows + row) * 2]);
        float ls = 0.f;
        if (mm != -INFINITY) {
          ls = l * ex2(m - mm);
#pragma unroll
          for (int o = 1; o < WG; ++o)
            ls += mrg[((o - 1) * kTileRows + row) * 2 + 1] * ex2(mrg[((o - 1) * kTileRows + row) * 2] - mm);
        }
        const float kLn2 = 0.6931471805599453f;
        p.lse[(size_t)w.res_head * p.tq + q] = ls > 0.f ? (mm + lg2(ls)) * kLn2 : -INFINITY;
      }
    }
    if (!ok) atomicOr(p.err, TKV_DEVERR_TIMEOUT);
  }

  // every TMEM read and MMA of the CTA has completed: free the accumulators
  tc_fence_before();
  __syncthreads();
  if (warp == kProdWarp) {
    tc_fence_after();
    tmem_free(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- block means
__global__ void block_mean_kernel(const float* token_mass, int tk, int block_size, float inv_count,
                                  float* block_scores) {
  const int blk = blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = (tk + block_size - 1) / block_size;
  if (blk >= nb) return;
  const int k0 = blk * block_size, k1 = min(tk, k0 + block_size);
  float sum = 0.f;
  for (int kk = k0; kk < k1; ++kk) sum += token_mass[kk] * inv_count;
  block_scores[blk] = sum / (float)(k1 - k0);
}

cudaError_t prefill_error_word(uint32_t** out) {
  return cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_tkv_prefill_err);
}

template <int D, bool kCols>
static cudaError_t launch_umma(PrefillParams p, const CUtensorMap maps[2], long long grid,
                               cudaStream_t stream) {
  constexpr int WG = kCols ? TKV_PF_WG_COLS : TKV_PF_WG_LSE;
  using L = PfLayout<D, WG>;
  if (grid <= 0 || grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  cudaError_t e = prefill_error_word(&p.err);
  if (e != cudaSuccess) return e;
  auto kern = umma_pass_kernel<D, kCols, WG>;
  // the shared-memory opt-in is per function and device; it is idempotent
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)grid, PfWarps<WG>::kThreads, L::kBytes, stream>>>(p, maps[0], maps[1]);
  return cudaGetLastError();
}

cudaError_t launch_prefill_lse(const PrefillParams& p, const CUtensorMap maps[2],
                               cudaStream_t stream) {
  const long long grid = (long long)((p.tq + kTileRows - 1) / kTileRows) * p.batch * p.num_heads;
  if (p.head_dim == 128) return launch_umma<128, false>(p, maps, grid, stream);
  if (p.head_dim == 64) return launch_umma<64, false>(p, maps, grid, stream);
  return cudaErrorInvalidValue;
}

// Items (query head, query tile) per column-pass CTA: enough to amortise the
// CTA's resident-tile load and TMEM setup, few enough that the longest key
// tiles split over several SMs.
constexpr int kColsPartItems = 32;

cudaError_t launch_prefill_scores(const PrefillParams& p_in, const CUtensorMap maps[2],
                                  cudaStream_t stream) {
  PrefillParams p = p_in;
  cudaError_t e = cudaMemsetAsync(p.token_mass, 0, sizeof(float) * (size_t)p.tk, stream);
  if (e != cudaSuccess) return e;
  const int nqt = (p.tq + kTileRows - 1) / kTileRows;
  const int nkt = (p.tk + kTileRows - 1) / kTileRows;
  p.part_items = kColsPartItems;
  p.parts = (p.groups * nqt + p.part_items - 1) / p.part_items;
  const long long grid = (long long)nkt * p.parts * p.batch * p.kv_heads;
  if (p.head_dim == 128) e = launch_umma<128, true>(p, maps, grid, stream);
  else if (p.head_dim == 64) e = launch_umma<64, true>(p, maps, grid, stream);
  else return cudaErrorInvalidValue;
  if (e != cudaSuccess) return e;
  const int nb = (p.tk + p.block_size - 1) / p.block_size;
  const float inv = 1.f / ((float)p.batch * (float)p.num_heads * (float)p.tq);
  block_mean_kernel<<<(nb + 127) / 128, 128, 0, stream>>>(p.token_mass, p.tk, p.block_size, inv,
                                                          p.block_scores);
  return cudaGetLastError();
}

}  // namespace tkv
