// tkv_decode.cu -- tiered paged decode attention for sm_100a.
//
// Replaces the Triton kernels of xiaoMartintin/Paged_TierKV
// (tierkv_triton.py:45-145 single pass + score pass, 147-264 split + reduce).
//
// One CTA per (split, kv head, sequence); the splits of a (sequence, kv head)
// claim block ranges of up to 8, 16 or 32 blocks (the maximum chosen per
// launch by the planner) from a shared counter.  Warp 0 is the producer: it
// reads the block table one range (a lane per entry) at a time, skips COLD
// blocks (their valid tokens
// only add the analytic term n * exp(0 - m) to the softmax denominator), and
// streams each HOT / WARM block tile of this kv head through a ring of shared
// memory stages with TMA (128-byte swizzled boxes; no multicast), completing
// on an mbarrier per stage.  The other warps consume tiles round-robin: each tile
// is one logical block (16 or 32 tokens x head_dim) for all query heads of
// the GQA group, so K/V are read from HBM once per kv head.
//   S^T[tok, h] = K[tok, :] . Q[h, :]       mma.m16n8k16 (M = tokens, N = heads)
//   O^T[d, h]  += V^T[d, tok] . P^T[tok, h] mma.m16n8k16 (M = head_dim rows)
// HOT tiles feed ldmatrix directly; WARM tiles (uint8 codes) are expanded in
// registers with byte permutes into exact fp16 (code - zero) values, the
// per-token scale being applied to the logits (K) and folded into P (V).
// Online softmax runs in the log2 domain in fp32.  Each consumer keeps its own
// (m, l, acc); the CTA merges them, then either writes the output (one split)
// or a normalised partial plus its LSE; the last CTA of a (sequence, kv head)
// merges the splits (split tickets reset themselves).
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <atomic>

#include "tkv_internal.h"
#include "tkv_ptx.cuh"

namespace tkv {

struct TileInfo {
  int32_t state;  // 0 HOT, 1 WARM, -1 end of stream
  int32_t len;    // valid tokens (1..bs)
  int32_t block;  // logical block index
  float ks;       // Format S: K scale of the tile
  float vs;       // Format S: V scale of the tile
  int32_t pad[3];
};

// Pipeline shape: consumer warps per CTA, ring depth for stages of <= 8 KB and
// of 16 KB, and the CTAs per SM the register budget is sized for.
#ifndef TKV_CONSUMERS
#define TKV_CONSUMERS 3
#endif
#ifndef TKV_STAGES_8K
#define TKV_STAGES_8K 6
#endif
#ifndef TKV_STAGES_16K
#define TKV_STAGES_16K 3
#endif
#ifndef TKV_MIN_CTAS
#define TKV_MIN_CTAS 4
#endif
// A consumer hands its stage back as soon as the tile's V fragments are in
// registers (before the softmax and the PV products) instead of at the end.
#ifndef TKV_EARLY_RELEASE
#define TKV_EARLY_RELEASE 1
#endif
// Launch decode kernels with programmatic stream serialization (see launch_one).
#ifndef TKV_PDL
#define TKV_PDL 1
#endif
// The first-wave CTAs prefetch the tiles that fill their ring into L2 before
// their dependency wait (0: off).  Measured on B200: configuration 4 1.538 ->
// 1.513 ms per step, an 8-GPU shard's launch 17.5 -> 16.6 us, 8 sequences of
// configuration 3 -2 %, configuration 5 unchanged; prefetching the whole
// first chunk (32 tiles) instead was slower everywhere (+3 % on
// configuration 4), and prefetching in every wave cost configuration 5 1 %.
#ifndef TKV_PREFETCH
#define TKV_PREFETCH 1
#endif


template <int D, int BS, int FMT, int QT>
struct DecodeCfg {
  static constexpr int kConsumers = TKV_CONSUMERS;
  static constexpr int kThreads = 32 * (kConsumers + 1);
  static constexpr int kHotBytes = BS * D * 2;            // one K (or V) HOT tile
  static constexpr int kStageBytes = 2 * kHotBytes;       // K + V, multiple of 1024
  static constexpr int kStages = (kStageBytes <= 8192) ? TKV_STAGES_8K : TKV_STAGES_16K;
  static_assert(kStages % kConsumers == 0, "each consumer must own a fixed subset of stages");
  static constexpr int kMetaBytes = (FMT == kFmtR) ? 4 * BS * 2 : 16;
  static constexpr int kKS = D / 16;                      // 16-wide steps over head_dim
  static constexpr int kSub = BS / 16;                    // 16-token sub-tiles per block
  static constexpr int kWarmSwz = (D == 128) ? 7 : 3;     // SWIZZLE_128B / SWIZZLE_64B
  // layout of dynamic shared memory (after aligning the base to 1024); bulk
  // copy destinations (the meta area) must start on 16-byte boundaries
  static constexpr int align_to(int x, int a) { return (x + a - 1) / a * a; }
  static constexpr int kOffBars = kStages * kStageBytes;
  static constexpr int kOffInfo = align_to(kOffBars + 2 * kStages * 8, 16);
  static constexpr int kOffMeta = align_to(kOffInfo + kStages * (int)sizeof(TileInfo), 128);
  static constexpr int kOffMisc = align_to(kOffMeta + kStages * kMetaBytes, 16);
  static_assert(kOffMeta % 128 == 0 && kMetaBytes % 16 == 0 && (BS * 2) % 16 == 0,
                "every meta bulk-copy destination must be 16-byte aligned");
  static_assert(kStageBytes % 1024 == 0 && kHotBytes % 1024 == 0,
                "swizzled TMA boxes need 1024-byte aligned destinations");
  // query of the GQA group, fp16, twice: standard d order (HOT K) and the
  // permuted order of the register-expanded WARM K; rows padded by 16 bytes
  static constexpr int kQStride = D + 8;
  static constexpr int kOffQ = kOffMisc + 128;  // misc: 32 words
  static constexpr int kQBytes = kMaxGroups * kQStride * 2;
  static constexpr int kSmemBytes = 1024 + kOffQ + 2 * kQBytes;
  // the end-of-kernel merge scratch aliases the stage ring
  static constexpr int kMergeFloats = kConsumers * (2 * kMaxGroups + kMaxGroups * D);
  static_assert(kMergeFloats * 4 <= kStages * kStageBytes, "merge scratch must fit the ring");
  static_assert(kMaxGroups * (kMaxSplits + 2) * 4 <= kStages * kStageBytes,
                "split-merge scratch must fit the ring");
};

__device__ __forceinline__ void store_out(void* out, int dtype, size_t idx, float v) {
  if (dtype == kDtF16) {
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  } else if (dtype == kDtBF16) {
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<float*>(out)[idx] = v;
  }
}

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// Stages the query heads of this kv head in shared memory.  Rows n >= G are
// zero.
//  sqh[n][d]        standard d order, for ldmatrix-fed HOT K fragments
//  sqw[n][pw(d)]    permuted so that a standard ldmatrix of k-step s hands lane
//                   t the dims t*D/4 + 4s + {0,1} (b0) and + {2,3} (b1), the
//                   order of the register-expanded WARM K codes
// bf16 queries are rescaled per head by 2^-e (exact) so they fit fp16; the
// factor 2^e is returned through sexp[0..8) and folded into the logit scale;
// sexp[8..16) receives the per-head sums of the staged values as floats.
// Only the NC consumer warps take part (the producer is already streaming
// tiles meanwhile); each thread moves one 16-byte vector of the query per
// step, and the call ends with named barrier 1 over the consumer warps.
template <int D, int QT, int NC>
__device__ __forceinline__ void stage_query(const DecodeParams& p, int seq, int kvh,
                                            __half* sqh, __half* sqw, int* sexp) {
  constexpr int QS = D + 8;
  constexpr int NT = NC * 32;
  constexpr int VPR = D / 8;                  // 16-byte vectors per head row
  constexpr int kVecs = kMaxGroups * VPR;
  const int G = p.groups;
  const int tid = threadIdx.x - 32;           // consumer thread
  const int cw = tid >> 5, lane = tid & 31;
  const size_t row0 = (size_t)seq * p.num_heads + (size_t)kvh * G;
  if (QT == kDtBF16) {
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.query);
    for (int n = cw; n < kMaxGroups; n += NC) {
      float amax = 0.f;
      if (n < G)
        for (int d = lane; d < D; d += 32)
          amax = fmaxf(amax, fabsf(__bfloat162float(q[(row0 + n) * D + d])));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      int k = 0;
      frexpf(amax, &k);  // amax < 2^k
      if (lane == 0) sexp[n] = max(0, k - 15);
    }
    named_barrier(1, NT);
  } else if (tid < kMaxGroups) {
    sexp[tid] = 0;
  }
  float* qsum = reinterpret_cast<float*>(sexp + 8);
  // the loop is warp-uniform: a row's VPR vectors lie in one aligned lane group
  for (int base = cw * 32; base < kVecs; base += NT) {
    const int e = base + lane;
    const int n = e / VPR;
    const int c = e % VPR;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (e < kVecs && n < G)
      raw = __ldg(reinterpret_cast<const uint4*>(p.query) + ((row0 + n) * D) / 8 + c);
    __align__(16) __half h[8];
    if (QT == kDtF16) {
      *reinterpret_cast<uint4*>(h) = raw;
    } else {
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&raw);
      const int ex = n < kMaxGroups ? sexp[n] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(ldexpf(__bfloat162float(b[j]), -ex));
    }
    float sum = 0.f;
    if (e < kVecs) {
      *reinterpret_cast<uint4*>(sqh + n * QS + 8 * c) = *reinterpret_cast<const uint4*>(h);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = 8 * c + j;
        const int tq = d / (D / 4);
        const int s = (d % (D / 4)) / 4;
        const int jj = d & 3;
        sqw[n * QS + 16 * s + 2 * tq + (jj & 1) + 8 * (jj >> 1)] = h[j];
        sum += __half2float(h[j]);
      }
    }
    // per-head sum of the staged fp16 values (the WARM K zero-point correction)
#pragma unroll
    for (int off = VPR / 2; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (e < kVecs && c == 0) qsum[n] = sum;
  }
  named_barrier(1, NT);
}

// B fragments (k = head_dim, n = query head) of k-steps 2m and 2m+1 from a
// staged query block: lane (g, t) receives rows n = g, dims 16ks + 2t (+8).
template <int D>
__device__ __forceinline__ void load_qfrag(uint32_t sq, int lane, int m, uint32_t& b00,
                                           uint32_t& b01, uint32_t& b10, uint32_t& b11) {
  constexpr int QS = D + 8;
  const uint32_t addr = sq + ((lane & 7) * QS + 32 * m + 8 * (lane >> 3)) * 2;
  ldsm_x4(addr, b00, b01, b10, b11);
}

// ---------------------------------------------------------------- exchange
// Rank q's inbox as mapped in this process: o words [2][rows_cap][world][D]
// and lse words [2][rows_cap][world] (epoch parity), each word the epoch of
// the call that wrote it (high half) and an fp32 value (low half).  A word is
// valid for a call when its epoch is the call's: the value and its epoch
// travel in one single-copy-atomic 8-byte store, so no flag and no release
// fence are needed, and a reader polls the words themselves.  The epoch of
// the call is read once per CTA at kernel start (thread 0: the value in the
// parameters, or a plain global load from x_epoch_dev, which nothing writes
// while the launch runs) and handed to these helpers by value.
template <int D>
__device__ __forceinline__ uint64_t* x_o(const DecodeParams& p, int q, uint32_t epoch) {
  return reinterpret_cast<uint64_t*>(p.x_inbox[q]) +
         (size_t)(epoch & 1u) * p.x_rows_cap * p.x_world * D;
}
template <int D>
__device__ __forceinline__ uint64_t* x_lse(const DecodeParams& p, int q, uint32_t epoch) {
  return reinterpret_cast<uint64_t*>(p.x_inbox[q] + xchg_o_bytes(p.x_world, p.x_rows_cap, D)) +
         (size_t)(epoch & 1u) * p.x_rows_cap * p.x_world;
}
__device__ __forceinline__ uint64_t x_word(float v, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ bool x_valid(uint64_t w, uint32_t epoch) {
  return (uint32_t)(w >> 32) == epoch;
}
__device__ __forceinline__ float x_value(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Merges `cnt` normalised partials (o, LSE) of the G rows row0.. of a
// (sequence, kv head): part j of row r at po + ((r * rstride) + j0 + j) * D
// and plse[r * rstride + j0 + j].  The result goes to the final output
// (p.out / p.out_lse / p.lse_final) when dst_o is null, else to the fp32
// partial slot dj of rows with stride dstride.  wsl is shared scratch of
// G * cnt floats.  One warp per head, no CTA barrier: a lane owns 4 dims (a
// float4 of every part's row) and, for head_dim 64, every other part; each
// round keeps kMergeDepth independent 16-byte loads in flight, the first
// round together with the row's LSEs (kMergeLseDepth per lane per round).
// (Measured on B200 against three CTA-wide phases -- LSEs, max and sum,
// weights -- each behind a CTA barrier and a full fence around the ticket:
// the 74-way merge of a 131072-token layer 5.3 -> 3.3 us, an 8-GPU shard's
// launch 18.8 -> 17.3 us.)
// Partial rows each lane loads per round of the split merge (the merge is
// latency-bound: one round trip per round).
#ifndef TKV_MERGE_DEPTH
#define TKV_MERGE_DEPTH 16
#endif
constexpr int kMergeDepth = TKV_MERGE_DEPTH;
constexpr int kMergeLseDepth = 4;
// WARM tiles a consumer warp takes between two removals of the V offset sum
#ifndef TKV_VCORR_FLUSH
#define TKV_VCORR_FLUSH 8
#endif
constexpr int kVcorrFlush = TKV_VCORR_FLUSH;

// Stores the merged row (o: this lane's float4 of dims 4v..4v+3).
template <int D>
__device__ __forceinline__ void merged_row_out(const DecodeParams& p, size_t row, int v, bool lead,
                                               int lane, float4 o, float lse, float* dst_o,
                                               float* dst_lse, int dstride, int dj, bool xout,
                                               uint32_t epoch) {
  if (dst_o != nullptr) {
    if (lead) reinterpret_cast<float4*>(dst_o + (row * dstride + dj) * D)[v] = o;
    if (lane == 0) dst_lse[row * dstride + dj] = lse;
  } else if (xout) {
    // this rank's partial of the row into every rank's inbox
    for (int q = 0; q < p.x_world; ++q) {
      if (lead) {
        uint64_t* dst = x_o<D>(p, q, epoch) + (row * p.x_world + p.x_rank) * D + 4 * v;
        st_relaxed_sys_v2(dst, x_word(o.x, epoch), x_word(o.y, epoch));
        st_relaxed_sys_v2(dst + 2, x_word(o.z, epoch), x_word(o.w, epoch));
      }
      if (lane == 0) st_relaxed_sys(x_lse<D>(p, q, epoch) + row * p.x_world + p.x_rank, x_word(lse, epoch));
    }
  } else {
    if (lead) {
      const size_t base = row * D + 4 * v;
      store_out(p.out, p.out_dtype, base + 0, o.x);
      store_out(p.out, p.out_dtype, base + 1, o.y);
      store_out(p.out, p.out_dtype, base + 2, o.z);
      store_out(p.out, p.out_dtype, base + 3, o.w);
    }
    if (lane == 0) {
      if (p.out_lse) p.out_lse[row] = lse;
      if (p.lse_final) p.lse_final[row] = lse;
    }
  }
}

// The warp of a head requests the first round of partial rows and the row's
// LSEs together, reduces max and sum over its lanes and keeps the weights in
// its own scratch row.
template <int D, int NT>
__device__ __forceinline__ void merge_parts(const float* po, const float* plse, int rstride,
                                            int j0, int cnt, size_t row0, int G, float* wsl,
                                            const DecodeParams& p, float* dst_o, float* dst_lse,
                                            int dstride, int dj, bool xout = false,
                                            uint32_t epoch = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kVecs = D / 4;                 // float4 per partial row
  constexpr int kLanesPerRow = kVecs < 32 ? kVecs : 32;
  constexpr int kSplitLanes = 32 / kLanesPerRow;
  const int v = lane % kLanesPerRow;
  const int sp0 = lane / kLanesPerRow;
  for (int h = warp; h < G; h += NT / 32) {
    const size_t row = row0 + h;
    float* wl = wsl + (size_t)h * cnt;
    const float4* src = reinterpret_cast<const float4*>(po + (row * rstride + j0) * D) + v;
    const float* lsrc = plse + row * rstride + j0;
    float4 x[kMergeDepth];
#pragma unroll
    for (int k = 0; k < kMergeDepth; ++k) {
      const int sidx = sp0 + k * kSplitLanes;
      x[k] = sidx < cnt ? __ldcg(src + (size_t)sidx * kVecs) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float M = -INFINITY;
    for (int e0 = lane; e0 < cnt; e0 += 32 * kMergeLseDepth) {
      float lv[kMergeLseDepth];
#pragma unroll
      for (int k = 0; k < kMergeLseDepth; ++k) {
        const int e = e0 + 32 * k;
        lv[k] = e < cnt ? __ldcg(lsrc + e) : -INFINITY;
      }
#pragma unroll
      for (int k = 0; k < kMergeLseDepth; ++k) {
        const int e = e0 + 32 * k;
        if (e < cnt) wl[e] = lv[k];
        M = fmaxf(M, lv[k]);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    // each lane turns its own LSEs into weights, then the warp reads them all
    float S = 0.f;
    if (M != -INFINITY) {
      for (int e = lane; e < cnt; e += 32) {
        const float w = ex2((wl[e] - M) * kLog2e);
        wl[e] = w;
        S += w;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S += __shfl_xor_sync(0xffffffffu, S, off);
    const bool live = M != -INFINITY && S > 0.f;
    for (int e = lane; e < cnt; e += 32) wl[e] = live ? wl[e] / S : 0.f;
    __syncwarp();
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    int sp = sp0;
    for (;;) {
#pragma unroll
      for (int k = 0; k < kMergeDepth; ++k) {
        const int sidx = sp + k * kSplitLanes;
        const float w = sidx < cnt ? wl[sidx] : 0.f;
        o.x += w * x[k].x; o.y += w * x[k].y; o.z += w * x[k].z; o.w += w * x[k].w;
      }
      sp += kMergeDepth * kSplitLanes;
      if (sp - sp0 >= cnt) break;
#pragma unroll
      for (int k = 0; k < kMergeDepth; ++k) {
        const int sidx = sp + k * kSplitLanes;
        x[k] = sidx < cnt ? __ldcg(src + (size_t)sidx * kVecs) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int off = kLanesPerRow; off < 32; off <<= 1) {
      o.x += __shfl_xor_sync(0xffffffffu, o.x, off);
      o.y += __shfl_xor_sync(0xffffffffu, o.y, off);
      o.z += __shfl_xor_sync(0xffffffffu, o.z, off);
      o.w += __shfl_xor_sync(0xffffffffu, o.w, off);
    }
    const float lse = live ? M + logf(S) : -INFINITY;
    merged_row_out<D>(p, row, v, sp0 == 0, lane, o, lse, dst_o, dst_lse, dstride, dj, xout, epoch);
  }
}

// The world partials of the G rows row0.. (this rank's inbox, epoch parity)
// merged into the output: one warp per head.  Every lane requests, in one
// round, its 4 dims of every rank's partial (and lane q < world rank q's LSE
// word); only words that do not carry the call's epoch yet are polled again.
// All polls share one deadline (timeout_ns, 2 s by default); past it they
// give up, record TKV_DEVERR_TIMEOUT and count the missing partials as empty.
template <int D, int NT>
__device__ __forceinline__ void x_merge(const DecodeParams& p, size_t row0, int G, uint32_t epoch) {
  constexpr int kVecs = D / 4;                 // float4 per row
  constexpr int kLanesPerRow = kVecs < 32 ? kVecs : 32;
  constexpr int kSplitLanes = 32 / kLanesPerRow;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = p.x_world;
  const uint64_t* xo = x_o<D>(p, p.x_rank, epoch);
  const uint64_t* xl = x_lse<D>(p, p.x_rank, epoch);
  const int v = lane % kLanesPerRow;
  const int q0 = lane / kLanesPerRow;
  const uint64_t limit = p.x_timeout_ns ? p.x_timeout_ns : 2000000000ull;
  const uint64_t t0 = globaltimer();
  bool late = false;  // this lane gave up on a word
  for (int h = warp; h < G; h += NT / 32) {
    const size_t row = row0 + h;
    const uint64_t* lsrc = xl + row * W + lane;
    uint64_t lw = lane < W ? ld_relaxed_sys(lsrc) : 0;
    uint64_t a[8][4];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < W && (q % kSplitLanes) == q0) {
        const uint64_t* src = xo + (row * W + q) * D + 4 * v;
        ld_relaxed_sys_v2(src, a[q][0], a[q][1]);
        ld_relaxed_sys_v2(src + 2, a[q][2], a[q][3]);
      } else {
        a[q][0] = a[q][1] = a[q][2] = a[q][3] = 0;
      }
    }
    if (lane < W) {
      while (!x_valid(lw, epoch) && !late) {
        if (globaltimer() - t0 > limit) {
          late = true;
        } else {
          __nanosleep(32);
          lw = ld_relaxed_sys(lsrc);
        }
      }
    }
    const float lq = (lane < W && x_valid(lw, epoch)) ? x_value(lw) : -INFINITY;
    float M = lq;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float wq = (M != -INFINITY && lq != -INFINITY) ? ex2((lq - M) * kLog2e) : 0.f;
    float S = wq;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) S += __shfl_xor_sync(0xffffffffu, S, off);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float w = __shfl_sync(0xffffffffu, wq, q);  // 0 for absent / empty partials
      if (q < W && (q % kSplitLanes) == q0 && w > 0.f) {
        bool ok = x_valid(a[q][0], epoch) && x_valid(a[q][1], epoch) &&
                  x_valid(a[q][2], epoch) && x_valid(a[q][3], epoch);
        while (!ok && !late) {
          if (globaltimer() - t0 > limit) {
            late = true;
          } else {
            __nanosleep(32);
            const uint64_t* src = xo + (row * W + q) * D + 4 * v;
            ld_relaxed_sys_v2(src, a[q][0], a[q][1]);
            ld_relaxed_sys_v2(src + 2, a[q][2], a[q][3]);
            ok = x_valid(a[q][0], epoch) && x_valid(a[q][1], epoch) &&
                 x_valid(a[q][2], epoch) && x_valid(a[q][3], epoch);
          }
        }
        if (ok) {
          acc.x += w * x_value(a[q][0]); acc.y += w * x_value(a[q][1]);
          acc.z += w * x_value(a[q][2]); acc.w += w * x_value(a[q][3]);
        }
      }
    }
#pragma unroll
    for (int off = kLanesPerRow; off < 32; off <<= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
    }
    const float inv = S > 0.f ? 1.f / S : 0.f;
    const float total = (M != -INFINITY && S > 0.f) ? M + logf(S) : -INFINITY;
    if (q0 == 0) {
      const size_t base = row * D + 4 * v;
      store_out(p.out, p.out_dtype, base + 0, acc.x * inv);
      store_out(p.out, p.out_dtype, base + 1, acc.y * inv);
      store_out(p.out, p.out_dtype, base + 2, acc.z * inv);
      store_out(p.out, p.out_dtype, base + 3, acc.w * inv);
    }
    if (lane == 0) {
      if (p.out_lse) p.out_lse[row] = total;
      if (p.lse_final) p.lse_final[row] = total;
    }
  }
  if (late) atomicOr(p.err, 0x2u);
}

// Merges the world partials of this unit (its own partial is already stored
// into every rank's inbox) and, with a device epoch, advances the epoch once
// the launch's last unit is done.
template <int D, int NT>
__device__ __forceinline__ void x_finish(const DecodeParams& p, size_t row0, int G,
                                         uint32_t epoch) {
  x_merge<D, NT>(p, row0, G, epoch);
  // A device epoch advances when the last unit of the launch is done: every
  // CTA of the launch has read the epoch by then (at its start).
  if (p.x_epoch_dev != nullptr && threadIdx.x == 0) {
    __threadfence();
    uint32_t* ticket = p.err + 1;
    const uint32_t units = (uint32_t)p.batch * (uint32_t)p.kv_heads;
    if (atomicAdd(ticket, 1u) == units - 1u) {
      atomicExch(ticket, 0u);
      atomicAdd(p.x_epoch_dev, 1u);
    }
  }
}

// Chunk c of a (sequence, kv head) with nb blocks and chunks of cmax blocks:
// blocks [base, base + cnt), front to back.  (Measured on B200 and rejected:
// handing the chunks out back to front or alternately from both ends, which
// makes every CTA stream HOT tiles at once and then WARM tiles at once
// instead of a mix, +4 % on configuration 4; short chunks for the last part
// of each context, -2 % on configuration 4 but +1 % on configuration 5 and
// +9 % on configuration 3 at 8 sequences.)
__device__ __forceinline__ void chunk_span(int c, int nb, int cmax, int& base, int& cnt) {
  base = c * cmax;
  cnt = max(0, min(cmax, nb - base));
}

constexpr uint32_t kMagic = 0x64646464u;  // fp16 exponent byte of 1024.0


template <int D, int BS, int FMT, int QT>
__global__ void __launch_bounds__(DecodeCfg<D, BS, FMT, QT>::kThreads, TKV_MIN_CTAS)
    decode_kernel(const __grid_constant__ DecodeParams p,
                  const __grid_constant__ CUtensorMap tm_hk,
                  const __grid_constant__ CUtensorMap tm_hv,
                  const __grid_constant__ CUtensorMap tm_wk,
                  const __grid_constant__ CUtensorMap tm_wv) {
  using Cfg = DecodeCfg<D, BS, FMT, QT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBars);
  uint64_t* empty_bar = full_bar + Cfg::kStages;
  TileInfo* info = reinterpret_cast<TileInfo*>(smem + Cfg::kOffInfo);
  uint8_t* meta = smem + Cfg::kOffMeta;
  // misc: [0] cold tokens, [1] last-CTA flag, [2] exchange epoch, [8..16) query exponents,
  // [16..24) per-head sums of the staged fp16 query (as float bits)
  int* misc = reinterpret_cast<int*>(smem + Cfg::kOffMisc);
  __half* sqh = reinterpret_cast<__half*>(smem + Cfg::kOffQ);
  __half* sqw = reinterpret_cast<__half*>(smem + Cfg::kOffQ + Cfg::kQBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int seq = blockIdx.z;
  const int G = p.groups;
  const int Hq = p.num_heads;

  // Set-up that reads no global memory (barriers, descriptor prefetch) runs
  // before the dependency wait, so that under programmatic dependent launch it
  // overlaps the previous kernel's tail; everything a previous kernel may have
  // written -- tables, block counts, query, workspace counters, the exchange
  // epoch -- is read after it.
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    fence_mbar_init();
  } else if (threadIdx.x == 32) {
    prefetch_tensormap(&tm_hk);
    prefetch_tensormap(&tm_hv);
    prefetch_tensormap(&tm_wk);
    prefetch_tensormap(&tm_wv);
  }
  pdl_launch_dependents();
#if TKV_PREFETCH
  // L2 prefetch of the first tiles of this CTA's first chunk before the
  // dependency wait, by the CTAs of the first wave: under programmatic
  // dependent launch they stream in during the previous kernel's tail.  The table entries read here may still
  // change until the wait; they only choose what is prefetched (a stale entry
  // costs a useless prefetch, never a wrong value), and everything the result
  // depends on is read again after the wait.
  if (warp == 1 && (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z)) <
                       p.prefetch_ctas) {
    const int nbg = max(0, min(p.nb_dev ? __ldcg(p.nb_dev + seq) : p.nb_uniform, p.max_blocks));
    const int i = (p.splits > 1 ? split * p.chunk : 0) + lane;
    if (lane < min(p.chunk, Cfg::kStages) && i < nbg) {
      const size_t toff = (size_t)seq * p.table_stride + i;
      const int slot = __ldcg(p.table + toff);
      const int st = __ldcg(p.states + toff);
      const int len = __ldcg(p.lengths + toff);
      if (len > 0 && slot >= 0) {
        const int32_t row = (slot * p.kv_heads + kvh) * BS;
        if (st == 0 && slot < p.hot_slots) {
#if TKV_HOT_3D
          tma_prefetch_3d(&tm_hk, 0, row, 0);
          tma_prefetch_3d(&tm_hv, 0, row, 0);
#else
#pragma unroll
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_prefetch_2d(&tm_hk, hh * 64, row);
            tma_prefetch_2d(&tm_hv, hh * 64, row);
          }
#endif
        } else if (st == 1 && slot < p.warm_slots) {
          tma_prefetch_2d(&tm_wk, 0, row);
          tma_prefetch_2d(&tm_wv, 0, row);
          if (FMT == kFmtR) {
            bulk_prefetch_l2(reinterpret_cast<const __half*>(p.k_scale) + row, BS * 2);
            bulk_prefetch_l2(reinterpret_cast<const __half*>(p.k_zero) + row, BS * 2);
            bulk_prefetch_l2(reinterpret_cast<const __half*>(p.v_scale) + row, BS * 2);
            bulk_prefetch_l2(reinterpret_cast<const __half*>(p.v_zero) + row, BS * 2);
          }
        }
      }
    }
  }
#endif
  pdl_wait();

  int nb = p.nb_dev ? p.nb_dev[seq] : p.nb_uniform;
  nb = max(0, min(nb, p.max_blocks));
  // Work is handed out in chunks of p.chunk (8, 16 or 32) blocks, one block
  // per producer lane.  With several splits, split s starts on chunk s and
  // then the CTAs of a (sequence, kv head) claim further chunks from a shared
  // atomic counter, so CTAs on less loaded SMs (or launched earlier) take more
  // of them and HOT-heavy chunks (sink, recent window) do not pile up on one
  // CTA; the merge is order-free.  (Measured: shrinking the claims towards the
  // end costs more in claim latency than it gains in balance.)  One split
  // walks the chunks in order.
  const int cmax = p.chunk;
  const bool dynamic = p.splits > 1;
  const size_t unit = (size_t)seq * p.kv_heads + kvh;
  uint32_t* chunk_ctr = p.counters + (size_t)p.batch * p.kv_heads + unit;
  const int32_t* trow = p.table + (size_t)seq * p.table_stride;
  const int32_t* srow = p.states + (size_t)seq * p.table_stride;
  const int32_t* lrow = p.lengths + (size_t)seq * p.table_stride;
  // the table entries of the producer's first chunk are requested before the
  // prologue; chunk `nchunk` = blocks [nbase, nbase + ncnt) is the one whose
  // entries are loading
  int nchunk = dynamic ? split : 0;
  int nbase = 0, ncnt = 0;
  int nslot = -1, nstate = 2, nlen = 0;
  if (warp == 0) {
    chunk_span(nchunk, nb, cmax, nbase, ncnt);
    if (lane < ncnt) {
      nslot = __ldg(trow + nbase + lane);
      nstate = __ldg(srow + nbase + lane);
      nlen = __ldg(lrow + nbase + lane);
    }
  }

  if (threadIdx.x == 0) {
    misc[0] = 0;
    misc[1] = 0;
    // the exchange epoch of this call (see x_o): a value, never an address,
    // is taken from the parameters
    uint32_t epoch = p.x_epoch;
    if (p.x_world > 0 && p.x_epoch_dev != nullptr) epoch = __ldcg(p.x_epoch_dev);
    misc[2] = (int)epoch;
  }
  __syncthreads();  // barriers initialised; the consumers stage the query below

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int tile = 0;
    int cold = 0;
    bool fail = false;
    // software-pipelined table reads: the next chunk is claimed and its entries
    // requested before the current chunk's tiles are issued
    while (ncnt > 0 && !fail) {
      const int base = nbase;
      const int i = base + lane;
      const bool mine = lane < ncnt;  // this lane's block of the chunk
      const int slot = nslot;
      const int st = nstate;
      const int len = max(0, min(nlen, BS));
      if (dynamic) {
        // claims beyond the first chunks of all splits
        int c = 0;
        if (lane == 0) c = (int)atomicAdd(chunk_ctr, 1u);
        nchunk = __shfl_sync(0xffffffffu, c, 0) + p.splits;
      } else {
        ++nchunk;
      }
      chunk_span(nchunk, nb, cmax, nbase, ncnt);
      nslot = -1;
      nstate = 2;
      nlen = 0;
      if (lane < ncnt) {
        nslot = __ldg(trow + nbase + lane);
        nstate = __ldg(srow + nbase + lane);
        nlen = __ldg(lrow + nbase + lane);
      }
      bool issue = mine && (st == 0 || st == 1) && len > 0;
      if (issue) {
        const int64_t cap = (st == 0) ? p.hot_slots : p.warm_slots;
        if (slot < 0 || (int64_t)slot >= cap) {
          issue = false;  // out-of-pool slot: read as zeros, reported
          atomicOr(p.err, 0x1u);
        }
      }
      if (mine && !issue) {
        cold += len;
        if (p.lse_blk != nullptr) {
          const float v = len > 0 ? logf((float)len) : -INFINITY;
          for (int h = 0; h < G; ++h)
            p.lse_blk[((size_t)seq * Hq + (size_t)kvh * G + h) * p.max_blocks + i] = v;
        }
      }
      float ks = 1.f, vs = 1.f;
      if (FMT == kFmtS && issue && st == 1) {
        const size_t mi = (size_t)slot * p.kv_heads + kvh;
        ks = __ldg(reinterpret_cast<const float*>(p.k_scale) + mi);
        vs = __ldg(reinterpret_cast<const float*>(p.v_scale) + mi);
      }
      // Lane-parallel issue: the tiles of this chunk take consecutive ring
      // positions in block order; every issuing lane handles its own tile, at
      // most kStages lanes (distinct stages) per round.
      const uint32_t mask = __ballot_sync(0xffffffffu, issue);
      const int n_issue = __popc(mask);
      const int rank = __popc(mask & ((1u << lane) - 1u));
      for (int r0 = 0; r0 < n_issue; r0 += Cfg::kStages) {
        int ok = 1;
        if (issue && rank >= r0 && rank < r0 + Cfg::kStages) {
          const int my = tile + rank;
          const int s = my % Cfg::kStages;
          const uint32_t ph = (uint32_t)(my / Cfg::kStages) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
            ok = 0;
          } else {
            const int jst = st, jlen = len, jslot = slot;
            TileInfo ti;
            ti.state = jst;
            ti.len = jlen;
            ti.block = i;
            ti.ks = ks;
            ti.vs = vs;
            info[s] = ti;
            const int32_t row = (jslot * p.kv_heads + kvh) * BS;
            uint8_t* kdst = stages + s * Cfg::kStageBytes;
            uint8_t* vdst = kdst + Cfg::kHotBytes;
            if (jst == 0) {
              mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::kHotBytes);
#if TKV_HOT_3D
              // one box {64, BS, D/64}: smem [D/64][BS][64], the same layout as
              // the per-half 2-D boxes below
              tma_load_3d(kdst, &tm_hk, 0, row, 0, &full_bar[s]);
              tma_load_3d(vdst, &tm_hv, 0, row, 0, &full_bar[s]);
#else
#pragma unroll
              for (int hh = 0; hh < D / 64; ++hh) {
                tma_load_2d(kdst + hh * BS * 128, &tm_hk, hh * 64, row, &full_bar[s]);
                tma_load_2d(vdst + hh * BS * 128, &tm_hv, hh * 64, row, &full_bar[s]);
              }
#endif
            } else {
              const uint32_t mbytes = (FMT == kFmtR) ? 4 * BS * 2 : 0;
              mbar_arrive_expect_tx(&full_bar[s], 2 * BS * D + mbytes);
              tma_load_2d(kdst, &tm_wk, 0, row, &full_bar[s]);
              tma_load_2d(vdst, &tm_wv, 0, row, &full_bar[s]);
              if (FMT == kFmtR) {
                uint8_t* md = meta + s * Cfg::kMetaBytes;
                const __half* src[4] = {reinterpret_cast<const __half*>(p.k_scale),
                                        reinterpret_cast<const __half*>(p.k_zero),
                                        reinterpret_cast<const __half*>(p.v_scale),
                                        reinterpret_cast<const __half*>(p.v_zero)};
#pragma unroll
                for (int m = 0; m < 4; ++m)
                  bulk_load(md + m * BS * 2, src[m] + row, BS * 2, &full_bar[s]);
              }
            }
          }
        }
        if (!__all_sync(0xffffffffu, ok)) {
          fail = true;
          break;
        }
      }
      tile += n_issue;
    }
    // one end-of-stream marker per consumer warp (kConsumers <= kStages lanes)
    if (!fail && lane < Cfg::kConsumers) {
      const int my = tile + lane;
      const int s = my % Cfg::kStages;
      const uint32_t ph = (uint32_t)(my / Cfg::kStages) & 1u;
      if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
        fail = true;
      } else {
        info[s].state = -1;
        mbar_arrive(&full_bar[s]);
      }
    }
    fail = __any_sync(0xffffffffu, fail);
    if (fail && lane == 0) atomicOr(p.err, 0x2u);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) cold += __shfl_xor_sync(0xffffffffu, cold, off);
    if (lane == 0) misc[0] = cold;
  }

  // ------------------------------------------------------------ consumers
  float m2[2] = {-INFINITY, -INFINITY};  // running max (log2 domain), heads 2t, 2t+1
  float l[2] = {0.f, 0.f};               // this lane's share of the denominator
  // O^T accumulator; m-tile 4kk+i holds rows d = 64kk + 8g + i (row g) and
  // 64kk + 8g + 4 + i (row g+8), columns = heads 2t, 2t+1
  float acc[Cfg::kKS][4];
#pragma unroll
  for (int i = 0; i < Cfg::kKS; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  // WARM V enters the tensor cores as exact fp16 (1024 + code), so acc also
  // collects sum_t w_t (1024 + zero_t) per head (w = P * V scale as the MMA
  // sees it, fp16); vcorr is this lane's share of that sum, heads 2t, 2t+1.
  // It is taken out of acc every kVcorrFlush WARM tiles and once more before
  // the merge.  Left in until the end, the offset (about 1024 x the weights)
  // grows with the tokens a warp walks, and the fp32 rounding of acc costs the
  // result bits in proportion.
  float vcorr[2] = {0.f, 0.f};
  int warm_run = 0;  // WARM tiles since vcorr was last taken out of acc

  const int g = lane >> 2;
  const int t = lane & 3;
  if (warp > 0) {
    const int cw = warp - 1;
    stage_query<D, QT, Cfg::kConsumers>(p, seq, kvh, sqh, sqw, misc + 8);
    const uint32_t sqh_u = smem_u32(sqh);
    const uint32_t sqw_u = smem_u32(sqw);
    float qmul[2], qsum[2];  // logit scale (log2 domain) and query sum of heads 2t, 2t+1
    qmul[0] = ldexpf(p.scale_log2, misc[8 + 2 * t]);
    qmul[1] = ldexpf(p.scale_log2, misc[8 + 2 * t + 1]);
    qsum[0] = __int_as_float(misc[16 + 2 * t]);
    qsum[1] = __int_as_float(misc[16 + 2 * t + 1]);
    // Lazy rescaling: the running max only moves when a logit exceeds it by
    // more than 2^8 (log2 domain), so P stays <= 256 and most tiles skip the
    // cross-lane max and the accumulator rescale.
    constexpr float kLazy = 8.f;

    for (int it = cw;; it += Cfg::kConsumers) {
      const int s = it % Cfg::kStages;
      const uint32_t ph = (uint32_t)(it / Cfg::kStages) & 1u;
      if (!mbar_wait(&full_bar[s], ph)) {
        if (lane == 0) atomicOr(p.err, 0x2u);
        break;
      }
      const TileInfo ti = info[s];
      if (ti.state < 0) break;
      // every shared-memory fragment address of this tile depends on a token
      // taken after the wait, so no load of the stage (or of the staged
      // query) is scheduled before the data has landed
      const uint32_t tok = wait_token();
      const uint32_t kb = after(smem_u32(stages + s * Cfg::kStageBytes), tok);
      const uint32_t vb = kb + Cfg::kHotBytes;
      const uint32_t sqh_t = after(sqh_u, tok);
      const uint32_t sqw_t = after(sqw_u, tok);
      const __half* ms = reinterpret_cast<const __half*>(meta + s * Cfg::kMetaBytes);
      const bool hot = ti.state == 0;

      // ---- logits S^T[token, head] for this block
      float x[Cfg::kSub][4];
#pragma unroll
      for (int u = 0; u < Cfg::kSub; ++u) x[u][0] = x[u][1] = x[u][2] = x[u][3] = 0.f;
      if (hot) {
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const int r = 16 * u + (lane & 7) + (((lane >> 3) & 1) << 3);
          float xa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int m = 0; m < Cfg::kKS / 2; ++m) {
            uint32_t b00, b01, b10, b11;
            load_qfrag<D>(sqh_t, lane, m, b00, b01, b10, b11);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int ks = 2 * m + kk;
              const int ch = 2 * ks + (lane >> 4);
              const uint32_t addr =
                  kb + (ch >> 3) * (BS * 128) + r * 128 + ((((ch & 7) ^ (lane & 7))) << 4);
              uint32_t a0, a1, a2, a3;
              ldsm_x4(addr, a0, a1, a2, a3);
              if (kk)
                mma_16816(xa, a0, a1, a2, a3, b10, b11);
              else
                mma_16816(x[u], a0, a1, a2, a3, b00, b01);
            }
          }
          x[u][0] = (x[u][0] + xa[0]) * qmul[0];
          x[u][1] = (x[u][1] + xa[1]) * qmul[1];
          x[u][2] = (x[u][2] + xa[2]) * qmul[0];
          x[u][3] = (x[u][3] + xa[3]) * qmul[1];
        }
      } else {
        // codes enter the tensor cores as exact fp16 (1024 + code); the zero
        // point comes out as logit = s * (sum((1024 + q) Q) - (1024 + z) sum(Q))
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const int r0 = 16 * u + g;
          const int r1 = r0 + 8;
          float sc0, sc1, zc0, zc1;
          if (FMT == kFmtR) {
            sc0 = __half2float(ms[r0]);
            sc1 = __half2float(ms[r1]);
            zc0 = 1024.f + __half2float(ms[BS + r0]);
            zc1 = 1024.f + __half2float(ms[BS + r1]);
          } else {
            sc0 = sc1 = ti.ks;
            zc0 = zc1 = 1152.f;  // 1024 + 128: int8 codes are flipped to biased bytes
          }
          uint32_t w0[Cfg::kKS], w1[Cfg::kKS];
#pragma unroll
          for (int j = 0; j < D / 64; ++j) {
            const uint32_t c = (D == 128) ? (2 * t + j) : t;
            const uint4 v0 = lds128(kb + swz<Cfg::kWarmSwz>(r0 * D + c * 16));
            const uint4 v1 = lds128(kb + swz<Cfg::kWarmSwz>(r1 * D + c * 16));
            w0[4 * j + 0] = v0.x; w0[4 * j + 1] = v0.y; w0[4 * j + 2] = v0.z; w0[4 * j + 3] = v0.w;
            w1[4 * j + 0] = v1.x; w1[4 * j + 1] = v1.y; w1[4 * j + 2] = v1.z; w1[4 * j + 3] = v1.w;
          }
          float xa[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int m = 0; m < Cfg::kKS / 2; ++m) {
            uint32_t bq[2][2];
            load_qfrag<D>(sqw_t, lane, m, bq[0][0], bq[0][1], bq[1][0], bq[1][1]);
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int ks = 2 * m + kk;
              uint32_t c0 = w0[ks], c1 = w1[ks];
              if (FMT == kFmtS) {
                c0 ^= 0x80808080u;
                c1 ^= 0x80808080u;
              }
              const uint32_t a0 = __byte_perm(c0, kMagic, 0x4140);
              const uint32_t a2 = __byte_perm(c0, kMagic, 0x4342);
              const uint32_t a1 = __byte_perm(c1, kMagic, 0x4140);
              const uint32_t a3 = __byte_perm(c1, kMagic, 0x4342);
              if (kk)
                mma_16816(xa, a0, a1, a2, a3, bq[1][0], bq[1][1]);
              else
                mma_16816(x[u], a0, a1, a2, a3, bq[0][0], bq[0][1]);
            }
          }
          x[u][0] = (x[u][0] + xa[0] - zc0 * qsum[0]) * (qmul[0] * sc0);
          x[u][1] = (x[u][1] + xa[1] - zc0 * qsum[1]) * (qmul[1] * sc0);
          x[u][2] = (x[u][2] + xa[2] - zc1 * qsum[0]) * (qmul[0] * sc1);
          x[u][3] = (x[u][3] + xa[3] - zc1 * qsum[1]) * (qmul[1] * sc1);
        }
      }

      // ---- V fragments to registers; then the stage can be handed back.
      // Lane (g, t) needs dims 64kk + 8g .. +7 of tokens 2t, 2t+1, 2t+8, 2t+9:
      // one 16-byte load per token (HOT fp16) or one 8-byte load (WARM codes,
      // plus the per-token V scale and (1024 + zero)).
      uint32_t vf[Cfg::kSub][D / 64][16];
      float vsc[Cfg::kSub][2];
      float vzc[Cfg::kSub][2];  // 1024 + V zero point of tokens g, g + 8
      if (hot) {
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const int r0 = 16 * u + 2 * t;
#pragma unroll
          for (int kk = 0; kk < D / 64; ++kk) {
            const int rr[4] = {r0, r0 + 1, r0 + 8, r0 + 9};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 v = lds128(vb + swz<7>((kk * BS + rr[j]) * 128 + 16 * g));
              vf[u][kk][4 * j + 0] = v.x;
              vf[u][kk][4 * j + 1] = v.y;
              vf[u][kk][4 * j + 2] = v.z;
              vf[u][kk][4 * j + 3] = v.w;
            }
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const int r0 = 16 * u + 2 * t;
          if (FMT == kFmtR) {
            vsc[u][0] = __half2float(ms[2 * BS + 16 * u + g]);
            vsc[u][1] = __half2float(ms[2 * BS + 16 * u + g + 8]);
            vzc[u][0] = 1024.f + __half2float(ms[3 * BS + 16 * u + g]);
            vzc[u][1] = 1024.f + __half2float(ms[3 * BS + 16 * u + g + 8]);
          } else {
            vsc[u][0] = vsc[u][1] = ti.vs;
            vzc[u][0] = vzc[u][1] = 1152.f;  // int8 codes are flipped to biased bytes
          }
#pragma unroll
          for (int kk = 0; kk < D / 64; ++kk) {
            const int rr[4] = {r0, r0 + 1, r0 + 8, r0 + 9};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint2 v = lds64(vb + swz<Cfg::kWarmSwz>(rr[j] * D + 64 * kk + 8 * g));
              vf[u][kk][2 * j] = v.x;
              vf[u][kk][2 * j + 1] = v.y;
            }
          }
        }
      }
#if TKV_EARLY_RELEASE
      // the stage's data must be in registers before the stage is handed
      // back: the logits (K) and the V fragments are inputs of the release
#pragma unroll
      for (int u = 0; u < Cfg::kSub; ++u) {
#pragma unroll
        for (int j = 0; j < 4; ++j) hold(x[u][j]);
#pragma unroll
        for (int kk = 0; kk < D / 64; ++kk)
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (hot || j < 8) hold(vf[u][kk][j]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
#endif

      // ---- mask tokens >= len, online softmax (log2 domain)
      float lm[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int u = 0; u < Cfg::kSub; ++u) {
        if (16 * u + g >= ti.len) x[u][0] = x[u][1] = -INFINITY;
        if (16 * u + g + 8 >= ti.len) x[u][2] = x[u][3] = -INFINITY;
        lm[0] = fmaxf(lm[0], fmaxf(x[u][0], x[u][2]));
        lm[1] = fmaxf(lm[1], fmaxf(x[u][1], x[u][3]));
      }
      const bool grow = lm[0] > m2[0] + kLazy || lm[1] > m2[1] + kLazy;
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          lm[0] = fmaxf(lm[0], __shfl_xor_sync(0xffffffffu, lm[0], off));
          lm[1] = fmaxf(lm[1], __shfl_xor_sync(0xffffffffu, lm[1], off));
        }
        float alpha[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float mn = fmaxf(m2[j], lm[j]);
          alpha[j] = ex2(m2[j] - mn);
          m2[j] = mn;
          l[j] *= alpha[j];
        }
#pragma unroll
        for (int i = 0; i < Cfg::kKS; ++i) {
          acc[i][0] *= alpha[0]; acc[i][1] *= alpha[1];
          acc[i][2] *= alpha[0]; acc[i][3] *= alpha[1];
        }
        vcorr[0] *= alpha[0];
        vcorr[1] *= alpha[1];
      }
      float pr[Cfg::kSub][4];
      float ps[2] = {0.f, 0.f};
#pragma unroll
      for (int u = 0; u < Cfg::kSub; ++u) {
        pr[u][0] = ex2(x[u][0] - m2[0]);
        pr[u][1] = ex2(x[u][1] - m2[1]);
        pr[u][2] = ex2(x[u][2] - m2[0]);
        pr[u][3] = ex2(x[u][3] - m2[1]);
        ps[0] += pr[u][0] + pr[u][2];
        ps[1] += pr[u][1] + pr[u][3];
      }
      l[0] += ps[0];
      l[1] += ps[1];
      if (p.lse_blk != nullptr) {
        float bsum[2] = {ps[0], ps[1]};
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          bsum[0] += __shfl_xor_sync(0xffffffffu, bsum[0], off);
          bsum[1] += __shfl_xor_sync(0xffffffffu, bsum[1], off);
        }
        if (g == 0) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int h = 2 * t + j;
            if (h < G)
              p.lse_blk[((size_t)seq * Hq + (size_t)kvh * G + h) * p.max_blocks + ti.block] =
                  (m2[j] + lg2(bsum[j])) * kLn2;
          }
        }
      }

      // ---- O^T += V^T P^T (V fragments are already in registers)
      // m-tile 4kk+i: A rows g / g+8 are dims 64kk + 8g + i / + 4 + i, A columns
      // are the token pairs (2t, 2t+1) and (2t+8, 2t+9).
      if (hot) {
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const uint32_t pb0 = movmatrix_t(pack_half2(pr[u][0], pr[u][1]));
          const uint32_t pb1 = movmatrix_t(pack_half2(pr[u][2], pr[u][3]));
#pragma unroll
          for (int kk = 0; kk < D / 64; ++kk) {
            const uint32_t* f = vf[u][kk];  // token j: dims (0,1) (2,3) (4,5) (6,7) at 4j..4j+3
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
              const int w = i >> 1;
              const uint32_t a0 = __byte_perm(f[0 + w], f[4 + w], sel);
              const uint32_t a1 = __byte_perm(f[2 + w], f[6 + w], sel);
              const uint32_t a2 = __byte_perm(f[8 + w], f[12 + w], sel);
              const uint32_t a3 = __byte_perm(f[10 + w], f[14 + w], sel);
              mma_16816(acc[4 * kk + i], a0, a1, a2, a3, pb0, pb1);
            }
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < Cfg::kSub; ++u) {
          const uint32_t w01 = pack_half2(pr[u][0] * vsc[u][0], pr[u][1] * vsc[u][0]);
          const uint32_t w23 = pack_half2(pr[u][2] * vsc[u][1], pr[u][3] * vsc[u][1]);
          const uint32_t pb0 = movmatrix_t(w01);
          const uint32_t pb1 = movmatrix_t(w23);
          {
            const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&w01));
            const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&w23));
            vcorr[0] = fmaf(f01.x, vzc[u][0], fmaf(f23.x, vzc[u][1], vcorr[0]));
            vcorr[1] = fmaf(f01.y, vzc[u][0], fmaf(f23.y, vzc[u][1], vcorr[1]));
          }
#pragma unroll
          for (int kk = 0; kk < D / 64; ++kk) {
            // token j: codes of dims 0..3 in word 2j, dims 4..7 in word 2j+1
            uint32_t f[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) f[k] = vf[u][kk][k];
            if (FMT == kFmtS) {
#pragma unroll
              for (int k = 0; k < 8; ++k) f[k] ^= 0x80808080u;
            }
            // interleave the two tokens of each k pair byte by byte
            const uint32_t xl[2] = {__byte_perm(f[0], f[2], 0x5140), __byte_perm(f[0], f[2], 0x7362)};
            const uint32_t xh[2] = {__byte_perm(f[1], f[3], 0x5140), __byte_perm(f[1], f[3], 0x7362)};
            const uint32_t yl[2] = {__byte_perm(f[4], f[6], 0x5140), __byte_perm(f[4], f[6], 0x7362)};
            const uint32_t yh[2] = {__byte_perm(f[5], f[7], 0x5140), __byte_perm(f[5], f[7], 0x7362)};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t sel = (i & 1) ? 0x4342u : 0x4140u;
              const uint32_t a0 = __byte_perm(xl[i >> 1], kMagic, sel);
              const uint32_t a1 = __byte_perm(xh[i >> 1], kMagic, sel);
              const uint32_t a2 = __byte_perm(yl[i >> 1], kMagic, sel);
              const uint32_t a3 = __byte_perm(yh[i >> 1], kMagic, sel);
              mma_16816(acc[4 * kk + i], a0, a1, a2, a3, pb0, pb1);
            }
          }
        }
        if (++warm_run == kVcorrFlush) {
          warm_run = 0;
          float vc0 = vcorr[0], vc1 = vcorr[1];
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            vc0 += __shfl_xor_sync(0xffffffffu, vc0, off);
            vc1 += __shfl_xor_sync(0xffffffffu, vc1, off);
          }
#pragma unroll
          for (int i = 0; i < Cfg::kKS; ++i) {
            acc[i][0] -= vc0; acc[i][1] -= vc1;
            acc[i][2] -= vc0; acc[i][3] -= vc1;
          }
          vcorr[0] = 0.f;
          vcorr[1] = 0.f;
        }
      }
#if !TKV_EARLY_RELEASE
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
#endif
    }
  }

  // ------------------------------------------------------------ CTA merge
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], off);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], off);
    vcorr[0] += __shfl_xor_sync(0xffffffffu, vcorr[0], off);
    vcorr[1] += __shfl_xor_sync(0xffffffffu, vcorr[1], off);
  }
#pragma unroll
  for (int i = 0; i < Cfg::kKS; ++i) {
    acc[i][0] -= vcorr[0]; acc[i][1] -= vcorr[1];
    acc[i][2] -= vcorr[0]; acc[i][3] -= vcorr[1];
  }
  __syncthreads();  // every stage is drained: the ring becomes merge scratch
  float* sm_m = reinterpret_cast<float*>(stages);
  float* sm_l = sm_m + Cfg::kConsumers * kMaxGroups;
  float* sm_acc = sm_l + Cfg::kConsumers * kMaxGroups;
  if (warp > 0) {
    const int cw = warp - 1;
    if (g == 0) {
      sm_m[cw * kMaxGroups + 2 * t] = m2[0];
      sm_m[cw * kMaxGroups + 2 * t + 1] = m2[1];
      sm_l[cw * kMaxGroups + 2 * t] = l[0];
      sm_l[cw * kMaxGroups + 2 * t + 1] = l[1];
    }
    float* a = sm_acc + (size_t)cw * kMaxGroups * D;
#pragma unroll
    for (int kk = 0; kk < D / 64; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int dlo = 64 * kk + 8 * g + i;
        const int dhi = dlo + 4;
        a[(2 * t) * D + dlo] = acc[4 * kk + i][0];
        a[(2 * t + 1) * D + dlo] = acc[4 * kk + i][1];
        a[(2 * t) * D + dhi] = acc[4 * kk + i][2];
        a[(2 * t + 1) * D + dhi] = acc[4 * kk + i][3];
      }
    }
  }
  __syncthreads();
  const int cold = misc[0];
  const int nsplit = p.splits;
  for (int e = threadIdx.x; e < G * D; e += Cfg::kThreads) {
    const int h = e / D;
    const int d = e - h * D;
    float M = cold > 0 ? 0.f : -INFINITY;
#pragma unroll
    for (int c = 0; c < Cfg::kConsumers; ++c) M = fmaxf(M, sm_m[c * kMaxGroups + h]);
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int c = 0; c < Cfg::kConsumers; ++c) {
      const float mc = sm_m[c * kMaxGroups + h];
      if (mc != -INFINITY) {
        const float w = ex2(mc - M);
        L += sm_l[c * kMaxGroups + h] * w;
        o += sm_acc[((size_t)c * kMaxGroups + h) * D + d] * w;
      }
    }
    if (cold > 0) L += (float)cold * ex2(-M);
    const float on = L > 0.f ? o / L : 0.f;
    const float lse = L > 0.f ? (M + lg2(L)) * kLn2 : -INFINITY;
    const size_t row = (size_t)seq * Hq + (size_t)kvh * G + h;
    if (nsplit == 1 && p.x_world > 0) {
      const uint32_t epoch = (uint32_t)misc[2];
      for (int q = 0; q < p.x_world; ++q) {
        st_relaxed_sys(x_o<D>(p, q, epoch) + (row * p.x_world + p.x_rank) * D + d, x_word(on, epoch));
        if (d == 0)
          st_relaxed_sys(x_lse<D>(p, q, epoch) + row * p.x_world + p.x_rank, x_word(lse, epoch));
      }
    } else if (nsplit == 1) {
      store_out(p.out, p.out_dtype, row * D + d, on);
      if (d == 0) {
        if (p.out_lse) p.out_lse[row] = lse;
        if (p.lse_final) p.lse_final[row] = lse;
      }
    } else {
      p.part_o[(row * nsplit + split) * D + d] = on;
      if (d == 0) p.part_lse[row * nsplit + split] = lse;
    }
  }
  if (nsplit == 1) {
    if (p.x_world > 0)
      x_finish<D, Cfg::kThreads>(p, (size_t)seq * Hq + (size_t)kvh * G, G, (uint32_t)misc[2]);
    return;
  }

  // ------------------------------------------------------------ split merge
  // The last CTA of each group of group_size splits merges the group's
  // partials; with more than one group, the last group's merger then merges
  // the group partials.  Tickets reset themselves, as does the chunk counter
  // once every CTA of the unit is done claiming.
  const int gsz = p.group_size;
  const int ngroups = (nsplit + gsz - 1) / gsz;
  const int group = split / gsz;
  const int gfirst = group * gsz;
  const int gcount = min(gsz, nsplit - gfirst);
  const size_t row0 = (size_t)seq * Hq + (size_t)kvh * G;
  float* wsl = reinterpret_cast<float*>(stages);  // merge scratch aliases the ring
  uint32_t* ticket = ngroups > 1 ? p.counters + 2 * (size_t)p.batch * p.kv_heads +
                                       unit * (size_t)ngroups + group
                                 : p.counters + unit;
  // thread 0's acquire-release increment publishes the CTA's partials (the
  // barrier orders every thread's stores before it) and, for the last CTA,
  // acquires everyone else's; the next barrier hands that on to the CTA
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atom_add_acq_rel_gpu(ticket, 1u);
    misc[1] = (prev == (uint32_t)(gcount - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (misc[1] == 0) return;
  if (ngroups == 1) {
    if (threadIdx.x == 0) {
      atomicExch(ticket, 0u);
      atomicExch(chunk_ctr, 0u);
    }
    const uint32_t epoch = (uint32_t)misc[2];
    merge_parts<D, Cfg::kThreads>(p.part_o, p.part_lse, nsplit, 0, nsplit, row0, G, wsl, p,
                                  nullptr, nullptr, 0, 0, p.x_world > 0, epoch);
    if (p.x_world > 0) x_finish<D, Cfg::kThreads>(p, row0, G, epoch);
    return;
  }
  if (threadIdx.x == 0) atomicExch(ticket, 0u);
  merge_parts<D, Cfg::kThreads>(p.part_o, p.part_lse, nsplit, gfirst, gcount, row0, G, wsl, p,
                                p.gpart_o, p.gpart_lse, ngroups, group);
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atom_add_acq_rel_gpu(p.counters + unit, 1u);
    misc[1] = (prev == (uint32_t)(ngroups - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (misc[1] == 0) return;
  if (threadIdx.x == 0) {
    atomicExch(p.counters + unit, 0u);
    atomicExch(chunk_ctr, 0u);
  }
  const uint32_t epoch = (uint32_t)misc[2];
  merge_parts<D, Cfg::kThreads>(p.gpart_o, p.gpart_lse, ngroups, 0, ngroups, row0, G, wsl, p,
                                nullptr, nullptr, 0, 0, p.x_world > 0, epoch);
  if (p.x_world > 0) x_finish<D, Cfg::kThreads>(p, row0, G, epoch);
}

// ---------------------------------------------------------------- dispatch
template <int D, int BS, int FMT, int QT>
static cudaError_t launch_one(const DecodeParams& p, const CUtensorMap maps[4],
                              cudaStream_t stream) {
  using Cfg = DecodeCfg<D, BS, FMT, QT>;
  auto kern = decode_kernel<D, BS, FMT, QT>;
  // the shared-memory opt-in is per function and device; set it once per device
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (!bit || !(attr_set.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set.fetch_or(bit, std::memory_order_relaxed);
  }
  // Programmatic dependent launch: the kernel may start while the previous
  // kernel of the stream finishes (it waits with griddepcontrol.wait before
  // touching memory that kernel could have written).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.kv_heads, p.batch);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = TKV_PDL ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, p, maps[0], maps[1], maps[2], maps[3]);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <int D, int BS, int FMT, int QT>
static cudaError_t occupancy_one(int* ctas) {
  using Cfg = DecodeCfg<D, BS, FMT, QT>;
  auto kern = decode_kernel<D, BS, FMT, QT>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, kern, Cfg::kThreads, Cfg::kSmemBytes);
}

#define TKV_DISPATCH(FN, ...)                                                       \
  do {                                                                              \
    const int key = ((head_dim == 128) << 3) | ((block_size == 32) << 2) |          \
                    ((format == kFmtS) << 1) | (query_dtype == kDtBF16);             \
    switch (key) {                                                                  \
      case 0: return FN<64, 16, kFmtR, kDtF16>(__VA_ARGS__);                        \
      case 1: return FN<64, 16, kFmtR, kDtBF16>(__VA_ARGS__);                       \
      case 2: return FN<64, 16, kFmtS, kDtF16>(__VA_ARGS__);                        \
      case 3: return FN<64, 16, kFmtS, kDtBF16>(__VA_ARGS__);                       \
      case 4: return FN<64, 32, kFmtR, kDtF16>(__VA_ARGS__);                        \
      case 5: return FN<64, 32, kFmtR, kDtBF16>(__VA_ARGS__);                       \
      case 6: return FN<64, 32, kFmtS, kDtF16>(__VA_ARGS__);                        \
      case 7: return FN<64, 32, kFmtS, kDtBF16>(__VA_ARGS__);                       \
      case 8: return FN<128, 16, kFmtR, kDtF16>(__VA_ARGS__);                       \
      case 9: return FN<128, 16, kFmtR, kDtBF16>(__VA_ARGS__);                      \
      case 10: return FN<128, 16, kFmtS, kDtF16>(__VA_ARGS__);                      \
      case 11: return FN<128, 16, kFmtS, kDtBF16>(__VA_ARGS__);                     \
      case 12: return FN<128, 32, kFmtR, kDtF16>(__VA_ARGS__);                      \
      case 13: return FN<128, 32, kFmtR, kDtBF16>(__VA_ARGS__);                     \
      case 14: return FN<128, 32, kFmtS, kDtF16>(__VA_ARGS__);                      \
      default: return FN<128, 32, kFmtS, kDtBF16>(__VA_ARGS__);                     \
    }                                                                               \
  } while (0)

cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap maps[4], int head_dim,
                          int block_size, int format, int query_dtype, cudaStream_t stream) {
  TKV_DISPATCH(launch_one, p, maps, stream);
}

cudaError_t decode_occupancy(int head_dim, int block_size, int format, int query_dtype,
                             int* ctas_per_sm) {
  TKV_DISPATCH(occupancy_one, ctas_per_sm);
}

// ---------------------------------------------------------------- merge (K2)
// One warp per row: LSE merge of `parts` normalised partials.
__global__ void merge_kernel(const MergeParams p) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  float M = -INFINITY;
  for (int i = lane; i < p.parts; i += 32) M = fmaxf(M, p.part_lse[(size_t)i * p.lse_stride + row]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float S = 0.f;
  if (M != -INFINITY)
    for (int i = lane; i < p.parts; i += 32)
      S += ex2((p.part_lse[(size_t)i * p.lse_stride + row] - M) * kLog2e);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) S += __shfl_xor_sync(0xffffffffu, S, off);
  const bool empty = !(M != -INFINITY && S > 0.f);
  for (int d = lane; d < p.head_dim; d += 32) {
    float o = 0.f;
    if (!empty) {
      for (int i = 0; i < p.parts; ++i) {
        const float l = p.part_lse[(size_t)i * p.lse_stride + row];
        if (l != -INFINITY)
          o += ex2((l - M) * kLog2e) * p.part_o[(size_t)i * p.o_stride + (size_t)row * p.head_dim + d];
      }
      o /= S;
    }
    store_out(p.out, p.out_dtype, (size_t)row * p.head_dim + d, o);
  }
  if (lane == 0 && p.out_lse) p.out_lse[row] = empty ? -INFINITY : M + logf(S);
}

cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream) {
  const int warps = 8;
  const int grid = (p.rows + warps - 1) / warps;
  merge_kernel<<<grid, warps * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- scores (K3)
// score_sums[row, b] = exp(lse_blk[row, b] - lse_final[row]) for b < nb, else 0
// (the per-block softmax mass of tierkv_triton.py:121-145 without a second K pass).
__global__ void scores_kernel(const ScoreParams p) {
  const int row = blockIdx.y;
  const int seq = row / p.num_heads;
  int nb = p.nb_dev ? p.nb_dev[seq] : p.nb_uniform;
  nb = max(0, min(nb, p.max_blocks));
  const float lf = p.lse_final[row];
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < p.max_blocks;
       b += gridDim.x * blockDim.x) {
    float v = 0.f;
    if (b < nb && lf != -INFINITY) {
      const float lb = p.lse_blk[(size_t)row * p.max_blocks + b];
      v = (lb == -INFINITY) ? 0.f : ex2((lb - lf) * kLog2e);
    }
    p.score_sums[(size_t)row * p.max_blocks + b] = v;
  }
}

cudaError_t launch_scores(const ScoreParams& p, cudaStream_t stream) {
  const int threads = 256;
  int gx = (p.max_blocks + threads - 1) / threads;
  gx = max(1, min(gx, 64));
  dim3 grid(gx, p.rows);
  scores_kernel<<<grid, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- block scores (a8)
__global__ void block_scores_kernel(const BlockScoreParams p) {
  const int seq = blockIdx.y;
  int nb = p.nb_dev ? p.nb_dev[seq] : p.nb_uniform;
  nb = max(0, min(nb, p.max_blocks));
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < p.max_blocks;
       b += gridDim.x * blockDim.x) {
    float v = 0.f;
    if (b < nb) {
      float s = 0.f;
      for (int h = 0; h < p.num_heads; ++h)
        s += p.score_sums[((size_t)seq * p.num_heads + h) * p.max_blocks + b];
      const int len = max(p.lengths[(size_t)seq * p.table_stride + b], 1);
      v = (s / (float)p.num_heads) / (float)len;
    }
    p.block_scores[(size_t)seq * p.max_blocks + b] = v;
  }
}

cudaError_t launch_block_scores(const BlockScoreParams& p, cudaStream_t stream) {
  const int threads = 256;
  int gx = (p.max_blocks + threads - 1) / threads;
  gx = max(1, min(gx, 64));
  dim3 grid(gx, p.batch);
  block_scores_kernel<<<grid, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace tkv
