// tkv_prefill.cu -- prefill block scores without materialising attention weights.
//
// The reference scores a prefilled layer's blocks from the eager attention
// weights: softmax(Q K^T * scaling + causal mask) over keys, averaged over
// (batch, heads, queries) per key, then per block of block_size keys
// (TierKVPolicyEngine.compute_block_scores, tierkv_policy.py:1378-1388, called
// from modeling_llama.py:281-289); with SDPA / flash prefill it falls back to
// a sink + recency proxy (modeling_llama.py:291-302) because the weights never
// exist.  Here the exact scores come from two tensor-core passes over Q K^T:
//   lse_kernel      per query row: LSE of the scaled, causally masked logits
//                   (skipped when the caller's flash attention returns it);
//   colsum_kernel   per key tile: sum over the group's query heads and every
//                   query row of exp(s * scaling - LSE_q) -- the attention
//                   mass each key receives -- accumulated per key;
//   block_mean_kernel  token mass / (batch * heads * queries), then the mean
//                   over each block's keys.
// Both passes use mma.m16n8k16 (f16 in, f32 accumulate) with ldmatrix-fed
// fragments; exponentials in the log2 domain.
#include <cuda_fp16.h>
#include <math.h>

#include "tkv_internal.h"
#include "tkv_ptx.cuh"

namespace tkv {

constexpr float kLog2eP = 1.4426950408889634f;

// A 64-row tile of fp16 rows [row0, row0 + 64) x D from `src` (row stride D)
// into shared memory with row stride D + 8 halves; rows >= rows_valid are zero.
template <int D>
__device__ __forceinline__ void stage_rows(__half* dst, const __half* src, int row0, int rows_valid) {
  constexpr int kVec = D / 8;  // 16-byte vectors per row
  for (int e = threadIdx.x; e < 64 * kVec; e += 128) {
    const int r = e / kVec, c = e % kVec;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row0 + r < rows_valid) v = __ldg(reinterpret_cast<const uint4*>(src + (size_t)(row0 + r) * D) + c);
    *reinterpret_cast<uint4*>(dst + r * (D + 8) + 8 * c) = v;
  }
}

// A fragments (16 rows x 16 dims, k-step ks) of a staged 64-row tile for the
// warp's rows [16 w, 16 w + 16).
template <int D>
__device__ __forceinline__ void load_afrag(uint32_t base, int w, int lane, int ks, uint32_t (&a)[4]) {
  const int j = lane >> 3, r = lane & 7;
  const uint32_t addr = base + ((16 * w + r + 8 * (j & 1)) * (D + 8) + 16 * ks + 8 * (j >> 1)) * 2;
  ldsm_x4(addr, a[0], a[1], a[2], a[3]);
}

// B fragments of k-steps 2m, 2m+1 for the 8 rows [8 n, 8 n + 8) of a staged tile.
template <int D>
__device__ __forceinline__ void load_bfrag(uint32_t base, int n, int lane, int m, uint32_t& b00,
                                           uint32_t& b01, uint32_t& b10, uint32_t& b11) {
  const uint32_t addr = base + ((8 * n + (lane & 7)) * (D + 8) + 32 * m + 8 * (lane >> 3)) * 2;
  ldsm_x4(addr, b00, b01, b10, b11);
}

// ---------------------------------------------------------------- LSE pass
// Grid (ceil(Tq / 64), num_heads, batch); warp w owns query rows 16 w .. 16 w + 15
// of the tile (the M dimension), keys run over 64-key tiles (8 n-tiles).
template <int D>
__global__ void __launch_bounds__(128) lse_kernel(const PrefillParams p) {
  __shared__ __align__(16) __half sq[64 * (D + 8)];
  __shared__ __align__(16) __half sk[64 * (D + 8)];
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int kvh = h / p.groups;
  const __half* q = reinterpret_cast<const __half*>(p.q) + ((size_t)b * p.num_heads + h) * p.tq * D;
  const __half* k = reinterpret_cast<const __half*>(p.k) + ((size_t)b * p.kv_heads + kvh) * p.tk * D;
  stage_rows<D>(sq, q, qt * 64, p.tq);
  __syncthreads();
  uint32_t afr[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) load_afrag<D>(smem_u32(sq), warp, lane, ks, afr[ks]);
  const float c = p.scaling * kLog2eP;
  // this thread's rows: query 16 w + g and 16 w + g + 8 (positions with the causal offset)
  const int q_lo = qt * 64 + 16 * warp + g, q_hi = q_lo + 8;
  const int pos_lo = q_lo + p.q_offset, pos_hi = q_hi + p.q_offset;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const int last_key = min(p.tk, (p.causal ? qt * 64 + 63 + p.q_offset + 1 : p.tk));
  for (int k0 = 0; k0 < last_key; k0 += 64) {
    __syncthreads();
    stage_rows<D>(sk, k, k0, p.tk);
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 4; ++i) s[n][i] = 0.f;
#pragma unroll
      for (int m = 0; m < D / 32; ++m) {
        uint32_t b00, b01, b10, b11;
        load_bfrag<D>(smem_u32(sk), n, lane, m, b00, b01, b10, b11);
        mma_16816(s[n], afr[2 * m][0], afr[2 * m][1], afr[2 * m][2], afr[2 * m][3], b00, b01);
        mma_16816(s[n], afr[2 * m + 1][0], afr[2 * m + 1][1], afr[2 * m + 1][2], afr[2 * m + 1][3],
                  b10, b11);
      }
    }
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int key = k0 + 8 * n + 2 * t + i;
        const bool ok_lo = key < p.tk && (!p.causal || key <= pos_lo);
        const bool ok_hi = key < p.tk && (!p.causal || key <= pos_hi);
        s[n][i] = ok_lo ? s[n][i] * c : -INFINITY;
        s[n][2 + i] = ok_hi ? s[n][2 + i] * c : -INFINITY;
        mx_lo = fmaxf(mx_lo, s[n][i]);
        mx_hi = fmaxf(mx_hi, s[n][2 + i]);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float nm_lo = fmaxf(m_lo, mx_lo), nm_hi = fmaxf(m_hi, mx_hi);
    if (nm_lo != -INFINITY) l_lo *= ex2(m_lo - nm_lo);
    if (nm_hi != -INFINITY) l_hi *= ex2(m_hi - nm_hi);
    m_lo = nm_lo;
    m_hi = nm_hi;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (m_lo != -INFINITY) l_lo += ex2(s[n][i] - m_lo);
        if (m_hi != -INFINITY) l_hi += ex2(s[n][2 + i] - m_hi);
      }
    }
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  if (t == 0) {
    float* out = p.lse + ((size_t)b * p.num_heads + h) * p.tq;
    const float kLn2 = 0.6931471805599453f;
    if (q_lo < p.tq) out[q_lo] = l_lo > 0.f ? (m_lo + lg2(l_lo)) * kLn2 : -INFINITY;
    if (q_hi < p.tq) out[q_hi] = l_hi > 0.f ? (m_hi + lg2(l_hi)) * kLn2 : -INFINITY;
  }
}

// ---------------------------------------------------------------- column sums
// Grid (ceil(Tk / 64), kv_heads, batch); warp w owns keys 16 w .. 16 w + 15 of
// the tile (the M dimension of S^T = K Q^T); the loop runs over the group's
// query heads and the 64-row query tiles that can see the tile's keys.
template <int D>
__global__ void __launch_bounds__(128) colsum_kernel(const PrefillParams p) {
  __shared__ __align__(16) __half sk[64 * (D + 8)];
  __shared__ __align__(16) __half sq[64 * (D + 8)];
  __shared__ float slse[64];
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const __half* k = reinterpret_cast<const __half*>(p.k) + ((size_t)b * p.kv_heads + kvh) * p.tk * D;
  stage_rows<D>(sk, k, kt * 64, p.tk);
  __syncthreads();
  uint32_t afr[D / 16][4];
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) load_afrag<D>(smem_u32(sk), warp, lane, ks, afr[ks]);
  const float c = p.scaling * kLog2eP;
  const int key_lo = kt * 64 + 16 * warp + g, key_hi = key_lo + 8;
  float sum_lo = 0.f, sum_hi = 0.f;
  // the first query that sees this tile's first key
  const int q_first = p.causal ? max(0, kt * 64 - p.q_offset) : 0;
  for (int hh = 0; hh < p.groups; ++hh) {
    const int h = kvh * p.groups + hh;
    const __half* q = reinterpret_cast<const __half*>(p.q) + ((size_t)b * p.num_heads + h) * p.tq * D;
    const float* lse = p.lse + ((size_t)b * p.num_heads + h) * p.tq;
    for (int q0 = (q_first / 64) * 64; q0 < p.tq; q0 += 64) {
      __syncthreads();
      stage_rows<D>(sq, q, q0, p.tq);
      if (threadIdx.x < 64) {
        const int qi = q0 + threadIdx.x;
        slse[threadIdx.x] = qi < p.tq ? lse[qi] * kLog2eP : INFINITY;  // +inf: no mass
      }
      __syncthreads();
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int m = 0; m < D / 32; ++m) {
          uint32_t b00, b01, b10, b11;
          load_bfrag<D>(smem_u32(sq), n, lane, m, b00, b01, b10, b11);
          mma_16816(s, afr[2 * m][0], afr[2 * m][1], afr[2 * m][2], afr[2 * m][3], b00, b01);
          mma_16816(s, afr[2 * m + 1][0], afr[2 * m + 1][1], afr[2 * m + 1][2], afr[2 * m + 1][3],
                    b10, b11);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int ql = 8 * n + 2 * t + i;          // query row in the tile
          const int pos = q0 + ql + p.q_offset;      // its position
          const float l2 = slse[ql];
          if (key_lo < p.tk && (!p.causal || key_lo <= pos)) sum_lo += ex2(s[i] * c - l2);
          if (key_hi < p.tk && (!p.causal || key_hi <= pos)) sum_hi += ex2(s[2 + i] * c - l2);
        }
      }
    }
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    sum_lo += __shfl_xor_sync(0xffffffffu, sum_lo, off);
    sum_hi += __shfl_xor_sync(0xffffffffu, sum_hi, off);
  }
  if (t == 0) {
    if (key_lo < p.tk) atomicAdd(p.token_mass + key_lo, sum_lo);
    if (key_hi < p.tk) atomicAdd(p.token_mass + key_hi, sum_hi);
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

cudaError_t launch_prefill_lse(const PrefillParams& p, cudaStream_t stream) {
  const dim3 grid((unsigned)((p.tq + 63) / 64), (unsigned)p.num_heads, (unsigned)p.batch);
  if (p.head_dim == 128) lse_kernel<128><<<grid, 128, 0, stream>>>(p);
  else if (p.head_dim == 64) lse_kernel<64><<<grid, 128, 0, stream>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_prefill_scores(const PrefillParams& p, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(p.token_mass, 0, sizeof(float) * (size_t)p.tk, stream);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((p.tk + 63) / 64), (unsigned)p.kv_heads, (unsigned)p.batch);
  if (p.head_dim == 128) colsum_kernel<128><<<grid, 128, 0, stream>>>(p);
  else if (p.head_dim == 64) colsum_kernel<64><<<grid, 128, 0, stream>>>(p);
  else return cudaErrorInvalidValue;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int nb = (p.tk + p.block_size - 1) / p.block_size;
  const float inv = 1.f / ((float)p.batch * (float)p.num_heads * (float)p.tq);
  block_mean_kernel<<<(nb + 127) / 128, 128, 0, stream>>>(p.token_mass, p.tk, p.block_size, inv,
                                                          p.block_scores);
  return cudaGetLastError();
}

}  // namespace tkv
