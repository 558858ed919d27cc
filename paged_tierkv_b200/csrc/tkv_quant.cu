// tkv_quant.cu -- HOT<->WARM conversion kernels for sm_100a.
//
// Format R (the reference's WARM layout): per token row asymmetric uint8 with
// fp16 scale and zero point, bit-exact with quantize_fp16_to_int8 /
// dequantize_int8_to_fp16 of xiaoMartintin/Paged_TierKV (tierkv_policy.py:21-44).
// Every step is one PyTorch fp16 op: evaluated in fp32, rounded to nearest-even
// fp16; torch.round is round-half-even (rintf).
//
// These kernels move bytes: one row of head_dim fp16 values is split over a
// few lanes that each load several 16-byte chunks before computing (memory
// parallelism), and the per-element work is one multiply by the scale's
// reciprocal plus exact fp16 steps.  Rows are independent; the grid strides
// over rows.
#include <algorithm>
#include <cuda_fp16.h>
#include <math.h>

#include "tkv_internal.h"

namespace tkv {

__device__ __forceinline__ float to_h(float x) { return __half2float(__float2half_rn(x)); }

// fp16(x / s) of the reference (PyTorch divides two fp16 tensors in fp32 and
// rounds to fp16: RN16(RN32(x / s))) computed as RN16(x * RN32(1/s)).  The two
// agree for all fp16 x and s > 0 whenever |x / s| >= 2^-14:
//  * x / s is never an fp16 rounding midpoint there: a midpoint is K * 2^c with
//    K odd in [2^11, 2^12), so x = K * 2^c * s would need an odd significand
//    factor >= 2049 in x, whose significand has 11 bits;
//  * it is more than 2 fp32 ulps from every midpoint: |x - M s| is a nonzero
//    multiple of 2^(c + exponent of s's last bit), i.e. |x / s - M| > 2^c / 2^11
//    = 2 ulp32(M);
//  * q = RN32(x * RN32(1/s)) is within 1.5 ulp32 of x / s (the reciprocal adds
//    at most 2^-24 relative error, the product rounding half an ulp), and so is
//    RN32(x / s) (half an ulp): no midpoint separates them from x / s.
// Below 2^-14 (fp16 subnormal results) only the sign matters to the callers:
// they round the quotient to an integer, and |q| < 0.25 rounds to a zero of
// q's sign either way.  Infinities and NaNs propagate as in the division
// (s = +inf gives r = 0 and x * 0 = x / inf for finite x).
__device__ __forceinline__ float div_by(float x, float r) { return __fmul_rn(x, r); }

constexpr float kInv255 = 1.0f / 255.0f;  // RN32(1/255)

// Scale, zero point and the scale's reciprocal of one row (tierkv_policy.py:25-33):
// scale = h(h(max - min) / 255), 1 where that is 0; zp = h(-rint(h(min / scale))).
__device__ __forceinline__ void row_params(float mn, float mx, float& scale, float& zp,
                                           float& rcp) {
  const float diff = to_h(mx - mn);
  float s = to_h(div_by(diff, kInv255));
  if (s == 0.f) s = 1.f;
  scale = s;
  rcp = __frcp_rn(s);
  zp = to_h(-rintf(to_h(div_by(mn, rcp))));
}

// Row minimum and maximum over V 16-byte chunks of fp16 per lane and LPR lanes
// per row, NaN-propagating like torch.min / torch.max.  The pair travels as one
// half2 (min, -max) so one shuffle and one min serve both per level.
template <int LPR, int V>
__device__ __forceinline__ void row_min_max(const uint4 (&raw)[V], float& mn, float& mx) {
  const __half2* h = reinterpret_cast<const __half2*>(raw);
  __half2 lo = h[0], hi = h[0];
#pragma unroll
  for (int j = 1; j < 4 * V; ++j) {
    lo = __hmin2_nan(lo, h[j]);
    hi = __hmax2_nan(hi, h[j]);
  }
  const __half2 nhi = __hneg2(hi);
  __half2 m = __hmin2_nan(__lows2half2(lo, nhi), __highs2half2(lo, nhi));
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) {
    uint32_t w = *reinterpret_cast<const uint32_t*>(&m);
    w = __shfl_xor_sync(0xffffffffu, w, off);
    m = __hmin2_nan(m, *reinterpret_cast<const __half2*>(&w));
  }
  mn = __low2float(m);
  mx = -__high2float(m);
}

// Codes of one 16-byte chunk (8 fp16 values) packed in a uint2
// (tierkv_policy.py:34: uint8(clamp(h(rint(h(x / scale)) + zp), 0, 255))).
// After the division every step is exact in fp16: rint, the sum of two
// integers, the clamp (a NaN row gives code 0, as the reference's CUDA cast
// does), and +1024 leaves the code in the low byte.
__device__ __forceinline__ uint2 quant_chunk(const uint4 raw, float rcp, __half hz) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
  const __half2 zp2 = __half2half2(hz);
  const __half2 lo2 = __float2half2_rn(0.f);
  const __half2 hi2 = __float2half2_rn(255.f);
  const __half2 bias2 = __float2half2_rn(1024.f);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    const __half2 t = __floats2half2_rn(div_by(f.x, rcp), div_by(f.y, rcp));
    const __half2 c = __hadd2(__hmin2(__hmax2(__hadd2(h2rint(t), zp2), lo2), hi2), bias2);
    w[i] = *reinterpret_cast<const uint32_t*>(&c);
  }
  uint2 out;
  out.x = __byte_perm(w[0], w[1], 0x6420);
  out.y = __byte_perm(w[2], w[3], 0x6420);
  return out;
}

// Lane layout shared by the row kernels: a row of D fp16 values is 2D bytes,
// LPR lanes per row, lane `sub` holding the 16-byte chunks sub + LPR * v,
// v < V = D / (8 LPR); load v of a warp then covers LPR * 16 contiguous bytes
// of each of its 32 / LPR rows.
template <int D, int LPR>
struct RowLayout {
  static constexpr int V = D / (8 * LPR);
  static constexpr int RPW = 32 / LPR;
  static_assert(V >= 1 && V * 8 * LPR == D, "head_dim must be a multiple of 8 * LPR");
};

// Lanes per row for head_dim D: TKV_QUANT_CHUNKS 16-byte chunks per lane, so
// the per-row work (reduction, scale, zero point) is shared by few lanes.
#ifndef TKV_QUANT_CHUNKS
#define TKV_QUANT_CHUNKS 4
#endif
template <int D>
__host__ __device__ constexpr int lanes_per_row() {
  return (D / 8) / TKV_QUANT_CHUNKS < 1 ? 1 : (D / 8) / TKV_QUANT_CHUNKS;
}

// Quantizes the row this lane group holds and stores its codes (and, from the
// group's first lane, the row's scale and zero point).
template <int D, int LPR>
__device__ __forceinline__ void quantize_store(const uint4 (&raw)[RowLayout<D, LPR>::V],
                                               uint8_t* codes, __half* scale, __half* zero,
                                               bool store, int sub) {
  using L = RowLayout<D, LPR>;
  float mn, mx, s, zp, rcp;
  row_min_max<LPR, L::V>(raw, mn, mx);
  row_params(mn, mx, s, zp, rcp);
  const __half hz = __float2half_rn(zp);
  if (!store) return;
#pragma unroll
  for (int v = 0; v < L::V; ++v)
    *reinterpret_cast<uint2*>(codes + (sub + LPR * v) * 8) = quant_chunk(raw[v], rcp, hz);
  if (sub == 0) {
    *scale = __float2half_rn(s);
    *zero = hz;
  }
}

// ---------------------------------------------------------------- plain rows
template <int D>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __half* __restrict__ x,
                                                            int64_t rows,
                                                            uint8_t* __restrict__ codes,
                                                            __half* __restrict__ scale,
                                                            __half* __restrict__ zero) {
  constexpr int LPR = lanes_per_row<D>();
  using L = RowLayout<D, LPR>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = warp * L::RPW; r0 < rows; r0 += nwarps * L::RPW) {
    const int64_t r = r0 + lane / LPR;
    const bool ok = r < rows;
    uint4 raw[L::V];
    const __half* xp = x + r * D + sub * 8;
#pragma unroll
    for (int v = 0; v < L::V; ++v)
      raw[v] = ok ? *reinterpret_cast<const uint4*>(xp + v * LPR * 8) : make_uint4(0u, 0u, 0u, 0u);
    quantize_store<D, LPR>(raw, codes + r * D, scale + r, zero + r, ok, sub);
  }
}

cudaError_t launch_quantize_rows(const void* x, int64_t rows, int dim, void* codes, void* scale,
                                 void* zero, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  auto* xs = reinterpret_cast<const __half*>(x);
  auto* cs = reinterpret_cast<uint8_t*>(codes);
  auto* ss = reinterpret_cast<__half*>(scale);
  auto* zs = reinterpret_cast<__half*>(zero);
  auto grid = [&](int lpr) {
    const int64_t per_block = (int64_t)threads / lpr;
    const int64_t b = (rows + per_block - 1) / per_block;
    return (unsigned)(b < (int64_t)sms * 16 ? b : (int64_t)sms * 16);
  };
#define TKV_QROWS(DIM)                                                                         \
  case DIM:                                                                                    \
    quantize_rows_kernel<DIM><<<grid(lanes_per_row<DIM>()), threads, 0, stream>>>(xs, rows, cs, \
                                                                                  ss, zs);     \
    break;
  switch (dim) {
    TKV_QROWS(16)
    TKV_QROWS(32)
    TKV_QROWS(64)
    TKV_QROWS(128)
    TKV_QROWS(256)
    default: return cudaErrorInvalidValue;
  }
#undef TKV_QROWS
  return cudaGetLastError();
}

// ---------------------------------------------------------------- demotion, Format R
// The launch's rows are r = (2 i + kind) * R + rr for demoted block i, tensor
// kind (K = 0, V = 1) and rr = kv_head * block_size + t < R = kv_heads *
// block_size: the R rows of one (block, tensor) are contiguous in both the HOT
// slot and the WARM slot.  rows < 2^31 per launch (the host splits larger
// calls), so the row arithmetic is 32-bit.  Rows with t < length are
// quantized; tail rows are cleared (code 0, scale 1, zero 0) only when
// clear_tail is set.
template <int D>
__global__ void __launch_bounds__(256) demote_r_kernel(const DemoteParams p, uint32_t rows) {
  constexpr int LPR = lanes_per_row<D>();
  using L = RowLayout<D, LPR>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const uint32_t bs = (uint32_t)p.block_size;
  const uint32_t R = (uint32_t)p.kv_heads * bs;
  const uint32_t warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const uint32_t wstride = gridDim.x * (blockDim.x >> 5) * L::RPW;
  for (uint32_t r0 = warp * L::RPW; r0 < rows; r0 += wstride) {
    const uint32_t r = r0 + lane / LPR;
    bool ok = r < rows;
    uint32_t rr = 0;
    int kind = 0, len = 0;
    int64_t src = 0, dst = 0;
    if (ok) {
      const uint32_t item = r / R;
      rr = r - item * R;
      const uint32_t i = item >> 1;
      kind = (int)(item & 1u);
      src = p.src[i];
      dst = p.dst[i];
      len = max(0, min(p.lengths[i], (int)bs));
      ok = src >= 0 && src < p.hot_slots && dst >= 0 && dst < p.warm_slots;
    }
    const bool valid = ok && (int)(rr % bs) < len;
    const int64_t in_row = src * R + rr;
    const int64_t out_row = dst * R + rr;
    uint4 raw[L::V];
    const __half* hp = reinterpret_cast<const __half*>(kind ? p.hot_v : p.hot_k) + in_row * D + sub * 8;
#pragma unroll
    for (int v = 0; v < L::V; ++v)
      raw[v] = valid ? *reinterpret_cast<const uint4*>(hp + v * LPR * 8) : make_uint4(0u, 0u, 0u, 0u);
    uint8_t* wp = reinterpret_cast<uint8_t*>(kind ? p.warm_v : p.warm_k) + out_row * D;
    __half* sp = reinterpret_cast<__half*>(kind ? p.v_scale : p.k_scale) + out_row;
    __half* zp = reinterpret_cast<__half*>(kind ? p.v_zero : p.k_zero) + out_row;
    quantize_store<D, LPR>(raw, wp, sp, zp, valid, sub);
    if (ok && !valid && p.clear_tail) {
#pragma unroll
      for (int v = 0; v < L::V; ++v)
        *reinterpret_cast<uint2*>(wp + (sub + LPR * v) * 8) = make_uint2(0u, 0u);
      if (sub == 0) {
        *sp = __float2half_rn(1.f);
        *zp = __float2half_rn(0.f);
      }
    }
  }
}

// ---------------------------------------------------------------- demotion, Format S
// One warp per (block, tensor, kv head) tile: absmax over the valid rows, one
// fp32 scale, codes clamp(rint(x / s), -127, 127); tail rows get code 0.
template <int D>
__global__ void demote_s_kernel(const DemoteParams p) {
  const int lane = threadIdx.x & 31;
  const int bs = p.block_size;
  const int64_t tiles = (int64_t)p.count * 2 * p.kv_heads;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  constexpr int kVecPerRow = D / 8;
  for (int64_t w = warp; w < tiles; w += nwarps) {
    const int i = (int)(w / (2 * p.kv_heads));
    const int rem = (int)(w - (int64_t)i * 2 * p.kv_heads);
    const int kind = rem / p.kv_heads;
    const int kvh = rem - kind * p.kv_heads;
    const int64_t src = p.src[i], dst = p.dst[i];
    if (src < 0 || src >= p.hot_slots || dst < 0 || dst >= p.warm_slots) continue;
    const int len = max(0, min(p.lengths[i], bs));
    const __half* hp = reinterpret_cast<const __half*>(kind ? p.hot_v : p.hot_k) +
                       (src * p.kv_heads + kvh) * bs * D;
    int8_t* wp = reinterpret_cast<int8_t*>(kind ? p.warm_v : p.warm_k) +
                 (dst * p.kv_heads + kvh) * bs * D;
    float amax = 0.f;
    for (int v = lane; v < len * kVecPerRow; v += 32) {
      const uint4 raw = *reinterpret_cast<const uint4*>(hp + v * 8);
      const __half* h = reinterpret_cast<const __half*>(&raw);
#pragma unroll
      for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(__half2float(h[k])));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    float s = __fdiv_rn(amax, 127.f);
    if (s == 0.f) s = 1.f;
    for (int v = lane; v < bs * kVecPerRow; v += 32) {
      uint2 out = make_uint2(0u, 0u);
      if (v < len * kVecPerRow) {
        const uint4 raw = *reinterpret_cast<const uint4*>(hp + v * 8);
        const __half* h = reinterpret_cast<const __half*>(&raw);
        uint32_t b[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float q = fminf(fmaxf(rintf(__fdiv_rn(__half2float(h[k]), s)), -127.f), 127.f);
          b[k] = (uint32_t)(int32_t)q & 0xffu;
        }
        out.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        out.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
      }
      *reinterpret_cast<uint2*>(wp + v * 8) = out;
    }
    if (lane == 0) reinterpret_cast<float*>(kind ? p.v_scale : p.k_scale)[dst * p.kv_heads + kvh] = s;
  }
}

cudaError_t launch_demote(const DemoteParams& p, int format, cudaStream_t stream) {
  if (p.count <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  if (format == kFmtR) {
    if (p.head_dim != 64 && p.head_dim != 128) return cudaErrorInvalidValue;
    const int lpr = p.head_dim == 64 ? lanes_per_row<64>() : lanes_per_row<128>();
    const int64_t rows_per_item = 2LL * p.kv_heads * p.block_size;  // rows of one demoted block
    const int64_t max_items = ((1LL << 31) - 1) / rows_per_item;
    for (int64_t first = 0; first < p.count; first += max_items) {
      DemoteParams q = p;
      q.count = (int32_t)(p.count - first < max_items ? p.count - first : max_items);
      q.src = p.src + first;
      q.dst = p.dst + first;
      q.lengths = p.lengths + first;
      const int64_t rows = (int64_t)q.count * rows_per_item;
      const int64_t per_block = threads / lpr;
      int64_t blocks = (rows + per_block - 1) / per_block;
      blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
      if (p.head_dim == 64)
        demote_r_kernel<64><<<(unsigned)blocks, threads, 0, stream>>>(q, (uint32_t)rows);
      else
        demote_r_kernel<128><<<(unsigned)blocks, threads, 0, stream>>>(q, (uint32_t)rows);
    }
  } else {
    const int64_t tiles = (int64_t)p.count * 2 * p.kv_heads;
    int64_t blocks = (tiles + (threads / 32) - 1) / (threads / 32);
    blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
    switch (p.head_dim) {
      case 64: demote_s_kernel<64><<<blocks, threads, 0, stream>>>(p); break;
      case 128: demote_s_kernel<128><<<blocks, threads, 0, stream>>>(p); break;
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- promotion, Format R
// HOT[dst] rows [0, length) = h(h(h(code) - zero) * scale)  (tierkv_policy.py:39-44).
// h(code) - zero is evaluated in fp32 and rounded, as the reference does; the
// product of two fp16 values is exact in fp32, so the fp16 multiply (one
// rounding of the exact product) equals the reference's fp32 multiply + cast.
__device__ __forceinline__ uint4 dequant_chunk(const uint2 c, float z, __half2 s2) {
  const __half2 bias2 = __float2half2_rn(1024.f);
  const uint32_t w[2] = {c.x, c.y};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // (1024 + code) as fp16: the code in the low byte of the significand
    const uint32_t x = __byte_perm(w[i >> 1], 0x64646464u, (i & 1) ? 0x4342u : 0x4140u);
    const float2 q = __half22float2(__hsub2(*reinterpret_cast<const __half2*>(&x), bias2));
    const __half2 h = __hmul2(__floats2half2_rn(q.x - z, q.y - z), s2);
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Rows as in demote_r_kernel, with src a WARM slot and dst a HOT slot.
template <int D>
__global__ void __launch_bounds__(256) promote_r_kernel(const DemoteParams p, uint32_t rows) {
  constexpr int LPR = lanes_per_row<D>();
  using L = RowLayout<D, LPR>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const uint32_t bs = (uint32_t)p.block_size;
  const uint32_t R = (uint32_t)p.kv_heads * bs;
  const uint32_t warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const uint32_t wstride = gridDim.x * (blockDim.x >> 5) * L::RPW;
  for (uint32_t r0 = warp * L::RPW; r0 < rows; r0 += wstride) {
    const uint32_t r = r0 + lane / LPR;
    if (r >= rows) continue;
    const uint32_t item = r / R;
    const uint32_t rr = r - item * R;
    const uint32_t i = item >> 1;
    const int kind = (int)(item & 1u);
    const int64_t src = p.src[i], dst = p.dst[i];
    const int len = max(0, min(p.lengths[i], (int)bs));
    if (src < 0 || src >= p.warm_slots || dst < 0 || dst >= p.hot_slots || (int)(rr % bs) >= len)
      continue;
    const int64_t in_row = src * R + rr;
    const int64_t out_row = dst * R + rr;
    const uint8_t* wp = reinterpret_cast<const uint8_t*>(kind ? p.warm_v : p.warm_k) + in_row * D;
    uint2 c[L::V];
#pragma unroll
    for (int v = 0; v < L::V; ++v) c[v] = *reinterpret_cast<const uint2*>(wp + (sub + LPR * v) * 8);
    const __half hs = reinterpret_cast<const __half*>(kind ? p.v_scale : p.k_scale)[in_row];
    const float z = __half2float(reinterpret_cast<const __half*>(kind ? p.v_zero : p.k_zero)[in_row]);
    const __half2 s2 = __half2half2(hs);
    __half* hp = reinterpret_cast<__half*>(const_cast<void*>(kind ? p.hot_v : p.hot_k)) + out_row * D;
#pragma unroll
    for (int v = 0; v < L::V; ++v)
      *reinterpret_cast<uint4*>(hp + (sub + LPR * v) * 8) = dequant_chunk(c[v], z, s2);
  }
}

cudaError_t launch_promote(const DemoteParams& p, cudaStream_t stream) {
  if (p.count <= 0) return cudaSuccess;
  if (p.head_dim != 64 && p.head_dim != 128) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  const int lpr = p.head_dim == 64 ? lanes_per_row<64>() : lanes_per_row<128>();
  const int64_t rows_per_item = 2LL * p.kv_heads * p.block_size;
  const int64_t max_items = ((1LL << 31) - 1) / rows_per_item;
  for (int64_t first = 0; first < p.count; first += max_items) {
    DemoteParams q = p;
    q.count = (int32_t)(p.count - first < max_items ? p.count - first : max_items);
    q.src = p.src + first;
    q.dst = p.dst + first;
    q.lengths = p.lengths + first;
    const int64_t rows = (int64_t)q.count * rows_per_item;
    const int64_t per_block = threads / lpr;
    int64_t blocks = (rows + per_block - 1) / per_block;
    blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
    if (p.head_dim == 64)
      promote_r_kernel<64><<<(unsigned)blocks, threads, 0, stream>>>(q, (uint32_t)rows);
    else
      promote_r_kernel<128><<<(unsigned)blocks, threads, 0, stream>>>(q, (uint32_t)rows);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- decode append
// One CTA per (kv head, K/V): rows [start, start + tokens) of the HOT slot get
// the new rows, rows [start + tokens, block_size) are zeroed
// (tierkv_policy.py:954-958), 16 bytes per thread-step; CTA (0, 0) also writes
// the block-table cells.
__global__ void __launch_bounds__(128) append_kernel(const AppendParams p) {
  const int h = blockIdx.x;
  const int kind = blockIdx.y;
  const int vpr = p.head_dim / 8;  // 16-byte vectors per row
  uint4* dst = reinterpret_cast<uint4*>(kind ? p.hot_v : p.hot_k) +
               ((p.slot * p.kv_heads + h) * p.block_size + p.start) * vpr;
  const uint4* src = reinterpret_cast<const uint4*>(kind ? p.value : p.key) +
                     (size_t)h * p.tokens * vpr;
  const int n = (p.block_size - p.start) * vpr;
  const int fill = p.tokens * vpr;
  for (int e = threadIdx.x; e < n; e += blockDim.x)
    dst[e] = e < fill ? __ldg(src + e) : make_uint4(0u, 0u, 0u, 0u);
  if (h == 0 && kind == 0 && threadIdx.x < p.n_cells) *p.cell_ptr[threadIdx.x] = p.cell_val[threadIdx.x];
}

cudaError_t launch_append(const AppendParams& p, cudaStream_t stream) {
  append_kernel<<<dim3((unsigned)p.kv_heads, 2), 128, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- prefill store
// The launch's rows are r = (2 e + kind) * R + rr for entry e, tensor kind
// (K = 0, V = 1) and rr = kv_head * block_size + t < R = kv_heads *
// block_size.  Row t < length of an entry reads input row (kv_head, first +
// t); HOT entries store it (rows past the length store zeros), WARM entries
// quantize it (rows past the length get code 0, scale 1, zero 0).  Every lane
// runs the row quantizer, whose lanes exchange values by shuffles, and stores
// only for WARM rows.  rows < 2^31 per launch (the host splits), so the row
// arithmetic is 32-bit.
template <int D>
__global__ void __launch_bounds__(256) store_prefill_kernel(const PrefillStoreParams p,
                                                            uint32_t rows) {
  constexpr int LPR = lanes_per_row<D>();
  using L = RowLayout<D, LPR>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const uint32_t bs = (uint32_t)p.block_size;
  const uint32_t R = (uint32_t)p.kv_heads * bs;
  const uint32_t warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const uint32_t wstride = gridDim.x * (blockDim.x >> 5) * L::RPW;
  for (uint32_t r0 = warp * L::RPW; r0 < rows; r0 += wstride) {
    const uint32_t r = r0 + lane / LPR;
    bool ok = r < rows;
    int state = -1, kind = 0, len = 0, first = 0;
    int64_t slot = 0;
    uint32_t rr = 0;
    if (ok) {
      const uint32_t item = r / R;
      rr = r - item * R;
      const int32_t* e = p.blocks + 4 * (size_t)(item >> 1);
      kind = (int)(item & 1u);
      state = e[0];
      slot = e[1];
      first = e[2];
      len = e[3];
      ok = ((state == 0 && slot >= 0 && slot < p.hot_slots) ||
            (state == 1 && slot >= 0 && slot < p.warm_slots)) &&
           len >= 0 && len <= (int)bs && first >= 0 && first <= p.tokens - len;
    }
    const uint32_t head = rr / bs, t = rr - (rr / bs) * bs;
    const bool valid = ok && (int)t < len;
    uint4 raw[L::V];
    const __half* src = reinterpret_cast<const __half*>(kind ? p.value : p.key) +
                        ((int64_t)head * p.tokens + first + (int64_t)t) * D + sub * 8;
#pragma unroll
    for (int v = 0; v < L::V; ++v)
      raw[v] = valid ? *reinterpret_cast<const uint4*>(src + v * LPR * 8) : make_uint4(0u, 0u, 0u, 0u);
    const bool warm = ok && state == 1;
    const int64_t out_row = (ok ? slot : 0) * R + rr;
    uint8_t* wp = warm ? reinterpret_cast<uint8_t*>(kind ? p.warm_v : p.warm_k) + out_row * D : nullptr;
    __half* sp = warm ? reinterpret_cast<__half*>(kind ? p.v_scale : p.k_scale) + out_row : nullptr;
    __half* zp = warm ? reinterpret_cast<__half*>(kind ? p.v_zero : p.k_zero) + out_row : nullptr;
    quantize_store<D, LPR>(raw, wp, sp, zp, warm && valid, sub);
    if (warm && !valid) {
#pragma unroll
      for (int v = 0; v < L::V; ++v)
        *reinterpret_cast<uint2*>(wp + (sub + LPR * v) * 8) = make_uint2(0u, 0u);
      if (sub == 0) {
        *sp = __float2half_rn(1.f);
        *zp = __float2half_rn(0.f);
      }
    }
    if (ok && state == 0) {
      __half* hp = reinterpret_cast<__half*>(kind ? p.hot_v : p.hot_k) + out_row * D + sub * 8;
#pragma unroll
      for (int v = 0; v < L::V; ++v) *reinterpret_cast<uint4*>(hp + v * LPR * 8) = raw[v];
    }
  }
}

cudaError_t launch_store_prefill(const PrefillStoreParams& p_in, cudaStream_t stream) {
  if (p_in.count <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_entry = 2 * (int64_t)p_in.kv_heads * p_in.block_size;
  const int64_t max_entries = 0x7fffffffLL / per_entry;
  const int threads = 256;
  for (int64_t e0 = 0; e0 < p_in.count; e0 += max_entries) {
    PrefillStoreParams p = p_in;
    p.blocks = p_in.blocks + 4 * e0;
    p.count = (int32_t)std::min<int64_t>(max_entries, p_in.count - e0);
    const uint32_t rows = (uint32_t)(p.count * per_entry);
    auto grid = [&](int lpr) {
      const int64_t per_block = (int64_t)threads / lpr;
      const int64_t b = ((int64_t)rows + per_block - 1) / per_block;
      return (unsigned)(b < (int64_t)sms * 16 ? b : (int64_t)sms * 16);
    };
    switch (p.head_dim) {
      case 64: store_prefill_kernel<64><<<grid(lanes_per_row<64>()), threads, 0, stream>>>(p, rows); break;
      case 128: store_prefill_kernel<128><<<grid(lanes_per_row<128>()), threads, 0, stream>>>(p, rows); break;
      default: return cudaErrorInvalidValue;
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace tkv
