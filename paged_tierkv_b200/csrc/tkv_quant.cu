// tkv_quant.cu -- HOT<->WARM conversion kernels for sm_100a.
//
// Format R (the reference's WARM layout): per token row asymmetric uint8 with
// fp16 scale and zero point, bit-exact with quantize_fp16_to_int8 /
// dequantize_int8_to_fp16 of xiaoMartintin/Paged_TierKV (tierkv_policy.py:21-44).
// Every step is one PyTorch fp16 op: evaluated in fp32, rounded to nearest-even
// fp16; torch.round is round-half-even (rintf).
//
// These kernels move bytes: one row of head_dim fp16 values is split over
// head_dim/8 lanes that each load 16 bytes, so a warp reads 512 contiguous
// bytes per step.  Rows are independent; the grid strides over rows.
#include <cuda_fp16.h>
#include <math.h>

#include "tkv_internal.h"

namespace tkv {

__device__ __forceinline__ float hmin_nan(float a, float b) { return (a != a || a < b) ? a : b; }
__device__ __forceinline__ float hmax_nan(float a, float b) { return (a != a || a > b) ? a : b; }
__device__ __forceinline__ float to_h(float x) { return __half2float(__float2half_rn(x)); }

// Scale and zero point of one row (tierkv_policy.py:25-33).
__device__ __forceinline__ void row_params(float mn, float mx, float& scale, float& zp) {
  const float diff = to_h(mx - mn);
  float s = to_h(__fdiv_rn(diff, 255.0f));
  if (s == 0.f) s = 1.f;
  scale = s;
  zp = to_h(-rintf(to_h(__fdiv_rn(mn, s))));
}

// fp16(fp32 x / s), the reference's `tensor / scale` (x, s fp16 values, s > 0
// finite or 1).  q = x * RN(1/s) is within 2.5 fp32 ulps of RN(x / s), so
// both round to the same fp16 value unless q lies within 3 ulps of an fp16
// rounding midpoint (fp32 mantissa bits [12:0] near 0x1000) or outside the
// range where fp16 is normal; only those take the IEEE division.
__device__ __forceinline__ __half div_to_half(float x, float s, float r) {
  const float q = __fmul_rn(x, r);
  const uint32_t b = __float_as_uint(q);
  const uint32_t e = (b >> 23) & 0xffu;
  const bool fast = e >= 113u && e <= 141u && ((b - 0x0ffdu) & 0x1fffu) > 6u;
  return __float2half_rn(fast ? q : __fdiv_rn(x, s));
}

// Quantizes one row held as 8 fp16 values per lane over LPR lanes; returns
// the 8 codes packed in a uint2 and the row's scale / zero point
// (tierkv_policy.py:34: uint8(clamp(h(rint(h(x / scale)) + zp), 0, 255))).
// After the division every step is exact in fp16: rint, the sum of two
// integers, the clamp (a NaN row gives code 0, as the reference's CUDA cast
// does), and +1024 leaves the code in the low byte.
template <int LPR>
__device__ __forceinline__ uint2 quant_row(const uint4 raw, __half& hs, __half& hz) {
  const __half* h = reinterpret_cast<const __half*>(&raw);
  float v[8];
  float mn, mx;
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __half2float(h[i]);
  mn = v[0];
  mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = hmin_nan(mn, v[i]);
    mx = hmax_nan(mx, v[i]);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) {
    mn = hmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = hmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  float scale, zp;
  row_params(mn, mx, scale, zp);
  hs = __float2half_rn(scale);
  hz = __float2half_rn(zp);
  const float rcp = __frcp_rn(scale);
  const __half2 zp2 = __half2half2(hz);
  const __half2 lo2 = __float2half2_rn(0.f);
  const __half2 hi2 = __float2half2_rn(255.f);
  const __half2 bias2 = __float2half2_rn(1024.f);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 t = __halves2half2(div_to_half(v[2 * i], scale, rcp),
                                     div_to_half(v[2 * i + 1], scale, rcp));
    const __half2 c = __hadd2(__hmin2(__hmax2(__hadd2(h2rint(t), zp2), lo2), hi2), bias2);
    w[i] = *reinterpret_cast<const uint32_t*>(&c);
  }
  uint2 out;
  out.x = __byte_perm(w[0], w[1], 0x6420);
  out.y = __byte_perm(w[2], w[3], 0x6420);
  return out;
}

// ---------------------------------------------------------------- plain rows
template <int LPR>
__global__ void quantize_rows_kernel(const __half* __restrict__ x, int64_t rows,
                                     uint8_t* __restrict__ codes, __half* __restrict__ scale,
                                     __half* __restrict__ zero) {
  constexpr int D = LPR * 8;
  constexpr int RPW = 32 / LPR;  // rows per warp step
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = warp * RPW; r0 < rows; r0 += nwarps * RPW) {
    const int64_t r = r0 + lane / LPR;
    const bool ok = r < rows;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (ok) raw = *reinterpret_cast<const uint4*>(x + r * D + sub * 8);
    __half hs, hz;
    const uint2 c = quant_row<LPR>(raw, hs, hz);
    if (ok) {
      *reinterpret_cast<uint2*>(codes + r * D + sub * 8) = c;
      if (sub == 0) {
        scale[r] = hs;
        zero[r] = hz;
      }
    }
  }
}

cudaError_t launch_quantize_rows(const void* x, int64_t rows, int dim, void* codes, void* scale,
                                 void* zero, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  const int64_t rows_per_block = (threads / 32) * (32 / (dim / 8));
  int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
  auto* xs = reinterpret_cast<const __half*>(x);
  auto* cs = reinterpret_cast<uint8_t*>(codes);
  auto* ss = reinterpret_cast<__half*>(scale);
  auto* zs = reinterpret_cast<__half*>(zero);
  switch (dim) {
    case 16: quantize_rows_kernel<2><<<blocks, threads, 0, stream>>>(xs, rows, cs, ss, zs); break;
    case 32: quantize_rows_kernel<4><<<blocks, threads, 0, stream>>>(xs, rows, cs, ss, zs); break;
    case 64: quantize_rows_kernel<8><<<blocks, threads, 0, stream>>>(xs, rows, cs, ss, zs); break;
    case 128: quantize_rows_kernel<16><<<blocks, threads, 0, stream>>>(xs, rows, cs, ss, zs); break;
    case 256: quantize_rows_kernel<32><<<blocks, threads, 0, stream>>>(xs, rows, cs, ss, zs); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- demotion, Format R
// Row r of the launch = (block i, tensor K/V, kv head, token t).  Rows with
// t < length are quantized from the HOT slot into the WARM slot; tail rows are
// cleared (code 0, scale 1, zero 0) only when clear_tail is set.
template <int LPR>
__global__ void demote_r_kernel(const DemoteParams p) {
  constexpr int D = LPR * 8;
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const int bs = p.block_size;
  const int64_t rows_per_block = 2LL * p.kv_heads * bs;
  const int64_t rows = (int64_t)p.count * rows_per_block;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = warp * RPW; r0 < rows; r0 += nwarps * RPW) {
    const int64_t r = r0 + lane / LPR;
    bool ok = r < rows;
    int i = 0, kind = 0, kvh = 0, t = 0, len = 0;
    int64_t src = -1, dst = -1;
    if (ok) {
      i = (int)(r / rows_per_block);
      int64_t rem = r - (int64_t)i * rows_per_block;
      kind = (int)(rem / ((int64_t)p.kv_heads * bs));
      rem -= (int64_t)kind * p.kv_heads * bs;
      kvh = (int)(rem / bs);
      t = (int)(rem - (int64_t)kvh * bs);
      src = p.src[i];
      dst = p.dst[i];
      len = max(0, min(p.lengths[i], bs));
      ok = src >= 0 && src < p.hot_slots && dst >= 0 && dst < p.warm_slots;
    }
    const bool valid = ok && t < len;
    const int64_t in_row = ((src * p.kv_heads + kvh) * bs + t);
    const int64_t out_row = ((dst * p.kv_heads + kvh) * bs + t);
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (valid) {
      const __half* hp = reinterpret_cast<const __half*>(kind ? p.hot_v : p.hot_k);
      raw = *reinterpret_cast<const uint4*>(hp + in_row * D + sub * 8);
    }
    __half hs, hz;
    const uint2 c = quant_row<LPR>(raw, hs, hz);
    uint8_t* wp = reinterpret_cast<uint8_t*>(kind ? p.warm_v : p.warm_k);
    __half* sp = reinterpret_cast<__half*>(kind ? p.v_scale : p.k_scale);
    __half* zp = reinterpret_cast<__half*>(kind ? p.v_zero : p.k_zero);
    if (valid) {
      *reinterpret_cast<uint2*>(wp + out_row * D + sub * 8) = c;
      if (sub == 0) {
        sp[out_row] = hs;
        zp[out_row] = hz;
      }
    } else if (ok && p.clear_tail) {
      *reinterpret_cast<uint2*>(wp + out_row * D + sub * 8) = make_uint2(0u, 0u);
      if (sub == 0) {
        sp[out_row] = __float2half_rn(1.f);
        zp[out_row] = __float2half_rn(0.f);
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
    const int lpr = p.head_dim / 8;
    const int64_t rows = (int64_t)p.count * 2 * p.kv_heads * p.block_size;
    const int64_t per_block = (threads / 32) * (32 / lpr);
    int64_t blocks = (rows + per_block - 1) / per_block;
    blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
    switch (p.head_dim) {
      case 64: demote_r_kernel<8><<<blocks, threads, 0, stream>>>(p); break;
      case 128: demote_r_kernel<16><<<blocks, threads, 0, stream>>>(p); break;
      default: return cudaErrorInvalidValue;
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
template <int LPR>
__global__ void promote_r_kernel(const DemoteParams p) {
  constexpr int D = LPR * 8;
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;
  const int bs = p.block_size;
  const int64_t rows_per_block = 2LL * p.kv_heads * bs;
  const int64_t rows = (int64_t)p.count * rows_per_block;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r0 = warp * RPW; r0 < rows; r0 += nwarps * RPW) {
    const int64_t r = r0 + lane / LPR;
    if (r >= rows) continue;
    const int i = (int)(r / rows_per_block);
    int64_t rem = r - (int64_t)i * rows_per_block;
    const int kind = (int)(rem / ((int64_t)p.kv_heads * bs));
    rem -= (int64_t)kind * p.kv_heads * bs;
    const int kvh = (int)(rem / bs);
    const int t = (int)(rem - (int64_t)kvh * bs);
    const int64_t src = p.src[i], dst = p.dst[i];  // src: WARM slot, dst: HOT slot
    const int len = max(0, min(p.lengths[i], bs));
    if (src < 0 || src >= p.warm_slots || dst < 0 || dst >= p.hot_slots || t >= len) continue;
    const int64_t in_row = (src * p.kv_heads + kvh) * bs + t;
    const int64_t out_row = (dst * p.kv_heads + kvh) * bs + t;
    const uint8_t* wp = reinterpret_cast<const uint8_t*>(kind ? p.warm_v : p.warm_k);
    const __half* sp = reinterpret_cast<const __half*>(kind ? p.v_scale : p.k_scale);
    const __half* zp = reinterpret_cast<const __half*>(kind ? p.v_zero : p.k_zero);
    const uint2 c = *reinterpret_cast<const uint2*>(wp + in_row * D + sub * 8);
    const float s = __half2float(sp[in_row]);
    const float z = __half2float(zp[in_row]);
    const uint32_t w[2] = {c.x, c.y};
    __half o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float q = (float)((w[k >> 2] >> (8 * (k & 3))) & 0xffu);
      o[k] = __float2half_rn(to_h(q - z) * s);
    }
    __half* hp = reinterpret_cast<__half*>(kind ? const_cast<void*>(p.hot_v) : const_cast<void*>(p.hot_k));
    *reinterpret_cast<uint4*>(hp + out_row * D + sub * 8) = *reinterpret_cast<const uint4*>(o);
  }
}

cudaError_t launch_promote(const DemoteParams& p, cudaStream_t stream) {
  if (p.count <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  const int lpr = p.head_dim / 8;
  const int64_t rows = (int64_t)p.count * 2 * p.kv_heads * p.block_size;
  const int64_t per_block = (threads / 32) * (32 / lpr);
  int64_t blocks = (rows + per_block - 1) / per_block;
  blocks = blocks < (int64_t)sms * 16 ? blocks : (int64_t)sms * 16;
  switch (p.head_dim) {
    case 64: promote_r_kernel<8><<<blocks, threads, 0, stream>>>(p); break;
    case 128: promote_r_kernel<16><<<blocks, threads, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace tkv
