// tkv_api.cu -- the extern "C" boundary declared in include/tierkv_b200.h.
//
// Validates arguments the way the reference wrapper does
// (tierkv_triton.py:290-304; errors become status codes instead of Python
// exceptions), plans the split-KV partition, carves the caller's workspace,
// encodes the TMA descriptors of the four data pools and launches the sm_100a
// kernels on the caller's stream.  Nothing here allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>

#include "tierkv_b200.h"
#include "tkv_internal.h"

using namespace tkv;

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D tiled map over a pool viewed as [rows, head_dim] elements.
bool encode_pool_map(CUtensorMap* map, void* base, bool fp16, int64_t rows, int head_dim,
                     int box_inner, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int esize = fp16 ? 2 : 1;
  cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)head_dim * esize};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const int inner_bytes = box_inner * esize;
  CUtensorMapSwizzle swz = inner_bytes == 128   ? CU_TENSOR_MAP_SWIZZLE_128B
                           : inner_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = fn(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                  base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

constexpr int kMaxDevices = 64;

// SM count of the current device, cached per device (0 = not an sm_100 part).
int current_device_sms(int* sms) {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TKV_ERR_NO_DEVICE;
  if (dev >= 0 && dev < kMaxDevices) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) {
      *sms = c;
      return TKV_OK;
    }
  }
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return TKV_ERR_NO_DEVICE;
  if (major != 10) return TKV_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return TKV_ERR_NO_DEVICE;
  if (dev >= 0 && dev < kMaxDevices) cache[dev].store(*sms, std::memory_order_relaxed);
  return TKV_OK;
}

// CTAs per SM of one decode kernel instance, cached per (device, instance).
bool cached_occupancy(int head_dim, int block_size, int format, int query_dtype, int* ctas) {
  static std::atomic<int> cache[kMaxDevices][16];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const int key = ((head_dim == 128) << 3) | ((block_size == 32) << 2) |
                  ((format == TKV_FORMAT_S) << 1) | (query_dtype == TKV_DTYPE_BF16);
  const bool cacheable = dev >= 0 && dev < kMaxDevices;
  if (cacheable) {
    const int c = cache[dev][key].load(std::memory_order_relaxed);
    if (c > 0) {
      *ctas = c;
      return true;
    }
  }
  if (decode_occupancy(head_dim, block_size, format, query_dtype, ctas) != cudaSuccess) return false;
  if (cacheable && *ctas > 0) cache[dev][key].store(*ctas, std::memory_order_relaxed);
  return true;
}

int32_t check_pools(const tkv_pools* pl, bool need_meta) {
  if (!pl) return TKV_ERR_INVALID;
  if (pl->format != TKV_FORMAT_R && pl->format != TKV_FORMAT_S) return TKV_ERR_UNSUPPORTED;
  if (pl->head_dim != 64 && pl->head_dim != 128) return TKV_ERR_UNSUPPORTED;
  if (pl->block_size != 16 && pl->block_size != 32) return TKV_ERR_UNSUPPORTED;
  if (pl->kv_heads <= 0 || pl->hot_slots <= 0 || pl->warm_slots <= 0) return TKV_ERR_INVALID;
  if (!pl->hot_k || !pl->hot_v || !pl->warm_k || !pl->warm_v) return TKV_ERR_INVALID;
  if (!aligned(pl->hot_k, 16) || !aligned(pl->hot_v, 16) || !aligned(pl->warm_k, 16) ||
      !aligned(pl->warm_v, 16))
    return TKV_ERR_INVALID;
  const int64_t max_rows = std::max(pl->hot_slots, pl->warm_slots) * pl->kv_heads * pl->block_size;
  if (max_rows >= (int64_t(1) << 31)) return TKV_ERR_INVALID;
  if (need_meta) {
    if (!pl->k_scale || !pl->v_scale) return TKV_ERR_INVALID;
    if (pl->format == TKV_FORMAT_R) {
      if (!pl->k_zero || !pl->v_zero) return TKV_ERR_INVALID;
      if (!aligned(pl->k_scale, 16) || !aligned(pl->k_zero, 16) || !aligned(pl->v_scale, 16) ||
          !aligned(pl->v_zero, 16))
        return TKV_ERR_INVALID;
    } else if (!aligned(pl->k_scale, 4) || !aligned(pl->v_scale, 4)) {
      return TKV_ERR_INVALID;
    }
  }
  return TKV_OK;
}

// 3-D tiled map over an fp16 HOT pool: dims {64, rows, head_dim/64} with
// strides {head_dim*2, 128} bytes, box {64, bs, head_dim/64}.  One box is a
// whole [bs, head_dim] tile landing as [head_dim/64][bs][64] in shared memory.
bool encode_hot_map_3d(CUtensorMap* map, void* base, int64_t rows, int head_dim, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(head_dim / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)(head_dim / 64)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Workspace layout, a function of the workspace's size W alone: [0, 256) the
// device error word, [256, 256 + R) the counters with R = W / 8 rounded down
// to 256 bytes, then the data regions (partials, per-block LSE).  Every launch
// returns its counters to zero and no data region reaches below 256 + R, so
// one workspace, zero-filled once, serves calls of any shape in any order.
inline size_t counter_reserve(size_t w) { return (w / 8) / kAlign * kAlign; }
inline size_t data_base(size_t w) { return kAlign + counter_reserve(w); }
inline bool layout_fits(size_t w, size_t counters, size_t data) {
  return counter_reserve(w) >= counters && data_base(w) + data <= w;
}
size_t required_workspace(size_t counters, size_t data) {
  constexpr size_t kStep = 8 * kAlign;
  size_t w = std::max(8 * align_up(counters), (data + kAlign) * 8 / 7 + kAlign);
  w = (w + kStep - 1) / kStep * kStep;
  while (!layout_fits(w, counters, data)) w += kStep;
  return w;
}

struct Plan {
  int splits = 1;
  int chunk = 32;
  int group_size = 1;  // splits per merge group; = splits when the merge has one level
  size_t counters_bytes = 0, data_bytes = 0;
  // offsets of the data regions from the data base
  size_t off_part_o = 0, off_part_lse = 0, off_gpart_o = 0, off_gpart_lse = 0,
         off_lse_final = 0, off_lse_blk = 0;
  size_t total = 0;  // smallest workspace that holds this layout
};

// Splits beyond this count are merged in two levels: groups of about
// sqrt(splits) partials, then the group results.  Each level costs a ticket,
// a round of LSE loads and three CTA barriers (measured: at 74 splits one
// level is 1.3 us faster per launch), so only very wide merges use two.
#ifndef TKV_TREE_MERGE_SPLITS
#define TKV_TREE_MERGE_SPLITS 128
#endif
constexpr int kTreeMergeSplits = TKV_TREE_MERGE_SPLITS;

int32_t make_plan(const tkv_pools* pl, const tkv_decode_args* a, Plan* plan) {
  int32_t st = check_pools(pl, true);
  if (st != TKV_OK) return st;
  if (!a) return TKV_ERR_INVALID;
  if (a->batch <= 0 || a->num_heads <= 0 || a->num_kv_groups <= 0) return TKV_ERR_INVALID;
  if (a->num_kv_groups > kMaxGroups) return TKV_ERR_UNSUPPORTED;
  if ((int64_t)pl->kv_heads * a->num_kv_groups != a->num_heads) return TKV_ERR_INVALID;
  if (a->query_dtype != TKV_DTYPE_F16 && a->query_dtype != TKV_DTYPE_BF16) return TKV_ERR_UNSUPPORTED;
  if (a->out_dtype != TKV_DTYPE_F16 && a->out_dtype != TKV_DTYPE_BF16 && a->out_dtype != TKV_DTYPE_F32)
    return TKV_ERR_UNSUPPORTED;
  if (a->num_blocks < 0 || a->max_blocks < 0 || a->num_blocks > a->max_blocks) return TKV_ERR_INVALID;
  if (a->table_stride < a->max_blocks) return TKV_ERR_INVALID;
  if (a->num_splits < 0 || a->num_splits > kMaxSplits) return TKV_ERR_INVALID;
  if ((a->flags & ~TKV_FLAG_CHUNK_MASK) != 0) return TKV_ERR_INVALID;
  const int forced_chunk = a->flags & TKV_FLAG_CHUNK_MASK;
  if (forced_chunk != 0 && forced_chunk != 8 && forced_chunk != 16 && forced_chunk != 32)
    return TKV_ERR_INVALID;
  int splits = a->num_splits;
  int chunk = forced_chunk != 0 ? forced_chunk : 32;
  if (splits == 0 || forced_chunk == 0) {
    // with the split count given, the waves do not depend on the chunk size:
    // the choice needs no device
    int64_t slots = 1;
    if (splits == 0) {
      int sms = 0;
      st = current_device_sms(&sms);
      if (st != TKV_OK) return st;
      int ctas = 0;
      if (!cached_occupancy(pl->head_dim, pl->block_size, pl->format, a->query_dtype, &ctas) ||
          ctas <= 0)
        return TKV_ERR_CUDA;
      slots = (int64_t)sms * ctas;
    }
    const int64_t units = (int64_t)a->batch * pl->kv_heads;
    // The CTAs of a (sequence, kv head) claim `chunk`-block pieces of its
    // table; cost ~ waves * (blocks of the busiest CTA + its chunk claims + a
    // fixed per-CTA overhead: prologue, pipeline fill and drain, merge).
    // Smaller chunks even out the CTAs' shares when there are few chunks per
    // CTA (one long context, small batches).
    double best = 1e300;
    for (int c = 32; c >= 8; c >>= 1) {
      if (forced_chunk != 0 && c != forced_chunk) continue;
      const int chunks = std::max(1, (a->num_blocks + c - 1) / c);
      const int lo = a->num_splits > 0 ? a->num_splits : 1;
      const int hi = a->num_splits > 0 ? a->num_splits : std::min(kMaxSplits, chunks);
      for (int s = lo; s <= hi; ++s) {
        const int64_t ctas_total = units * s;
        const double waves = (double)((ctas_total + slots - 1) / slots);
        // dynamic claiming evens the CTAs' shares to within about one chunk
        const double per_chunks = (double)chunks / s + 0.5;
        const double cost = waves * (per_chunks * (c + (double)TKV_CHUNK_OVERHEAD_BLOCKS) +
                                     (double)TKV_CTA_OVERHEAD_BLOCKS);
        if (cost < best - 1e-9) {
          best = cost;
          splits = s;
          chunk = c;
        }
      }
    }
  }
  plan->splits = std::max(1, splits);
  plan->chunk = chunk;
  plan->group_size = plan->splits;
  if (plan->splits > kTreeMergeSplits) {
    int g = (int)std::ceil(std::sqrt((double)plan->splits));
    while (g * g < plan->splits) ++g;
    plan->group_size = g;
  }
  const int ngroups = (plan->splits + plan->group_size - 1) / plan->group_size;
  const size_t rows = (size_t)a->batch * a->num_heads;
  const size_t units = (size_t)a->batch * pl->kv_heads;
  // counters: split (or group) tickets and chunk counters, one each per
  // (sequence, kv head), then the group tickets
  plan->counters_bytes = sizeof(uint32_t) * units * (2 + (ngroups > 1 ? ngroups : 0));
  size_t off = 0;
  if (plan->splits > 1) {
    plan->off_part_o = off;
    off = align_up(off + sizeof(float) * rows * plan->splits * pl->head_dim);
    plan->off_part_lse = off;
    off = align_up(off + sizeof(float) * rows * plan->splits);
  }
  if (ngroups > 1) {
    plan->off_gpart_o = off;
    off = align_up(off + sizeof(float) * rows * ngroups * pl->head_dim);
    plan->off_gpart_lse = off;
    off = align_up(off + sizeof(float) * rows * ngroups);
  }
  if (a->score_sums) {
    plan->off_lse_final = off;
    off = align_up(off + sizeof(float) * rows);
    plan->off_lse_blk = off;
    off = align_up(off + sizeof(float) * rows * std::max(1, a->max_blocks));
  }
  plan->data_bytes = off;
  plan->total = required_workspace(plan->counters_bytes, plan->data_bytes);
  return TKV_OK;
}

inline int32_t cuda_status(cudaError_t e) { return e == cudaSuccess ? TKV_OK : TKV_ERR_CUDA; }

}  // namespace

bool tkv::encode_head_rows_map(CUtensorMap* map, const void* base, int64_t heads, int64_t rows,
                               int head_dim) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {64, (cuuint64_t)rows, (cuuint64_t)(head_dim / 64), (cuuint64_t)heads};
  cuuint64_t strides[3] = {(cuuint64_t)head_dim * 2, 128, (cuuint64_t)rows * head_dim * 2};
  cuuint32_t box[4] = {64, 128, (cuuint32_t)(head_dim / 64), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

extern "C" {

int32_t tkv_get_version(void) { return TKV_ABI_VERSION; }

const char* tkv_status_string(int32_t status) {
  switch (status) {
    case TKV_OK: return "ok";
    case TKV_ERR_INVALID: return "invalid argument (pointer, shape, stride or alignment)";
    case TKV_ERR_UNSUPPORTED: return "unsupported geometry, dtype or WARM format";
    case TKV_ERR_WORKSPACE: return "workspace missing or smaller than tkv_decode_plan() requires";
    case TKV_ERR_CUDA: return "CUDA error while encoding or launching";
    case TKV_ERR_NO_DEVICE: return "no usable sm_100 (B200) device is current";
    case TKV_ERR_SCRATCH_LIMIT:
      return "call needs more scratch than the library's fixed array (TKV_NOALLOC_SCRATCH_BYTES); "
             "use tkv_decode_attention with a caller workspace";
    default: return "unknown status";
  }
}

int32_t tkv_decode_plan(const tkv_pools* pools, const tkv_decode_args* args,
                        int32_t* num_splits_out, size_t* workspace_bytes_out) {
  Plan plan;
  const int32_t st = make_plan(pools, args, &plan);
  if (st != TKV_OK) return st;
  if (num_splits_out) *num_splits_out = plan.splits;
  if (workspace_bytes_out) *workspace_bytes_out = plan.total;
  return TKV_OK;
}

// The four TMA descriptors of a pool set.  Serving loops decode against the
// same pools layer after layer, and encoding costs host time on every call,
// so the last few sets of this thread are kept, keyed by every input of the
// encoding.
static bool pool_maps(const tkv_pools* pools, CUtensorMap maps[4]) {
  struct Entry {
    const void* ptr[4];
    int64_t hot_rows, warm_rows;
    int d, bs, valid;
    CUtensorMap maps[4];
  };
  thread_local Entry cache[4] = {};
  thread_local int next = 0;
  const int bs = pools->block_size, d = pools->head_dim, hkv = pools->kv_heads;
  const int64_t hot_rows = pools->hot_slots * hkv * bs;
  const int64_t warm_rows = pools->warm_slots * hkv * bs;
  const void* ptr[4] = {pools->hot_k, pools->hot_v, pools->warm_k, pools->warm_v};
  for (Entry& e : cache) {
    if (e.valid && e.hot_rows == hot_rows && e.warm_rows == warm_rows && e.d == d && e.bs == bs &&
        e.ptr[0] == ptr[0] && e.ptr[1] == ptr[1] && e.ptr[2] == ptr[2] && e.ptr[3] == ptr[3]) {
      std::memcpy(maps, e.maps, sizeof(e.maps));
      return true;
    }
  }
#if TKV_HOT_3D
  const bool hot_ok = encode_hot_map_3d(&maps[0], pools->hot_k, hot_rows, d, bs) &&
                      encode_hot_map_3d(&maps[1], pools->hot_v, hot_rows, d, bs);
#else
  const bool hot_ok = encode_pool_map(&maps[0], pools->hot_k, true, hot_rows, d, 64, bs) &&
                      encode_pool_map(&maps[1], pools->hot_v, true, hot_rows, d, 64, bs);
#endif
  if (!hot_ok || !encode_pool_map(&maps[2], pools->warm_k, false, warm_rows, d, d, bs) ||
      !encode_pool_map(&maps[3], pools->warm_v, false, warm_rows, d, d, bs))
    return false;
  Entry& e = cache[next];
  next = (next + 1) % 4;
  for (int i = 0; i < 4; ++i) e.ptr[i] = ptr[i];
  e.hot_rows = hot_rows;
  e.warm_rows = warm_rows;
  e.d = d;
  e.bs = bs;
  e.valid = 1;
  std::memcpy(e.maps, maps, sizeof(e.maps));
  return true;
}

static int32_t decode_impl(const tkv_pools* pools, const tkv_decode_args* a,
                           const tkv_exchange* xc, void* stream) {
  Plan plan;
  int32_t st = make_plan(pools, a, &plan);
  if (st != TKV_OK) return st;
  if (!a->query || !a->out || !aligned(a->query, 16)) return TKV_ERR_INVALID;
  if (a->max_blocks > 0 && (!a->block_table || !a->block_states || !a->block_lengths))
    return TKV_ERR_INVALID;
  if (!a->workspace || !layout_fits(a->workspace_bytes, plan.counters_bytes, plan.data_bytes) ||
      !aligned(a->workspace, 256))
    return TKV_ERR_WORKSPACE;
  if (pools->hot_slots * pools->kv_heads * pools->block_size >= (int64_t(1) << 31))
    return TKV_ERR_INVALID;
  int sms = 0;
  st = current_device_sms(&sms);
  if (st != TKV_OK) return st;

  CUtensorMap maps[4];
  if (!pool_maps(pools, maps)) return TKV_ERR_CUDA;
  const int bs = pools->block_size, d = pools->head_dim, hkv = pools->kv_heads;

  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.query = a->query;
  p.table = a->block_table;
  p.states = a->block_states;
  p.lengths = a->block_lengths;
  p.nb_dev = a->num_blocks_dev;
  p.k_scale = pools->k_scale;
  p.k_zero = pools->k_zero;
  p.v_scale = pools->v_scale;
  p.v_zero = pools->v_zero;
  p.out = a->out;
  p.out_lse = a->out_lse;
  p.err = reinterpret_cast<uint32_t*>(ws);
  p.counters = reinterpret_cast<uint32_t*>(ws + kAlign);
  uint8_t* data = ws + data_base(a->workspace_bytes);
  if (plan.splits > 1) {
    p.part_o = reinterpret_cast<float*>(data + plan.off_part_o);
    p.part_lse = reinterpret_cast<float*>(data + plan.off_part_lse);
  }
  if (plan.group_size < plan.splits) {
    p.gpart_o = reinterpret_cast<float*>(data + plan.off_gpart_o);
    p.gpart_lse = reinterpret_cast<float*>(data + plan.off_gpart_lse);
  }
  if (a->score_sums) {
    p.lse_final = reinterpret_cast<float*>(data + plan.off_lse_final);
    p.lse_blk = reinterpret_cast<float*>(data + plan.off_lse_blk);
  }
  p.table_stride = a->table_stride;
  p.hot_slots = pools->hot_slots;
  p.warm_slots = pools->warm_slots;
  p.nb_uniform = a->num_blocks;
  p.batch = a->batch;
  p.kv_heads = hkv;
  p.num_heads = a->num_heads;
  p.groups = a->num_kv_groups;
  p.max_blocks = a->max_blocks;
  p.splits = plan.splits;
  p.chunk = plan.chunk;
  p.group_size = plan.group_size;
  {
    // the first wave of CTAs (those resident at once) prefetches before its
    // dependency wait; later waves start after the previous kernel is done
    int ctas = 0;
    if (!cached_occupancy(d, bs, pools->format, a->query_dtype, &ctas) || ctas <= 0)
      return TKV_ERR_CUDA;
    p.prefetch_ctas = sms * ctas;
  }
  p.out_dtype = a->out_dtype;
  p.scale_log2 = a->scaling * kLog2e;
  if (xc) {
    p.x_world = xc->world;
    p.x_rank = xc->rank;
    p.x_epoch = xc->epoch;
    p.x_rows_cap = xc->rows_cap;
    p.x_units_cap = xc->units_cap;
    p.x_timeout_ns = xc->timeout_ns;
    p.x_epoch_dev = xc->epoch_dev;
    for (int q = 0; q < xc->world; ++q) p.x_inbox[q] = reinterpret_cast<uint8_t*>(xc->inbox[q]);
  }

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  st = cuda_status(launch_decode(p, maps, d, bs, pools->format, a->query_dtype, s));
  if (st != TKV_OK || !a->score_sums) return st;
  ScoreParams sp;
  sp.lse_blk = p.lse_blk;
  sp.lse_final = p.lse_final;
  sp.nb_dev = a->num_blocks_dev;
  sp.score_sums = a->score_sums;
  sp.nb_uniform = a->num_blocks;
  sp.num_heads = a->num_heads;
  sp.max_blocks = a->max_blocks;
  sp.rows = a->batch * a->num_heads;
  if (a->max_blocks == 0) return TKV_OK;
  return cuda_status(launch_scores(sp, s));
}

int32_t tkv_decode_attention(const tkv_pools* pools, const tkv_decode_args* a, void* stream) {
  return decode_impl(pools, a, nullptr, stream);
}

size_t tkv_exchange_bytes(int32_t world, int32_t rows, int32_t units, int32_t head_dim) {
  if (world < 1 || world > TKV_EXCHANGE_MAX_RANKS || rows < 1 || units < 1 || head_dim < 1) return 0;
  return xchg_total_bytes(world, rows, units, head_dim);
}

int32_t tkv_exchange_alloc(size_t bytes, void** ptr_out, void* ipc_handle_out) {
  if (!ptr_out || !ipc_handle_out || bytes == 0) return TKV_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == TKV_IPC_HANDLE_BYTES, "IPC handle size");
  void* ptr = nullptr;
  if (cudaMalloc(&ptr, bytes) != cudaSuccess) return TKV_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) {
    cudaFree(ptr);
    return TKV_ERR_CUDA;
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *ptr_out = ptr;
  return TKV_OK;
}

int32_t tkv_exchange_open(const void* ipc_handle, void** ptr_out) {
  if (!ipc_handle || !ptr_out) return TKV_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* ptr = nullptr;
  if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return TKV_ERR_CUDA;
  *ptr_out = ptr;
  return TKV_OK;
}

int32_t tkv_exchange_close(void* mapped_ptr) {
  if (!mapped_ptr) return TKV_ERR_INVALID;
  return cudaIpcCloseMemHandle(mapped_ptr) == cudaSuccess ? TKV_OK : TKV_ERR_CUDA;
}

int32_t tkv_exchange_free(void* ptr) {
  if (!ptr) return TKV_ERR_INVALID;
  return cudaFree(ptr) == cudaSuccess ? TKV_OK : TKV_ERR_CUDA;
}

int32_t tkv_decode_attention_exchange(const tkv_pools* pools, const tkv_decode_args* a,
                                      const tkv_exchange* xc, void* stream) {
  if (!xc || !a || !pools) return TKV_ERR_INVALID;
  if (xc->world < 1 || xc->world > TKV_EXCHANGE_MAX_RANKS || xc->rank < 0 || xc->rank >= xc->world ||
      (xc->epoch == 0 && !xc->epoch_dev))
    return TKV_ERR_INVALID;
  if (xc->epoch_dev && !aligned(xc->epoch_dev, 4)) return TKV_ERR_INVALID;
  for (int q = 0; q < xc->world; ++q)
    if (!xc->inbox[q] || !aligned(xc->inbox[q], 256)) return TKV_ERR_INVALID;
  const int64_t rows = (int64_t)a->batch * a->num_heads;
  const int64_t units = (int64_t)a->batch * pools->kv_heads;
  if (rows > xc->rows_cap || units > xc->units_cap) return TKV_ERR_INVALID;
  // every unit's last CTA waits for the peers while holding an SM slot; the
  // other CTAs must always find free slots
  int sms = 0;
  int32_t st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  int ctas = 0;
  if (!cached_occupancy(pools->head_dim, pools->block_size, pools->format, a->query_dtype, &ctas) ||
      ctas <= 0)
    return TKV_ERR_CUDA;
  if (units * 2 > (int64_t)sms * ctas) return TKV_ERR_UNSUPPORTED;
  return decode_impl(pools, a, xc, stream);
}

int32_t tkv_merge_partials(const float* part_o, int64_t o_part_stride, const float* part_lse,
                           int64_t lse_part_stride, int32_t parts, int32_t rows,
                           int32_t head_dim, void* out, int32_t out_dtype, float* out_lse,
                           void* stream) {
  if (!part_o || !part_lse || !out || parts <= 0 || rows < 0 || head_dim <= 0)
    return TKV_ERR_INVALID;
  if (parts > 1 && (o_part_stride < (int64_t)rows * head_dim || lse_part_stride < rows))
    return TKV_ERR_INVALID;
  if (out_dtype != TKV_DTYPE_F16 && out_dtype != TKV_DTYPE_BF16 && out_dtype != TKV_DTYPE_F32)
    return TKV_ERR_UNSUPPORTED;
  if (rows == 0) return TKV_OK;
  int sms = 0;
  int32_t st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  MergeParams p{part_o, part_lse, o_part_stride, lse_part_stride, out, out_lse,
                parts, rows, head_dim, out_dtype};
  return cuda_status(launch_merge(p, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_block_scores(const float* score_sums, const int32_t* block_lengths,
                         int64_t table_stride, const int32_t* num_blocks_dev, int32_t num_blocks,
                         int32_t batch, int32_t num_heads, int32_t max_blocks,
                         float* block_scores, void* stream) {
  if (!score_sums || !block_lengths || !block_scores || batch <= 0 || num_heads <= 0 ||
      max_blocks < 0 || num_blocks < 0 || num_blocks > max_blocks || table_stride < max_blocks)
    return TKV_ERR_INVALID;
  if (max_blocks == 0) return TKV_OK;
  int sms = 0;
  int32_t st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  BlockScoreParams p{score_sums, block_lengths, num_blocks_dev, block_scores, table_stride,
                     num_blocks,  batch,         num_heads,      max_blocks};
  return cuda_status(launch_block_scores(p, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_quantize_rows_r(const void* x, int64_t rows, int32_t dim, void* codes, void* scale,
                            void* zero, void* stream) {
  if (rows < 0 || !x || !codes || !scale || !zero) return TKV_ERR_INVALID;
  if (dim != 16 && dim != 32 && dim != 64 && dim != 128 && dim != 256) return TKV_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(codes, 8) || !aligned(scale, 2) || !aligned(zero, 2))
    return TKV_ERR_INVALID;
  if (rows == 0) return TKV_OK;
  int sms = 0;
  int32_t st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  return cuda_status(
      launch_quantize_rows(x, rows, dim, codes, scale, zero, reinterpret_cast<cudaStream_t>(stream)));
}

static int32_t fill_demote(const tkv_pools* pl, const int32_t* src, const int32_t* dst,
                           const int32_t* lengths, int32_t count, int32_t clear_tail,
                           DemoteParams* p) {
  int32_t st = check_pools(pl, true);
  if (st != TKV_OK) return st;
  if (count < 0) return TKV_ERR_INVALID;
  if (count > 0 && (!src || !dst || !lengths)) return TKV_ERR_INVALID;
  p->hot_k = pl->hot_k;
  p->hot_v = pl->hot_v;
  p->warm_k = pl->warm_k;
  p->warm_v = pl->warm_v;
  p->k_scale = pl->k_scale;
  p->k_zero = pl->k_zero;
  p->v_scale = pl->v_scale;
  p->v_zero = pl->v_zero;
  p->src = src;
  p->dst = dst;
  p->lengths = lengths;
  p->hot_slots = pl->hot_slots;
  p->warm_slots = pl->warm_slots;
  p->count = count;
  p->kv_heads = pl->kv_heads;
  p->block_size = pl->block_size;
  p->head_dim = pl->head_dim;
  p->clear_tail = clear_tail;
  return TKV_OK;
}

int32_t tkv_demote_to_warm(const tkv_pools* pools, const int32_t* src_hot_slots,
                           const int32_t* dst_warm_slots, const int32_t* lengths, int32_t count,
                           int32_t clear_tail, void* stream) {
  DemoteParams p;
  int32_t st = fill_demote(pools, src_hot_slots, dst_warm_slots, lengths, count, clear_tail, &p);
  if (st != TKV_OK) return st;
  if (count == 0) return TKV_OK;
  int sms = 0;
  st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  return cuda_status(launch_demote(p, pools->format, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_promote_to_hot(const tkv_pools* pools, const int32_t* src_warm_slots,
                           const int32_t* dst_hot_slots, const int32_t* lengths, int32_t count,
                           void* stream) {
  if (pools && pools->format != TKV_FORMAT_R) return TKV_ERR_UNSUPPORTED;
  DemoteParams p;
  int32_t st = fill_demote(pools, src_warm_slots, dst_hot_slots, lengths, count, 0, &p);
  if (st != TKV_OK) return st;
  if (count == 0) return TKV_OK;
  int sms = 0;
  st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  return cuda_status(launch_promote(p, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_append_hot_tokens(const tkv_pools* pools, int32_t hot_slot, int32_t start,
                              int32_t tokens, const void* key, const void* value,
                              const tkv_table_cell* cells, int32_t n_cells, void* stream) {
  if (!pools || !pools->hot_k || !pools->hot_v || !key || !value) return TKV_ERR_INVALID;
  if (pools->kv_heads <= 0 || pools->block_size <= 0 || pools->hot_slots <= 0) return TKV_ERR_INVALID;
  if (pools->head_dim <= 0 || pools->head_dim % 8 != 0) return TKV_ERR_UNSUPPORTED;
  if (hot_slot < 0 || hot_slot >= pools->hot_slots) return TKV_ERR_INVALID;
  if (start < 0 || tokens < 1 || start + tokens > pools->block_size) return TKV_ERR_INVALID;
  if (!aligned(pools->hot_k, 16) || !aligned(pools->hot_v, 16) || !aligned(key, 16) ||
      !aligned(value, 16))
    return TKV_ERR_INVALID;
  if (n_cells < 0 || n_cells > TKV_APPEND_MAX_CELLS || (n_cells > 0 && !cells)) return TKV_ERR_INVALID;
  AppendParams p;
  std::memset(&p, 0, sizeof(p));
  p.hot_k = pools->hot_k;
  p.hot_v = pools->hot_v;
  p.key = key;
  p.value = value;
  p.slot = hot_slot;
  p.start = start;
  p.tokens = tokens;
  p.kv_heads = pools->kv_heads;
  p.block_size = pools->block_size;
  p.head_dim = pools->head_dim;
  p.n_cells = n_cells;
  for (int i = 0; i < n_cells; ++i) {
    if (!cells[i].table || cells[i].index < 0 || !aligned(cells[i].table, 4)) return TKV_ERR_INVALID;
    p.cell_ptr[i] = cells[i].table + cells[i].index;
    p.cell_val[i] = cells[i].value;
  }
  int sms = 0;
  const int32_t st = current_device_sms(&sms);
  if (st != TKV_OK) return st;
  return cuda_status(launch_append(p, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_store_prefill_blocks(const tkv_pools* pools, const void* key, const void* value,
                                 int32_t tokens, const int32_t* blocks, int32_t count,
                                 void* stream) {
  if (!pools || !key || !value || tokens < 0 || count < 0 || (count > 0 && !blocks))
    return TKV_ERR_INVALID;
  if (pools->format != TKV_FORMAT_R) return TKV_ERR_UNSUPPORTED;
  if (pools->head_dim != 64 && pools->head_dim != 128) return TKV_ERR_UNSUPPORTED;
  if (pools->kv_heads <= 0 || pools->block_size <= 0 || pools->hot_slots < 0 ||
      pools->warm_slots < 0)
    return TKV_ERR_INVALID;
  if (pools->hot_slots > 0 && (!pools->hot_k || !pools->hot_v || !aligned(pools->hot_k, 16) ||
                               !aligned(pools->hot_v, 16)))
    return TKV_ERR_INVALID;
  if (pools->warm_slots > 0 &&
      (!pools->warm_k || !pools->warm_v || !pools->k_scale || !pools->k_zero || !pools->v_scale ||
       !pools->v_zero || !aligned(pools->warm_k, 16) || !aligned(pools->warm_v, 16) ||
       !aligned(pools->k_scale, 2) || !aligned(pools->k_zero, 2) || !aligned(pools->v_scale, 2) ||
       !aligned(pools->v_zero, 2)))
    return TKV_ERR_INVALID;
  if (!aligned(key, 16) || !aligned(value, 16) || (count > 0 && !aligned(blocks, 4)))
    return TKV_ERR_INVALID;
  if (count == 0) return TKV_OK;
  PrefillStoreParams p;
  std::memset(&p, 0, sizeof(p));
  p.key = key;
  p.value = value;
  p.hot_k = pools->hot_k;
  p.hot_v = pools->hot_v;
  p.warm_k = pools->warm_k;
  p.warm_v = pools->warm_v;
  p.k_scale = pools->k_scale;
  p.k_zero = pools->k_zero;
  p.v_scale = pools->v_scale;
  p.v_zero = pools->v_zero;
  p.blocks = blocks;
  p.hot_slots = pools->hot_slots;
  p.warm_slots = pools->warm_slots;
  p.count = count;
  p.tokens = tokens;
  p.kv_heads = pools->kv_heads;
  p.block_size = pools->block_size;
  p.head_dim = pools->head_dim;
  return cuda_status(launch_store_prefill(p, reinterpret_cast<cudaStream_t>(stream)));
}

static bool prefill_maps(const PrefillParams& p, CUtensorMap maps[2]) {
  return encode_head_rows_map(&maps[0], p.q, (int64_t)p.batch * p.num_heads, p.tq, p.head_dim) &&
         encode_head_rows_map(&maps[1], p.k, (int64_t)p.batch * p.kv_heads, p.tk, p.head_dim);
}

static int32_t prefill_params(const void* q, const void* k, int32_t batch, int32_t num_heads,
                              int32_t kv_heads, int32_t tq, int32_t tk, int32_t head_dim,
                              float scaling, int32_t causal, PrefillParams* p) {
  if (!q || !k || !aligned(q, 16) || !aligned(k, 16)) return TKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return TKV_ERR_UNSUPPORTED;
  if (batch < 1 || num_heads < 1 || kv_heads < 1 || num_heads % kv_heads != 0 || tq < 1 || tk < 1)
    return TKV_ERR_INVALID;
  if (causal && tk < tq) return TKV_ERR_INVALID;
  if (!(scaling > 0.f) || !std::isfinite(scaling)) return TKV_ERR_INVALID;
  std::memset(p, 0, sizeof(*p));
  p->q = q;
  p->k = k;
  p->batch = batch;
  p->num_heads = num_heads;
  p->kv_heads = kv_heads;
  p->groups = num_heads / kv_heads;
  p->tq = tq;
  p->tk = tk;
  p->head_dim = head_dim;
  p->q_offset = tk - tq;
  p->causal = causal ? 1 : 0;
  p->scaling = scaling;
  int sms = 0;
  return current_device_sms(&sms);
}

int32_t tkv_prefill_lse(const void* q, const void* k, int32_t batch, int32_t num_heads,
                        int32_t kv_heads, int32_t tq, int32_t tk, int32_t head_dim, float scaling,
                        int32_t causal, float* lse, void* stream) {
  PrefillParams p;
  int32_t st = prefill_params(q, k, batch, num_heads, kv_heads, tq, tk, head_dim, scaling, causal, &p);
  if (st != TKV_OK) return st;
  if (!lse) return TKV_ERR_INVALID;
  p.lse = lse;
  CUtensorMap maps[2];
  if (!prefill_maps(p, maps)) return TKV_ERR_CUDA;
  return cuda_status(launch_prefill_lse(p, maps, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_prefill_block_scores(const void* q, const void* k, const float* lse, int32_t batch,
                                 int32_t num_heads, int32_t kv_heads, int32_t tq, int32_t tk,
                                 int32_t head_dim, float scaling, int32_t causal,
                                 int32_t block_size, float* token_mass, float* block_scores,
                                 void* stream) {
  PrefillParams p;
  int32_t st = prefill_params(q, k, batch, num_heads, kv_heads, tq, tk, head_dim, scaling, causal, &p);
  if (st != TKV_OK) return st;
  if (!lse || !token_mass || !block_scores || block_size < 1) return TKV_ERR_INVALID;
  p.lse = const_cast<float*>(lse);
  p.token_mass = token_mass;
  p.block_scores = block_scores;
  p.block_size = block_size;
  CUtensorMap maps[2];
  if (!prefill_maps(p, maps)) return TKV_ERR_CUDA;
  return cuda_status(launch_prefill_scores(p, maps, reinterpret_cast<cudaStream_t>(stream)));
}

int32_t tkv_prefill_read_errors(uint32_t* bits_out, void* stream) {
  if (!bits_out) return TKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* word = nullptr;
  if (prefill_error_word(&word) != cudaSuccess) return TKV_ERR_CUDA;
  uint32_t bits = 0;
  if (cudaMemcpyAsync(&bits, word, sizeof(bits), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return TKV_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TKV_ERR_CUDA;
  if (cudaMemsetAsync(word, 0, sizeof(uint32_t), s) != cudaSuccess) return TKV_ERR_CUDA;
  *bits_out = bits;
  return TKV_OK;
}

int32_t tkv_read_device_errors(void* workspace, uint32_t* bits_out, void* stream) {
  if (!workspace || !bits_out) return TKV_ERR_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t bits = 0;
  if (cudaMemcpyAsync(&bits, workspace, sizeof(bits), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return TKV_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TKV_ERR_CUDA;
  if (cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s) != cudaSuccess) return TKV_ERR_CUDA;
  *bits_out = bits;
  return TKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without a caller workspace.
//
// Some callers cannot allocate device memory: a serving runtime that has
// already handed (nearly) all of HBM to its own KV-cache pools and forbids side
// allocations, or a host that reaches this library only through the C ABI with
// no device-allocation binding.  For them the split partials, split tickets,
// chunk counters and score scratch live in this fixed array instead.  Every
// GPU that loads the library's module holds TKV_NOALLOC_SCRATCH_BYTES of it
// until the process exits.  Host code must not use `g_tkv_noalloc_scratch` as
// a device address (on the host the name is only a stand-in); its device
// address is looked up per device with cudaGetSymbolAddress.
//
// Under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default of recent
// CUDA runtimes) the array is committed on a device only when this module is
// first loaded there, which the first cudaGetSymbolAddress does.
// tkv_noalloc_prepare() does that up front, before the caller hands HBM to its
// pools; otherwise the first no-alloc call on the device does it.
//
// Layout: the workspace layout of tkv_decode_attention over the whole array --
// [0, 256) the device error word (sticky: set by the kernels, cleared only by
// tkv_noalloc_read_device_errors), then the counters, then the data regions.
// ---------------------------------------------------------------------------
namespace {

__device__ __align__(256) uint8_t g_tkv_noalloc_scratch[TKV_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on device `dev`, which must be current;
// resolved on the first request for that device and kept.
int32_t noalloc_scratch_on(int dev, void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return TKV_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tkv_noalloc_scratch) != cudaSuccess || p == nullptr)
      return TKV_ERR_CUDA;
    addr[dev] = p;
  }
  *out = addr[dev];
  return TKV_OK;
}

int32_t noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TKV_ERR_NO_DEVICE;
  return noalloc_scratch_on(dev, out);
}

}  // namespace

extern "C" int32_t tkv_noalloc_prepare(int32_t device) {
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return TKV_ERR_NO_DEVICE;
  const int dev = device < 0 ? cur : device;
  if (dev != cur && cudaSetDevice(dev) != cudaSuccess) return TKV_ERR_NO_DEVICE;
  int sms = 0;
  int32_t st = current_device_sms(&sms);  // rejects devices that are not sm_100
  void* scratch = nullptr;
  if (st == TKV_OK) st = noalloc_scratch_on(dev, &scratch);
  if (dev != cur && cudaSetDevice(cur) != cudaSuccess && st == TKV_OK) st = TKV_ERR_CUDA;
  return st;
}

extern "C" int32_t tkv_noalloc_read_device_errors(uint32_t* bits_out, void* stream) {
  if (!bits_out) return TKV_ERR_INVALID;
  void* scratch = nullptr;
  const int32_t st = noalloc_scratch(&scratch);
  if (st != TKV_OK) return st;
  return tkv_read_device_errors(scratch, bits_out, stream);
}

extern "C" int32_t tkv_decode_attention_noalloc(const tkv_pools* pools,
                                                const tkv_decode_args* args, void* stream) {
  if (!args) return TKV_ERR_INVALID;
  Plan plan;
  int32_t st = make_plan(pools, args, &plan);
  if (st != TKV_OK) return st;
  if (plan.total > (size_t)TKV_NOALLOC_SCRATCH_BYTES) return TKV_ERR_SCRATCH_LIMIT;
  int sms = 0;
  st = current_device_sms(&sms);  // rejects devices that are not sm_100
  if (st != TKV_OK) return st;
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st != TKV_OK) return st;
  // The array keeps whatever the previous call left.  The split tickets and
  // chunk counters must start at zero (a call cut short by a timeout can
  // leave them set), so they are cleared first; the error word at offset 0
  // is left alone so that errors stay readable until
  // tkv_noalloc_read_device_errors clears them.
  if (cudaMemsetAsync(reinterpret_cast<uint8_t*>(scratch) + kAlign, 0, plan.counters_bytes,
                      reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return TKV_ERR_CUDA;
  tkv_decode_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = (size_t)TKV_NOALLOC_SCRATCH_BYTES;
  return tkv_decode_attention(pools, &a, stream);
}
