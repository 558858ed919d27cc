// tkv_internal.h -- parameter blocks shared by the host launchers and the
// sm_100a kernels of the tiered decode path (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

// HOT tiles: one 3-D TMA box per K/V tile instead of head_dim/64 2-D boxes.
#ifndef TKV_HOT_3D
#define TKV_HOT_3D 1
#endif

// Split planner: fixed cost of one decode CTA expressed in blocks of work.
#ifndef TKV_CTA_OVERHEAD_BLOCKS
#define TKV_CTA_OVERHEAD_BLOCKS 16
#endif
// ... and of claiming one work chunk (atomic ticket + table entries), as
// measured on a 131072-token context: 32-block chunks beat 16 and 8.
#ifndef TKV_CHUNK_OVERHEAD_BLOCKS
#define TKV_CHUNK_OVERHEAD_BLOCKS 6
#endif

namespace tkv {

constexpr int kFmtR = 0;
constexpr int kFmtS = 1;
constexpr int kDtF16 = 0;
constexpr int kDtBF16 = 1;
constexpr int kDtF32 = 2;
constexpr int kMaxGroups = 8;      // query heads per KV head handled by one CTA (mma N = 8)
constexpr int kMaxSplits = 512;    // split-KV partitions per (sequence, kv head)
constexpr float kLn2 = 0.693147180559945309f;
constexpr float kLog2e = 1.442695040888963387f;

// Everything one decode launch needs besides the four TMA descriptors.
struct DecodeParams {
  const void* query;          // [batch, num_heads, D]
  const int32_t* table;       // [batch, table_stride]
  const int32_t* states;
  const int32_t* lengths;
  const int32_t* nb_dev;      // optional [batch]
  const void* k_scale;        // Format R: fp16 [warm_slots*kv_heads*bs]; Format S: fp32 [warm_slots*kv_heads]
  const void* k_zero;
  const void* v_scale;
  const void* v_zero;
  void* out;                  // [batch, num_heads, D] out dtype
  float* out_lse;             // optional [batch, num_heads]
  float* part_o;              // [batch*num_heads, splits, D] (splits > 1)
  float* part_lse;            // [batch*num_heads, splits]
  float* gpart_o;             // [batch*num_heads, groups, D] (more than one split group)
  float* gpart_lse;           // [batch*num_heads, groups]
  uint32_t* counters;         // [batch*kv_heads] split (or group) tickets, [batch*kv_heads]
                              // chunk counters, then [batch*kv_heads][groups] group tickets
                              // (both reset by the last CTA of each sequence/kv head)
  float* lse_blk;             // optional [batch*num_heads, max_blocks]: per-block LSE
  float* lse_final;           // optional [batch*num_heads]: final LSE for the score pass
  uint32_t* err;              // device error bits; err[1]: exchange launch ticket
  int64_t table_stride;
  int64_t hot_slots;
  int64_t warm_slots;
  int32_t nb_uniform;
  int32_t batch;
  int32_t kv_heads;
  int32_t num_heads;
  int32_t groups;
  int32_t max_blocks;
  int32_t splits;
  int32_t chunk;              // blocks per claimed work chunk: 8, 16 or 32
  int32_t group_size;         // splits merged per group (= splits: one level)
  int32_t prefetch_ctas;      // CTAs with a smaller linear index prefetch before the
                              // dependency wait (the first wave)
  // context-sharded exchange (x_world > 0): inbox of rank q mapped at x_inbox[q];
  // layout: epoch-tagged 64-bit words, o [2][rows][world][D] then lse
  // [2][rows][world] (double-buffered by epoch parity; see xchg_total_bytes)
  int32_t x_world;
  int32_t x_rank;
  uint32_t x_epoch;
  int32_t x_rows_cap;
  int32_t x_units_cap;
  uint64_t x_timeout_ns;
  uint32_t* x_epoch_dev;      // when set, the epoch is read here and advanced by the launch
  uint8_t* x_inbox[8];
  int32_t out_dtype;
  float scale_log2;           // scaling * log2(e)
};

struct MergeParams {
  const float* part_o;        // part i at part_o + i * o_stride: [rows, D]
  const float* part_lse;      // part i at part_lse + i * lse_stride: [rows]
  int64_t o_stride;
  int64_t lse_stride;
  void* out;
  float* out_lse;
  int32_t parts;
  int32_t rows;
  int32_t head_dim;
  int32_t out_dtype;
};

struct ScoreParams {
  const float* lse_blk;       // [batch*num_heads, max_blocks]
  const float* lse_final;     // [batch*num_heads]
  const int32_t* nb_dev;
  float* score_sums;          // [batch*num_heads, max_blocks]
  int32_t nb_uniform;
  int32_t num_heads;
  int32_t max_blocks;
  int32_t rows;               // batch * num_heads
};

struct BlockScoreParams {
  const float* score_sums;    // [batch, num_heads, max_blocks]
  const int32_t* lengths;     // [batch, table_stride]
  const int32_t* nb_dev;
  float* block_scores;        // [batch, max_blocks]
  int64_t table_stride;
  int32_t nb_uniform;
  int32_t batch;
  int32_t num_heads;
  int32_t max_blocks;
};

struct DemoteParams {
  const void* hot_k;
  const void* hot_v;
  void* warm_k;
  void* warm_v;
  void* k_scale;
  void* k_zero;
  void* v_scale;
  void* v_zero;
  const int32_t* src;         // HOT slots (demote) / WARM slots (promote)
  const int32_t* dst;         // WARM slots (demote) / HOT slots (promote)
  const int32_t* lengths;
  int64_t hot_slots;
  int64_t warm_slots;
  int32_t count;
  int32_t kv_heads;
  int32_t block_size;
  int32_t head_dim;
  int32_t clear_tail;
};

// Host launchers (defined in the .cu files, called by tkv_api.cu).
cudaError_t launch_decode(const DecodeParams& p, const CUtensorMap maps[4], int head_dim,
                          int block_size, int format, int query_dtype, cudaStream_t stream);
cudaError_t decode_occupancy(int head_dim, int block_size, int format, int query_dtype,
                             int* ctas_per_sm);
cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream);
cudaError_t launch_scores(const ScoreParams& p, cudaStream_t stream);
cudaError_t launch_block_scores(const BlockScoreParams& p, cudaStream_t stream);
cudaError_t launch_quantize_rows(const void* x, int64_t rows, int dim, void* codes, void* scale,
                                 void* zero, cudaStream_t stream);
struct AppendParams {
  void* hot_k;
  void* hot_v;
  const void* key;            // [kv_heads, tokens, head_dim] fp16
  const void* value;
  int64_t slot;
  int32_t start;
  int32_t tokens;
  int32_t kv_heads;
  int32_t block_size;
  int32_t head_dim;
  int32_t n_cells;
  int32_t* cell_ptr[8];       // table + index, resolved on the host
  int32_t cell_val[8];
};

// Inbox layout of the context-sharded exchange (see DecodeParams::x_inbox):
// o words [2][rows][world][D], then LSE words [2][rows][world], double-buffered
// by epoch parity.  A word is 64 bits: the epoch of the call that wrote it in
// the high half, the fp32 value in the low half.  (`units` does not enter the
// layout.)
__host__ __device__ inline size_t xchg_o_bytes(int world, int rows, int d) {
  return (size_t)2 * rows * world * d * 8;
}
__host__ __device__ inline size_t xchg_total_bytes(int world, int rows, int units, int d) {
  (void)units;
  return xchg_o_bytes(world, rows, d) + ((size_t)2 * rows * world * 8 + 255) / 256 * 256;
}

struct PrefillParams {
  const void* q;              // [batch, num_heads, tq, head_dim] fp16
  const void* k;              // [batch, kv_heads, tk, head_dim] fp16
  float* lse;                 // [batch, num_heads, tq] natural log
  float* token_mass;          // [tk]
  float* block_scores;        // [ceil(tk / block_size)]
  int32_t batch;
  int32_t num_heads;
  int32_t kv_heads;
  int32_t groups;
  int32_t tq;
  int32_t tk;
  int32_t head_dim;
  int32_t q_offset;           // tk - tq: query i sits at position i + q_offset
  int32_t causal;
  int32_t block_size;
  float scaling;
  int32_t parts;              // column pass: CTAs per key tile
  int32_t part_items;         // column pass: (head, query tile) items per CTA
  uint32_t* err;              // the device's prefill error word (TKV_DEVERR_*)
};

// maps[0]: Q as [batch * num_heads][tq][head_dim]; maps[1]: K as
// [batch * kv_heads][tk][head_dim] (encode_head_rows_map).
cudaError_t launch_prefill_lse(const PrefillParams& p, const CUtensorMap maps[2],
                               cudaStream_t stream);
cudaError_t launch_prefill_scores(const PrefillParams& p, const CUtensorMap maps[2],
                                  cudaStream_t stream);
cudaError_t prefill_error_word(uint32_t** out);
// 4-D tiled map over fp16 rows [heads][rows][head_dim]: dims {64, rows,
// head_dim / 64, heads}, box {64, 128, head_dim / 64, 1}, 128-byte swizzle; a
// box lands as [head_dim / 64][128][64] and rows past `rows` read as zero.
bool encode_head_rows_map(CUtensorMap* map, const void* base, int64_t heads, int64_t rows,
                          int head_dim);

cudaError_t launch_demote(const DemoteParams& p, int format, cudaStream_t stream);
cudaError_t launch_append(const AppendParams& p, cudaStream_t stream);

// tkv_store_prefill_blocks: entries (state, slot, first token, length).
struct PrefillStoreParams {
  const void* key;            // [kv_heads, tokens, head_dim] fp16
  const void* value;
  void* hot_k;
  void* hot_v;
  void* warm_k;
  void* warm_v;
  void* k_scale;
  void* k_zero;
  void* v_scale;
  void* v_zero;
  const int32_t* blocks;      // [count][4]
  int64_t hot_slots;
  int64_t warm_slots;
  int32_t count;
  int32_t tokens;
  int32_t kv_heads;
  int32_t block_size;
  int32_t head_dim;
};
cudaError_t launch_store_prefill(const PrefillStoreParams& p, cudaStream_t stream);
cudaError_t launch_promote(const DemoteParams& p, cudaStream_t stream);

}  // namespace tkv
