/*
 * tierkv_b200.h -- C ABI of the B200-native (sm_100a) tiered paged
 * decode-attention path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * passed as `void*` (NULL = legacy default stream); no framework types cross
 * this boundary.  Calls are asynchronous on the given stream and never
 * synchronize.  They return a tkv_status code and never abort the process.
 * No call retains a pointer after it returns; pools may be reallocated by the
 * caller between calls.
 *
 * The functions replace, one for one, the pieces of xiaoMartintin/Paged_TierKV
 * that sit on the decode hot path (file:line references are into that
 * project):
 *
 *   tkv_decode_attention   tierkv_triton.py:272-465  tierkv_decode_attention()
 *                          (kernels tierkv_triton.py:45-145, split + reduce
 *                          tierkv_triton.py:147-264)
 *   tkv_merge_partials     tierkv_triton.py:231-264  split-KV LSE reduce,
 *                          also used after the cross-GPU all-gather
 *   tkv_block_scores       tierkv_policy.py:1905-1912
 *                          TieredKVRuntime.block_scores_from_probability_sums()
 *   tkv_quantize_rows_r    tierkv_policy.py:21-36    quantize_fp16_to_int8()
 *   tkv_demote_to_warm     tierkv_policy.py:1042-1068 (compact pool) and
 *                          329-361 (dense pool) demote_to_warm(), batched
 *   tkv_promote_to_hot     tierkv_policy.py:1087-1115 (compact) and 375-402
 *                          (dense) promote_to_hot(), batched
 *   tkv_decode_attention_exchange
 *                          the survey's context-sharded decode (one context
 *                          split by block range over GPUs): decode, exchange
 *                          of the (o, LSE) partials over NVLink peer memory
 *                          and their merge in one launch per rank
 *   tkv_prefill_lse /      modeling_llama.py:281-302 compute_prefill_block_scores()
 *   tkv_prefill_block_scores  with tierkv_policy.py:1378-1388 compute_block_scores():
 *                          exact prefill block scores without materialising
 *                          the attention weights
 *   tkv_append_hot_tokens  tierkv_policy.py:934-967 write_hot_tokens() tensor
 *                          work plus the block-table writes of _set_metadata
 *                          (917-926) and set_block_entry (1016-1035), fused
 *   tkv_store_prefill_blocks  tierkv_policy.py:1722-1766
 *                          append_prefill_with_policy(): the tensor work of its
 *                          per-block write_hot_tokens (934-967) and
 *                          write_warm_block (969-1002) calls, one launch
 *
 * Pool layout (the reference's, tierkv_policy.py:129-135 and 835-841):
 *   hot_k / hot_v     [hot_slots,  kv_heads, block_size, head_dim] fp16
 *   warm_k / warm_v   [warm_slots, kv_heads, block_size, head_dim]
 *                       Format R: uint8 codes (the reference layout)
 *                       Format S: int8 codes
 *   k_scale/k_zero/v_scale/v_zero
 *                       Format R: [warm_slots, kv_heads, block_size(, 1)] fp16
 *                       Format S: k_scale/v_scale [warm_slots, kv_heads] fp32,
 *                                 k_zero/v_zero unused (may be NULL)
 * Tables (per sequence row, `table_stride` int32 apart):
 *   block_table[b]   slot of logical block b in the HOT pool when
 *                    block_states[b] == 0, in the WARM pool when == 1;
 *                    ignored (never dereferenced) for COLD blocks
 *   block_states[b]  0 HOT, 1 WARM, anything else COLD (evicted)
 *   block_lengths[b] valid tokens of logical block b (clamped to [0, bs])
 */
#ifndef TIERKV_B200_H
#define TIERKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TKV_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------ */
#define TKV_OK                 0
#define TKV_ERR_INVALID        1  /* bad pointer / shape / size   -> ValueError  */
#define TKV_ERR_UNSUPPORTED    2  /* geometry or format not built -> ValueError  */
#define TKV_ERR_WORKSPACE      3  /* workspace missing or too small -> ValueError */
#define TKV_ERR_CUDA           4  /* CUDA driver / launch failure -> RuntimeError */
#define TKV_ERR_NO_DEVICE      5  /* no usable sm_100 device       -> RuntimeError */
#define TKV_ERR_SCRATCH_LIMIT  6  /* call needs more than the fixed no-alloc scratch -> ValueError */

/* Size of the library-owned device array used by tkv_decode_attention_noalloc. */
#define TKV_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* ---- enums --------------------------------------------------------------- */
#define TKV_STATE_HOT   0
#define TKV_STATE_WARM  1
#define TKV_STATE_COLD  2

#define TKV_FORMAT_R    0  /* uint8, asymmetric, fp16 scale + zero per token row */
#define TKV_FORMAT_S    1  /* int8, symmetric absmax, fp32 scale per (block, kv head) */

#define TKV_DTYPE_F16   0
#define TKV_DTYPE_BF16  1
#define TKV_DTYPE_F32   2

/* Device-side error bits, reported through tkv_read_device_errors(). */
#define TKV_DEVERR_BAD_SLOT  0x1u  /* HOT/WARM block whose slot is outside its pool */
#define TKV_DEVERR_TIMEOUT   0x2u  /* a bounded pipeline wait gave up            */

/* tkv_decode_args.flags: blocks per work chunk (0 = chosen by the planner) */
#define TKV_FLAG_CHUNK_MASK  0xff

typedef struct tkv_pools {
    void*   hot_k;
    void*   hot_v;
    void*   warm_k;
    void*   warm_v;
    void*   k_scale;
    void*   k_zero;
    void*   v_scale;
    void*   v_zero;
    int64_t hot_slots;
    int64_t warm_slots;
    int32_t kv_heads;
    int32_t block_size;   /* 16 or 32 */
    int32_t head_dim;     /* 64 or 128 */
    int32_t format;       /* TKV_FORMAT_R / TKV_FORMAT_S */
} tkv_pools;

typedef struct tkv_decode_args {
    const void*    query;          /* [batch, num_heads, head_dim] (query_len 1),
                                      16-byte aligned */
    int32_t        query_dtype;    /* TKV_DTYPE_F16 / TKV_DTYPE_BF16 */
    int32_t        out_dtype;      /* TKV_DTYPE_F16 / BF16 / F32 */
    int32_t        batch;
    int32_t        num_heads;
    int32_t        num_kv_groups;  /* num_heads / kv_heads, 1..8 */
    int32_t        max_blocks;     /* columns of score_sums (block_table length) */
    const int32_t* block_table;    /* [batch, table_stride] */
    const int32_t* block_states;
    const int32_t* block_lengths;
    int64_t        table_stride;
    const int32_t* num_blocks_dev; /* optional device [batch] block counts */
    int32_t        num_blocks;     /* uniform count, or upper bound of num_blocks_dev */
    float          scaling;
    void*          out;            /* [batch, num_heads, head_dim] out_dtype; with
                                      out_dtype F32 the row is the normalised
                                      partial o of a context shard */
    float*         out_lse;        /* optional [batch, num_heads] natural-log LSE */
    float*         score_sums;     /* optional [batch, num_heads, max_blocks] */
    int32_t        num_splits;     /* 0 = automatic */
    int32_t        flags;          /* bits 0-7: blocks per work chunk (0 = planned,
                                      else 8, 16 or 32); other bits 0 */
    void*          workspace;      /* zero-filled once by the owner, see below */
    size_t         workspace_bytes;
} tkv_decode_args;

/* Library version (TKV_ABI_VERSION) and a static message for a status. */
int32_t     tkv_get_version(void);
const char* tkv_status_string(int32_t status);

/* Number of splits the launch will use and the workspace it needs.
 * The workspace must be zero-filled once when it is allocated.  Its first
 * eighth holds the work counters, which every launch returns to zero; the
 * partial results live above them, so one workspace serves calls of any
 * shape in any order.  Concurrent calls on different streams need different
 * workspaces.
 * Replaces the partial-buffer allocations of tierkv_triton.py:316-325. */
int32_t tkv_decode_plan(const tkv_pools* pools, const tkv_decode_args* args,
                        int32_t* num_splits_out, size_t* workspace_bytes_out);

/* Tiered paged decode attention, one query token per sequence.
 * HOT tiles are read as fp16, WARM tiles dequantized in registers, COLD
 * tiles never read (each valid COLD token adds logit 0 / value 0, as in the
 * reference).  Optional per-block softmax mass (score_sums) as in
 * tierkv_triton.py:121-145 (zero for blocks >= num_blocks).
 * Replaces tierkv_triton.py:272-465. */
int32_t tkv_decode_attention(const tkv_pools* pools, const tkv_decode_args* args, void* stream);

/* LSE merge of `parts` normalised partials.  Partial i is the fp32 block
 * part_o + i * o_part_stride ([rows, head_dim]) with its natural-log LSEs at
 * part_lse + i * lse_part_stride ([rows], -inf = empty); strides are in
 * elements, so one all-gathered [parts, rows*head_dim + rows] buffer can be
 * merged in place.  Writes out [rows, head_dim] (out_dtype) and optionally
 * out_lse [rows].
 * Replaces tierkv_triton.py:231-264 (and merges context shards). */
int32_t tkv_merge_partials(const float* part_o, int64_t o_part_stride, const float* part_lse,
                           int64_t lse_part_stride, int32_t parts, int32_t rows,
                           int32_t head_dim, void* out, int32_t out_dtype, float* out_lse,
                           void* stream);

/* Per-block importance: block_scores[s, b] = mean_h score_sums[s, h, b] /
 * max(block_lengths[s, b], 1) for b < num_blocks(s), 0 beyond.
 * score_sums [batch, num_heads, max_blocks]; block_scores [batch, max_blocks].
 * Replaces tierkv_policy.py:1905-1912. */
int32_t tkv_block_scores(const float* score_sums, const int32_t* block_lengths,
                         int64_t table_stride, const int32_t* num_blocks_dev,
                         int32_t num_blocks, int32_t batch, int32_t num_heads,
                         int32_t max_blocks, float* block_scores, void* stream);

/* Format R quantization of `rows` contiguous fp16 rows of `dim` values,
 * bit-exact with quantize_fp16_to_int8 (tierkv_policy.py:21-36):
 * codes [rows, dim] uint8, scale / zero [rows] fp16. */
int32_t tkv_quantize_rows_r(const void* x, int64_t rows, int32_t dim, void* codes,
                            void* scale, void* zero, void* stream);

/* Batched HOT->WARM demotion of whole blocks (all kv heads, K and V):
 * block i reads HOT slot src_hot_slots[i] rows [0, lengths[i]) and writes
 * WARM slot dst_warm_slots[i].  Format R: bit-exact with demote_to_warm;
 * clear_tail != 0 additionally sets rows >= length to code 0 / scale 1 /
 * zero 0 (dense pool, tierkv_policy.py:350-356); clear_tail == 0 leaves them
 * (compact pool, tierkv_policy.py:1058-1063).  Format S: one fp32 scale per
 * (block, kv head) over the valid rows; tail rows get code 0.
 * Slot lists and lengths are device int32 arrays of `count` entries.
 * Replaces tierkv_policy.py:1042-1068 / 329-361. */
int32_t tkv_demote_to_warm(const tkv_pools* pools, const int32_t* src_hot_slots,
                           const int32_t* dst_warm_slots, const int32_t* lengths,
                           int32_t count, int32_t clear_tail, void* stream);

/* Batched WARM->HOT promotion (Format R), bit-exact with
 * dequantize_int8_to_fp16 (tierkv_policy.py:39-44) as used by promote_to_hot
 * (tierkv_policy.py:1087-1115): rows [0, lengths[i]) of WARM slot
 * src_warm_slots[i] are written to HOT slot dst_hot_slots[i].
 * Replaces tierkv_policy.py:1087-1115 / 375-402. */
int32_t tkv_promote_to_hot(const tkv_pools* pools, const int32_t* src_warm_slots,
                           const int32_t* dst_hot_slots, const int32_t* lengths,
                           int32_t count, void* stream);

/* One int32 table cell for tkv_append_hot_tokens: table[index] = value. */
typedef struct tkv_table_cell {
    int32_t* table;   /* device pointer to an int32 table */
    int64_t  index;   /* element index */
    int32_t  value;
    int32_t  reserved;
} tkv_table_cell;

#define TKV_APPEND_MAX_CELLS 8

/* Decode-time KV append in one launch: rows [start, start + tokens) of HOT
 * slot hot_slot get the new key / value rows ([kv_heads, tokens, head_dim]
 * fp16, contiguous, 16-byte aligned), rows [start + tokens, block_size) are
 * zeroed (as write_hot_tokens does, tierkv_policy.py:956-958), and up to
 * TKV_APPEND_MAX_CELLS block-table cells are written (the GPU-table updates of
 * _set_metadata and set_block_entry, passed by value: no host->device copy).
 * Replaces the tensor work of tierkv_policy.py:934-967 plus 917-926 and
 * 1016-1035; the slot bookkeeping stays with the caller. */
int32_t tkv_append_hot_tokens(const tkv_pools* pools, int32_t hot_slot, int32_t start,
                              int32_t tokens, const void* key, const void* value,
                              const tkv_table_cell* cells, int32_t n_cells, void* stream);

/* The data movement of a prefilled layer in one launch.  `blocks` is a
 * device int32 array of `count` entries of 4: (state, slot, first token,
 * length).  State 0 (HOT): rows [first, first + length) of key / value
 * ([kv_heads, tokens, head_dim] fp16, contiguous, 16-byte aligned) go to rows
 * [0, length) of HOT slot `slot` and its rows [length, block_size) are zeroed
 * (write_hot_tokens, tierkv_policy.py:934-967).  State 1 (WARM, Format R):
 * the same rows are quantized into WARM slot `slot` bit-exactly as
 * quantize_fp16_to_int8 (21-36) with per-row fp16 scale and zero point, and
 * rows [length, block_size) get code 0, scale 1, zero 0 (write_warm_block,
 * 969-1002).  0 <= length <= block_size and first + length <= tokens; an
 * entry with another state, a slot outside its pool or a token range outside
 * the input is skipped.  No two entries may name the same slot of a pool.
 * Pools absent from the call (no WARM entry) may have null pointers and 0
 * slots.  Replaces the tensor work of tierkv_policy.py:1722-1766; the slot
 * bookkeeping stays with the caller. */
int32_t tkv_store_prefill_blocks(const tkv_pools* pools, const void* key, const void* value,
                                 int32_t tokens, const int32_t* blocks, int32_t count,
                                 void* stream);

/* ---- context-sharded decode with a peer-memory exchange -------------------
 * Each rank holds a contiguous block range of the same sequences; every rank
 * launches tkv_decode_attention_exchange with its own tables and pools and
 * the same epoch.  The last CTA of each (sequence, kv head) writes its
 * normalised partial (o, LSE) into every rank's inbox through CUDA IPC
 * mappings (no multicast) as 64-bit words, each the call's epoch (high half)
 * and an fp32 value (low half) in one system-scope store; it then polls the
 * words of all ranks in its own inbox until each carries the epoch (bounded
 * by timeout_ns; TKV_DEVERR_TIMEOUT when it runs out, missing partials then
 * count as empty) and merges the world partials into args->out / out_lse
 * (and the global LSE the score pass normalises with).  Partials are
 * double-buffered by epoch parity, so a rank may run one call ahead of the
 * others.  Replaces the per-layer all-gather + merge. */
#define TKV_EXCHANGE_MAX_RANKS 8

typedef struct tkv_exchange {
    int32_t  world;        /* ranks sharing the contexts, 1..8 */
    int32_t  rank;
    uint32_t epoch;        /* +1 per call, equal on every rank, never 0 */
    int32_t  rows_cap;     /* the inboxes' capacity (their layout): rows ... */
    int32_t  units_cap;    /* ... and (sequence, kv head) units, as allocated */
    int32_t  reserved;
    uint64_t timeout_ns;   /* bound of the wait for the peers; 0 = 2 s */
    uint32_t* epoch_dev;   /* optional device word holding the epoch (read
                              instead of `epoch`, e.g. by CUDA graph replays);
                              the launch advances it by one when it is done */
    void*    inbox[TKV_EXCHANGE_MAX_RANKS];  /* rank q's inbox, mapped here */
} tkv_exchange;

/* Bytes of one rank's inbox for up to `rows` = batch * num_heads rows and
 * `units` = batch * kv_heads (sequence, kv head) pairs at head_dim; every
 * rank's inbox has the same capacities, passed in tkv_exchange. */
size_t  tkv_exchange_bytes(int32_t world, int32_t rows, int32_t units, int32_t head_dim);

/* Allocates a zeroed inbox of `bytes` on the current device and returns its
 * CUDA IPC handle (TKV_IPC_HANDLE_BYTES bytes) for the other ranks. */
#define TKV_IPC_HANDLE_BYTES 64
int32_t tkv_exchange_alloc(size_t bytes, void** ptr_out, void* ipc_handle_out);
/* Maps another rank's inbox into this process (peer access over NVLink). */
int32_t tkv_exchange_open(const void* ipc_handle, void** ptr_out);
int32_t tkv_exchange_close(void* mapped_ptr);
int32_t tkv_exchange_free(void* ptr);

int32_t tkv_decode_attention_exchange(const tkv_pools* pools, const tkv_decode_args* args,
                                      const tkv_exchange* xc, void* stream);

/* ---- prefill block scores ------------------------------------------------
 * q [batch, num_heads, tq, head_dim] and k [batch, kv_heads, tk, head_dim]
 * fp16, contiguous, 16-byte aligned; head_dim 64 or 128; num_heads a
 * multiple of kv_heads; scaling finite and > 0.  causal: key j is visible
 * to query i iff j <= i + (tk - tq) (requires tk >= tq).
 * tkv_prefill_lse writes lse [batch, num_heads, tq] fp32, the natural-log
 * LSE of the scaled, masked logits (what flash attention returns).
 * tkv_prefill_block_scores writes token_mass [tk] (the softmax mass each key
 * receives, summed over batch, heads and queries) and block_scores
 * [ceil(tk / block_size)]: token_mass / (batch * num_heads * tq) averaged over
 * each block's keys -- the reference's mean of the eager attention weights
 * over (batch, heads, queries), then per block (tierkv_policy.py:1378-1388). */
int32_t tkv_prefill_lse(const void* q, const void* k, int32_t batch, int32_t num_heads,
                        int32_t kv_heads, int32_t tq, int32_t tk, int32_t head_dim, float scaling,
                        int32_t causal, float* lse, void* stream);
int32_t tkv_prefill_block_scores(const void* q, const void* k, const float* lse, int32_t batch,
                                 int32_t num_heads, int32_t kv_heads, int32_t tq, int32_t tk,
                                 int32_t head_dim, float scaling, int32_t causal,
                                 int32_t block_size, float* token_mass, float* block_scores,
                                 void* stream);
/* Reads and clears the error bits (TKV_DEVERR_TIMEOUT) the prefill kernels of
 * the current device have recorded.  Synchronizes the stream. */
int32_t tkv_prefill_read_errors(uint32_t* bits_out, void* stream);

/* Reads and clears the device error bits (TKV_DEVERR_*) that decode calls
 * using this workspace have recorded.  Synchronizes the stream. */
int32_t tkv_read_device_errors(void* workspace, uint32_t* bits_out, void* stream);

/* Decode attention for callers that cannot allocate device memory -- a serving
 * runtime that has handed (nearly) all of HBM to its own pools and forbids side
 * allocations, or a host that reaches this library only through this C ABI
 * with no device-allocation binding of its own.  Same arguments and results as
 * tkv_decode_attention, except that args->workspace / workspace_bytes are
 * ignored: the scratch (split partials, split tickets, chunk counters, score
 * scratch, the device error word) lives in a library-owned device array of
 * TKV_NOALLOC_SCRATCH_BYTES that every GPU where the library's module is
 * loaded holds until the process exits.  The call itself allocates nothing
 * (no cudaMalloc/cudaFree, no allocating library routine); it clears the
 * counters it needs on `stream` before the launch.  Calls whose
 * tkv_decode_plan() workspace exceeds the array return TKV_ERR_SCRATCH_LIMIT.
 * The first call on a device looks up the array's device address with
 * cudaGetSymbolAddress while that device is current (see
 * tkv_noalloc_prepare); make that first call before any stream capture.  All
 * calls on a device share the one array, so calls that overlap on the GPU
 * (different streams, or different host threads) race and must be serialised
 * by the caller.  Device errors (TKV_DEVERR_*) accumulate in the array's error
 * word until tkv_noalloc_read_device_errors reads and clears them.
 * No counterpart in the reference (its wrapper allocates with torch). */
int32_t tkv_decode_attention_noalloc(const tkv_pools* pools, const tkv_decode_args* args,
                                     void* stream);

/* Resolves the no-alloc scratch array on `device` (< 0: the current device)
 * ahead of the first tkv_decode_attention_noalloc call.  Under lazy module
 * loading (CUDA_MODULE_LOADING=LAZY, the default of recent CUDA runtimes) the
 * array's TKV_NOALLOC_SCRATCH_BYTES are committed on a device when the
 * library's module is first loaded there, which this call does: call it at
 * start-up, before the runtime hands HBM to its own pools and before any
 * stream capture.  Idempotent; restores the current device.
 * No counterpart in the reference. */
int32_t tkv_noalloc_prepare(int32_t device);

/* Reads and clears the device error bits (TKV_DEVERR_*) that no-alloc decode
 * calls on the current device have recorded in the library's array (the
 * counterpart of tkv_read_device_errors for a caller workspace).
 * Synchronizes the stream.  No counterpart in the reference. */
int32_t tkv_noalloc_read_device_errors(uint32_t* bits_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TIERKV_B200_H */
