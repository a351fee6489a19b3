/*
 * paged_attention_b200.h — C ABI of the B200 (sm_100a) paged-attention hot path.
 *
 * Drop-in for the attention seam of akshajravi/llm-inference-server:
 *   inference_server/core/attention.py:73-88     paged_attention(query, k_pool, v_pool,
 *                                                block_tables, context_lens, query_lens, scale)
 *   inference_server/core/paged_executor.py:116-125  _PagedCache.update (KV append)
 *   inference_server/core/paged_executor.py:211-263  _pack (per-step ragged metadata)
 *   inference_server/core/kv_pool.py:142-182 and paged_executor.py:265-270  block swap
 *                                                and copy-on-write moves
 *
 * Plain C types only: device pointers, element strides, sizes and a dtype enum.  The
 * library owns no device memory: the caller allocates outputs, the packed metadata
 * buffer and the workspace.  Every launch is asynchronous on the caller's stream and
 * the entry points never synchronise the device.
 *
 * Pools use the reference layout bit for bit (inference_server/core/kv_pool.py:120):
 * one contiguous [num_blocks, block_size, num_kv_heads, head_dim] tensor per layer for
 * K and one for V.  A flat slot is block * block_size + offset
 * (inference_server/core/block_table.py:143-159).
 *
 * Return codes: PA_OK or one of PA_ERR_*; pa_last_error() gives the message of the
 * calling thread's most recent failure.  Contract violations use the reference's own
 * message texts (inference_server/core/attention.py:202-219).
 */
#ifndef PAGED_ATTENTION_B200_H
#define PAGED_ATTENTION_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PA_OK 0
#define PA_ERR_INVALID_ARGUMENT 1   /* contract violation; maps to ValueError */
#define PA_ERR_UNSUPPORTED 2        /* shape/dtype this build does not run */
#define PA_ERR_CUDA 3               /* a CUDA runtime/driver call failed */
#define PA_ERR_BUFFER_TOO_SMALL 4   /* metadata buffer or workspace too small */

/* Storage dtype of query, pools and output (all three must match). */
#define PA_DTYPE_F32 0
#define PA_DTYPE_F16 1
#define PA_DTYPE_BF16 2

/*
 * Per-step plan: sizes and the offsets (in int32 words) of every array inside the
 * packed metadata buffer that pa_plan_step fills.  One plan serves every layer of a
 * step, so the host builds and uploads metadata once per step, not once per layer.
 */
typedef struct pa_step_plan {
  int32_t num_seqs;            /* B */
  int32_t num_tokens;          /* T = sum(query_lens) */
  int32_t table_width;         /* W: blocks per row of the packed int32 block table */
  int32_t block_size;          /* tokens per pool block */
  int32_t num_decode_seqs;     /* sequences with query_len == 1 */
  int32_t num_prefill_seqs;    /* sequences with query_len > 1 */
  int32_t num_prefill_tokens;  /* tokens of those sequences */
  int32_t split_blocks;        /* pool blocks per decode split (split-K) */
  int32_t num_decode_items;    /* decode work items = (sequence, split) pairs */
  int32_t num_combine_seqs;    /* decode sequences with more than one split */
  int32_t max_context;         /* max(context_lens) */
  int32_t max_query_len;       /* max(query_lens) */
  int32_t prefill_tile_tokens; /* query rows per prefill work tile (0: no tile list) */
  int32_t num_prefill_tiles;   /* prefill work tiles = (sequence, first query row) */
  int64_t total_context;       /* sum(context_lens) */
  int64_t off_block_tables;    /* [B, W] physical block ids, 0-padded */
  int64_t off_context_lens;    /* [B] tokens in the cache after this pass */
  int64_t off_query_lens;      /* [B] new tokens per sequence */
  int64_t off_cu_query_lens;   /* [B+1] exclusive prefix sum of query_lens */
  int64_t off_seq_idx;         /* [T] sequence of each packed token */
  int64_t off_q_pos;           /* [T] logical position ctx - q_len + t of each token */
  int64_t off_slot_mapping;    /* [T] flat pool slot each new token's K/V is written to */
  int64_t off_decode_items;    /* [num_decode_items][4] seq, split, part, nsplit */
  int64_t off_combine;         /* [num_combine_seqs][4] seq, token, first part, nsplit */
  int64_t off_prefill_tiles;   /* [num_prefill_tiles][2] seq, first query row; most keys first */
  int64_t words;               /* int32 words used in the packed buffer */
} pa_step_plan;

/* Version of this ABI (bumped on any signature or struct change).  No reference
 * counterpart (the reference is one Python package). */
int32_t pa_abi_version(void);

/* Message of the calling thread's last failed call ("" if none).  No reference
 * counterpart: the reference raises; the Python binding turns this message into the
 * reference's exception (ValueError / NotImplementedError) with the same text. */
const char* pa_last_error(void);

/* Kernels launched by the calling thread's most recent pa_paged_attention_fwd or
 * pa_paged_attention_fwd_noalloc call (a bit mask of PA_LAUNCH_*); lets tests and
 * benchmarks confirm which kernel served which rows.  No counterpart in the reference. */
#define PA_LAUNCH_DECODE_MMA 1      /* tensor-pipe split-K decode (bf16/fp16) */
#define PA_LAUNCH_DECODE_SIMT 2     /* SIMT split-K decode */
#define PA_LAUNCH_COMBINE 4         /* split-K combine */
#define PA_LAUNCH_PREFILL_TC 8      /* tcgen05 varlen prefill */
#define PA_LAUNCH_GENERIC 16        /* generic ragged kernel */
#define PA_LAUNCH_PREFILL_PAIR 32   /* tcgen05 varlen prefill on CTA pairs (head_dim 128) */
#define PA_LAUNCH_PREFILL_PERSIST 64 /* persistent tcgen05 varlen prefill (P in TMEM, Q by TMA) */
int32_t pa_last_launches(void);

/*
 * Upper bound on the int32 words pa_plan_step writes for a step with num_seqs
 * sequences, num_tokens packed tokens and at most max_blocks_per_seq blocks per row.
 * No reference counterpart (sizes the packed buffer that replaces _pack's six tensors).
 */
int64_t pa_plan_words_bound(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks_per_seq);

/*
 * Validate one step's ragged batch and write its packed metadata into a HOST buffer
 * (pinned memory makes the single upload asynchronous).  Replaces the per-layer
 * validation of inference_server/core/attention.py:202-219 (_check), the per-token
 * tables of inference_server/core/attention_triton.py:129-150 (_token_map) and the
 * write-slot computation of inference_server/core/paged_executor.py:240-247.
 *
 *   context_lens, query_lens  host int64 [num_seqs]
 *   block_tables              host int64, row i at block_tables + i * table_row_stride,
 *                             table_cols entries per row (the reference's 0-padded rows)
 *   num_tokens                the query's token count (must equal sum(query_lens))
 *   pool_num_blocks           blocks in the pool; every block a sequence reads must be
 *                             in [0, pool_num_blocks)
 *   num_kv_heads, sm_count    used to size decode splits so the grid fills the GPU
 *   prefill_tile_tokens       query rows per prefill tile (0 = no prefill tile list)
 *   meta_out, meta_capacity   host int32 buffer and its size in words
 *
 * The upload of meta_out[0 .. plan->words) to a device buffer is the caller's (one
 * cudaMemcpyAsync); the device copy is what pa_paged_attention_fwd and
 * pa_reshape_and_cache read.
 */
int32_t pa_plan_step(const int64_t* context_lens, const int64_t* query_lens, int32_t num_seqs,
                     const int64_t* block_tables, int64_t table_row_stride, int32_t table_cols,
                     int32_t num_tokens, int64_t pool_num_blocks, int32_t block_size,
                     int32_t num_kv_heads, int32_t sm_count, int32_t prefill_tile_tokens,
                     int32_t* meta_out, int64_t meta_capacity, pa_step_plan* plan);

/*
 * A decode-step plan padded to a fixed shape, so that every launch parameter of
 * pa_reshape_and_cache / pa_paged_attention_fwd stays the same from step to step and a
 * CUDA graph captured once can be replayed with each step's metadata copied into the
 * same device buffer.  No reference counterpart (the reference launches per call);
 * the arrays are those of pa_plan_step for an all-decode batch (every query_len 1,
 * num_tokens = num_seqs), with the split size fixed to split_blocks, block tables
 * width_cap wide, and the decode-item and combine lists padded with null entries
 * (sequence -1, skipped by the kernels) to items_cap and combine_cap.  A step that does
 * not fit returns PA_ERR_BUFFER_TOO_SMALL ("bucket: ..."); the caller then picks a larger
 * bucket.  With meta_out NULL it only fills *plan (plan->words sizes the buffer).
 */
int32_t pa_plan_decode_padded(const int64_t* context_lens, int32_t num_seqs, const int64_t* block_tables,
                              int64_t table_row_stride, int32_t table_cols, int64_t pool_num_blocks,
                              int32_t block_size, int32_t num_kv_heads, int32_t split_blocks, int32_t width_cap,
                              int32_t items_cap, int32_t combine_cap, int32_t* meta_out, int64_t meta_capacity,
                              pa_step_plan* plan);

/* (token, query-head) rows of one tensor-core prefill tile at this head_dim (128: the
 * persistent tcgen05 kernel, or the single-CTA one when the environment variable
 * PA_PREFILL_KERNEL is "per_tile"): plan prefill steps with prefill_tile_tokens =
 * pa_prefill_tile_rows(head_dim) / (num_heads / num_kv_heads) so their rows take it.  At
 * head_dim 128 a plan tiled at 256 rows runs on the CTA-pair tcgen05 kernel instead (half
 * the K/V bytes per SM; measured slower on B200, so not the default).  No reference
 * counterpart. */
int32_t pa_prefill_tile_rows(int32_t head_dim);

/* Device workspace bytes pa_paged_attention_fwd needs for this plan and head shape.
 * No reference counterpart (the reference's gather path allocates per call). */
uint64_t pa_workspace_bytes(const pa_step_plan* plan, int32_t num_heads, int32_t head_dim);

/*
 * Causal paged attention over a ragged batch: the computation of
 * inference_server/core/attention.py:92-187 (paged_attention_gather), replacing the
 * Triton kernel of inference_server/core/attention_triton.py:156-305.
 *
 *   query    [num_tokens, num_heads, head_dim], any element strides
 *   k_pool   contiguous [pool_num_blocks, block_size, num_kv_heads, head_dim]
 *   v_pool   same shape as k_pool
 *   out      [num_tokens, num_heads, head_dim], strides out_stride_token/out_stride_head,
 *            unit stride along head_dim
 *   meta     device copy of the packed buffer pa_plan_step wrote for `plan`
 *   workspace  at least pa_workspace_bytes(plan, num_heads, head_dim) device bytes,
 *            256-byte aligned; it holds split-K partials and, in its first 4 bytes, a
 *            device error word the caller zeroes once when it allocates the workspace
 *   stream   cudaStream_t to launch on
 *
 * Token t of sequence i sits at position ctx_i - q_i + t and attends to keys 0..that.
 * Scores, softmax and accumulation are float32; the output is stored in `dtype`.
 */
int32_t pa_paged_attention_fwd(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                               int64_t q_stride_dim, int32_t num_tokens, int32_t num_heads,
                               int32_t head_dim, const void* k_pool, const void* v_pool,
                               int64_t pool_num_blocks, int32_t block_size, int32_t num_kv_heads,
                               int32_t dtype, float scale, const pa_step_plan* plan,
                               const int32_t* meta, void* out, int64_t out_stride_token,
                               int64_t out_stride_head, void* workspace, uint64_t workspace_bytes,
                               void* stream);

/* Size of the static scratch pa_paged_attention_fwd_noalloc uses (32 MiB per GPU). */
#define PA_NOALLOC_SCRATCH_BYTES (32u << 20)

/*
 * pa_paged_attention_fwd without a workspace argument, for callers that cannot
 * allocate device memory (a plug-in inside a host framework that owns all device
 * memory, a serving loop that cannot pay cudaMalloc's device-wide synchronisation).
 * No counterpart in the reference: its gather path allocates freely through torch.
 *
 * The split-K scratch lives in a static device array of PA_NOALLOC_SCRATCH_BYTES that
 * every GPU loading this library reserves until the process exits; steps whose
 * pa_workspace_bytes exceeds it are rejected with PA_ERR_BUFFER_TOO_SMALL (after the same
 * argument checks as pa_paged_attention_fwd, before anything is enqueued).  The first
 * call in each CUDA context looks the array's address up and zeroes its error word on
 * `stream` (make it before any stream capture).  All calls share the array, and calls
 * whose GPU work overlaps race on it.  The kernels' error word in it is sticky, as a
 * workspace's is: read and clear it with pa_noalloc_read_device_error.  Allocates
 * nothing.
 */
int32_t pa_paged_attention_fwd_noalloc(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                                       int64_t q_stride_dim, int32_t num_tokens, int32_t num_heads,
                                       int32_t head_dim, const void* k_pool, const void* v_pool,
                                       int64_t pool_num_blocks, int32_t block_size, int32_t num_kv_heads,
                                       int32_t dtype, float scale, const pa_step_plan* plan,
                                       const int32_t* meta, void* out, int64_t out_stride_token,
                                       int64_t out_stride_head, void* stream);

/*
 * Read (and clear, when clear != 0) the device error word inside the static scratch of
 * pa_paged_attention_fwd_noalloc, for callers that never see a workspace pointer: the
 * same bits pa_read_device_error reports for a workspace (an out-of-range block id
 * reached a kernel, a pipeline wait ran out of its limit), accumulated over every
 * no-allocation call in the current context since the last clear.  Synchronises
 * `stream`.  Allocates nothing.  No counterpart in the reference.
 */
int32_t pa_noalloc_read_device_error(int32_t clear, int32_t* error_word, void* stream);

/*
 * Fused K+V append: write the new tokens' keys and values into both pools at their
 * flat slots.  Replaces the two index_copy_ calls of
 * inference_server/core/paged_executor.py:116-125 (_PagedCache.update); the pool bytes
 * after the call are identical to the reference's.
 *
 *   key, value     [num_tokens, num_kv_heads, head_dim] with the given element strides
 *                  (unit stride along head_dim); same dtype as the pools
 *   slot_mapping   device int32 [num_tokens], each in [0, pool_num_blocks * block_size)
 */
int32_t pa_reshape_and_cache(const void* key, int64_t k_stride_token, int64_t k_stride_head,
                             const void* value, int64_t v_stride_token, int64_t v_stride_head,
                             int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                             int32_t dtype, void* k_pool, void* v_pool, int64_t pool_num_blocks,
                             int32_t block_size, const int32_t* slot_mapping, void* stream);

/*
 * Whole-block moves across every layer's K and V pools, one launch per 128 layers.
 * The pools are the reference layout; block_bytes = block_size * num_kv_heads * head_dim
 * * element size (a multiple of 16; pools and staging 16-byte aligned).  k_pools and
 * v_pools are HOST arrays of num_layers device pointers.  Block ids are device int32;
 * an id outside [0, pool_num_blocks) sets bit 1 of *error_word (device int32, required)
 * and that block is skipped.  The moves are bitwise and asynchronous on `stream`.
 *
 * pa_copy_blocks: pool[dst] = pool[src] in every layer, for pairs [num_pairs][2]
 * (src, dst).  Replaces inference_server/core/paged_executor.py:265-270 (_copy_block,
 * the copy-on-write move BlockTable.ensure_private asks for, one block and one layer at
 * a time).  Precondition: the destinations are distinct and none is also a source (the
 * pairs run concurrently).
 */
int32_t pa_copy_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                       int64_t block_bytes, const int32_t* pairs, int32_t num_pairs, int32_t* error_word,
                       void* stream);

/*
 * pa_gather_blocks: copy blocks[0..num_blocks) of every layer into `staging`, laid out
 * [num_layers][K, V][num_blocks][block_bytes] — each [layer][K or V] slice is the
 * reference's per-layer host tensor [num_blocks, block_size, Hkv, D].  Replaces the
 * per-layer index_select of inference_server/core/kv_pool.py:142-166 (swap_out); the
 * caller then moves staging to host memory with one copy.
 *
 * pa_scatter_blocks: the inverse, staging -> blocks (inference_server/core/kv_pool.py:
 * 168-182, swap_in's per-layer index_copy_).  Precondition: the blocks are distinct.
 */
int32_t pa_gather_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                         int64_t block_bytes, const int32_t* blocks, int32_t num_blocks, void* staging,
                         int32_t* error_word, void* stream);
int32_t pa_scatter_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                          int64_t block_bytes, const int32_t* blocks, int32_t num_blocks, const void* staging,
                          int32_t* error_word, void* stream);

/*
 * CUDA IPC for the peer all-reduce's buffers (no reference counterpart).
 * pa_ipc_export: the 64-byte handle of the allocation holding dev_ptr and dev_ptr's byte
 * offset in it.  pa_ipc_open: map a peer's handle into the calling device's context (peer
 * access enabled on demand) and return the peer's pointer (allocation base + offset).
 * pa_ipc_close: unmap a pointer pa_ipc_open returned (same offset).
 */
#define PA_IPC_HANDLE_BYTES 64
int32_t pa_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
int32_t pa_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out);
int32_t pa_ipc_close(void* dev_ptr, int64_t offset);

/*
 * Sum `count` elements across the `world` ranks of one node (<= 8) in place, over peer
 * memory.  No counterpart in the reference, which has no multi-GPU path: it replaces the
 * torch.distributed.all_reduce that follows the row-split o_proj in KV-head tensor
 * parallelism.
 *
 *   bases         HOST array of `world` device pointers: every rank's buffer, mapped into
 *                 this process (CUDA IPC), all allocated with the same layout
 *   data_offset   byte offset of this call's data (the caller's partial, overwritten with
 *                 the sum on every rank); 16-byte aligned, count * element size a multiple
 *                 of 16
 *   flags_offset  byte offset of a zero-initialised 128-byte flag area owned by this
 *                 collective (it also counts the calls, so a captured CUDA graph of the
 *                 call replays correctly)
 *   timeout_s     bound on each of the kernel's two barrier waits; on expiry bit 4 of
 *                 *error_word is set and the collective (and its buffer) must not be
 *                 used again
 *
 * Every rank must make the same sequence of calls with the same arguments except rank and
 * the mapping of bases;
 * the kernel returns on each rank once all ranks' sums are in place.  Asynchronous on
 * `stream`; the caller's partial must be written before it on that stream.
 */
int32_t pa_peer_allreduce(void* const* bases, int32_t world, int32_t rank, int64_t data_offset, int64_t flags_offset,
                          int64_t count, int32_t dtype, double timeout_s, int32_t* error_word, void* stream);

/*
 * The row-split o_proj GEMM fused with its all-reduce, over peer memory: every rank ends
 * with out[rows, n] = sum over ranks of round(a_r . w_r^T) (each rank's product rounded to
 * the storage dtype, then summed in float32 in rank order and rounded once).  No
 * counterpart in the reference (no multi-GPU path): it replaces `attn @ w_o` plus
 * torch.distributed.all_reduce in KV-head tensor parallelism.  bf16 or fp16 only.
 *
 *   a             this rank's [rows, k] activations (row stride a_row_stride elements,
 *                 a multiple of 8; 16-byte aligned)
 *   w             this rank's o_proj slice, K-major [n, k] contiguous (16-byte aligned)
 *   k, n          k a multiple of 64; n a multiple of 256 * world
 *   bases         HOST array of `world` device pointers: every rank's buffer (CUDA IPC),
 *                 same layout on all ranks: a staging area of rows * n elements at
 *                 stage_offset, the output [rows, n] at out_offset, a zero-initialised
 *                 128-byte flag area at flags_offset (offsets 16-byte aligned)
 *   timeout_s     bound on each wait for a peer; on expiry bit 4 of *error_word is set
 *                 and the buffer must not be used again
 *
 * Two launches on `stream` (the GEMM, whose epilogue stores each output tile into the
 * staging area of the rank owning its columns, then the owners' sums stored into every
 * rank's output).  Every rank must make the same sequence of calls with the same rows,
 * k, n and offsets; the output is complete on this rank when the second launch ends.
 */
int32_t pa_oproj_allreduce(const void* a, int64_t a_row_stride, int32_t rows, int32_t k, const void* w, int32_t n,
                           int32_t dtype, void* const* bases, int32_t world, int32_t rank, int64_t stage_offset,
                           int64_t out_offset, int64_t flags_offset, double timeout_s, int32_t* error_word,
                           void* stream);

/*
 * Read (and clear, when clear != 0) the device error word a workspace carries.  It is
 * set by kernels that met an out-of-range block id or slot (the host checks make this
 * unreachable for planned steps) or a pipeline wait that ran out of its iteration
 * limit.  Synchronises `stream`.  Returns PA_OK and stores the word in *error_word.
 * No reference counterpart (the reference's torch ops raise on the host).
 */
int32_t pa_read_device_error(void* workspace, int32_t clear, int32_t* error_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_ATTENTION_B200_H */
