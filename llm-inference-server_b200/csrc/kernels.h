// Host-side launchers of the device kernels (internal to the library).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pa {

// Split-K decode over (sequence, split) work items, one CTA per item and KV head.
struct DecodeParams {
  const void* q;
  int64_t q_st, q_sh;         // element strides of query (unit stride along head_dim)
  void* out;
  int64_t o_st, o_sh;         // element strides of out (unit stride along head_dim)
  const int32_t* tables;      // [B, width]
  int32_t width;
  const int32_t* ctx_lens;    // [B]
  const int32_t* cu_q;        // [B+1]
  const int4* items;          // [num_items] seq, split, part, nsplit
  int32_t num_items;
  float* part_o;              // [parts, Hq, D]
  float2* part_ml;            // [parts, Hq]: running max (log2 domain) and denominator
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t split_blocks;
  int32_t pool_blocks;
  float qscale;               // softmax scale * log2(e)
  int* err;
};

struct CombineParams {
  void* out;
  int64_t o_st, o_sh;
  const int4* combine;        // [num_combine] seq, token, first part, nsplit
  int32_t num_combine;
  const float* part_o;
  const float2* part_ml;
  int32_t num_heads;
  int32_t head_dim;
};

// Generic kernel: any block size, head_dim <= 256, any strides; one warp per
// (token, head).  Serves shapes outside the fast paths and prefill rows.
struct GenericParams {
  const void* q;
  int64_t q_st, q_sh, q_sd;
  void* out;
  int64_t o_st, o_sh;
  const void* k_pool;
  const void* v_pool;
  int32_t block_size, num_kv_heads, head_dim, num_heads;
  const int32_t* tables;
  int32_t width;
  const int32_t* seq_idx;
  const int32_t* q_pos;
  const int32_t* query_lens;
  int32_t num_tokens;
  int32_t skip_decode;        // 1: tokens of query_len == 1 sequences are done elsewhere
  int32_t skip_prefill;       // 1: tokens of query_len > 1 sequences are done elsewhere
  int64_t pool_blocks;
  float qscale;
  int* err;
};

// tcgen05 varlen prefill over (sequence, first query row) tiles, one CTA per tile and KV head.
struct PrefillParams {
  const void* q;
  int64_t q_st, q_sh;         // element strides of query (unit stride along head_dim)
  void* out;
  int64_t o_st, o_sh;
  const int32_t* tables;      // [B, width]
  int32_t width;
  const int32_t* ctx_lens;    // [B]
  const int32_t* query_lens;  // [B]
  const int32_t* cu_q;        // [B+1]
  const int2* tiles;          // [num_tiles] seq, first query row
  int32_t num_tiles;
  int32_t num_heads, num_kv_heads;
  int32_t pool_blocks;
  float qscale;
  int* err;
};

struct AppendParams {
  const uint8_t* key;
  int64_t k_st, k_sh;         // byte strides
  const uint8_t* value;
  int64_t v_st, v_sh;
  int32_t num_tokens, num_kv_heads;
  int32_t row_bytes;          // head_dim * element size
  uint8_t* k_pool;
  uint8_t* v_pool;
  int64_t num_slots;
  const int32_t* slots;
};

// Whole-block moves over every layer's K and V pools (copy-on-write, swap gather/scatter).
constexpr int kCopyLayers = 128;  // layers per launch (pool pointers travel in the parameters)
enum BlockMoveMode : int32_t { kBlockCopy = 0, kBlockGather = 1, kBlockScatter = 2 };
struct BlockCopyParams {
  uint8_t* k[kCopyLayers];
  uint8_t* v[kCopyLayers];
  int32_t num_layers;         // layers in this launch
  int32_t layer0;             // index of k[0] among all layers (staging offset)
  int32_t mode;               // BlockMoveMode
  int32_t n;                  // pairs (copy) or blocks (gather / scatter)
  int64_t block_bytes;        // block_size * Hkv * D * element size, a multiple of 16
  int64_t pool_blocks;
  const int32_t* ids;         // copy: [n][2] (src, dst); gather / scatter: [n]
  uint8_t* staging;           // [all layers][K, V][n][block_bytes]
  int* err;
};

// All-reduce over peer memory (tensor-parallel o_proj).  Each rank's mapped buffer holds
// data slots and, at flags_offset, a uint32 flag area: [kPeerReady + p] and
// [kPeerDone + p] are written by rank p, [kPeerCounter] counts finished CTAs,
// [kPeerEpoch] holds the last completed call's epoch.
constexpr int kPeerMax = 8;
constexpr int kPeerThreads = 512;
constexpr int kPeerReady = 0, kPeerDone = 8, kPeerCounter = 16, kPeerEpoch = 17, kPeerFlagWords = 32;
struct PeerReduceParams {
  uint8_t* base[kPeerMax];    // every rank's buffer, mapped into this process
  int64_t data_offset;        // byte offset of this call's data slot (16-byte aligned)
  int64_t flags_offset;       // byte offset of the flag area
  int64_t count;              // elements; count * element size is a multiple of 16
  int32_t world, rank;
  uint64_t timeout_ns;        // bound on every wait
  int* err;
};

// The o_proj GEMM fused with its all-reduce (oproj_allreduce.cu).  Each rank's mapped
// buffer holds a staging area [world][rows][n / world] (16-bit partials pushed by every
// rank into the owner of those columns), output slots [rows][n] and the flag area above;
// the gather launch counts its finished CTAs in [kPeerCounter2].
constexpr int kPeerCounter2 = 18;
constexpr int kOprojTile = 128;       // output rows of one GEMM CTA
constexpr int kOprojTileN = 256;      // output columns of one GEMM CTA
constexpr int kOprojKStep = 64;       // k per pipeline stage (one 128-byte swizzled row)
struct OprojParams {
  uint8_t* base[kPeerMax];
  int64_t stage_offset;       // byte offset of the staging area
  int64_t out_offset;         // byte offset of this call's output slot
  int64_t flags_offset;
  int32_t rows, k, n;         // a is [rows, k], w is [n, k] (K-major), the output [rows, n]
  int32_t world, rank;
  uint64_t timeout_ns;
  int* err;
};

// Returns true when the fast decode kernel has an instantiation for this shape.
bool decode_supported(int dtype, int head_dim, int group, int block_size);
// Dynamic shared memory bytes of the decode kernel.
int decode_smem_bytes(int dtype, int head_dim, int group);
cudaError_t launch_decode(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                          const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_combine(int dtype, const CombineParams& p, cudaStream_t stream);
// Tensor-pipe decode (bf16/fp16): pools described with 64-element boxes and 128B swizzle.
bool decode_mma_supported(int dtype, int head_dim, int group, int block_size);
cudaError_t launch_decode_mma(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                              const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_generic(int dtype, const GenericParams& p, cudaStream_t stream);
// tcgen05 prefill (bf16/fp16): tiles of prefill_tile_rows() (token, head) rows.
bool prefill_tc_supported(int dtype, int head_dim, int group, int block_size);
int prefill_tile_rows();
cudaError_t launch_prefill_tc(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                              const PrefillParams& p, cudaStream_t stream);
// tcgen05 prefill on CTA pairs (cta_group::2, head_dim 128): tiles of
// prefill_pair_tile_rows() rows, one cluster of two CTAs per tile and KV head.
bool prefill_pair_supported(int dtype, int head_dim, int group, int block_size);
int prefill_pair_tile_rows();
cudaError_t launch_prefill_pair(int dtype, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                                const PrefillParams& p, cudaStream_t stream);
// Persistent tcgen05 prefill over the same 128-row tiles: two CTAs per SM, Q by TMA from
// `tq` (the query as (head_dim, num_heads, num_tokens), box (64, G, 128 / G), 128-byte
// swizzle), P kept in TMEM.
bool prefill_persist_supported(int dtype, int head_dim, int group, int block_size);
cudaError_t launch_prefill_persist(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                                   const CUtensorMap& tq, const PrefillParams& p, cudaStream_t stream);
cudaError_t launch_append(const AppendParams& p, cudaStream_t stream);
cudaError_t launch_block_copy(const BlockCopyParams& p, cudaStream_t stream);
cudaError_t launch_peer_allreduce(int dtype, const PeerReduceParams& p, int grid, cudaStream_t stream);
// ta: a as (k, rows), box (64, 128); tw: w as (k, n), box (64, 256); tw_half: the same map
// with box (64, 128) (the CTA-pair GEMM, used when rows > 128); 128-byte swizzle.
cudaError_t launch_oproj_allreduce(int dtype, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tw_half,
                                   const OprojParams& p, int gather_grid, cudaStream_t stream);

}  // namespace pa
