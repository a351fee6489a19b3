// extern "C" entry points declared in include/paged_attention_b200.h: argument checks,
// TMA descriptor encoding (cached per pool), workspace layout and kernel dispatch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "kernels.h"
#include "pa_common.cuh"
#include "pa_host.h"

namespace pa {

// Workspace layout: [0, 256) device error word + padding, then split-K partials
// (float2 (m, l) per part and head, then float[head_dim] per part and head).
constexpr uint64_t kWsHeader = 256;

static uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

static int elem_size(int dtype) { return dtype == PA_DTYPE_F32 ? 4 : 2; }

static CUtensorMapDataType tma_dtype(int dtype) {
  switch (dtype) {
    case PA_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    case PA_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// cuMemGetAddressRange (allocation base of a device pointer) through the same route.
static PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  });
  return fn;
}

struct MapKey {
  uintptr_t base;
  int64_t blocks;
  int32_t bs, hkv, dim, dtype, box_inner, swizzle;
  bool operator==(const MapKey& o) const {
    return base == o.base && blocks == o.blocks && bs == o.bs && hkv == o.hkv && dim == o.dim &&
           dtype == o.dtype && box_inner == o.box_inner && swizzle == o.swizzle;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.base) ^ (std::hash<int64_t>()(k.blocks) * 31) ^ (size_t(k.dim) << 7) ^
           (size_t(k.hkv) << 17) ^ size_t(k.dtype) ^ (size_t(k.box_inner) << 27) ^ (size_t(k.swizzle) << 40);
  }
};

// The pool [NB, BS, Hkv, D] as a 3-D tensor (D, Hkv, NB*BS); box (box_inner, 1, BS) is
// (part of) one block of one KV head: the whole row without swizzle for the SIMT kernel,
// 64-element (128-byte) column halves with 128B swizzle for the tensor-pipe kernel.
// Descriptors are cached by pool address and shape: a serving process has 2 pools per
// layer and encodes each once.
static int32_t pool_tensor_map(const void* pool, int64_t num_blocks, int bs, int hkv, int dim, int dtype,
                               int box_inner, bool swizzle128, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(pool), num_blocks, bs, hkv, dim, dtype, box_inner, swizzle128 ? 1 : 0};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return PA_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  const int es = elem_size(dtype);
  cuuint64_t gdim[3] = {cuuint64_t(dim), cuuint64_t(hkv), cuuint64_t(num_blocks) * cuuint64_t(bs)};
  cuuint64_t gstride[2] = {cuuint64_t(dim) * es, cuuint64_t(hkv) * dim * es};
  cuuint32_t box[3] = {cuuint32_t(box_inner), 1u, cuuint32_t(bs)};
  cuuint32_t estride[3] = {1u, 1u, 1u};
  CUtensorMap map;
  CUresult r = fn(&map, tma_dtype(dtype), 3, const_cast<void*>(pool), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return PA_OK;
}

// The query as a 3-D TMA map (head_dim, num_heads, num_tokens) with a box of 64 elements x
// `group` heads x `rows / group` tokens, 128-byte swizzle: one box is the 128 (token, head)
// rows of a prefill tile for one 64-column half.
static int32_t query_tensor_map(const void* query, int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                                int64_t q_stride_token, int64_t q_stride_head, int dtype, int group, int rows,
                                CUtensorMap* out) {
  auto fn = encode_fn();
  if (!fn) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  const int es = elem_size(dtype);
  cuuint64_t gdim[3] = {cuuint64_t(head_dim), cuuint64_t(num_heads), cuuint64_t(num_tokens)};
  cuuint64_t gstride[2] = {cuuint64_t(q_stride_head) * es, cuuint64_t(q_stride_token) * es};
  cuuint32_t box[3] = {64u, cuuint32_t(group), cuuint32_t(rows / group)};
  cuuint32_t estride[3] = {1u, 1u, 1u};
  CUresult r = fn(out, tma_dtype(dtype), 3, const_cast<void*>(query), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled (query) failed (CUresult %d)", int(r));
  return PA_OK;
}

// Which kernel serves 128-row prefill tiles: the persistent kernel unless
// PA_PREFILL_KERNEL is "per_tile" (one CTA per tile).  Read on every call, so one process
// can run both.
static bool prefill_persistent_selected() {
  const char* v = getenv("PA_PREFILL_KERNEL");
  return !(v && strcmp(v, "per_tile") == 0);
}

static thread_local int32_t g_last_launches = 0;

static int32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(PA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void reset_last_launches() { g_last_launches = 0; }

int32_t check_attention_args(int32_t num_tokens, int32_t num_heads, int32_t head_dim, int32_t block_size,
                             int32_t num_kv_heads, int32_t dtype, const pa_step_plan* plan) {
  if (!plan) return fail(PA_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_UNSUPPORTED, "dtype code %d is not float32, float16 or bfloat16", dtype);
  if (num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "heads and head_dim must be positive");
  if (num_heads % num_kv_heads)
    return fail(PA_ERR_INVALID_ARGUMENT, "%d query heads not divisible by %d kv heads", num_heads, num_kv_heads);
  if (head_dim > 256) return fail(PA_ERR_UNSUPPORTED, "head_dim %d > 256 is not supported", head_dim);
  if (plan->num_tokens != num_tokens)
    return fail(PA_ERR_INVALID_ARGUMENT, "plan was built for %d tokens, query has %d", plan->num_tokens, num_tokens);
  if (plan->block_size != block_size)
    return fail(PA_ERR_INVALID_ARGUMENT, "plan was built for block_size %d, pool has %d", plan->block_size,
                block_size);
  return PA_OK;
}

}  // namespace pa

extern "C" {

int32_t pa_last_launches(void) { return pa::g_last_launches; }

uint64_t pa_workspace_bytes(const pa_step_plan* plan, int32_t num_heads, int32_t head_dim) {
  if (!plan) return 0;
  const uint64_t parts = uint64_t(plan->num_decode_items > 0 ? plan->num_decode_items : 0);
  const uint64_t ml = pa::align_up(parts * num_heads * sizeof(float2), 256);
  const uint64_t po = parts * num_heads * uint64_t(head_dim) * sizeof(float);
  return pa::kWsHeader + ml + po;
}

int32_t pa_paged_attention_fwd(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                               int64_t q_stride_dim, int32_t num_tokens, int32_t num_heads,
                               int32_t head_dim, const void* k_pool, const void* v_pool,
                               int64_t pool_num_blocks, int32_t block_size, int32_t num_kv_heads,
                               int32_t dtype, float scale, const pa_step_plan* plan,
                               const int32_t* meta, void* out, int64_t out_stride_token,
                               int64_t out_stride_head, void* workspace, uint64_t workspace_bytes,
                               void* stream_ptr) {
  using namespace pa;
  g_last_launches = 0;
  const int32_t bad = check_attention_args(num_tokens, num_heads, head_dim, block_size, num_kv_heads, dtype, plan);
  if (bad != PA_OK) return bad;
  if (num_tokens == 0) return PA_OK;
  if (!query || !k_pool || !v_pool || !out || !meta || !workspace)
    return fail(PA_ERR_INVALID_ARGUMENT, "NULL device pointer");
  const uint64_t need = pa_workspace_bytes(plan, num_heads, head_dim);
  if (workspace_bytes < need)
    return fail(PA_ERR_BUFFER_TOO_SMALL, "workspace holds %llu bytes, %llu needed",
                (unsigned long long)workspace_bytes, (unsigned long long)need);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(PA_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");

  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int* err = static_cast<int*>(workspace);
  const uint64_t parts = uint64_t(plan->num_decode_items);
  float2* part_ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + kWsHeader);
  float* part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWsHeader +
                                           align_up(parts * num_heads * sizeof(float2), 256));
  const int group = num_heads / num_kv_heads;
  const float qscale = scale * kLog2e;
  const int32_t* tables = meta + plan->off_block_tables;

  // Decode rows go to the split-K kernel when it has an instantiation for the shape and
  // the pool/query layouts meet its alignment needs; every other row goes to the
  // generic kernel.
  const bool fast_decode = plan->num_decode_seqs > 0 && decode_supported(dtype, head_dim, group, block_size) &&
                           q_stride_dim == 1 && reinterpret_cast<uintptr_t>(k_pool) % 16 == 0 &&
                           reinterpret_cast<uintptr_t>(v_pool) % 16 == 0;
  // 16-bit pools take the tensor-pipe kernel when q rows can be read as 32-bit pairs.
  const bool use_mma = fast_decode && decode_mma_supported(dtype, head_dim, group, block_size) &&
                       q_stride_token % 2 == 0 && q_stride_head % 2 == 0 &&
                       reinterpret_cast<uintptr_t>(query) % 4 == 0;
  if (fast_decode) {
    CUtensorMap tk, tv;
    const int box = use_mma ? 64 : head_dim;
    int32_t rc = pool_tensor_map(k_pool, pool_num_blocks, block_size, num_kv_heads, head_dim, dtype, box, use_mma,
                                 &tk);
    if (rc != PA_OK) return rc;
    rc = pool_tensor_map(v_pool, pool_num_blocks, block_size, num_kv_heads, head_dim, dtype, box, use_mma, &tv);
    if (rc != PA_OK) return rc;
    DecodeParams p{};
    p.q = query;
    p.q_st = q_stride_token;
    p.q_sh = q_stride_head;
    p.out = out;
    p.o_st = out_stride_token;
    p.o_sh = out_stride_head;
    p.tables = tables;
    p.width = plan->table_width;
    p.ctx_lens = meta + plan->off_context_lens;
    p.cu_q = meta + plan->off_cu_query_lens;
    p.items = reinterpret_cast<const int4*>(meta + plan->off_decode_items);
    p.num_items = plan->num_decode_items;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.num_heads = num_heads;
    p.num_kv_heads = num_kv_heads;
    p.split_blocks = plan->split_blocks;
    p.pool_blocks = int32_t(pool_num_blocks);
    p.qscale = qscale;
    p.err = err;
    cudaError_t e = use_mma ? launch_decode_mma(dtype, head_dim, group, tk, tv, p, stream)
                            : launch_decode(dtype, head_dim, group, tk, tv, p, stream);
    if (e != cudaSuccess) return cuda_fail(e, "split-K decode launch");
    if (p.num_items > 0) g_last_launches |= use_mma ? PA_LAUNCH_DECODE_MMA : PA_LAUNCH_DECODE_SIMT;
    if (plan->num_combine_seqs > 0) {
      CombineParams c{};
      c.out = out;
      c.o_st = out_stride_token;
      c.o_sh = out_stride_head;
      c.combine = reinterpret_cast<const int4*>(meta + plan->off_combine);
      c.num_combine = plan->num_combine_seqs;
      c.part_o = part_o;
      c.part_ml = part_ml;
      c.num_heads = num_heads;
      c.head_dim = head_dim;
      e = launch_combine(dtype, c, stream);
      if (e != cudaSuccess) return cuda_fail(e, "split-K combine launch");
      g_last_launches |= PA_LAUNCH_COMBINE;
    }
  }
  // Prefill rows go to a tcgen05 kernel when the plan's tiles fit one and query/out rows
  // are 16-byte aligned: 128-row tiles to the persistent kernel (or the single-CTA kernel
  // under PA_PREFILL_KERNEL=per_tile), 256-row tiles to the CTA-pair kernel (head_dim 128).
  const int es = elem_size(dtype);
  const int tile_rows = plan->prefill_tile_tokens * group;
  const bool persist_prefill = prefill_persist_supported(dtype, head_dim, group, block_size) &&
                               tile_rows == prefill_tile_rows() && prefill_persistent_selected();
  const bool pair_prefill = prefill_pair_supported(dtype, head_dim, group, block_size) &&
                            tile_rows == prefill_pair_tile_rows();
  const bool single_prefill = !persist_prefill && prefill_tc_supported(dtype, head_dim, group, block_size) &&
                              tile_rows == prefill_tile_rows();
  const bool tc_prefill = plan->num_prefill_tiles > 0 && (persist_prefill || pair_prefill || single_prefill) &&
                          q_stride_dim == 1 &&
                          (q_stride_token * es) % 16 == 0 && (q_stride_head * es) % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(query) % 16 == 0 && (out_stride_token * es) % 16 == 0 &&
                          (out_stride_head * es) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(k_pool) % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(v_pool) % 16 == 0;
  if (tc_prefill) {
    CUtensorMap tk, tv;
    int32_t rc = pool_tensor_map(k_pool, pool_num_blocks, block_size, num_kv_heads, head_dim, dtype, 64, true, &tk);
    if (rc != PA_OK) return rc;
    rc = pool_tensor_map(v_pool, pool_num_blocks, block_size, num_kv_heads, head_dim, dtype, 64, true, &tv);
    if (rc != PA_OK) return rc;
    PrefillParams f{};
    f.q = query;
    f.q_st = q_stride_token;
    f.q_sh = q_stride_head;
    f.out = out;
    f.o_st = out_stride_token;
    f.o_sh = out_stride_head;
    f.tables = tables;
    f.width = plan->table_width;
    f.ctx_lens = meta + plan->off_context_lens;
    f.query_lens = meta + plan->off_query_lens;
    f.cu_q = meta + plan->off_cu_query_lens;
    f.tiles = reinterpret_cast<const int2*>(meta + plan->off_prefill_tiles);
    f.num_tiles = plan->num_prefill_tiles;
    f.num_heads = num_heads;
    f.num_kv_heads = num_kv_heads;
    f.pool_blocks = int32_t(pool_num_blocks);
    f.qscale = qscale;
    f.err = err;
    cudaError_t e;
    if (persist_prefill) {
      CUtensorMap tq;
      rc = query_tensor_map(query, num_tokens, num_heads, head_dim, q_stride_token, q_stride_head, dtype, group,
                            tile_rows, &tq);
      if (rc != PA_OK) return rc;
      e = launch_prefill_persist(dtype, head_dim, group, tk, tv, tq, f, stream);
    } else if (pair_prefill) {
      e = launch_prefill_pair(dtype, group, tk, tv, f, stream);
    } else {
      e = launch_prefill_tc(dtype, head_dim, group, tk, tv, f, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 prefill launch");
    g_last_launches |= persist_prefill ? PA_LAUNCH_PREFILL_PERSIST
                                       : (pair_prefill ? PA_LAUNCH_PREFILL_PAIR : PA_LAUNCH_PREFILL_TC);
  }
  const bool decode_left = plan->num_decode_seqs > 0 && !fast_decode;
  const bool prefill_left = plan->num_prefill_tokens > 0 && !tc_prefill;
  if (decode_left || prefill_left) {
    GenericParams g{};
    g.q = query;
    g.q_st = q_stride_token;
    g.q_sh = q_stride_head;
    g.q_sd = q_stride_dim;
    g.out = out;
    g.o_st = out_stride_token;
    g.o_sh = out_stride_head;
    g.k_pool = k_pool;
    g.v_pool = v_pool;
    g.block_size = block_size;
    g.num_kv_heads = num_kv_heads;
    g.head_dim = head_dim;
    g.num_heads = num_heads;
    g.tables = tables;
    g.width = plan->table_width;
    g.seq_idx = meta + plan->off_seq_idx;
    g.q_pos = meta + plan->off_q_pos;
    g.query_lens = meta + plan->off_query_lens;
    g.num_tokens = num_tokens;
    g.skip_decode = decode_left ? 0 : 1;
    g.skip_prefill = prefill_left ? 0 : 1;
    g.pool_blocks = pool_num_blocks;
    g.qscale = qscale;
    g.err = err;
    cudaError_t e = launch_generic(dtype, g, stream);
    if (e != cudaSuccess) return cuda_fail(e, "generic attention launch");
    g_last_launches |= PA_LAUNCH_GENERIC;
  }
  return PA_OK;
}

int32_t pa_reshape_and_cache(const void* key, int64_t k_stride_token, int64_t k_stride_head,
                             const void* value, int64_t v_stride_token, int64_t v_stride_head,
                             int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim,
                             int32_t dtype, void* k_pool, void* v_pool, int64_t pool_num_blocks,
                             int32_t block_size, const int32_t* slot_mapping, void* stream_ptr) {
  using namespace pa;
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_UNSUPPORTED, "dtype code %d is not float32, float16 or bfloat16", dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "bad append shape");
  if (num_tokens == 0) return PA_OK;
  if (!key || !value || !k_pool || !v_pool || !slot_mapping)
    return fail(PA_ERR_INVALID_ARGUMENT, "NULL device pointer");
  const int es = elem_size(dtype);
  AppendParams p{};
  p.key = static_cast<const uint8_t*>(key);
  p.k_st = k_stride_token * es;
  p.k_sh = k_stride_head * es;
  p.value = static_cast<const uint8_t*>(value);
  p.v_st = v_stride_token * es;
  p.v_sh = v_stride_head * es;
  p.num_tokens = num_tokens;
  p.num_kv_heads = num_kv_heads;
  p.row_bytes = head_dim * es;
  p.k_pool = static_cast<uint8_t*>(k_pool);
  p.v_pool = static_cast<uint8_t*>(v_pool);
  p.num_slots = pool_num_blocks * block_size;
  p.slots = slot_mapping;
  cudaError_t e = launch_append(p, static_cast<cudaStream_t>(stream_ptr));
  if (e != cudaSuccess) return cuda_fail(e, "reshape_and_cache launch");
  return PA_OK;
}

static int32_t block_move(int32_t mode, void* const* k_pools, void* const* v_pools, int32_t num_layers,
                          int64_t pool_num_blocks, int64_t block_bytes, const int32_t* ids, int32_t n,
                          const void* staging, int32_t* error_word, void* stream_ptr, const char* what) {
  using namespace pa;
  if (num_layers < 0 || n < 0 || pool_num_blocks <= 0 || block_bytes <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "%s: bad sizes (layers %d, count %d, pool %lld blocks of %lld bytes)", what,
                num_layers, n, (long long)pool_num_blocks, (long long)block_bytes);
  if (block_bytes % 16 != 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "%s: block_bytes %lld is not a multiple of 16", what, (long long)block_bytes);
  if (n == 0 || num_layers == 0) return PA_OK;
  if (!k_pools || !v_pools || !ids || !error_word || (mode != kBlockCopy && !staging))
    return fail(PA_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (reinterpret_cast<uintptr_t>(staging) % 16 != 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "%s: staging buffer is not 16-byte aligned", what);
  BlockCopyParams p{};
  p.mode = mode;
  p.n = n;
  p.block_bytes = block_bytes;
  p.pool_blocks = pool_num_blocks;
  p.ids = ids;
  p.staging = static_cast<uint8_t*>(const_cast<void*>(staging));
  p.err = error_word;
  for (int32_t l0 = 0; l0 < num_layers; l0 += kCopyLayers) {
    p.layer0 = l0;
    p.num_layers = std::min<int32_t>(kCopyLayers, num_layers - l0);
    for (int32_t l = 0; l < p.num_layers; ++l) {
      p.k[l] = static_cast<uint8_t*>(k_pools[l0 + l]);
      p.v[l] = static_cast<uint8_t*>(v_pools[l0 + l]);
      if (!p.k[l] || !p.v[l] || reinterpret_cast<uintptr_t>(p.k[l]) % 16 || reinterpret_cast<uintptr_t>(p.v[l]) % 16)
        return fail(PA_ERR_INVALID_ARGUMENT, "%s: layer %d pool pointer is NULL or not 16-byte aligned", what, l0 + l);
    }
    cudaError_t e = launch_block_copy(p, static_cast<cudaStream_t>(stream_ptr));
    if (e != cudaSuccess) return cuda_fail(e, what);
  }
  return PA_OK;
}

int32_t pa_copy_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                       int64_t block_bytes, const int32_t* pairs, int32_t num_pairs, int32_t* error_word,
                       void* stream) {
  return block_move(pa::kBlockCopy, k_pools, v_pools, num_layers, pool_num_blocks, block_bytes, pairs, num_pairs,
                    nullptr, error_word, stream, "copy_blocks");
}

int32_t pa_gather_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                         int64_t block_bytes, const int32_t* blocks, int32_t num_blocks, void* staging,
                         int32_t* error_word, void* stream) {
  return block_move(pa::kBlockGather, k_pools, v_pools, num_layers, pool_num_blocks, block_bytes, blocks, num_blocks,
                    staging, error_word, stream, "gather_blocks");
}

int32_t pa_scatter_blocks(void* const* k_pools, void* const* v_pools, int32_t num_layers, int64_t pool_num_blocks,
                          int64_t block_bytes, const int32_t* blocks, int32_t num_blocks, const void* staging,
                          int32_t* error_word, void* stream) {
  return block_move(pa::kBlockScatter, k_pools, v_pools, num_layers, pool_num_blocks, block_bytes, blocks,
                    num_blocks, staging, error_word, stream, "scatter_blocks");
}

int32_t pa_prefill_tile_rows(int32_t head_dim) {
  (void)head_dim;  // 128-row tiles serve every head_dim by default (the 256-row pair kernel measured slower)
  return pa::prefill_tile_rows();
}

int32_t pa_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  using namespace pa;
  if (!dev_ptr || !handle_out || !offset_out) return fail(PA_ERR_INVALID_ARGUMENT, "ipc_export: NULL pointer");
  auto fn = range_fn();
  if (!fn) return fail(PA_ERR_CUDA, "cuMemGetAddressRange is not available from the CUDA driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return fail(PA_ERR_INVALID_ARGUMENT, "ipc_export: %p is not device memory", dev_ptr);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<uintptr_t>(dev_ptr) - uintptr_t(base));
  return PA_OK;
}

int32_t pa_ipc_open(const void* handle, int64_t offset, void** dev_ptr_out) {
  using namespace pa;
  if (!handle || !dev_ptr_out || offset < 0) return fail(PA_ERR_INVALID_ARGUMENT, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *dev_ptr_out = static_cast<uint8_t*>(base) + offset;
  return PA_OK;
}

int32_t pa_ipc_close(void* dev_ptr, int64_t offset) {
  using namespace pa;
  if (!dev_ptr || offset < 0) return fail(PA_ERR_INVALID_ARGUMENT, "ipc_close: bad argument");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return PA_OK;
}

int32_t pa_peer_allreduce(void* const* bases, int32_t world, int32_t rank, int64_t data_offset, int64_t flags_offset,
                          int64_t count, int32_t dtype, double timeout_s, int32_t* error_word, void* stream_ptr) {
  using namespace pa;
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(PA_ERR_INVALID_ARGUMENT, "peer_allreduce: rank %d of %d (at most %d ranks)", rank, world, kPeerMax);
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_UNSUPPORTED, "peer_allreduce: dtype code %d", dtype);
  const int es = elem_size(dtype);
  if (count < 0 || (count * es) % 16 != 0)
    return fail(PA_ERR_UNSUPPORTED, "peer_allreduce: %lld elements is not a whole number of 16-byte vectors",
                (long long)count);
  if (!bases || !error_word || data_offset % 16 || flags_offset % 16 || data_offset < 0 || flags_offset < 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "peer_allreduce: NULL pointer or unaligned offset");
  if (!(timeout_s > 0.0) || timeout_s > 600.0)
    return fail(PA_ERR_INVALID_ARGUMENT, "peer_allreduce: timeout must be in (0, 600] seconds");
  PeerReduceParams p{};
  for (int r = 0; r < world; ++r) {
    p.base[r] = static_cast<uint8_t*>(bases[r]);
    if (!p.base[r] || reinterpret_cast<uintptr_t>(p.base[r]) % 16)
      return fail(PA_ERR_INVALID_ARGUMENT, "peer_allreduce: buffer of rank %d is NULL or not 16-byte aligned", r);
  }
  p.data_offset = data_offset;
  p.flags_offset = flags_offset;
  p.count = count;
  p.world = world;
  p.rank = rank;
  p.timeout_ns = uint64_t(timeout_s * 1e9);
  p.err = error_word;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // At most one CTA per SM, so every CTA of the call is resident and the barrier's
  // signalling CTA always runs.
  const int64_t vecs = count * es / 16, per = (vecs + world - 1) / world;
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(sms, (per + kPeerThreads - 1) / kPeerThreads)));
  cudaError_t e = launch_peer_allreduce(dtype, p, grid, static_cast<cudaStream_t>(stream_ptr));
  if (e != cudaSuccess) return cuda_fail(e, "peer_allreduce launch");
  return PA_OK;
}

int32_t pa_oproj_allreduce(const void* a, int64_t a_row_stride, int32_t rows, int32_t k, const void* w, int32_t n,
                           int32_t dtype, void* const* bases, int32_t world, int32_t rank, int64_t stage_offset,
                           int64_t out_offset, int64_t flags_offset, double timeout_s, int32_t* error_word,
                           void* stream_ptr) {
  using namespace pa;
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: rank %d of %d (at most %d ranks)", rank, world, kPeerMax);
  if (dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_UNSUPPORTED, "oproj_allreduce: dtype code %d (bf16 or fp16 only)", dtype);
  if (rows < 0 || k <= 0 || k % kOprojKStep || n <= 0 || n % (kOprojTileN * world))
    return fail(PA_ERR_UNSUPPORTED, "oproj_allreduce: rows %d, k %d, n %d (k a multiple of %d, n of %d x %d ranks)",
                rows, k, n, kOprojKStep, kOprojTileN, world);
  if (a_row_stride < k || a_row_stride % 8 || a_row_stride > (int64_t(1) << 32))
    return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: a row stride %lld for k %d (a multiple of 8, >= k)",
                (long long)a_row_stride, k);
  if (!a || !w || !bases || !error_word || reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(w) % 16)
    return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: NULL or unaligned pointer");
  if (stage_offset < 0 || out_offset < 0 || flags_offset < 0 || stage_offset % 16 || out_offset % 16 ||
      flags_offset % 16)
    return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: offsets must be non-negative multiples of 16");
  if (!(timeout_s > 0.0) || timeout_s > 600.0)
    return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: timeout must be in (0, 600] seconds");
  OprojParams p{};
  for (int r = 0; r < world; ++r) {
    p.base[r] = static_cast<uint8_t*>(bases[r]);
    if (!p.base[r] || reinterpret_cast<uintptr_t>(p.base[r]) % 16)
      return fail(PA_ERR_INVALID_ARGUMENT, "oproj_allreduce: buffer of rank %d is NULL or not 16-byte aligned", r);
  }
  if (rows == 0) return PA_OK;
  auto fn = encode_fn();
  if (!fn) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the CUDA driver");
  // a as (k, rows) and w as (k, n): one stage is a (64, 128) box of a and a (64, 256) box
  // of w, 128-byte swizzle (rows past `rows` read as zeros).
  auto kmajor = [&](const void* base, int64_t outer, int64_t stride, int box_rows, CUtensorMap* map) -> int32_t {
    cuuint64_t gdim[2] = {cuuint64_t(k), cuuint64_t(outer)};
    cuuint64_t gstride[1] = {cuuint64_t(stride) * 2};
    cuuint32_t box[2] = {cuuint32_t(kOprojKStep), cuuint32_t(box_rows)};
    cuuint32_t estride[2] = {1u, 1u};
    CUresult r = fn(map, tma_dtype(dtype), 2, const_cast<void*>(base), gdim, gstride, box, estride,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    return PA_OK;
  };
  CUtensorMap ta, tw, tw_half;
  int32_t st = kmajor(a, rows, a_row_stride, kOprojTile, &ta);
  if (st != PA_OK) return st;
  st = kmajor(w, n, k, kOprojTileN, &tw);
  if (st != PA_OK) return st;
  st = kmajor(w, n, k, kOprojTileN / 2, &tw_half);
  if (st != PA_OK) return st;
  p.stage_offset = stage_offset;
  p.out_offset = out_offset;
  p.flags_offset = flags_offset;
  p.rows = rows;
  p.k = k;
  p.n = n;
  p.world = world;
  p.rank = rank;
  p.timeout_ns = uint64_t(timeout_s * 1e9);
  p.err = error_word;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t vecs = int64_t(rows) * (n / world) * 2 / 16;  // 16-byte vectors of this rank's slice
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(sms, (vecs + kPeerThreads - 1) / kPeerThreads)));
  cudaError_t e = launch_oproj_allreduce(dtype, ta, tw, tw_half, p, grid, static_cast<cudaStream_t>(stream_ptr));
  if (e != cudaSuccess) return cuda_fail(e, "oproj_allreduce launch");
  return PA_OK;
}

int32_t pa_read_device_error(void* workspace, int32_t clear, int32_t* error_word, void* stream_ptr) {
  using namespace pa;
  if (!workspace || !error_word) return fail(PA_ERR_INVALID_ARGUMENT, "NULL pointer");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, workspace, sizeof(word), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (clear) {
    e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), stream);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  *error_word = word;
  return PA_OK;
}

}  // extern "C"
