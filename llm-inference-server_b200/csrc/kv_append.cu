// Fused K+V append ("reshape and cache"): one CTA per new token copies that token's
// [num_kv_heads, head_dim] key row and value row into both pools at its flat slot.
// The copy is bitwise, so the pool bytes equal those of the reference's two
// index_copy_ calls (inference_server/core/paged_executor.py:116-125).
#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

template <int VEC>
struct Chunk;
template <> struct Chunk<16> { using T = uint4; };
template <> struct Chunk<8> { using T = uint2; };
template <> struct Chunk<4> { using T = uint32_t; };
template <> struct Chunk<2> { using T = uint16_t; };

template <int VEC>
__global__ void __launch_bounds__(128) reshape_and_cache_kernel(const AppendParams p) {
  using C = typename Chunk<VEC>::T;
  const int t = blockIdx.x;
  const int32_t slot = p.slots[t];
  if (slot < 0 || int64_t(slot) >= p.num_slots) return;  // planned steps never get here
  const int per_head = p.row_bytes / VEC;
  const int per_tensor = p.num_kv_heads * per_head;
  const int64_t dst_row = int64_t(slot) * p.num_kv_heads * p.row_bytes;
  for (int c = threadIdx.x; c < 2 * per_tensor; c += blockDim.x) {
    const bool is_v = c >= per_tensor;
    const int cc = is_v ? c - per_tensor : c;
    const int h = cc / per_head, j = cc - h * per_head;
    const uint8_t* src = is_v ? p.value + t * p.v_st + h * p.v_sh : p.key + t * p.k_st + h * p.k_sh;
    uint8_t* dst = (is_v ? p.v_pool : p.k_pool) + dst_row + int64_t(h) * p.row_bytes;
    *reinterpret_cast<C*>(dst + j * VEC) = *reinterpret_cast<const C*>(src + j * VEC);
  }
}

cudaError_t launch_append(const AppendParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  auto aligned = [&](int v) {
    auto ok = [v](int64_t x) { return x % v == 0; };
    return ok(p.row_bytes) && ok(p.k_st) && ok(p.k_sh) && ok(p.v_st) && ok(p.v_sh) &&
           ok(reinterpret_cast<uintptr_t>(p.key)) && ok(reinterpret_cast<uintptr_t>(p.value)) &&
           ok(reinterpret_cast<uintptr_t>(p.k_pool)) && ok(reinterpret_cast<uintptr_t>(p.v_pool));
  };
  dim3 grid(p.num_tokens), block(128);
  if (aligned(16))
    reshape_and_cache_kernel<16><<<grid, block, 0, stream>>>(p);
  else if (aligned(8))
    reshape_and_cache_kernel<8><<<grid, block, 0, stream>>>(p);
  else if (aligned(4))
    reshape_and_cache_kernel<4><<<grid, block, 0, stream>>>(p);
  else
    reshape_and_cache_kernel<2><<<grid, block, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace pa
