// pa_paged_attention_fwd_noalloc: paged attention for callers that cannot allocate
// device memory.
//
// Some callers cannot call cudaMalloc: a plug-in running inside a host framework that
// owns every byte of device memory and forbids allocation from its callbacks, or a
// latency-critical serving loop that cannot afford cudaMalloc's implicit device-wide
// synchronisation.  They still own their inputs and outputs, but the split-K decode
// also needs scratch for its per-split partial results.  This entry point gives that
// scratch a fixed home: a file-scope device array of PA_NOALLOC_SCRATCH_BYTES that the
// CUDA runtime reserves on every GPU where this library's code is loaded, and keeps
// until the process exits.
//
// The host cannot use the array's name as a device address (in host code it names a
// host-side stand-in), so the first call on each device, with that device current,
// looks the address up with cudaGetSymbolAddress and caches it; make that first call
// before any stream capture.  Every call shares the one array and finds the previous
// call's contents in it: the error word that kernels OR into is cleared at the start of
// each call, and the partials are always written before they are read.  Two calls whose
// work overlaps on the GPU (different streams, or different host threads on one device)
// race on the array; serialise them.
#include <cuda_runtime.h>

#include <mutex>

#include "paged_attention_b200.h"
#include "pa_host.h"

namespace pa {

static __device__ __align__(256) unsigned char g_noalloc_scratch[PA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
static int32_t noalloc_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(PA_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(PA_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(PA_ERR_CUDA, "cudaGetSymbolAddress of the static scratch: %s", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return PA_OK;
}

}  // namespace pa

extern "C" int32_t pa_paged_attention_fwd_noalloc(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int64_t q_stride_dim, int32_t num_tokens,
    int32_t num_heads, int32_t head_dim, const void* k_pool, const void* v_pool, int64_t pool_num_blocks,
    int32_t block_size, int32_t num_kv_heads, int32_t dtype, float scale, const pa_step_plan* plan,
    const int32_t* meta, void* out, int64_t out_stride_token, int64_t out_stride_head, void* stream) {
  using namespace pa;
  if (!plan) return fail(PA_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  const uint64_t need = pa_workspace_bytes(plan, num_heads, head_dim);
  if (need > uint64_t(PA_NOALLOC_SCRATCH_BYTES))
    return fail(PA_ERR_BUFFER_TOO_SMALL,
                "this step needs %llu bytes of split-K scratch but the static scratch holds %llu; "
                "plan a smaller batch or call pa_paged_attention_fwd with a workspace",
                (unsigned long long)need, (unsigned long long)PA_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int32_t rc = noalloc_scratch_address(&scratch);
  if (rc != PA_OK) return rc;
  cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(int32_t), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(PA_ERR_CUDA, "clearing the scratch error word: %s", cudaGetErrorString(e));
  return pa_paged_attention_fwd(query, q_stride_token, q_stride_head, q_stride_dim, num_tokens, num_heads, head_dim,
                                k_pool, v_pool, pool_num_blocks, block_size, num_kv_heads, dtype, scale, plan, meta,
                                out, out_stride_token, out_stride_head, scratch, PA_NOALLOC_SCRATCH_BYTES, stream);
}
