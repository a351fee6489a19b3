// pa_paged_attention_fwd_noalloc: paged attention for callers that cannot allocate
// device memory, and pa_noalloc_read_device_error, which reads its error word.
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
// host-side stand-in), so the first call in each CUDA context, with that context
// current, looks the address up with cudaGetSymbolAddress, zeroes the array's error
// word once and caches the address under the context's process-unique id (a context
// destroyed and re-created, e.g. by cudaDeviceReset, gets a new id and a fresh
// look-up).  Make that first call before any stream capture.
//
// Every call shares the one array and finds the previous call's contents in it.  The
// split-K partials are always written before they are read.  The first 4 bytes are the
// device error word the kernels OR their reports into (an out-of-range block id, a
// pipeline wait that ran out of its limit); like a caller's workspace word it is
// sticky, accumulating over calls until pa_noalloc_read_device_error clears it.  Two
// calls whose work overlaps on the GPU (different streams, or different host threads on
// one device) race on the array; serialise them.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "paged_attention_b200.h"
#include "pa_host.h"

namespace pa {

static __device__ __align__(256) unsigned char g_noalloc_scratch[PA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxContexts = 64;

template <typename Fn>
static Fn driver_fn(const char* name, unsigned version) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &ptr, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(ptr);
}

// Device address of g_noalloc_scratch in the current context (looked up, and its error
// word zeroed on `stream`, once per context).
static int32_t noalloc_scratch_address(cudaStream_t stream, void** out) {
  static std::mutex mu;
  static unsigned long long ids[kMaxContexts] = {};
  static void* addrs[kMaxContexts] = {};
  static int used = 0;
  static PFN_cuCtxGetCurrent_v4000 get_ctx = driver_fn<PFN_cuCtxGetCurrent_v4000>("cuCtxGetCurrent", 4000);
  static PFN_cuCtxGetId_v12000 get_id = driver_fn<PFN_cuCtxGetId_v12000>("cuCtxGetId", 12000);
  if (!get_ctx || !get_id) return fail(PA_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are not available from the driver");

  // The runtime makes the device's primary context current on its first call in this
  // thread; cudaGetDevice alone does not, so a thread that has made no CUDA call yet
  // sees no context and the symbol look-up below initialises it.
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuCtxGetCurrent failed");
  void* p = nullptr;
  if (!ctx) {
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(PA_ERR_CUDA, "cudaGetSymbolAddress of the static scratch: %s", cudaGetErrorString(e));
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return fail(PA_ERR_CUDA, "no current CUDA context");
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return fail(PA_ERR_CUDA, "cuCtxGetId failed");

  std::lock_guard<std::mutex> g(mu);
  for (int i = 0; i < used; ++i)
    if (ids[i] == id) {
      *out = addrs[i];
      return PA_OK;
    }
  if (!p) {
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(PA_ERR_CUDA, "cudaGetSymbolAddress of the static scratch: %s", cudaGetErrorString(e));
  }
  cudaError_t e = cudaMemsetAsync(p, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return fail(PA_ERR_CUDA, "zeroing the static scratch's error word: %s", cudaGetErrorString(e));
  if (used == kMaxContexts) used = 0;  // a process that cycles through contexts: start over
  ids[used] = id;
  addrs[used] = p;
  ++used;
  *out = p;
  return PA_OK;
}

}  // namespace pa

extern "C" int32_t pa_paged_attention_fwd_noalloc(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, int64_t q_stride_dim, int32_t num_tokens,
    int32_t num_heads, int32_t head_dim, const void* k_pool, const void* v_pool, int64_t pool_num_blocks,
    int32_t block_size, int32_t num_kv_heads, int32_t dtype, float scale, const pa_step_plan* plan,
    const int32_t* meta, void* out, int64_t out_stride_token, int64_t out_stride_head, void* stream) {
  using namespace pa;
  reset_last_launches();
  const int32_t bad = check_attention_args(num_tokens, num_heads, head_dim, block_size, num_kv_heads, dtype, plan);
  if (bad != PA_OK) return bad;
  const uint64_t need = pa_workspace_bytes(plan, num_heads, head_dim);
  if (need > uint64_t(PA_NOALLOC_SCRATCH_BYTES))
    return fail(PA_ERR_BUFFER_TOO_SMALL,
                "this step needs %llu bytes of split-K scratch but the static scratch holds %llu; "
                "plan a smaller batch or call pa_paged_attention_fwd with a workspace",
                (unsigned long long)need, (unsigned long long)PA_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int32_t rc = noalloc_scratch_address(static_cast<cudaStream_t>(stream), &scratch);
  if (rc != PA_OK) return rc;
  return pa_paged_attention_fwd(query, q_stride_token, q_stride_head, q_stride_dim, num_tokens, num_heads, head_dim,
                                k_pool, v_pool, pool_num_blocks, block_size, num_kv_heads, dtype, scale, plan, meta,
                                out, out_stride_token, out_stride_head, scratch, PA_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int32_t pa_noalloc_read_device_error(int32_t clear, int32_t* error_word, void* stream) {
  using namespace pa;
  if (!error_word) return fail(PA_ERR_INVALID_ARGUMENT, "NULL pointer");
  void* scratch = nullptr;
  int32_t rc = noalloc_scratch_address(static_cast<cudaStream_t>(stream), &scratch);
  if (rc != PA_OK) return rc;
  return pa_read_device_error(scratch, clear, error_word, stream);
}
