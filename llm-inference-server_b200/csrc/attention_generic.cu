// Generic paged attention: one warp per (query token, head), any block size, any
// head_dim up to 256, any query strides, any GQA group.  It covers every shape the
// reference's contract admits (its tests use block sizes 4 and 6 and head_dims 8 and
// 12, tests/test_paged_attention_triton.py:74-128) and serves prefill rows that no
// shape-specialised kernel takes.
//
// Semantics follow inference_server/core/attention.py:92-187: token t of sequence i sits
// at q_pos = ctx_i - q_i + t and attends to keys 0..q_pos through the block table; GQA
// head h reads KV head h / (Hq / Hkv) (attention_triton.py:181).  Keys are walked in
// chunks of 32 (one per lane) with a float32 online softmax in the log2 domain.
#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

constexpr int kGenericMaxDim = 256;
constexpr int kGenericWarps = 4;

template <typename T>
__global__ void __launch_bounds__(32 * kGenericWarps) paged_attention_generic_kernel(const GenericParams p) {
  __shared__ float qs[kGenericWarps][kGenericMaxDim];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pair = int64_t(blockIdx.x) * kGenericWarps + warp;
  if (pair >= int64_t(p.num_tokens) * p.num_heads) return;
  const int tok = int(pair / p.num_heads), h = int(pair % p.num_heads);
  const int seq = p.seq_idx[tok];
  if (p.skip_decode && p.query_lens[seq] == 1) return;
  if (p.skip_prefill && p.query_lens[seq] > 1) return;
  const int n_keys = p.q_pos[tok] + 1;
  const int kvh = h / (p.num_heads / p.num_kv_heads);
  const int D = p.head_dim;

  const T* q = static_cast<const T*>(p.q) + tok * p.q_st + h * p.q_sh;
  for (int d = lane; d < D; d += 32) qs[warp][d] = to_float(q[d * p.q_sd]) * p.qscale;
  __syncwarp();

  const T* kp = static_cast<const T*>(p.k_pool);
  const T* vp = static_cast<const T*>(p.v_pool);
  const int32_t* row = p.tables + int64_t(seq) * p.width;
  const int64_t head_stride = D, slot_stride = int64_t(p.num_kv_heads) * D;

  float m = -INFINITY, l = 0.f, acc[kGenericMaxDim / 32];
#pragma unroll
  for (int i = 0; i < kGenericMaxDim / 32; ++i) acc[i] = 0.f;

  for (int k0 = 0; k0 < n_keys; k0 += 32) {
    const int key = k0 + lane;
    float s = -INFINITY;
    int64_t slot = 0;
    if (key < n_keys) {
      int64_t phys = row[key / p.block_size];
      if (phys < 0 || phys >= p.pool_blocks) {  // host-validated; never taken
        set_error(p.err, kErrBlockId);
        phys = 0;
      }
      slot = phys * p.block_size + key % p.block_size;
      const T* kr = kp + slot * slot_stride + kvh * head_stride;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(qs[warp][d], to_float(kr[d]), dot);
      s = dot;
    }
    float cmax = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
    const float m_new = fmaxf(m, cmax);
    const float alpha = exp2f(m - m_new);
    const float pr = key < n_keys ? exp2f(s - m_new) : 0.f;
    float psum = pr;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * alpha + psum;
#pragma unroll
    for (int i = 0; i < kGenericMaxDim / 32; ++i) acc[i] *= alpha;
    const int nk = min(32, n_keys - k0);
    for (int j = 0; j < nk; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pr, j);
      const int64_t sj = __shfl_sync(0xffffffffu, slot, j);
      const T* vr = vp + sj * slot_stride + kvh * head_stride;
#pragma unroll
      for (int i = 0; i < kGenericMaxDim / 32; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] = fmaf(pj, to_float(vr[d]), acc[i]);
      }
    }
    m = m_new;
  }
  T* o = static_cast<T*>(p.out) + tok * p.o_st + h * p.o_sh;
  const float inv = 1.f / l;
#pragma unroll
  for (int i = 0; i < kGenericMaxDim / 32; ++i) {
    const int d = lane + 32 * i;
    if (d < D) o[d] = from_float<T>(acc[i] * inv);
  }
}

cudaError_t launch_generic(int dtype, const GenericParams& p, cudaStream_t stream) {
  const int64_t pairs = int64_t(p.num_tokens) * p.num_heads;
  if (pairs == 0) return cudaSuccess;
  dim3 grid(unsigned((pairs + kGenericWarps - 1) / kGenericWarps)), block(32 * kGenericWarps);
  switch (dtype) {
    case PA_DTYPE_F32: paged_attention_generic_kernel<float><<<grid, block, 0, stream>>>(p); break;
    case PA_DTYPE_F16: paged_attention_generic_kernel<__half><<<grid, block, 0, stream>>>(p); break;
    case PA_DTYPE_BF16: paged_attention_generic_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pa
