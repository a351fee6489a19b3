// Whole-block KV moves across every layer in one launch: copy-on-write copies, and the
// gather / scatter halves of swap-out and swap-in.
//
// Reference behaviour restated:
//   copy     inference_server/core/paged_executor.py:265-270 (_copy_block: for each layer
//            pool[dst] = pool[src], K then V), called per shared block by
//            BlockTable.ensure_private.  Here one launch moves any number of blocks.
//   gather   inference_server/core/kv_pool.py:142-166 (swap_out: per layer
//            index_select(0, blocks) into a host tensor [n, block_size, Hkv, D]).  Here the
//            blocks of all layers land in one staging buffer laid out
//            [layer][K, V][n][block] (each [layer][K or V] slice is exactly the reference's
//            per-layer host tensor), so the device-to-host transfer is a single copy.
//   scatter  inference_server/core/kv_pool.py:168-182 (swap_in: per layer
//            index_copy_(0, blocks, host)), from the same staging layout.
//
// Each CTA moves one (block, K or V, layer) unit with 16-byte vector loads and stores;
// units of one layer and kind are consecutive in the grid, so a gather's writes (and a
// scatter's reads) of the staging buffer are contiguous across neighbouring CTAs.  Block
// ids are checked against the pool; a bad id sets kErrBlockId in the error word and its
// unit is skipped.  The copy is bitwise for every dtype.
#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

__global__ void __launch_bounds__(256) block_copy_kernel(const BlockCopyParams p) {
  const int64_t unit = blockIdx.x;
  const int i = int(unit % p.n);
  const int kind = int((unit / p.n) % 2);  // 0 = K, 1 = V
  const int layer = int(unit / (2 * int64_t(p.n)));
  uint8_t* pool = kind == 0 ? p.k[layer] : p.v[layer];
  const uint4* src;
  uint4* dst;
  if (p.mode == kBlockCopy) {
    const int s = p.ids[2 * i], d = p.ids[2 * i + 1];
    if (s < 0 || s >= p.pool_blocks || d < 0 || d >= p.pool_blocks) {
      if (threadIdx.x == 0) set_error(p.err, kErrBlockId);
      return;
    }
    src = reinterpret_cast<const uint4*>(pool + int64_t(s) * p.block_bytes);
    dst = reinterpret_cast<uint4*>(pool + int64_t(d) * p.block_bytes);
  } else {
    const int b = p.ids[i];
    if (b < 0 || b >= p.pool_blocks) {
      if (threadIdx.x == 0) set_error(p.err, kErrBlockId);
      return;
    }
    uint8_t* stage = p.staging + (((int64_t(p.layer0) + layer) * 2 + kind) * p.n + i) * p.block_bytes;
    uint8_t* blk = pool + int64_t(b) * p.block_bytes;
    src = reinterpret_cast<const uint4*>(p.mode == kBlockGather ? blk : stage);
    dst = reinterpret_cast<uint4*>(p.mode == kBlockGather ? stage : blk);
  }
  // Eight 16-byte loads in flight per thread before their stores (a 32 KB block is
  // exactly one such round at 256 threads).
  const int64_t chunks = p.block_bytes / 16;
  const int64_t step = blockDim.x;
  int64_t c = threadIdx.x;
  for (; c + 7 * step < chunks; c += 8 * step) {
    uint4 r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) r[u] = src[c + u * step];
#pragma unroll
    for (int u = 0; u < 8; ++u) dst[c + u * step] = r[u];
  }
  for (; c < chunks; c += step) dst[c] = src[c];
}

cudaError_t launch_block_copy(const BlockCopyParams& p, cudaStream_t stream) {
  if (p.n == 0 || p.num_layers == 0) return cudaSuccess;
  const int64_t units = int64_t(p.n) * 2 * p.num_layers;
  block_copy_kernel<<<dim3(unsigned(units)), dim3(256), 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace pa
