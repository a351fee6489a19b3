// All-reduce over NVLink peer memory for the KV-head tensor-parallel output projection:
// the `world` ranks of one node each hold a [rows, cols] partial o_proj product in a
// buffer every peer has mapped (CUDA IPC; plain peer loads and stores, no multicast), and
// one kernel leaves the elementwise sum in every rank's buffer.
//
// Two-shot, in place: rank r owns the r-th of `world` contiguous slices.  After an entry
// barrier (every rank's partial is complete), rank r reads its slice from all ranks'
// buffers, sums in float32 (in rank order, so every rank's result is bitwise identical),
// rounds to the storage dtype and writes the sum into that slice of every rank's
// buffer.  Slices are disjoint, so no location is read after another rank wrote it in
// the same call.  An exit barrier then holds each rank's kernel until all peers have
// finished writing into its buffer, so the stream's next work sees the full result and a
// later partial never overwrites a slice a peer is still reading.
//
// Barriers are epoch counters in a small flag area of each buffer: a call's epoch is one
// more than the previous call's, kept in device memory (so a captured CUDA graph replays
// correctly); rank p release-stores the epoch into slot p of every rank's flag area and
// waiters acquire-load their own (local) flags.  Every wait is
// bounded by a %globaltimer deadline; on expiry the kernel sets kErrWaitTimeout in the
// error word and stops waiting, so a missing peer ends the call with an error instead of
// a hang.  The collective replaces torch.distributed.all_reduce (NCCL) in
// tensor_parallel.KVHeadParallelAttention; the reference has no multi-GPU path.
#include "peer_common.cuh"

namespace pa {

// WMAX: the world-size bucket (2, 4 or 8); U = 16 / WMAX vectors per thread per round,
// so every thread has 16 peer loads in flight before it reduces.
template <typename T, int WMAX>
__global__ void __launch_bounds__(kPeerThreads) peer_allreduce_kernel(const PeerReduceParams p) {
  constexpr int U = 16 / WMAX;
  const int world = p.world, rank = p.rank;
  const uint64_t deadline = global_ns() + p.timeout_ns;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(p.base[rank] + p.flags_offset);
  // This call's epoch: the previous call (earlier on this stream) stored its own.
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags + kPeerEpoch) + 1;

  // ---- entry barrier: my partial is complete (it was written before this kernel on my
  // stream); tell every rank, then wait until every rank has told me.
  if (blockIdx.x == 0 && threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(p.base[threadIdx.x] + p.flags_offset) + kPeerReady + rank, epoch);
  }
  if (!wait_flags(my_flags + kPeerReady, world, epoch, deadline)) {
    if (threadIdx.x == 0) set_error(p.err, kErrWaitTimeout);
    return;
  }

  // ---- my slice: sum over ranks in rank order, write the sum into every rank's buffer.
  const int64_t vecs = p.count / Pack8<T>::N;                 // 16-byte vectors in the tensor
  const int64_t per = (vecs + world - 1) / world;
  const int64_t v0 = int64_t(rank) * per, v1 = min(vecs, v0 + per);
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t v = v0 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < v1; v += U * stride) {
    uint4 in[U][WMAX];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world && v + u * stride < v1) in[u][r] = ld_cg(p.base[r] + p.data_offset + (v + u * stride) * 16);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (v + u * stride >= v1) break;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world) Pack8<T>::add(acc, in[u][r]);
      const uint4 out = Pack8<T>::pack(acc);
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world) *reinterpret_cast<uint4*>(p.base[r] + p.data_offset + (v + u * stride) * 16) = out;
    }
  }

  // ---- exit barrier: the last CTA to finish announces that this rank's writes into
  // every buffer are done, then waits for all ranks to announce the same.  The CTA
  // barrier orders every thread's stores before thread 0's system-scope fence.
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    uint32_t* counter = my_flags + kPeerCounter;
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0;  // ready for the next call (stream-ordered)
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(p.base[threadIdx.x] + p.flags_offset) + kPeerDone + rank, epoch);
  }
  const bool ok = wait_flags(my_flags + kPeerDone, world, epoch, deadline);
  if (threadIdx.x == 0) {
    if (!ok) set_error(p.err, kErrWaitTimeout);
    my_flags[kPeerEpoch] = epoch;  // read by the next call on this stream
  }
}

template <int WMAX>
static void launch_w(int dtype, const PeerReduceParams& p, int grid, cudaStream_t stream) {
  switch (dtype) {
    case PA_DTYPE_BF16: peer_allreduce_kernel<__nv_bfloat16, WMAX><<<grid, kPeerThreads, 0, stream>>>(p); break;
    case PA_DTYPE_F16: peer_allreduce_kernel<__half, WMAX><<<grid, kPeerThreads, 0, stream>>>(p); break;
    default: peer_allreduce_kernel<float, WMAX><<<grid, kPeerThreads, 0, stream>>>(p); break;
  }
}

cudaError_t launch_peer_allreduce(int dtype, const PeerReduceParams& p, int grid, cudaStream_t stream) {
  if (dtype != PA_DTYPE_BF16 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_F32) return cudaErrorInvalidValue;
  if (p.world <= 2)
    launch_w<2>(dtype, p, grid, stream);
  else if (p.world <= 4)
    launch_w<4>(dtype, p, grid, stream);
  else
    launch_w<8>(dtype, p, grid, stream);
  return cudaGetLastError();
}

}  // namespace pa
