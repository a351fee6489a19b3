// The tensor-parallel output projection fused with its all-reduce over NVLink peer memory.
//
// Rank r holds a_r, the attention output of its query heads ([rows, k], row stride in
// elements), and w_r, its row slice of o_proj stored K-major ([n, k], n = d_model); the
// layer output is sum_r a_r . w_r^T, identical on every rank.  Columns are split into
// `world` contiguous slices of n / world; rank s owns slice s.  Two launches per call,
// and every access to another GPU's memory is a plain 16-byte store:
//
//   oproj_push_kernel   one CTA per 128 x 256 output tile (one CTA per SM).  Warp 4
//     streams 64-wide k steps of a and w with TMA (128-byte swizzle) into a 4-stage ring,
//     warp 5 issues tcgen05 MMAs (M = 128, N = 256, both operands K-major) into a
//     256-column TMEM accumulator, and warps 0-3 round the finished tile to the storage
//     dtype, stage it in the freed ring and store it, 512-byte row pieces at a time, into
//     the staging area of the rank owning those columns: the reduce-scatter is the GEMM's
//     epilogue.  128 x 256 moves a quarter fewer bytes per flop than 128 x 128 tiles,
//     which were measured slower in this kernel.  The last CTA to finish releases this
//     rank's "ready" flag into every rank's flag area.
//   oproj_push_pair_kernel  the same GEMM on CTA pairs (rows > 128): a cluster of two CTAs
//     computes one 256 x 256 tile with M = 256 tcgen05 MMAs (cta_group::2).  Each CTA loads
//     its own 128 rows of a and 128 of the tile's 256 rows of w (K-major) into its 6-stage
//     ring, so an SM moves a third fewer operand bytes per flop than with 128 x 256 tiles
//     (whose TMA delivery the profile shows the single-CTA GEMM waiting on); the leader's
//     MMA warp issues for both and commits to both CTAs' barriers, and each CTA's epilogue
//     pushes its own 128 x 256 accumulator exactly as above.  No load uses multicast.
//   oproj_gather_kernel the owner waits for every rank's ready flag, sums its slice over
//     the `world` staged partials in rank order in float32 (so every rank receives the
//     same bytes), rounds once and stores the sum into every rank's output slot: the
//     all-gather.  An exit barrier ("done" flags) holds each rank until every owner has
//     written its slice, so the stream's next work sees the whole output and the next
//     call's pushes cannot reach a staging area an owner is still reading.
//
// The numerics are those of the unfused path (a GEMM whose output is rounded to the
// storage dtype, then a float32 rank-order sum rounded once), with this kernel's own
// accumulation order inside the GEMM.  Flags carry a per-call epoch kept in device memory,
// as in peer_allreduce.cu, and every wait on a peer is bounded by a %globaltimer deadline
// (kErrWaitTimeout); mbarrier waits are bounded by kWaitLimit polls.  The reference has no
// multi-GPU path; this replaces the row-split o_proj GEMM plus torch.distributed.all_reduce.
#include "peer_common.cuh"
#include "tc_common.cuh"
#include "tc_pair.cuh"

namespace pa {

constexpr int kOpStages = 4;
constexpr int kOpThreads = 192;
constexpr int kOpBoxA = kOprojTile * 128;       // 128 rows x 64 elements (16-bit)
constexpr int kOpBoxW = kOprojTileN * 128;      // 256 rows x 64 elements
constexpr int kOpStage = kOpBoxA + kOpBoxW;     // a box, then w box
constexpr int kOpPitch = kOprojTileN * 2 + 16;  // staged output row: 512 bytes + 16 (bank spread)
constexpr int kOpBarOff = kOpStages * kOpStage;
constexpr int kOpSmem = kOpBarOff + 128;
static_assert(kOprojTile * kOpPitch <= kOpBarOff, "the output tile reuses the ring");
static_assert(kOpSmem <= 227 * 1024, "shared memory per CTA");

struct OpBars {
  uint64_t full[kOpStages], empty[kOpStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  uint32_t last;
};
static_assert(sizeof(OpBars) <= 128, "barrier area");

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(uint32_t lo, uint32_t hi);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kOpThreads, 1)
    oproj_push_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                      const __grid_constant__ OprojParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  OpBars* bars = reinterpret_cast<OpBars*>(smem + kOpBarOff);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kOprojTileN, m0 = blockIdx.y * kOprojTile;
  const int ksteps = p.k / kOprojKStep;

  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, kOprojTileN);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kOpStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tacc = bars->tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      bool ok = true;
      for (int j = 0; j < ksteps; ++j) {
        const int s = j % kOpStages;
        if (j >= kOpStages && !mbar_wait(&bars->empty[s], ((j / kOpStages) - 1) & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kOpStage;
        mbar_arrive_expect_tx(&bars->full[s], kOpStage);
        tma_load_2d(st, &ta, j * kOprojKStep, m0, &bars->full[s]);
        tma_load_2d(st + kOpBoxA, &tw, j * kOprojKStep, n0, &bars->full[s]);
      }
      if (!ok) set_error(p.err, kErrWaitTimeout);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16<T>(kOprojTile, kOprojTileN, false);
      bool ok = true;
      for (int j = 0; j < ksteps; ++j) {
        const int s = j % kOpStages;
        if (!mbar_wait(&bars->full[s], (j / kOpStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * kOpStage), w0 = a0 + kOpBoxA;
#pragma unroll
        for (int kk = 0; kk < kOprojKStep / 16; ++kk)
          umma_f16(tacc, smem_desc_sw128(a0 + kk * 32, 16, 1024), smem_desc_sw128(w0 + kk * 32, 16, 1024), idesc,
                   (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars->empty[s]);
      }
      if (!ok) set_error(p.err, kErrWaitTimeout);
      umma_commit(&bars->acc_full);  // also after an error, so the epilogue is not left waiting
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 0-3)
    // Row r of the tile is TMEM lane r; every MMA and every TMA load has completed once
    // acc_full fires, so the ring's shared memory is free for the staged tile.
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full, 0));
    if (got) {
      tc_fence_after();
      const int r = warp * 32 + lane;
      const uint32_t lane_base = uint32_t(warp * 32) << 16;
#pragma unroll
      for (int c = 0; c < kOprojTileN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tacc + lane_base + 32 * c, v);
        tmem_wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(smem + r * kOpPitch + c * 64);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_pair<T>(v[8 * q], v[8 * q + 1]), pack_pair<T>(v[8 * q + 2], v[8 * q + 3]),
                              pack_pair<T>(v[8 * q + 4], v[8 * q + 5]), pack_pair<T>(v[8 * q + 6], v[8 * q + 7]));
      }
    } else if (lane == 0) {
      set_error(p.err, kErrWaitTimeout);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
    if (got) {
      // One warp per 512-byte row piece; destination: staging[rank][row][col0 ..] of the
      // owner of columns n0 .. n0 + 255.
      const int slice = p.n / p.world, owner = n0 / slice, col0 = n0 - owner * slice;
      uint8_t* dst = p.base[owner] + p.stage_offset + (int64_t(p.rank) * p.rows * slice + col0) * 2;
      const int ch = tid & 31;
#pragma unroll 4
      for (int row = tid >> 5; row < kOprojTile; row += 4) {
        if (m0 + row < p.rows) {
          const uint4 v = *reinterpret_cast<const uint4*>(smem + row * kOpPitch + ch * 16);
          *reinterpret_cast<uint4*>(dst + int64_t(m0 + row) * slice * 2 + ch * 16) = v;
        }
      }
    }
  }

  // ---- completion: the last CTA to finish tells every owner that this rank's pushes are
  // complete.  The CTA barrier orders every thread's stores before thread 0's system-scope
  // fence and count.
  tc_fence_before();
  __syncthreads();
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(p.base[p.rank] + p.flags_offset);
  if (tid == 0) {
    __threadfence_system();
    uint32_t* counter = my_flags + kPeerCounter;
    const uint32_t last = atomicAdd(counter, 1u) == gridDim.x * gridDim.y - 1 ? 1u : 0u;
    if (last) *counter = 0;  // ready for the next call (stream-ordered)
    bars->last = last;
  }
  __syncthreads();
  if (bars->last && tid < p.world) {
    __threadfence_system();
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags + kPeerEpoch) + 1;
    st_release_sys(reinterpret_cast<uint32_t*>(p.base[tid] + p.flags_offset) + kPeerReady + p.rank, epoch);
  }
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tacc, kOprojTileN);
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM
constexpr int kOp2Stages = 6;
constexpr int kOp2Box = 128 * 128;                 // 128 rows x 64 k (16-bit), a or w
constexpr int kOp2Stage = 2 * kOp2Box;             // this CTA's a box, then its w box
constexpr int kOp2BarOff = kOp2Stages * kOp2Stage;
constexpr int kOp2Smem = kOp2BarOff + 128;
static_assert(kOprojTile * kOpPitch <= kOp2BarOff, "the output tile reuses the ring");
static_assert(kOp2Smem <= 227 * 1024, "shared memory per CTA");

struct OpBars2 {
  uint64_t full[kOp2Stages], empty[kOp2Stages];
  uint64_t acc_full;
  uint32_t tmem_base;
  uint32_t last;
};
static_assert(sizeof(OpBars2) <= 128, "barrier area");

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kOpThreads, 1)
    oproj_push_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                           const __grid_constant__ OprojParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  OpBars2* bars = reinterpret_cast<OpBars2*>(smem + kOp2BarOff);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int n0 = (blockIdx.x >> 1) * kOprojTileN;                   // the pair's 256 output columns
  const int m0 = blockIdx.y * 2 * kOprojTile + int(rank) * kOprojTile;  // this CTA's 128 rows
  const int wrow0 = n0 + int(rank) * (kOprojTileN / 2);             // this CTA's half of w's rows
  const int ksteps = p.k / kOprojKStep;

  if (warp == 5) {
    tmem_alloc_pair(&bars->tmem_base, kOprojTileN);
    tmem_relinquish_pair();
  }
  if (tid == 0) {
    for (int s = 0; s < kOp2Stages; ++s) {
      mbar_init(&bars->full[s], 2);     // both CTAs' expect-tx arrivals (leader's copy is used)
      mbar_init(&bars->empty[s], 1);    // the leader's MMA commit, multicast to both CTAs
    }
    mbar_init(&bars->acc_full, 1);
    fence_mbar_init();
  }
  // Both CTAs' barriers and TMEM exist before any cross-CTA arrival, load or MMA.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tacc = bars->tmem_base;
  auto leader_bar = [&](uint64_t* b) { return mapa_rank(smem_u32(b), 0); };

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      bool ok = true;
      for (int j = 0; j < ksteps; ++j) {
        const int s = j % kOp2Stages;
        if (j >= kOp2Stages && !mbar_wait(&bars->empty[s], ((j / kOp2Stages) - 1) & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kOp2Stage;
        if (leader)
          mbar_arrive_expect_tx(&bars->full[s], kOp2Stage);
        else
          mbar_arrive_expect_tx_remote(leader_bar(&bars->full[s]), kOp2Stage);
        tma_load_2d_pair(st, &ta, j * kOprojKStep, m0, leader_bar(&bars->full[s]));
        tma_load_2d_pair(st + kOp2Box, &tw, j * kOprojKStep, wrow0, leader_bar(&bars->full[s]));
      }
      if (!ok) set_error(p.err, kErrWaitTimeout);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16<T>(2 * kOprojTile, kOprojTileN, false);
      bool ok = true;
      for (int j = 0; j < ksteps; ++j) {
        const int s = j % kOp2Stages;
        if (!mbar_wait(&bars->full[s], (j / kOp2Stages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * kOp2Stage), w0 = a0 + kOp2Box;
#pragma unroll
        for (int kk = 0; kk < kOprojKStep / 16; ++kk)
          umma_pair_ss(tacc, smem_desc_sw128(a0 + kk * 32, 16, 1024), smem_desc_sw128(w0 + kk * 32, 16, 1024),
                       idesc, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair(&bars->empty[s]);
      }
      if (!ok) set_error(p.err, kErrWaitTimeout);
      umma_commit_pair(&bars->acc_full);  // also after an error, so neither epilogue is left waiting
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 0-3)
    // This CTA's 128 rows of the tile are its TMEM lanes; every MMA and every TMA load has
    // completed once acc_full fires, so the ring's shared memory is free for the staged tile.
    const bool got = __all_sync(0xffffffffu, mbar_wait(&bars->acc_full, 0));
    if (got) {
      tc_fence_after();
      const int r = warp * 32 + lane;
      const uint32_t lane_base = uint32_t(warp * 32) << 16;
#pragma unroll
      for (int c = 0; c < kOprojTileN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tacc + lane_base + 32 * c, v);
        tmem_wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(smem + r * kOpPitch + c * 64);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_pair<T>(v[8 * q], v[8 * q + 1]), pack_pair<T>(v[8 * q + 2], v[8 * q + 3]),
                              pack_pair<T>(v[8 * q + 4], v[8 * q + 5]), pack_pair<T>(v[8 * q + 6], v[8 * q + 7]));
      }
    } else if (lane == 0) {
      set_error(p.err, kErrWaitTimeout);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
    if (got) {
      const int slice = p.n / p.world, owner = n0 / slice, col0 = n0 - owner * slice;
      uint8_t* dst = p.base[owner] + p.stage_offset + (int64_t(p.rank) * p.rows * slice + col0) * 2;
      const int ch = tid & 31;
#pragma unroll 4
      for (int row = tid >> 5; row < kOprojTile; row += 4) {
        if (m0 + row < p.rows) {
          const uint4 v = *reinterpret_cast<const uint4*>(smem + row * kOpPitch + ch * 16);
          *reinterpret_cast<uint4*>(dst + int64_t(m0 + row) * slice * 2 + ch * 16) = v;
        }
      }
    }
  }

  // ---- completion, as in oproj_push_kernel: the last CTA releases this rank's ready flag.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(p.base[p.rank] + p.flags_offset);
  if (tid == 0) {
    __threadfence_system();
    uint32_t* counter = my_flags + kPeerCounter;
    const uint32_t last = atomicAdd(counter, 1u) == gridDim.x * gridDim.y - 1 ? 1u : 0u;
    if (last) *counter = 0;  // ready for the next call (stream-ordered)
    bars->last = last;
  }
  __syncthreads();
  if (bars->last && tid < p.world) {
    __threadfence_system();
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags + kPeerEpoch) + 1;
    st_release_sys(reinterpret_cast<uint32_t*>(p.base[tid] + p.flags_offset) + kPeerReady + p.rank, epoch);
  }
  // Neither CTA frees TMEM or leaves while the pair's MMAs may still read its peer.
  cluster_sync_all();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tacc, kOprojTileN);
  }
}

// WMAX: the world-size bucket (1, 2, 4 or 8); U = 16 / WMAX vectors per thread per round
// (8 for a single rank), so each thread has up to 16 staged loads in flight before it
// reduces.
template <typename T, int WMAX>
__global__ void __launch_bounds__(kPeerThreads) oproj_gather_kernel(const __grid_constant__ OprojParams p) {
  constexpr int U = WMAX == 1 ? 8 : 16 / WMAX;
  const int world = p.world, rank = p.rank;
  const uint64_t deadline = global_ns() + p.timeout_ns;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(p.base[rank] + p.flags_offset);
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(my_flags + kPeerEpoch) + 1;

  // ---- every rank's partial of my slice is in my staging area
  if (!wait_flags(my_flags + kPeerReady, world, epoch, deadline)) {
    if (threadIdx.x == 0) set_error(p.err, kErrWaitTimeout);
    return;
  }

  const int slice = p.n / world;
  const int64_t vrow = int64_t(slice) * 2 / 16;               // 16-byte vectors per slice row
  const int64_t total = int64_t(p.rows) * vrow;
  const int64_t src_bytes = int64_t(p.rows) * slice * 2;      // one rank's staged partial
  const uint8_t* stage = p.base[rank] + p.stage_offset;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < total; v += U * stride) {
    uint4 in[U][WMAX];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world && v + u * stride < total) in[u][r] = ld_cg(stage + r * src_bytes + (v + u * stride) * 16);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t vv = v + u * stride;
      if (vv >= total) break;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world) Pack8<T>::add(acc, in[u][r]);
      const uint4 out = Pack8<T>::pack(acc);
      const int64_t row = vv / vrow, cv = vv - row * vrow;
      const int64_t off = p.out_offset + (row * p.n + int64_t(rank) * slice) * 2 + cv * 16;
#pragma unroll
      for (int r = 0; r < WMAX; ++r)
        if (r < world) *reinterpret_cast<uint4*>(p.base[r] + off) = out;
    }
  }

  // ---- exit barrier (as in peer_allreduce_kernel): the last CTA announces that this
  // rank's slice is in every output, then waits until every owner has done the same.
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    uint32_t* counter = my_flags + kPeerCounter2;
    last = atomicAdd(counter, 1u) == gridDim.x - 1;
    if (last) *counter = 0;
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

template <typename T>
static cudaError_t launch_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tw_half,
                            const OprojParams& p, int gather_grid, cudaStream_t stream) {
  auto push = oproj_push_kernel<T>;
  auto push2 = oproj_push_pair_kernel<T>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(push, cudaFuncAttributeMaxDynamicSharedMemorySize, kOpSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(push, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(push2, cudaFuncAttributeMaxDynamicSharedMemorySize, kOp2Smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(push2, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  if (p.rows > kOprojTile) {  // CTA pairs: 256 x 256 tiles
    dim3 grid(2 * (p.n / kOprojTileN), (p.rows + 2 * kOprojTile - 1) / (2 * kOprojTile));
    push2<<<grid, kOpThreads, kOp2Smem, stream>>>(ta, tw_half, p);
  } else {
    dim3 grid(p.n / kOprojTileN, (p.rows + kOprojTile - 1) / kOprojTile);
    push<<<grid, kOpThreads, kOpSmem, stream>>>(ta, tw, p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.world <= 1)
    oproj_gather_kernel<T, 1><<<gather_grid, kPeerThreads, 0, stream>>>(p);
  else if (p.world <= 2)
    oproj_gather_kernel<T, 2><<<gather_grid, kPeerThreads, 0, stream>>>(p);
  else if (p.world <= 4)
    oproj_gather_kernel<T, 4><<<gather_grid, kPeerThreads, 0, stream>>>(p);
  else
    oproj_gather_kernel<T, 8><<<gather_grid, kPeerThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_oproj_allreduce(int dtype, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& tw_half,
                                   const OprojParams& p, int gather_grid, cudaStream_t stream) {
  if (dtype == PA_DTYPE_BF16) return launch_t<__nv_bfloat16>(ta, tw, tw_half, p, gather_grid, stream);
  if (dtype == PA_DTYPE_F16) return launch_t<__half>(ta, tw, tw_half, p, gather_grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
