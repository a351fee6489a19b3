// Split-K paged decode for sm_100a (query_len == 1 rows).
//
// Work: one CTA per (sequence, split) item and KV head.  A split is `split_blocks`
// consecutive 16-token blocks of one sequence's context; the host planner sizes it so
// the grid covers the GPU several times over whatever the context-length mix.  All
// G = Hq / Hkv query heads of a KV head are served by the same CTA, so each K/V byte is
// read from HBM once per step (the reference's gather re-reads it once per query head
// after `repeat_interleave`, inference_server/core/attention.py:141-142, 190-199).
//
// Data movement: each of the 4 warps owns two pipeline stages; its elected lane loads a
// block's K tile and V tile ([16, head_dim] each, one KV head) with two TMA tiled loads
// (cp.async.bulk.tensor.3d) completing on the stage's mbarrier, and refills the stage
// with the warp's next-but-one block as soon as the warp has consumed it.  Warp w takes
// blocks w, w+4, w+8, ... of the split.  The pool is described to TMA as the 3-D tensor
// [num_blocks*16 slots, num_kv_heads, head_dim], so a block's tile is the box
// (head_dim, 1, 16) at slot coordinate block*16: the block table is consumed as a TMA
// coordinate and never materialised.
//
// Math (all float32, scores pre-scaled by scale*log2(e) so exp2 is the softmax base):
//   scores   lane L owns head_dim/32 contiguous dims of q for all G heads; per token it
//            forms G partial dot products, and a reduce-scatter butterfly over the 32
//            lanes turns 32 partials per lane into one finished score per lane
//            (token t = chunk*TC + L/G, head L%G).
//   softmax  warp-shuffle max and sum over the lanes of the same head; online update of
//            (m, l) per head across blocks, as in attention_triton.py:218-228.
//   P.V      probabilities go through a 16xG warp-private shared buffer; each lane
//            accumulates its dims of all G heads over the block's valid tokens.
// At the end the 4 warps' (m, l, acc) are merged through shared memory.  A sequence with
// one split writes its normalised output directly; otherwise the unnormalised partial
// and (m, l) go to the workspace and the combine kernel finishes them.
//
// Masking follows attention.py:147-150: key j is real iff j < context_len; tokens past it
// in the last block get probability 0 and their V rows are never read.
#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

constexpr int kDecodeBS = 16;     // tokens per pool block (the fast path's block size)
constexpr int kDecodeWarps = 4;
constexpr int kDecodeStages = 2;  // pipeline stages per warp

template <typename T, int D, int G>
struct DecodeCfg {
  static constexpr int DL = D / 32;                              // dims per lane
  static constexpr int TILE_ELEMS = kDecodeBS * D;
  static constexpr int TILE_BYTES = TILE_ELEMS * sizeof(T);
  static constexpr int TC = (32 / G) < kDecodeBS ? (32 / G) : kDecodeBS;  // tokens per score chunk
  static constexpr int NCHUNK = kDecodeBS / TC;
  static constexpr int NV = TC * G;                              // partials per lane per chunk
  static constexpr int TILES_BYTES = kDecodeWarps * kDecodeStages * 2 * TILE_BYTES;
  static constexpr int BAR_BYTES = kDecodeWarps * kDecodeStages * 8;
  static constexpr int PBUF_FLOATS = kDecodeWarps * kDecodeBS * G;
  static constexpr int MERGE_FLOATS = kDecodeWarps * G * (D + 2);
  static_assert(MERGE_FLOATS * 4 <= TILES_BYTES, "merge scratch aliases the stage buffers");
  static constexpr int SMEM = TILES_BYTES + BAR_BYTES + PBUF_FLOATS * 4;
};

// Reduce-scatter across lanes: on entry each lane holds N partial sums v[0..N-1] of the
// same N quantities; on exit v[0] holds the full sum of quantity (lane * N / 32) when
// N >= 32, or of quantity (lane >> (log2(32/N))) when N < 32 (duplicated across the
// lanes of that group).
template <int N, int MASK>
__device__ __forceinline__ void reduce_scatter(float* v, int lane) {
  if constexpr (MASK > 0) {
    if constexpr (N >= 2) {
      constexpr int H = N / 2;
      const bool upper = (lane & MASK) != 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = upper ? v[i] : v[i + H];
        const float keep = upper ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, MASK);
      }
      reduce_scatter<H, MASK / 2>(v, lane);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], MASK);
      reduce_scatter<1, MASK / 2>(v, lane);
    }
  }
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(32 * kDecodeWarps)
    paged_decode_splitk_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                               const DecodeParams p) {
  using C = DecodeCfg<T, D, G>;
  constexpr int DL = C::DL, TC = C::TC, NCHUNK = C::NCHUNK, NV = C::NV;
  extern __shared__ __align__(128) uint8_t smem[];
  T* tiles = reinterpret_cast<T*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TILES_BYTES);
  float* pbuf_all = reinterpret_cast<float*>(smem + C::TILES_BYTES + C::BAR_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // KV head fastest: the heads of one work item run side by side, so the row slices of
  // each pool block they read reach DRAM close together.
  const int4 item = p.items[blockIdx.x / p.num_kv_heads];
  const int seq = item.x, split = item.y, part = item.z, nsplit = item.w;
  if (seq < 0) return;  // padding of a bucketed (CUDA-graph) plan
  const int kvh = blockIdx.x % p.num_kv_heads;
  const int ctx = p.ctx_lens[seq];
  const int tok = p.cu_q[seq];
  const int b0 = split * p.split_blocks;
  const int nb = min(p.split_blocks, (ctx + kDecodeBS - 1) / kDecodeBS - b0);
  const int32_t* row = p.tables + int64_t(seq) * p.width + b0;

  T* my_tiles = tiles + warp * kDecodeStages * 2 * C::TILE_ELEMS;
  uint64_t* my_bars = bars + warp * kDecodeStages;
  float* pbuf = pbuf_all + warp * kDecodeBS * G;
  const int my_n = nb > warp ? (nb - warp + kDecodeWarps - 1) / kDecodeWarps : 0;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kDecodeStages; ++s) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Lane 0 only: load local block `i` of this warp (block warp + 4*i of the split).
  auto issue = [&](int i, int s) {
    int phys = row[warp + kDecodeWarps * i];
    if (phys < 0 || phys >= p.pool_blocks) {  // the host planner rejects these
      set_error(p.err, kErrBlockId);
      phys = 0;
    }
    mbar_arrive_expect_tx(&my_bars[s], 2 * C::TILE_BYTES);
    tma_load_3d(my_tiles + (2 * s + 0) * C::TILE_ELEMS, &tk, 0, kvh, phys * kDecodeBS, &my_bars[s]);
    tma_load_3d(my_tiles + (2 * s + 1) * C::TILE_ELEMS, &tv, 0, kvh, phys * kDecodeBS, &my_bars[s]);
  };
  if (lane == 0) {
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
#pragma unroll
    for (int s = 0; s < kDecodeStages; ++s)
      if (s < my_n) issue(s, s);
  }

  // q for the G heads of this KV head, this lane's dims, pre-scaled.
  float q[G][DL];
  {
    const T* qp = static_cast<const T*>(p.q) + int64_t(tok) * p.q_st + int64_t(kvh * G) * p.q_sh + lane * DL;
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int d = 0; d < DL; ++d) q[h][d] = to_float(qp[h * p.q_sh + d]) * p.qscale;
  }

  float m[G], l[G], acc[G][DL];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) acc[h][d] = 0.f;
  }
  // This lane's finished-score head (G >= 2) and its token within a chunk.
  const int my_head = G >= 2 ? lane % G : 0;
  const int my_tok = G >= 2 ? lane / G : lane >> 1;
  constexpr int FIRST_MASK = G >= 2 ? G : 2;

  for (int i = 0; i < my_n; ++i) {
    const int s = i % kDecodeStages;
    if (!mbar_wait(&my_bars[s], (i / kDecodeStages) & 1)) {
      if (lane == 0) set_error(p.err, kErrWaitTimeout);
      break;
    }
    const T* Kt = my_tiles + (2 * s + 0) * C::TILE_ELEMS;
    const T* Vt = my_tiles + (2 * s + 1) * C::TILE_ELEMS;
    const int nvalid = min(kDecodeBS, ctx - (b0 + warp + kDecodeWarps * i) * kDecodeBS);

    // ---- scores: one finished score per lane per chunk
    float sc[NCHUNK];
#pragma unroll
    for (int c = 0; c < NCHUNK; ++c) {
      float v[NV];
#pragma unroll
      for (int tl = 0; tl < TC; ++tl) {
        float kf[DL];
        VecLoad<T, DL>::run(Kt + (c * TC + tl) * D + lane * DL, kf);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float a = 0.f;
#pragma unroll
          for (int d = 0; d < DL; ++d) a = fmaf(q[h][d], kf[d], a);
          v[tl * G + h] = a;
        }
      }
      reduce_scatter<NV, 16>(v, lane);
      sc[c] = (c * TC + my_tok < nvalid) ? v[0] : -INFINITY;
    }

    // ---- block max of my head, then every head's max on every lane
    float bm = sc[0];
#pragma unroll
    for (int c = 1; c < NCHUNK; ++c) bm = fmaxf(bm, sc[c]);
#pragma unroll
    for (int mask = FIRST_MASK; mask < 32; mask <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, mask));
    float m_new[G], alpha[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float bh = G >= 2 ? __shfl_sync(0xffffffffu, bm, h) : bm;
      m_new[h] = fmaxf(m[h], bh);
      alpha[h] = exp2f(m[h] - m_new[h]);
    }
    float my_m = m_new[0];
#pragma unroll
    for (int h = 1; h < G; ++h)
      if (my_head == h) my_m = m_new[h];

    // ---- probabilities, their per-head sums, and the shared buffer for P.V
    float ps = 0.f;
#pragma unroll
    for (int c = 0; c < NCHUNK; ++c) {
      const float pr = exp2f(sc[c] - my_m);
      ps += pr;
      if (G >= 2)
        pbuf[c * 32 + lane] = pr;
      else if ((lane & 1) == 0)
        pbuf[c * TC + my_tok] = pr;
    }
#pragma unroll
    for (int mask = FIRST_MASK; mask < 32; mask <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, mask);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float sh = G >= 2 ? __shfl_sync(0xffffffffu, ps, h) : ps;
      l[h] = l[h] * alpha[h] + sh;
#pragma unroll
      for (int d = 0; d < DL; ++d) acc[h][d] *= alpha[h];
      m[h] = m_new[h];
    }
    __syncwarp();

    // ---- P.V over the valid tokens of the block
#pragma unroll
    for (int t = 0; t < kDecodeBS; ++t) {
      if (t < nvalid) {
        float pv[G];
#pragma unroll
        for (int h = 0; h < G; ++h) pv[h] = pbuf[t * G + h];
        float vf[DL];
        VecLoad<T, DL>::run(Vt + t * D + lane * DL, vf);
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
          for (int d = 0; d < DL; ++d) acc[h][d] = fmaf(pv[h], vf[d], acc[h][d]);
      }
    }
    __syncwarp();  // stage s and pbuf fully consumed by every lane
    if (lane == 0 && i + kDecodeStages < my_n) {
      fence_proxy_async_smem();
      issue(i + kDecodeStages, s);
    }
  }

  // ---- merge the 4 warps (scratch aliases the stage buffers, now idle)
  __syncthreads();
  float* mrg = reinterpret_cast<float*>(smem);           // [warps][G][D] then [warps][G][2]
  float* mrg_ml = mrg + kDecodeWarps * G * D;
#pragma unroll
  for (int h = 0; h < G; ++h)
#pragma unroll
    for (int d = 0; d < DL; ++d) mrg[(warp * G + h) * D + lane * DL + d] = acc[h][d];
  if (lane < G) {
    float mm = m[0], ll = l[0];
#pragma unroll
    for (int h = 1; h < G; ++h)
      if (lane == h) { mm = m[h]; ll = l[h]; }
    mrg_ml[(warp * G + lane) * 2 + 0] = mm;
    mrg_ml[(warp * G + lane) * 2 + 1] = ll;
  }
  __syncthreads();

  const int head0 = kvh * G;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, mrg_ml[(w * G + h) * 2]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float sw = exp2f(mrg_ml[(w * G + h) * 2] - M);
      L += mrg_ml[(w * G + h) * 2 + 1] * sw;
      O += mrg[(w * G + h) * D + d] * sw;
    }
    if (nsplit == 1) {
      T* o = static_cast<T*>(p.out) + int64_t(tok) * p.o_st + int64_t(head0 + h) * p.o_sh;
      o[d] = from_float<T>(O / L);
    } else {
      const int64_t ph = int64_t(part) * p.num_heads + head0 + h;
      p.part_o[ph * D + d] = O;
      if (d == 0) p.part_ml[ph] = make_float2(M, L);
    }
  }
}

// Finish sequences whose context was split: weight each split's partial by
// exp2(m_split - M) and normalise by the weighted denominators.
template <typename T>
__global__ void __launch_bounds__(128) paged_decode_combine_kernel(const CombineParams p) {
  const int4 c = p.combine[blockIdx.x];
  if (c.x < 0) return;  // padding of a bucketed (CUDA-graph) plan
  const int tok = c.y, first = c.z, ns = c.w;
  const int h = blockIdx.y;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.part_ml[int64_t(first + s) * p.num_heads + h].x);
  float L = 0.f;
  for (int s = 0; s < ns; ++s) {
    const float2 ml = p.part_ml[int64_t(first + s) * p.num_heads + h];
    L += ml.y * exp2f(ml.x - M);
  }
  const float inv = 1.f / L;
  T* o = static_cast<T*>(p.out) + int64_t(tok) * p.o_st + int64_t(h) * p.o_sh;
  for (int d = threadIdx.x; d < p.head_dim; d += blockDim.x) {
    float O = 0.f;
    for (int s = 0; s < ns; ++s) {
      const int64_t ph = int64_t(first + s) * p.num_heads + h;
      O += p.part_o[ph * p.head_dim + d] * exp2f(p.part_ml[ph].x - M);
    }
    o[d] = from_float<T>(O * inv);
  }
}

// ------------------------------------------------------------------ dispatch
template <typename T, int D, int G>
static cudaError_t launch_one(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                              cudaStream_t stream) {
  using C = DecodeCfg<T, D, G>;
  auto kern = paged_decode_splitk_kernel<T, D, G>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    // Largest shared-memory carveout, so the designed number of CTAs fits on every SM
    // whatever the driver would otherwise pick for this launch.
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(p.num_items * p.num_kv_heads), block(32 * kDecodeWarps);
  kern<<<grid, block, C::SMEM, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t by_group(int group, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                            cudaStream_t s) {
  switch (group) {
    case 1: return launch_one<T, D, 1>(tk, tv, p, s);
    case 2: return launch_one<T, D, 2>(tk, tv, p, s);
    case 4: return launch_one<T, D, 4>(tk, tv, p, s);
    case 8: return launch_one<T, D, 8>(tk, tv, p, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t by_dim(int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                          const DecodeParams& p, cudaStream_t s) {
  switch (head_dim) {
    case 64: return by_group<T, 64>(group, tk, tv, p, s);
    case 128: return by_group<T, 128>(group, tk, tv, p, s);
    default: return cudaErrorInvalidValue;
  }
}

bool decode_supported(int dtype, int head_dim, int group, int block_size) {
  const bool dt = dtype == PA_DTYPE_F32 || dtype == PA_DTYPE_F16 || dtype == PA_DTYPE_BF16;
  const bool g = group == 1 || group == 2 || group == 4 || group == 8;
  return dt && g && (head_dim == 64 || head_dim == 128) && block_size == kDecodeBS;
}

template <typename T>
static int smem_for(int head_dim, int group) {
  auto pick = [&](auto d_tag) -> int {
    constexpr int D = decltype(d_tag)::value;
    switch (group) {
      case 1: return DecodeCfg<T, D, 1>::SMEM;
      case 2: return DecodeCfg<T, D, 2>::SMEM;
      case 4: return DecodeCfg<T, D, 4>::SMEM;
      default: return DecodeCfg<T, D, 8>::SMEM;
    }
  };
  return head_dim == 64 ? pick(std::integral_constant<int, 64>{}) : pick(std::integral_constant<int, 128>{});
}

int decode_smem_bytes(int dtype, int head_dim, int group) {
  switch (dtype) {
    case PA_DTYPE_F32: return smem_for<float>(head_dim, group);
    case PA_DTYPE_F16: return smem_for<__half>(head_dim, group);
    default: return smem_for<__nv_bfloat16>(head_dim, group);
  }
}

cudaError_t launch_decode(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                          const DecodeParams& p, cudaStream_t stream) {
  if (p.num_items == 0) return cudaSuccess;
  switch (dtype) {
    case PA_DTYPE_F32: return by_dim<float>(head_dim, group, tk, tv, p, stream);
    case PA_DTYPE_F16: return by_dim<__half>(head_dim, group, tk, tv, p, stream);
    case PA_DTYPE_BF16: return by_dim<__nv_bfloat16>(head_dim, group, tk, tv, p, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_combine(int dtype, const CombineParams& p, cudaStream_t stream) {
  if (p.num_combine == 0) return cudaSuccess;
  dim3 grid(p.num_combine, p.num_heads), block(128);
  switch (dtype) {
    case PA_DTYPE_F32: paged_decode_combine_kernel<float><<<grid, block, 0, stream>>>(p); break;
    case PA_DTYPE_F16: paged_decode_combine_kernel<__half><<<grid, block, 0, stream>>>(p); break;
    case PA_DTYPE_BF16: paged_decode_combine_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pa
