// Split-K paged decode with the Q.K^T and P.V contractions on the tensor pipe
// (bf16 / fp16 pools; query_len == 1 rows).
//
// Same work decomposition and data movement as the SIMT kernel in decode_splitk.cu:
// one CTA per (sequence, split) item and KV head, 4 warps, each warp owning two TMA
// pipeline stages and taking blocks w, w+4, ... of the split.  What changes is the
// math, which made the SIMT kernel issue-bound (about 1,270 warp instructions per
// 16-token block):
//
//   * The pool is described to TMA with 128-byte swizzle and 64-element boxes, so a
//     block's [16, head_dim] K (or V) tile lands as head_dim/64 swizzled 2 KB halves and
//     ldmatrix reads it without bank conflicts.
//   * S = Q K^T per block is 2 x (head_dim/16) m16n8k16 MMAs: A = the G query heads of
//     this KV head as rows (rows G..15 are zero and never stored), B = K rows via
//     ldmatrix (K is [token][dim], exactly the "col" B operand).  Q stays in registers
//     for the whole item, unscaled; the float32 scores are scaled by scale*log2(e).
//   * Online softmax on the accumulator fragments: each row's 16 scores sit in one lane
//     quad, so the row max is two shuffles; the running denominator stays per lane and
//     is summed over the quad once at the end.
//   * O += P V is head_dim/8 MMAs with P taken straight from the S fragments (rounded to
//     the pool dtype, as the reference casts probabilities to the V dtype before its
//     P.V, inference_server/core/attention.py:152) and V through ldmatrix.trans.
// About 130 warp instructions per block, so the kernel is bound by HBM, not issue.
//
// The last block of a sequence may hold fewer than 16 real tokens: their scores are
// masked to -inf and their V rows are zeroed in shared memory before the P.V MMA, so
// stale pool contents never reach the output (attention.py:147-150).
#include "kernels.h"
#include "pa_common.cuh"

namespace pa {

constexpr int kMmaBS = 16;
constexpr int kMmaWarps = 4;
constexpr int kMmaStages = 2;
constexpr int kHalfBytes = kMmaBS * 128;  // one 64-element-wide swizzled half of a tile

template <int D, int G>
struct MmaCfg {
  static constexpr int NH = D / 64;                       // swizzled halves per tile
  static constexpr int TILE_BYTES = NH * kHalfBytes;      // K or V tile of one block
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int TILES_BYTES = kMmaWarps * kMmaStages * STAGE_BYTES;
  static constexpr int BAR_BYTES = kMmaWarps * kMmaStages * 8;
  static constexpr int SMEM = TILES_BYTES + BAR_BYTES;
  static constexpr int KSTEPS = D / 16;
  static constexpr int NTO = D / 8;                       // output n-tiles
  static_assert(kMmaWarps * G * (D + 2) * 4 <= TILES_BYTES, "merge scratch aliases the stages");
};

template <typename T> struct Mma16;
template <> struct Mma16<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float& d0, float& d1, uint32_t a0, uint32_t a2, uint32_t b0,
                                             uint32_t b1) {
    float x, y;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, "
        "{%0,%1,%9,%9};"
        : "+f"(d0), "+f"(d1), "=f"(x), "=f"(y)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.f));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
};
template <> struct Mma16<__half> {
  __device__ __forceinline__ static void mma(float& d0, float& d1, uint32_t a0, uint32_t a2, uint32_t b0,
                                             uint32_t b1) {
    float x, y;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%5}, {%7,%8}, "
        "{%0,%1,%9,%9};"
        : "+f"(d0), "+f"(d1), "=f"(x), "=f"(y)
        : "r"(a0), "r"(0u), "r"(a2), "r"(b0), "r"(b1), "f"(0.f));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Byte offset of 16-byte chunk `chunk` (0..7) of token row `row` in a 128B-swizzled half.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(32 * kMmaWarps)
    paged_decode_mma_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                            const DecodeParams p) {
  using C = MmaCfg<D, G>;
  using M = Mma16<T>;
  constexpr int NH = C::NH, KSTEPS = C::KSTEPS, NTO = C::NTO;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TILES_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  // KV head fastest: the heads of one work item run side by side, so the row slices of
  // each pool block they read reach DRAM close together.
  const int4 item = p.items[blockIdx.x / p.num_kv_heads];
  const int seq = item.x, split = item.y, part = item.z, nsplit = item.w;
  if (seq < 0) return;  // padding of a bucketed (CUDA-graph) plan
  const int kvh = blockIdx.x % p.num_kv_heads;
  const int ctx = p.ctx_lens[seq];
  const int tok = p.cu_q[seq];
  const int b0 = split * p.split_blocks;
  const int nb = min(p.split_blocks, (ctx + kMmaBS - 1) / kMmaBS - b0);
  const int32_t* row = p.tables + int64_t(seq) * p.width + b0;

  uint8_t* my_stages = smem + warp * kMmaStages * C::STAGE_BYTES;
  uint64_t* my_bars = bars + warp * kMmaStages;
  const int my_n = nb > warp ? (nb - warp + kMmaWarps - 1) / kMmaWarps : 0;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kMmaStages; ++s) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto issue = [&](int i, int s) {  // lane 0: local block i of this warp into stage s
    int phys = row[warp + kMmaWarps * i];
    if (phys < 0 || phys >= p.pool_blocks) {  // the host planner rejects these
      set_error(p.err, kErrBlockId);
      phys = 0;
    }
    uint8_t* st = my_stages + s * C::STAGE_BYTES;
    mbar_arrive_expect_tx(&my_bars[s], C::STAGE_BYTES);
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      tma_load_3d(st + h * kHalfBytes, &tk, 64 * h, kvh, phys * kMmaBS, &my_bars[s]);
      tma_load_3d(st + C::TILE_BYTES + h * kHalfBytes, &tv, 64 * h, kvh, phys * kMmaBS, &my_bars[s]);
    }
  };
  if (lane == 0) {
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
#pragma unroll
    for (int s = 0; s < kMmaStages; ++s)
      if (s < my_n) issue(s, s);
  }

  // Q as MMA A fragments (row g = query head kvh*G + g; rows >= G stay zero).
  uint32_t qa[KSTEPS][2];
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk) qa[kk][0] = qa[kk][1] = 0u;
  if (g < G) {
    const T* qr = static_cast<const T*>(p.q) + int64_t(tok) * p.q_st + int64_t(kvh * G + g) * p.q_sh + 2 * tig;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      qa[kk][0] = *reinterpret_cast<const uint32_t*>(qr + 16 * kk);
      qa[kk][1] = *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8);
    }
  }

  float o[NTO][2];
#pragma unroll
  for (int j = 0; j < NTO; ++j) o[j][0] = o[j][1] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  // ldmatrix lane roles: matrix mi = lane / 8, row ri = lane % 8.
  const int mi = lane >> 3, ri = lane & 7;

  for (int i = 0; i < my_n; ++i) {
    const int s = i % kMmaStages;
    if (!mbar_wait(&my_bars[s], (i / kMmaStages) & 1)) {
      if (lane == 0) set_error(p.err, kErrWaitTimeout);
      break;
    }
    uint8_t* st = my_stages + s * C::STAGE_BYTES;
    const uint32_t kb = smem_u32(st), vb = smem_u32(st + C::TILE_BYTES);
    const int nvalid = min(kMmaBS, ctx - (b0 + warp + kMmaWarps * i) * kMmaBS);
    if (nvalid < kMmaBS) {  // zero the V rows past the context (last block only)
#pragma unroll
      for (int c = lane; c < kMmaBS * 8 * NH; c += 32) {
        const int r = (c >> 3) & (kMmaBS - 1), h = c >> 7;
        if (r >= nvalid) *reinterpret_cast<uint4*>(st + C::TILE_BYTES + h * kHalfBytes + r * 128 + (c & 7) * 16) =
            make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }

    // ---- S = Q K^T: two n-tiles of 8 tokens
    float sc[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float d0 = 0.f, d1 = 0.f;
      const int trow = nt * 8 + ri;  // token row this lane addresses
#pragma unroll
      for (int kk = 0; kk < KSTEPS; kk += 2) {
        // matrices: (kk, lo), (kk, hi), (kk+1, lo), (kk+1, hi) -> 16-byte chunks 2kk'..2kk'+3 of a half
        const int h = kk / 4, c0 = 2 * (kk % 4) + mi;
        uint32_t b0r, b1r, b2r, b3r;
        ldsm_x4(kb + h * kHalfBytes + sw128(trow, c0), b0r, b1r, b2r, b3r);
        M::mma(d0, d1, qa[kk][0], qa[kk][1], b0r, b1r);
        M::mma(d0, d1, qa[kk + 1][0], qa[kk + 1][1], b2r, b3r);
      }
      sc[nt][0] = d0;
      sc[nt][1] = d1;
    }

    // ---- online softmax on row g (tokens 8nt + 2tig + e)
    float bm = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tig + e;
        sc[nt][e] = t < nvalid ? sc[nt][e] * p.qscale : -INFINITY;
        bm = fmaxf(bm, sc[nt][e]);
      }
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    const float m_new = fmaxf(m_run, bm);
    const float alpha = exp2f(m_run - m_new);
    float pr[2][2], ps = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pr[nt][e] = exp2f(sc[nt][e] - m_new);
        ps += pr[nt][e];
      }
    l_run = l_run * alpha + ps;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < NTO; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
    }
    const uint32_t pa0 = M::pack(pr[0][0], pr[0][1]);  // P[g][2tig..2tig+1]
    const uint32_t pa1 = M::pack(pr[1][0], pr[1][1]);  // P[g][8+2tig..]

    // ---- O += P V: V^T fragments through ldmatrix.trans, two dim tiles per load
#pragma unroll
    for (int j = 0; j < NTO; j += 2) {
      const int chunk = j + (mi >> 1);          // 8-dim chunk 0..D/8-1
      const int trow = (mi & 1) * 8 + ri;       // token row
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(vb + (chunk >> 3) * kHalfBytes + sw128(trow, chunk & 7), v0, v1, v2, v3);
      M::mma(o[j][0], o[j][1], pa0, pa1, v0, v1);
      M::mma(o[j + 1][0], o[j + 1][1], pa0, pa1, v2, v3);
    }
    __syncwarp();  // stage s fully consumed
    if (lane == 0 && i + kMmaStages < my_n) {
      fence_proxy_async_smem();
      issue(i + kMmaStages, s);
    }
  }

  // ---- merge the 4 warps (scratch aliases the stages, now idle)
  float l_q = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_q += __shfl_xor_sync(0xffffffffu, l_q, 2);
  __syncthreads();
  float* mrg = reinterpret_cast<float*>(smem);
  float* mrg_ml = mrg + kMmaWarps * G * D;
  if (g < G) {
#pragma unroll
    for (int j = 0; j < NTO; ++j) {
      mrg[(warp * G + g) * D + 8 * j + 2 * tig + 0] = o[j][0];
      mrg[(warp * G + g) * D + 8 * j + 2 * tig + 1] = o[j][1];
    }
    if (tig == 0) {
      mrg_ml[(warp * G + g) * 2 + 0] = m_run;
      mrg_ml[(warp * G + g) * 2 + 1] = l_q;
    }
  }
  __syncthreads();

  const int head0 = kvh * G;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int h = e / D, d = e - h * D;
    float Mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) Mx = fmaxf(Mx, mrg_ml[(w * G + h) * 2]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kMmaWarps; ++w) {
      const float sw = exp2f(mrg_ml[(w * G + h) * 2] - Mx);
      L += mrg_ml[(w * G + h) * 2 + 1] * sw;
      O += mrg[(w * G + h) * D + d] * sw;
    }
    if (nsplit == 1) {
      T* out = static_cast<T*>(p.out) + int64_t(tok) * p.o_st + int64_t(head0 + h) * p.o_sh;
      out[d] = from_float<T>(O / L);
    } else {
      const int64_t ph = int64_t(part) * p.num_heads + head0 + h;
      p.part_o[ph * D + d] = O;
      if (d == 0) p.part_ml[ph] = make_float2(Mx, L);
    }
  }
}

// ------------------------------------------------------------------ dispatch
template <typename T, int D, int G>
static cudaError_t launch_mma_one(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                                  cudaStream_t stream) {
  using C = MmaCfg<D, G>;
  auto kern = paged_decode_mma_kernel<T, D, G>;
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
  dim3 grid(p.num_items * p.num_kv_heads), block(32 * kMmaWarps);
  kern<<<grid, block, C::SMEM, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t mma_by_group(int group, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                                cudaStream_t s) {
  switch (group) {
    case 1: return launch_mma_one<T, D, 1>(tk, tv, p, s);
    case 2: return launch_mma_one<T, D, 2>(tk, tv, p, s);
    case 4: return launch_mma_one<T, D, 4>(tk, tv, p, s);
    case 8: return launch_mma_one<T, D, 8>(tk, tv, p, s);
    default: return cudaErrorInvalidValue;
  }
}

bool decode_mma_supported(int dtype, int head_dim, int group, int block_size) {
  const bool g = group == 1 || group == 2 || group == 4 || group == 8;
  return (dtype == PA_DTYPE_BF16 || dtype == PA_DTYPE_F16) && g && (head_dim == 64 || head_dim == 128) &&
         block_size == kMmaBS;
}

cudaError_t launch_decode_mma(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                              const DecodeParams& p, cudaStream_t stream) {
  if (p.num_items == 0) return cudaSuccess;
  if (dtype == PA_DTYPE_BF16)
    return head_dim == 64 ? mma_by_group<__nv_bfloat16, 64>(group, tk, tv, p, stream)
                          : mma_by_group<__nv_bfloat16, 128>(group, tk, tv, p, stream);
  if (dtype == PA_DTYPE_F16)
    return head_dim == 64 ? mma_by_group<__half, 64>(group, tk, tv, p, stream)
                          : mma_by_group<__half, 128>(group, tk, tv, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
