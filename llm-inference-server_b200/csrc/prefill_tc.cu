// Varlen paged prefill on the 5th-generation tensor cores (tcgen05), bf16 / fp16.
//
// Semantics are the reference's ragged loop (inference_server/core/attention.py:156-187):
// query token t of sequence i sits at q_pos = ctx_i - q_i + t and attends to keys
// 0..q_pos, read through the block table; prefill (q_i == ctx_i), prefix-cache hits
// (q_i < ctx_i) and recompute all take this path.
//
// Work: one CTA per (prefill tile, KV head).  A tile is 128 // G consecutive query
// tokens of one sequence; its 128 rows are the (token, query head) pairs of those tokens
// and the G = Hq / Hkv query heads sharing the KV head (row r = token r / G, head r % G),
// so every K/V byte a CTA loads serves all G heads.  KV is walked in tiles of 64 keys
// (4 pool blocks) up to the causal limit of the tile's last token.  Q lives in TMEM (the
// A operand of S = Q.K^T comes straight from tensor memory), so shared memory holds only
// P and 3-deep K and V rings: 112 KB of shared memory and 256 TMEM columns at head_dim
// 128 let two CTAs share an SM, so one CTA's softmax and latencies overlap the other's
// MMAs.
//
// Roles (192 threads):
//   warps 0-3  one thread per row: write Q into TMEM (overlapping the first K/V loads),
//              softmax, O rescale, epilogue.  Row r lives in TMEM lane r, so row max and row sum
//              are thread-local.
//   warp 4     TMA producer: per KV tile, 4 blocks x (head_dim/64) boxes of K and of V
//              (128-byte swizzle) into 3-stage rings, one box per lane so a single warp
//              instruction issues a tile's copies; block ids come from the table, read 8
//              tiles at a time one group ahead of use.
//   warp 5     allocates TMEM (S: 64 columns, O: head_dim columns, Q: head_dim / 2
//              columns of packed pairs) and issues MMAs:
//              S = Q.K^T (M=128, N=64, K=16 per instruction; Q K-major from TMEM, K
//              K-major from shared memory) and
//              O += P.V (M=128, N=head_dim; P K-major from shared memory, V MN-major).
// Per KV tile j: TMA(K_j,V_j) -> MMA S_j -> softmax j reads S (s_consumed) while MMA
// may already start S_{j+1} -> softmax waits PV_{j-1}, writes P_j (bf16/fp16, swizzled)
// and rescales O in TMEM by exp2(m_old - m_new) (skipped when no row maximum of the warp
// moved) -> MMA PV_j.  Scores, softmax and the
// O accumulator are float32; P is rounded to the pool dtype as the reference rounds its
// probabilities to the V dtype before P.V (attention.py:184-185).
//
// Keys past the context in the last KV tile are masked to -inf and their V rows zeroed
// before the P.V MMA (blocks past the sequence's last block are not loaded at all).
// Every mbarrier wait is bounded; the TMEM allocation is released on every path.
#include "kernels.h"
#include "pa_common.cuh"
#include "tc_common.cuh"
#include "tc_softmax.cuh"

namespace pa {

constexpr int kPfRows = 128;
constexpr int kPfKeys = 64;
constexpr int kPfBlocks = kPfKeys / 16;
constexpr int kPfStages = 3;
constexpr int kPfThreads = 192;
constexpr int kPfSwHalf = kPfRows * 128;  // one 64-element-wide swizzled column half of a 128-row tile
constexpr int kPfKvHalf = kPfKeys * 128;  // the same for a 64-key K or V tile
constexpr float kLazyRescale = 8.f;        // raise the running row max only past 2^8 headroom

template <int D>
struct PfCfg {
  static constexpr int NH = D / 64;
  static constexpr int P_BYTES = kPfSwHalf;          // 128 rows x 64 keys
  static constexpr int K_BYTES = NH * kPfKvHalf;
  static constexpr int STAGE = 2 * K_BYTES;          // K tile then V tile
  static constexpr int OFF_P = 0;
  static constexpr int OFF_ST = OFF_P + P_BYTES;
  static constexpr int OFF_BAR = OFF_ST + kPfStages * STAGE;
  static constexpr int SMEM = OFF_BAR + 256;
  static constexpr uint32_t TMEM_COLS = 256;         // S (64), O (D), Q (D / 2)
  static_assert(kPfKeys + D + D / 2 <= 256, "TMEM budget");
};

struct PfBars {
  uint64_t k_full[kPfStages], k_empty[kPfStages];  // K ring: freed once S = Q.K^T retires
  uint64_t v_full[kPfStages], v_empty[kPfStages];  // V ring: freed once O += P.V retires
  uint64_t q_full, s_full, s_consumed, p_ready, pv_done;
  uint32_t tmem_base;
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(kPfThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                            const PrefillParams p) {
  using C = PfCfg<D>;
  constexpr int NH = C::NH;
  constexpr int TQ = kPfRows / G;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sP = smem + C::OFF_P;
  uint8_t* sST = smem + C::OFF_ST;
  PfBars* bars = reinterpret_cast<PfBars*>(smem + C::OFF_BAR);
  static_assert(sizeof(PfBars) <= 256, "barrier area");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 tile = p.tiles[blockIdx.x];
  const int seq = tile.x, t0 = tile.y;
  const int kvh = blockIdx.y;
  const int ctx = p.ctx_lens[seq], ql = p.query_lens[seq], tokbase = p.cu_q[seq];
  const int ntok = min(TQ, ql - t0);                  // valid query tokens in this tile
  const int n_keys = ctx - ql + t0 + ntok;            // causal limit of the last token + 1
  const int nkv = (n_keys + kPfKeys - 1) / kPfKeys;   // KV tiles to walk
  const int nblk_seq = (ctx + 15) / 16;
  const int32_t* trow = p.tables + int64_t(seq) * p.width;

  // Row of this thread (softmax warps): token t = r / G, query head kvh*G + r % G.
  const int r = tid;
  const int t_row = r / G, g_row = r % G;
  const bool row_valid = tid < kPfRows && t_row < ntok;
  const int t_eff = min(t_row, ntok - 1);
  const int qpos = ctx - ql + t0 + t_eff;

  // Softmax threads start their Q row loads before the setup barrier.  Rows past the
  // tile's tokens repeat its last token (finite scores; their outputs are never stored).
  uint32_t qw[D / 2];
  if (warp < 4) {
    const T* src = static_cast<const T*>(p.q) + int64_t(tokbase + t0 + t_eff) * p.q_st +
                   int64_t(kvh * G + g_row) * p.q_sh;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * c);
      qw[4 * c + 0] = v.x;
      qw[4 * c + 1] = v.y;
      qw[4 * c + 2] = v.z;
      qw[4 * c + 3] = v.w;
    }
  }
  // Producer warp: block ids of 8 KV tiles (32 blocks) per coalesced warp load, each group
  // read one group ahead of use.
  int ids_cur = 0, ids_nxt = 0;
  if (warp == 4) {
    ids_cur = lane < nblk_seq ? trow[lane] : 0;
    ids_nxt = 32 + lane < nblk_seq ? trow[32 + lane] : 0;
  }

  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->q_full, 128);
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->s_consumed, 128);
    mbar_init(&bars->p_ready, 128);
    mbar_init(&bars->pv_done, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t tS = tbase, tO = tbase + kPfKeys, tQ = tbase + kPfKeys + D;
  bool ok = true;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    // The whole warp walks the tiles.  Lane l < 4 * (head_dim / 64) owns box l of each K
    // and V tile (pool block l / NH, 64-column half l % NH), so one warp instruction issues
    // all of a tile's copies; block ids are shuffled out of the group registers.
    if (lane == 0) {
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
    }
    const int my_b = lane / NH, my_h = lane % NH;
    bool pok = true;
    for (int j = 0; j < nkv && pok; ++j) {
      const int s = j % kPfStages;
      const int b0 = j * kPfBlocks;
      const int nload = min(kPfBlocks, nblk_seq - b0);
      uint8_t* kst = sST + s * C::STAGE;
      uint8_t* vst = kst + C::K_BYTES;
      if (j > 0 && (j & 7) == 0) {
        ids_cur = ids_nxt;
        ids_nxt = b0 + 32 + lane < nblk_seq ? trow[b0 + 32 + lane] : 0;
      }
      const bool mine = lane < nload * NH;
      int phys = __shfl_sync(0xffffffffu, ids_cur, (j & 7) * kPfBlocks + (my_b & (kPfBlocks - 1)));
      if (mine && (phys < 0 || phys >= p.pool_blocks)) {  // the host planner rejects these
        set_error(p.err, kErrBlockId);
        phys = 0;
      }
      const uint32_t bytes = uint32_t(nload * NH * 2048);
      if (j >= kPfStages) pok = __all_sync(0xffffffffu, mbar_wait(&bars->k_empty[s], ((j / kPfStages) - 1) & 1));
      if (!pok) break;
      if (lane == 0) mbar_arrive_expect_tx(&bars->k_full[s], bytes);
      __syncwarp();
      if (mine) tma_load_3d(kst + my_h * kPfKvHalf + my_b * 2048, &tk, 64 * my_h, kvh, phys * 16, &bars->k_full[s]);
      if (j >= kPfStages) pok = __all_sync(0xffffffffu, mbar_wait(&bars->v_empty[s], ((j / kPfStages) - 1) & 1));
      if (!pok) break;
      if (lane == 0) mbar_arrive_expect_tx(&bars->v_full[s], bytes);
      __syncwarp();
      if (mine) tma_load_3d(vst + my_h * kPfKvHalf + my_b * 2048, &tv, 64 * my_h, kvh, phys * 16, &bars->v_full[s]);
    }
    if (!pok && lane == 0) set_error(p.err, kErrWaitTimeout);
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16<T>(kPfRows, kPfKeys, false);
      constexpr uint32_t idO = idesc_f16<T>(kPfRows, D, true);
      const uint32_t p0 = smem_u32(sP);
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(&bars->p_ready, i & 1) || !mbar_wait(&bars->v_full[i % kPfStages], (i / kPfStages) & 1))
          return false;
        tc_fence_after();
        const uint32_t v0 = smem_u32(sST + (i % kPfStages) * C::STAGE + C::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < kPfKeys / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(p0 + kk * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(v0 + kk * 2048, kPfKvHalf, 1024);
          umma_f16(tO, a, b, idO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done);
        umma_commit(&bars->v_empty[i % kPfStages]);
        return true;
      };
      if (!mbar_wait(&bars->q_full, 0)) {
        set_error(p.err, kErrWaitTimeout);
        ok = false;
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % kPfStages;
        if (!mbar_wait(&bars->k_full[s], (j / kPfStages) & 1) ||
            (j > 0 && !mbar_wait(&bars->s_consumed, (j - 1) & 1))) {
          set_error(p.err, kErrWaitTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k0 = smem_u32(sST + s * C::STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t b = smem_desc_sw128(k0 + (kk >> 2) * kPfKvHalf + (kk & 3) * 32, 16, 1024);
          umma_f16_ts(tS, tQ + 8 * kk, b, idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full);
        umma_commit(&bars->k_empty[s]);
        if (j > 0 && !issue_pv(j - 1)) {
          set_error(p.err, kErrWaitTimeout);
          ok = false;
          break;
        }
      }
      if (ok && !issue_pv(nkv - 1)) set_error(p.err, kErrWaitTimeout);
    }
  } else {
    // ------------------------------------------------------------ softmax (one row per thread)
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    {  // Q row -> TMEM lane r while the first K/V tiles load
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        tmem_st32(tQ + lane_base + 32 * c, *reinterpret_cast<const uint32_t(*)[32]>(&qw[32 * c]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->q_full);
    }
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full, j & 1));  // reconverge before .sync.aligned
      if (!ok) {
        if (lane == 0) set_error(p.err, kErrWaitTimeout);
        break;
      }
      tc_fence_after();
      uint32_t sr[kPfKeys];
      tmem_ld32_at<0>(tS + lane_base + 0, sr);
      tmem_ld32_at<32>(tS + lane_base + 32, sr);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars->s_consumed);

      // Last KV tile: zero the V rows past the context (and the blocks never loaded).
      const int kbase = j * kPfKeys;
      if (ctx - kbase < kPfKeys) {
        const int s = j % kPfStages;
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->v_full[s], (j / kPfStages) & 1));
        if (!ok) {
          if (lane == 0) set_error(p.err, kErrWaitTimeout);
          break;
        }
        uint8_t* vst = sST + s * C::STAGE + C::K_BYTES;
        const int first = ctx - kbase;
        for (int c = tid; c < (kPfKeys - first) * NH * 8; c += 128) {
          const int row = first + c / (NH * 8), rest = c % (NH * 8);
          *reinterpret_cast<uint4*>(vst + (rest >> 3) * kPfKvHalf + row * 128 + (rest & 7) * 16) =
              make_uint4(0, 0, 0, 0);
        }
      }

      const int lim = qpos - kbase;  // key column c is visible iff c <= lim
      // Four independent max / sum chains instead of one 64-long dependency chain.
      // Row maximum with three-input max (two scores per instruction, four chains).
      if (__any_sync(0xffffffffu, lim < kPfKeys - 1)) {  // the tile crosses the causal diagonal
#pragma unroll
        for (int c = 0; c < kPfKeys; ++c) sr[c] = c <= lim ? sr[c] : __float_as_uint(-INFINITY);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kPfKeys; c += 2)
        mx4[(c >> 1) & 3] = fmax3(mx4[(c >> 1) & 3], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      const float mx = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]);
      // Scores are raw q.k here; the softmax scale (> 0) is folded into the exponent.  The
      // subtracted maximum is only raised when the tile's maximum exceeds it by more than
      // kLazyRescale (log2 units): softmax is unchanged by the choice of that constant as
      // long as O and l share it, probabilities stay <= 2^kLazyRescale, and most tiles
      // then skip the rescale of O in TMEM.
      const float mx_s = mx * p.qscale;
      const bool grow = mx_s > m_run + kLazyRescale;
      const float m_new = grow ? mx_s : m_run;
      const float alpha = grow ? ex2(m_run - m_new) : 1.f;
      // Exponent arguments and the row sum on packed float pairs (one f32x2 FMA / add per
      // two scores; the same per-element rounding as scalar FMA / add).
      const uint64_t sc2 = f2pack(p.qscale, p.qscale), mn2 = f2pack(-m_new, -m_new);
      uint64_t rs2[2] = {0ull, 0ull};
      uint32_t pk[kPfKeys / 2];
#pragma unroll
      for (int c = 0; c < kPfKeys; c += 2) {
        float x0, x1;
        f2unpack(fma2(f2pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, mn2), x0, x1);
        const float e0 = ex2(x0), e1 = ex2(x1);
        rs2[(c >> 1) & 1] = add2(rs2[(c >> 1) & 1], f2pack(e0, e1));
        pk[c / 2] = pack2<T>(e0, e1);
      }
      float r0, r1, r2, r3;
      f2unpack(rs2[0], r0, r1);
      f2unpack(rs2[1], r2, r3);
      const float rs = (r0 + r1) + (r2 + r3);
      l_run = l_run * alpha + rs;
      m_run = m_new;

      if (j > 0) {  // PV_{j-1} must be done before P is overwritten and O rescaled
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (j - 1) & 1));
        if (!ok) {
          if (lane == 0) set_error(p.err, kErrWaitTimeout);
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < kPfKeys / 8; ++c)
        *reinterpret_cast<uint4*>(sP + sw_off(r, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {  // 64 columns per TMEM round trip
          uint32_t o[64];
          tmem_ld32_at<0>(tO + lane_base + 64 * c, o);
          tmem_ld32_at<32>(tO + lane_base + 64 * c + 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 64; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tO + lane_base + 64 * c, *reinterpret_cast<const uint32_t(*)[32]>(&o[0]));
          tmem_st32(tO + lane_base + 64 * c + 32, *reinterpret_cast<const uint32_t(*)[32]>(&o[32]));
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->p_ready);
    }
    // ---- epilogue: O / l -> out
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done, (nkv - 1) & 1));
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      T* dst = static_cast<T*>(p.out) + int64_t(tokbase + t0 + t_eff) * p.o_st + int64_t(kvh * G + g_row) * p.o_sh;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {  // 64 columns per TMEM round trip
        uint32_t o[64];
        tmem_ld32_at<0>(tO + lane_base + 64 * c, o);
        tmem_ld32_at<32>(tO + lane_base + 64 * c + 32, o);
        tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int e = 0; e < 64; e += 8) {
            uint4 w;
            w.x = pack2<T>(__uint_as_float(o[e + 0]) * inv, __uint_as_float(o[e + 1]) * inv);
            w.y = pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            w.z = pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            w.w = pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 64 * c + e) = w;
          }
        }
      }
    } else if (lane == 0) {
      set_error(p.err, kErrWaitTimeout);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ dispatch
template <typename T, int D, int G>
static cudaError_t launch_pf_one(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p,
                                 cudaStream_t stream) {
  using C = PfCfg<D>;
  auto kern = paged_prefill_tc_kernel<T, D, G>;
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
  dim3 grid(p.num_tiles, p.num_kv_heads), block(kPfThreads);
  kern<<<grid, block, C::SMEM, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t pf_by_group(int group, const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p,
                               cudaStream_t s) {
  switch (group) {
    case 1: return launch_pf_one<T, D, 1>(tk, tv, p, s);
    case 2: return launch_pf_one<T, D, 2>(tk, tv, p, s);
    case 4: return launch_pf_one<T, D, 4>(tk, tv, p, s);
    case 8: return launch_pf_one<T, D, 8>(tk, tv, p, s);
    default: return cudaErrorInvalidValue;
  }
}

bool prefill_tc_supported(int dtype, int head_dim, int group, int block_size) {
  const bool g = group == 1 || group == 2 || group == 4 || group == 8;
  return (dtype == PA_DTYPE_BF16 || dtype == PA_DTYPE_F16) && g && (head_dim == 64 || head_dim == 128) &&
         block_size == 16;
}

int prefill_tile_rows() { return kPfRows; }

cudaError_t launch_prefill_tc(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                              const PrefillParams& p, cudaStream_t stream) {
  if (p.num_tiles == 0) return cudaSuccess;
  if (dtype == PA_DTYPE_BF16)
    return head_dim == 64 ? pf_by_group<__nv_bfloat16, 64>(group, tk, tv, p, stream)
                          : pf_by_group<__nv_bfloat16, 128>(group, tk, tv, p, stream);
  if (dtype == PA_DTYPE_F16)
    return head_dim == 64 ? pf_by_group<__half, 64>(group, tk, tv, p, stream)
                          : pf_by_group<__half, 128>(group, tk, tv, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
