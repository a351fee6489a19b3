// Varlen paged prefill on CTA pairs (tcgen05 cta_group::2), bf16 / fp16, head_dim 128.
//
// Semantics are the reference's ragged loop (inference_server/core/attention.py:156-187):
// query token t of sequence i sits at q_pos = ctx_i - q_i + t and attends to keys
// 0..q_pos, read through the block table; keys past ctx_i are never part of the result
// (the reference slices them off, :171-172).
//
// Why pairs.  A 128-row tile holds only 128 / G query tokens (32 at the Llama-8B shape),
// so every K/V tile a sequence has is streamed into an SM once per 32 query tokens: on a
// 2,048-token prompt that is 64 re-reads of the whole prefix, and per-SM K/V delivery
// (16-row boxes from L2) bounded the single-CTA kernel.  Here two CTAs on the two SMs of
// a cluster run ONE M = 256 MMA per step: each CTA holds its own 128 rows (Q in its TMEM,
// P in its shared memory, S and O in its TMEM) and only HALF of every K/V tile — the
// MMA reads the B operand from both CTAs' shared memory (N / 2 columns each).  K/V bytes
// per SM per FLOP halve, the K/V re-reads halve, and each SM still holds two independent
// CTAs (two pairs), so one CTA's softmax overlaps the other's MMAs.  No load uses
// multicast: every CTA loads its own half from this GPU's pool.
//
// Work: one cluster per (pair tile, KV head).  A pair tile is 256 / G consecutive query
// tokens of one sequence; CTA rank r takes tokens [t0 + r*128/G, t0 + (r+1)*128/G), its
// row x = (token, head) with token x / G and query head kvh*G + x % G.  KV is walked in
// tiles of 64 keys (4 pool blocks) up to the causal limit of the pair's last token.
//   K tile (S = Q.K^T, N = 64 keys): CTA r loads keys [32r, 32r + 32) (2 blocks, both
//     64-column halves of head_dim), K-major, 128-byte swizzle.
//   V tile (O += P.V, N = head_dim 128): CTA r loads the 64-column half r of all 64 keys,
//     MN-major, 128-byte swizzle.
//
// Roles (192 threads per CTA):
//   warps 0-3  one thread per row: Q into TMEM, softmax, O rescale, epilogue (as in the
//              single-CTA kernel); their arrivals for the MMA go to the leader CTA.
//   warp 4     TMA producer: 8 boxes of 2 KB per tile (4 of K, 4 of V), completion
//              counted on the LEADER's full barriers (cta_group::2 loads).  The tile holding
//              the sequence's partial last block lands on a local barrier instead; the
//              producer zeroes that block's V rows past the context (stale pool data, which
//              the probabilities' zeros would otherwise multiply) before it arrives.
//   warp 5     both CTAs allocate TMEM together (cta_group::2); in the leader (rank 0)
//              lane 0 issues every MMA for the pair and commits them to both CTAs'
//              barriers (multicast commit).
// Every mbarrier wait is bounded; both CTAs meet at a cluster barrier before TMEM is freed
// and before either exits, so no CTA's shared memory or TMEM is released while its peer
// or the pair's MMAs may still use it.
#include "kernels.h"
#include "pa_common.cuh"
#include "tc_common.cuh"
#include "tc_pair.cuh"

namespace pa {

constexpr int kPrRows = 128;                 // rows per CTA; a pair covers 256
constexpr int kPrKeys = 64;                  // keys per KV tile
constexpr int kPrBlocks = kPrKeys / 16;
constexpr int kPrD = 128;
constexpr int kPrKStages = 5;
constexpr int kPrVStages = 5;
constexpr int kPrThreads = 192;
constexpr int kPrKHalf = 32 * 128;           // 32 keys x one 64-column half (128-byte rows)
constexpr int kPrKBytes = 2 * kPrKHalf;      // this CTA's half of a K tile
constexpr int kPrVBytes = kPrKeys * 128;     // all 64 keys x this CTA's 64-column half of V
constexpr int kPrPBytes = kPrRows * 128;     // 128 rows x 64 keys, 16-bit
constexpr int kPrOffP = 0;
constexpr int kPrOffK = kPrOffP + kPrPBytes;
constexpr int kPrOffV = kPrOffK + kPrKStages * kPrKBytes;
constexpr int kPrOffBar = kPrOffV + kPrVStages * kPrVBytes;
constexpr int kPrSmem = kPrOffBar + 256;
constexpr uint32_t kPrTmemCols = 256;        // S (64), O (128), Q (64 packed pairs)
constexpr float kPrLazyRescale = 8.f;

struct PrBars {
  uint64_t k_full[kPrKStages], k_empty[kPrKStages];
  uint64_t v_full[kPrVStages], v_empty[kPrVStages];
  uint64_t q_full, s_full, s_consumed, p_ready, pv_done, v_tail;
  uint32_t tmem_base;
};

__device__ __forceinline__ float pr_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <typename T>
__device__ __forceinline__ uint32_t pr_pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pr_pack2<__nv_bfloat16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <>
__device__ __forceinline__ uint32_t pr_pack2<__half>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T, int G>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPrThreads, 2)
    paged_prefill_pair_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                              const PrefillParams p) {
  constexpr int TQ = kPrRows / G;  // query tokens per CTA
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sP = smem + kPrOffP;
  uint8_t* sK = smem + kPrOffK;
  uint8_t* sV = smem + kPrOffV;
  PrBars* bars = reinterpret_cast<PrBars*>(smem + kPrOffBar);
  static_assert(sizeof(PrBars) <= 256, "barrier area");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int2 tile = p.tiles[blockIdx.x >> 1];
  const int seq = tile.x, t0 = tile.y;
  const int kvh = blockIdx.y;
  const int ctx = p.ctx_lens[seq], ql = p.query_lens[seq], tokbase = p.cu_q[seq];
  const int ntok_pair = min(2 * TQ, ql - t0);          // valid query tokens of the pair
  const int ntok = max(0, min(TQ, ntok_pair - int(rank) * TQ));  // ... of this CTA
  const int n_keys = ctx - ql + t0 + ntok_pair;        // causal limit of the pair's last token + 1
  const int nkv = (n_keys + kPrKeys - 1) / kPrKeys;
  const int nblk_seq = (ctx + 15) / 16;
  const int32_t* trow = p.tables + int64_t(seq) * p.width;

  // Row of this thread (softmax warps).  Rows past the CTA's tokens repeat the pair's last
  // token (finite scores; their outputs are never stored).
  const int t_row = tid / G, g_row = tid % G;
  const bool row_valid = tid < kPrRows && t_row < ntok;
  const int t_eff = min(int(rank) * TQ + t_row, ntok_pair - 1);  // token index within the pair
  const int qpos = ctx - ql + t0 + t_eff;

  uint32_t qw[kPrD / 2];
  if (warp < 4) {
    const T* src = static_cast<const T*>(p.q) + int64_t(tokbase + t0 + t_eff) * p.q_st +
                   int64_t(kvh * G + g_row) * p.q_sh;
#pragma unroll
    for (int c = 0; c < kPrD / 8; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * c);
      qw[4 * c + 0] = v.x;
      qw[4 * c + 1] = v.y;
      qw[4 * c + 2] = v.z;
      qw[4 * c + 3] = v.w;
    }
  }
  int ids_cur = 0, ids_nxt = 0;
  if (warp == 4) {
    ids_cur = lane < nblk_seq ? trow[lane] : 0;
    ids_nxt = 32 + lane < nblk_seq ? trow[32 + lane] : 0;
  }

  if (warp == 5) {
    tmem_alloc_pair(&bars->tmem_base, kPrTmemCols);
    tmem_relinquish_pair();
  }
  if (tid == 0) {
    for (int s = 0; s < kPrKStages; ++s) {
      mbar_init(&bars->k_full[s], 2);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < kPrVStages; ++s) {
      mbar_init(&bars->v_full[s], 2);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->q_full, 8);        // one arrival per softmax warp of both CTAs
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->s_consumed, 8);
    mbar_init(&bars->p_ready, 8);
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->v_tail, 1);
    fence_mbar_init();
  }
  // Both CTAs' barriers and TMEM exist before any cross-CTA arrival, load or MMA.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t tS = tbase, tO = tbase + kPrKeys, tQ = tbase + kPrKeys + kPrD;
  // Leader-CTA addresses of the barriers the MMA issuer waits on, and arrivals on them (a
  // local arrive in the leader, a remote one in the peer).
  auto leader_bar = [&](uint64_t* b) { return mapa_rank(smem_u32(b), 0); };
  auto arrive_leader = [&](uint64_t* b) {
    if (leader)
      mbar_arrive(b);
    else
      mbar_arrive_remote(leader_bar(b));
  };
  auto arrive_expect_leader = [&](uint64_t* b, uint32_t bytes) {
    if (leader)
      mbar_arrive_expect_tx(b, bytes);
    else
      mbar_arrive_expect_tx_remote(leader_bar(b), bytes);
  };
  bool ok = true;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
    }
    // Lane l < 4: K box (block 2*rank + l/2 of the tile, column half l%2) and V box (block
    // l of the tile, column half `rank`).
    const int kb = 2 * int(rank) + (lane >> 1), kh = lane & 1;
    const int tail_tile = (ctx % 16) ? (nblk_seq - 1) / kPrBlocks : -1;  // tile holding a partial block
    bool pok = true;
    for (int j = 0; j < nkv && pok; ++j) {
      const int ks = j % kPrKStages, vs = j % kPrVStages;
      const int b0 = j * kPrBlocks;
      const int nload = min(kPrBlocks, nblk_seq - b0);
      if (j > 0 && (j & 7) == 0) {
        ids_cur = ids_nxt;
        ids_nxt = b0 + 32 + lane < nblk_seq ? trow[b0 + 32 + lane] : 0;
      }
      int kphys = __shfl_sync(0xffffffffu, ids_cur, (j & 7) * kPrBlocks + (kb & 3));
      int vphys = __shfl_sync(0xffffffffu, ids_cur, (j & 7) * kPrBlocks + (lane & 3));
      const bool kmine = lane < 4 && kb < nload;
      const bool vmine = lane < 4 && lane < nload;
      if ((kmine && (kphys < 0 || kphys >= p.pool_blocks)) || (vmine && (vphys < 0 || vphys >= p.pool_blocks))) {
        set_error(p.err, kErrBlockId);  // the host planner rejects these
        kphys = (kphys < 0 || kphys >= p.pool_blocks) ? 0 : kphys;
        vphys = (vphys < 0 || vphys >= p.pool_blocks) ? 0 : vphys;
      }
      // K half: this CTA's blocks of the tile.
      if (j >= kPrKStages) pok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->k_empty[ks], ((j / kPrKStages) - 1) & 1));
      if (!pok) break;
      const uint32_t kbytes = uint32_t(max(0, min(2, nload - 2 * int(rank))) * 2 * 2048);
      if (lane == 0) arrive_expect_leader(&bars->k_full[ks], kbytes);
      __syncwarp();
      if (kmine)
        tma_load_3d_pair(sK + ks * kPrKBytes + kh * kPrKHalf + (kb & 1) * 2048, &tk, 64 * kh, kvh, kphys * 16,
                         leader_bar(&bars->k_full[ks]));
      // V half: this CTA's 64 columns of every block of the tile.
      if (j >= kPrVStages) pok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->v_empty[vs], ((j / kPrVStages) - 1) & 1));
      if (!pok) break;
      uint8_t* vst = sV + vs * kPrVBytes;
      const uint32_t vbytes = uint32_t(nload * 2048);
      if (j != tail_tile) {
        if (lane == 0) arrive_expect_leader(&bars->v_full[vs], vbytes);
        __syncwarp();
        if (vmine) tma_load_3d_pair(vst + lane * 2048, &tv, 64 * int(rank), kvh, vphys * 16, leader_bar(&bars->v_full[vs]));
      } else {
        // The sequence's partial last block: land locally, zero its rows past the context,
        // then release the stage to the MMA issuer.
        if (lane == 0) mbar_arrive_expect_tx(&bars->v_tail, vbytes);
        __syncwarp();
        if (vmine) tma_load_3d(vst + lane * 2048, &tv, 64 * int(rank), kvh, vphys * 16, &bars->v_tail);
        pok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->v_tail, 0));
        if (!pok) break;
        const int first = ctx - b0 * 16;  // first stale row of the tile (inside its last block)
        for (int c = lane; c < (nload * 16 - first) * 8; c += 32) {
          const int row = first + c / 8;
          *reinterpret_cast<uint4*>(vst + row * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_leader(&bars->v_full[vs]);
      }
    }
    if (!pok && lane == 0) set_error(p.err, kErrWaitTimeout);
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t idS = idesc_f16<T>(2 * kPrRows, kPrKeys, false);
      constexpr uint32_t idO = idesc_f16<T>(2 * kPrRows, kPrD, true);
      const uint32_t p0 = smem_u32(sP);
      auto issue_pv = [&](int i) -> bool {
        const int vs = i % kPrVStages;
        if (!mbar_wait_cl(&bars->p_ready, i & 1) || !mbar_wait_cl(&bars->v_full[vs], (i / kPrVStages) & 1))
          return false;
        tc_fence_after();
        const int nl = min(kPrBlocks, nblk_seq - i * kPrBlocks);  // blocks never loaded are skipped
        const uint32_t v0 = smem_u32(sV + vs * kPrVBytes);
        for (int kk = 0; kk < nl; ++kk) {
          const uint64_t a = smem_desc_sw128(p0 + kk * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(v0 + kk * 2048, kPrVBytes, 1024);
          umma_pair_ss(tO, a, b, idO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit_pair(&bars->pv_done);
        umma_commit_pair(&bars->v_empty[vs]);
        return true;
      };
      if (!mbar_wait_cl(&bars->q_full, 0)) {
        set_error(p.err, kErrWaitTimeout);
        ok = false;
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int ks = j % kPrKStages;
        if (!mbar_wait_cl(&bars->k_full[ks], (j / kPrKStages) & 1) ||
            (j > 0 && !mbar_wait_cl(&bars->s_consumed, (j - 1) & 1))) {
          set_error(p.err, kErrWaitTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k0 = smem_u32(sK + ks * kPrKBytes);
#pragma unroll
        for (int kk = 0; kk < kPrD / 16; ++kk) {
          const uint64_t b = smem_desc_sw128(k0 + (kk >> 2) * kPrKHalf + (kk & 3) * 32, 16, 1024);
          umma_pair_ts(tS, tQ + 8 * kk, b, idS, kk > 0 ? 1u : 0u);
        }
        umma_commit_pair(&bars->s_full);
        umma_commit_pair(&bars->k_empty[ks]);
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
      for (int c = 0; c < kPrD / 64; ++c)
        tmem_st32(tQ + lane_base + 32 * c, *reinterpret_cast<const uint32_t(*)[32]>(&qw[32 * c]));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&bars->q_full);
    }
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < nkv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->s_full, j & 1));
      if (!ok) {
        if (lane == 0) set_error(p.err, kErrWaitTimeout);
        break;
      }
      tc_fence_after();
      uint32_t sr[kPrKeys];
      tmem_ld32_at<0>(tS + lane_base + 0, sr);
      tmem_ld32_at<32>(tS + lane_base + 32, sr);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&bars->s_consumed);

      const int kbase = j * kPrKeys;
      const int lim = min(qpos, ctx - 1) - kbase;  // key column c is visible iff c <= lim
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (__any_sync(0xffffffffu, lim < kPrKeys - 1)) {  // the tile crosses the causal diagonal
#pragma unroll
        for (int c = 0; c < kPrKeys; ++c) {
          const float v = c <= lim ? __uint_as_float(sr[c]) : -INFINITY;
          sr[c] = __float_as_uint(v);
          mx4[c & 3] = fmaxf(mx4[c & 3], v);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kPrKeys; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], __uint_as_float(sr[c]));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // Raw q.k scores; the softmax scale (> 0) is folded into the exponent.  The running
      // maximum is raised only when the tile's exceeds it by more than kPrLazyRescale
      // (log2 units): softmax is unchanged by that choice as long as O and l share it,
      // probabilities stay <= 2^kPrLazyRescale, and most tiles skip the O rescale.
      const float mx_s = mx * p.qscale;
      const bool grow = mx_s > m_run + kPrLazyRescale;
      const float m_new = grow ? mx_s : m_run;
      const float alpha = grow ? pr_ex2(m_run - m_new) : 1.f;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[kPrKeys / 2];
#pragma unroll
      for (int c = 0; c < kPrKeys; c += 2) {
        const float e0 = pr_ex2(fmaf(__uint_as_float(sr[c]), p.qscale, -m_new));
        const float e1 = pr_ex2(fmaf(__uint_as_float(sr[c + 1]), p.qscale, -m_new));
        rs4[(c >> 1) & 3] += e0 + e1;
        pk[c / 2] = pr_pack2<T>(e0, e1);
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l_run = l_run * alpha + rs;
      m_run = m_new;

      if (j > 0) {  // PV_{j-1} must be done before P is overwritten and O rescaled
        ok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->pv_done, (j - 1) & 1));
        if (!ok) {
          if (lane == 0) set_error(p.err, kErrWaitTimeout);
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < kPrKeys / 8; ++c)
        *reinterpret_cast<uint4*>(sP + tid * 128 + ((c ^ (tid & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int c = 0; c < kPrD / 64; ++c) {
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
      __syncwarp();
      if (lane == 0) arrive_leader(&bars->p_ready);
    }
    // ---- epilogue: O / l -> out
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait_cl(&bars->pv_done, (nkv - 1) & 1));
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      T* dst = static_cast<T*>(p.out) + int64_t(tokbase + t0 + t_eff) * p.o_st + int64_t(kvh * G + g_row) * p.o_sh;
#pragma unroll
      for (int c = 0; c < kPrD / 64; ++c) {
        uint32_t o[64];
        tmem_ld32_at<0>(tO + lane_base + 64 * c, o);
        tmem_ld32_at<32>(tO + lane_base + 64 * c + 32, o);
        tmem_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int e = 0; e < 64; e += 8) {
            uint4 w;
            w.x = pr_pack2<T>(__uint_as_float(o[e + 0]) * inv, __uint_as_float(o[e + 1]) * inv);
            w.y = pr_pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            w.z = pr_pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            w.w = pr_pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 64 * c + e) = w;
          }
        }
      }
    } else if (lane == 0) {
      set_error(p.err, kErrWaitTimeout);
    }
  }

  // Both CTAs are done with TMEM, their shared memory and each other's barriers (the MMA
  // warp's lane 0 rejoins its warp here).
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, kPrTmemCols);
  }
}

// ------------------------------------------------------------------ dispatch
template <typename T, int G>
static cudaError_t launch_pr_one(const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p,
                                 cudaStream_t stream) {
  auto kern = paged_prefill_pair_kernel<T, G>;
  int dev = 0;
  cudaGetDevice(&dev);
  static bool configured[64] = {};
  if (dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPrSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(2 * p.num_tiles, p.num_kv_heads), block(kPrThreads);
  kern<<<grid, block, kPrSmem, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

bool prefill_pair_supported(int dtype, int head_dim, int group, int block_size) {
  const bool g = group == 1 || group == 2 || group == 4 || group == 8;
  return (dtype == PA_DTYPE_BF16 || dtype == PA_DTYPE_F16) && g && head_dim == kPrD && block_size == 16;
}

int prefill_pair_tile_rows() { return 2 * kPrRows; }

cudaError_t launch_prefill_pair(int dtype, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                                const PrefillParams& p, cudaStream_t stream) {
  if (p.num_tiles == 0) return cudaSuccess;
#define PR_BY_GROUP(T)                                  \
  switch (group) {                                      \
    case 1: return launch_pr_one<T, 1>(tk, tv, p, stream); \
    case 2: return launch_pr_one<T, 2>(tk, tv, p, stream); \
    case 4: return launch_pr_one<T, 4>(tk, tv, p, stream); \
    case 8: return launch_pr_one<T, 8>(tk, tv, p, stream); \
    default: return cudaErrorInvalidValue;              \
  }
  if (dtype == PA_DTYPE_BF16) PR_BY_GROUP(__nv_bfloat16)
  if (dtype == PA_DTYPE_F16) PR_BY_GROUP(__half)
#undef PR_BY_GROUP
  return cudaErrorInvalidValue;
}

}  // namespace pa
