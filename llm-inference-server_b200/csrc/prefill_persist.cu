// Persistent varlen paged prefill on tcgen05 with the probabilities kept in tensor memory,
// bf16 / fp16, head_dim 64 or 128.
//
// Semantics are those of the single-CTA prefill kernel (prefill_tc.cu) and of the
// reference's ragged loop (inference_server/core/attention.py:156-187): query token t of
// sequence i sits at q_pos = ctx_i - q_i + t and attends to keys 0..q_pos through the
// block table; probabilities are rounded to the pool dtype before P.V as the reference
// rounds them to the V dtype (attention.py:184-185).
//
// A work item is (prefill tile, KV head) over the planner's 128-row tiles: the (token,
// query head) pairs of 128 / G consecutive tokens of one sequence and the G query heads
// sharing the KV head.  Items = tiles x Hkv with the KV head fastest, so the planner's
// heaviest-first tile order is the items' order.  The grid is two CTAs per SM; CTA b takes
// items in a snake order (round k: b, or grid-1-b, + k*grid), which hands the heaviest
// items out first and evens the rounds' sums out.  A CTA keeps its TMEM, barriers and rings
// across items, so an item costs no setup, and the next item's Q and first K tiles load
// while the current item's last tiles are in the softmax.
//
// Data movement:
//   * Q by TMA: one {64, G, 128/G} box per 64 columns of head_dim (the tile's 128 rows
//     straight from the query tensor) into shared memory, reloaded once the item's last
//     S MMA has retired.
//   * K and V by TMA, one 16-row x 128-byte box per pool block and 64-column half, into
//     separate rings (a K stage frees when its S MMA retires, a V stage when its P.V does).
//   * P goes to TMEM (two 32-column buffers of packed pairs) and O += P.V takes it as the
//     A operand from tensor memory: no shared-memory P, no proxy fence per tile, and the
//     softmax waits on P.V only to reuse a P buffer two tiles later or to rescale O.
//
// Roles (256 threads): warps 0-3 softmax, one thread per row (TMEM lane r): the scores, the
// rare O rescale, the epilogue; warp 4: producer of item metadata (a 2-slot descriptor
// ring), Q and K (3-stage ring); warp 5: TMEM allocation and the S = Q.K^T issue (SS,
// M=128, N=64); warp 6: producer of V (2-stage ring); warp 7: the O += P.V issue (TS,
// M=128, N=head_dim).  MMA issue bounds the kernel, so S and P.V go out from two threads
// (neither waits behind the other's dependencies) with two commits per tile between them:
// "S retired" (one barrier per K stage, also freeing that stage) and "P.V retired" (one
// per P buffer, also freeing the V stage of the same index).
// TMEM columns: S [0, 64), O [64, 64 + D), P buffers [64 + D, 128 + D).
//
// Every mbarrier wait is bounded; the TMEM allocation is released on every path.
#include "kernels.h"
#include "pa_common.cuh"
#include "tc_common.cuh"
#include "tc_softmax.cuh"

namespace pa {

constexpr int kPpRows = 128;
constexpr int kPpKeys = 64;
constexpr int kPpBlocks = kPpKeys / 16;
constexpr int kPpKStages = 3;
constexpr int kPpVStages = 2;  // equal to the P buffer count: one "P.V retired" barrier frees both
constexpr int kPpThreads = 256;
constexpr int kPpQHalf = kPpRows * 128;   // 128 rows x 64 elements, 128-byte swizzle
constexpr int kPpKvHalf = kPpKeys * 128;  // 64 keys x 64 elements
constexpr int kPpDescConsumers = 7;       // 4 softmax warps, S and P.V issuers, V producer
constexpr float kPpLazyRescale = 8.f;

template <int D>
struct PpCfg {
  static constexpr int NH = D / 64;
  static constexpr int Q_BYTES = NH * kPpQHalf;
  static constexpr int KV_BYTES = NH * kPpKvHalf;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + kPpKStages * KV_BYTES;
  static constexpr int OFF_DESC = OFF_V + kPpVStages * KV_BYTES;
  static constexpr int OFF_BAR = OFF_DESC + 64;
  static constexpr int SMEM = OFF_BAR + 256;
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr uint32_t COL_O = kPpKeys, COL_P = kPpKeys + D;
  static_assert(COL_P + 2 * (kPpKeys / 2) <= TMEM_COLS, "TMEM budget");
};

struct PpItem {  // one work item, written by the producer, read by the other roles
  int32_t seq, t0, kvh, ntok, ctx, ql, tokbase, nkv;
};

struct PpBars {
  // S of tile g retired: s_full[g % kPpKStages], waited on by the softmax (the scores are
  // ready) and by the K producer (K stage g % kPpKStages is free again).
  uint64_t k_full[kPpKStages], s_full[kPpKStages];
  uint64_t v_full[kPpVStages];
  uint64_t q_full, q_empty, s_consumed;
  // P buffer written / the P.V that read it retired.  V stages and P buffers are both
  // indexed by tile % 2, so p_free[s] also frees V stage s for the V producer.
  uint64_t p_full[2], p_free[2];
  uint64_t d_full[2], d_empty[2];
  uint32_t tmem_base;
};

// Item k of CTA b in the snake order; -1 past the last item.
__device__ __forceinline__ int pp_item(int k, int b, int grid, int items) {
  const int it = k * grid + ((k & 1) ? grid - 1 - b : b);
  return it < items ? it : -1;
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kPpThreads, 2)
    paged_prefill_persist_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                                 const __grid_constant__ CUtensorMap tq, const PrefillParams p) {
  using C = PpCfg<D>;
  constexpr int NH = C::NH;
  constexpr int TQ = kPpRows / G;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* sQ = smem + C::OFF_Q;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  PpItem* desc = reinterpret_cast<PpItem*>(smem + C::OFF_DESC);
  PpBars* bars = reinterpret_cast<PpBars*>(smem + C::OFF_BAR);
  static_assert(sizeof(PpBars) <= 256, "barrier area");
  static_assert(2 * sizeof(PpItem) <= 64, "descriptor area");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int items = p.num_tiles * p.num_kv_heads;
  const int grid = gridDim.x, b = blockIdx.x;

  if (warp == 5) {
    tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kPpKStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->s_full[s], 1);
    }
    for (int s = 0; s < kPpVStages; ++s) {
      mbar_init(&bars->v_full[s], 1);
    }
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    mbar_init(&bars->s_consumed, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->p_full[s], 128);
      mbar_init(&bars->p_free[s], 1);
      mbar_init(&bars->d_full[s], 1);
      mbar_init(&bars->d_empty[s], kPpDescConsumers);
    }
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t tS = tbase, tO = tbase + C::COL_O, tP = tbase + C::COL_P;

  if (warp == 4) {
    // ------------------------------------------------------------ producer: items, Q, K
    if (lane == 0) {
      prefetch_tmap(&tk);
      prefetch_tmap(&tq);
    }
    const int my_b = lane / NH, my_h = lane % NH;
    bool pok = true;
    int g = 0;  // K tiles issued so far (all items)
    int it = pp_item(0, b, grid, items);
    int2 tile = it >= 0 ? p.tiles[it / p.num_kv_heads] : make_int2(0, 0);
    for (int k = 0; it >= 0 && pok; ++k) {
      const int kvh = it % p.num_kv_heads;
      const int seq = tile.x, t0 = tile.y;
      const int ctx = p.ctx_lens[seq], ql = p.query_lens[seq], tokbase = p.cu_q[seq];
      const int ntok = min(TQ, ql - t0);
      const int nkv = (ctx - ql + t0 + ntok + kPpKeys - 1) / kPpKeys;
      const int nblk_seq = (ctx + 15) / 16;
      const int32_t* trow = p.tables + int64_t(seq) * p.width;
      int ids_cur = lane < nblk_seq ? trow[lane] : 0;
      int ids_nxt = 32 + lane < nblk_seq ? trow[32 + lane] : 0;
      const int it_next = pp_item(k + 1, b, grid, items);
      const int2 tile_next = it_next >= 0 ? p.tiles[it_next / p.num_kv_heads] : make_int2(0, 0);

      const int slot = k & 1;
      if (k >= 2) pok = __all_sync(0xffffffffu, mbar_wait(&bars->d_empty[slot], ((k >> 1) - 1) & 1));
      if (!pok) break;
      if (lane == 0) {
        PpItem d;
        d.seq = seq;
        d.t0 = t0;
        d.kvh = kvh;
        d.ntok = ntok;
        d.ctx = ctx;
        d.ql = ql;
        d.tokbase = tokbase;
        d.nkv = nkv;
        desc[slot] = d;
        mbar_arrive(&bars->d_full[slot]);
      }
      for (int j = 0; j < nkv; ++j, ++g) {
        const int s = g % kPpKStages;
        const int b0 = j * kPpBlocks;
        const int nload = min(kPpBlocks, nblk_seq - b0);
        if (j > 0 && (j & 7) == 0) {
          ids_cur = ids_nxt;
          ids_nxt = b0 + 32 + lane < nblk_seq ? trow[b0 + 32 + lane] : 0;
        }
        const bool mine = lane < nload * NH;
        int phys = __shfl_sync(0xffffffffu, ids_cur, (j & 7) * kPpBlocks + (my_b & (kPpBlocks - 1)));
        if (mine && (phys < 0 || phys >= p.pool_blocks)) {  // the host planner rejects these
          set_error(p.err, kErrBlockId);
          phys = 0;
        }
        if (g >= kPpKStages)
          pok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[s], ((g / kPpKStages) - 1) & 1));
        if (!pok) break;
        if (lane == 0) mbar_arrive_expect_tx(&bars->k_full[s], uint32_t(nload * NH * 2048));
        __syncwarp();
        if (mine)
          tma_load_3d(sK + s * C::KV_BYTES + my_h * kPpKvHalf + my_b * 2048, &tk, 64 * my_h, kvh, phys * 16,
                      &bars->k_full[s]);
        if (j == 0) {
          // Q of this item, after its first K tile (whose stage frees earlier), once the
          // previous item's last S MMA has read the buffer.
          if (k >= 1) pok = __all_sync(0xffffffffu, mbar_wait(&bars->q_empty, (k - 1) & 1));
          if (!pok) break;
          if (lane == 0) mbar_arrive_expect_tx(&bars->q_full, uint32_t(C::Q_BYTES));
          __syncwarp();
          if (lane < NH) tma_load_3d(sQ + lane * kPpQHalf, &tq, 64 * lane, kvh * G, tokbase + t0, &bars->q_full);
        }
      }
      it = it_next;
      tile = tile_next;
    }
    if (!pok && lane == 0) set_error(p.err, kErrWaitTimeout);
  } else if (warp == 6) {
    // ------------------------------------------------------------ producer: V
    if (lane == 0) prefetch_tmap(&tv);
    const int my_b = lane / NH, my_h = lane % NH;
    bool pok = true;
    int g = 0;
    for (int k = 0; pok && pp_item(k, b, grid, items) >= 0; ++k) {
      const int slot = k & 1;
      pok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[slot], (k >> 1) & 1));
      if (!pok) break;
      const PpItem d = desc[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->d_empty[slot]);
      const int nblk_seq = (d.ctx + 15) / 16;
      const int32_t* trow = p.tables + int64_t(d.seq) * p.width;
      int ids_cur = lane < nblk_seq ? trow[lane] : 0;
      int ids_nxt = 32 + lane < nblk_seq ? trow[32 + lane] : 0;
      for (int j = 0; j < d.nkv; ++j, ++g) {
        const int s = g % kPpVStages;
        const int b0 = j * kPpBlocks;
        const int nload = min(kPpBlocks, nblk_seq - b0);
        if (j > 0 && (j & 7) == 0) {
          ids_cur = ids_nxt;
          ids_nxt = b0 + 32 + lane < nblk_seq ? trow[b0 + 32 + lane] : 0;
        }
        const bool mine = lane < nload * NH;
        int phys = __shfl_sync(0xffffffffu, ids_cur, (j & 7) * kPpBlocks + (my_b & (kPpBlocks - 1)));
        if (mine && (phys < 0 || phys >= p.pool_blocks)) phys = 0;  // reported by the K producer
        if (g >= kPpVStages)
          pok = __all_sync(0xffffffffu, mbar_wait(&bars->p_free[s], ((g / kPpVStages) - 1) & 1));
        if (!pok) break;
        if (lane == 0) mbar_arrive_expect_tx(&bars->v_full[s], uint32_t(nload * NH * 2048));
        __syncwarp();
        if (mine)
          tma_load_3d(sV + s * C::KV_BYTES + my_h * kPpKvHalf + my_b * 2048, &tv, 64 * my_h, d.kvh, phys * 16,
                      &bars->v_full[s]);
      }
    }
    if (!pok && lane == 0) set_error(p.err, kErrWaitTimeout);
  } else if (warp == 5) {
    // ------------------------------------------------------------ S issuer
    bool ok = true;
    int g = 0;  // tiles issued so far (all items)
    for (int k = 0; ok && pp_item(k, b, grid, items) >= 0; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[slot], (k >> 1) & 1));
      if (!ok) break;
      const int nkv = desc[slot].nkv;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars->d_empty[slot]);
        constexpr uint32_t idS = idesc_f16<T>(kPpRows, kPpKeys, false);
        const uint32_t q0 = smem_u32(sQ);
        if (!mbar_wait(&bars->q_full, k & 1)) ok = false;
        for (int j = 0; j < nkv && ok; ++j, ++g) {
          const int s = g % kPpKStages;
          if (!mbar_wait(&bars->k_full[s], (g / kPpKStages) & 1) ||
              (g > 0 && !mbar_wait(&bars->s_consumed, (g - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k0 = smem_u32(sK + s * C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(q0 + (kk >> 2) * kPpQHalf + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(k0 + (kk >> 2) * kPpKvHalf + (kk & 3) * 32, 16, 1024);
            umma_f16(tS, ad, bd, idS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars->s_full[s]);  // scores ready, K stage s free
          if (j == nkv - 1) umma_commit(&bars->q_empty);
        }
        if (!ok) set_error(p.err, kErrWaitTimeout);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      g = __shfl_sync(0xffffffffu, g, 0);
    }
  } else if (warp == 7) {
    // ------------------------------------------------------------ P.V issuer
    // O += P_h.V_h once the softmax has written P_h (after any rescale of O and, for the
    // item's first tile, after the previous item's epilogue read O) and V_h has landed;
    // the item's first P.V overwrites O.  S and P.V touch disjoint TMEM columns.
    bool ok = true;
    int g = 0;
    for (int k = 0; ok && pp_item(k, b, grid, items) >= 0; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[slot], (k >> 1) & 1));
      if (!ok) break;
      const int nkv = desc[slot].nkv;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars->d_empty[slot]);
        constexpr uint32_t idO = idesc_f16<T>(kPpRows, D, true);
        for (int j = 0; j < nkv && ok; ++j, ++g) {
          const int pb = g & 1, vs = g % kPpVStages;
          if (!mbar_wait(&bars->p_full[pb], (g >> 1) & 1) || !mbar_wait(&bars->v_full[vs], (g / kPpVStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v0 = smem_u32(sV + vs * C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < kPpKeys / 16; ++kk) {
            const uint64_t bd = smem_desc_sw128(v0 + kk * 2048, kPpKvHalf, 1024);
            umma_f16_ts(tO, tP + pb * (kPpKeys / 2) + 8 * kk, bd, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bars->p_free[pb]);  // also frees V stage vs (== pb)
        }
        if (!ok) set_error(p.err, kErrWaitTimeout);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      g = __shfl_sync(0xffffffffu, g, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax (one row per thread)
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    const int r = tid;
    const int t_row = r / G, g_row = r % G;
    bool ok = true;
    int g = 0;  // tiles consumed so far (all items)
    for (int k = 0; ok && pp_item(k, b, grid, items) >= 0; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->d_full[slot], (k >> 1) & 1));
      if (!ok) break;
      const PpItem d = desc[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->d_empty[slot]);
      const int t_eff = min(t_row, d.ntok - 1);
      const int qpos = d.ctx - d.ql + d.t0 + t_eff;

      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < d.nkv; ++j, ++g) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[g % kPpKStages], (g / kPpKStages) & 1));
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[kPpKeys];
        tmem_ld32_at<0>(tS + lane_base + 0, sr);
        tmem_ld32_at<32>(tS + lane_base + 32, sr);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&bars->s_consumed);

        // Last KV tile: zero the V rows past the context (and the blocks never loaded).
        const int kbase = j * kPpKeys;
        const bool zero_v = d.ctx - kbase < kPpKeys;
        if (zero_v) {
          const int vs = g % kPpVStages;
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->v_full[vs], (g / kPpVStages) & 1));
          if (!ok) break;
          uint8_t* vst = sV + vs * C::KV_BYTES;
          const int first = d.ctx - kbase;
          for (int c = tid; c < (kPpKeys - first) * NH * 8; c += 128) {
            const int row = first + c / (NH * 8), rest = c % (NH * 8);
            *reinterpret_cast<uint4*>(vst + (rest >> 3) * kPpKvHalf + row * 128 + (rest & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
        }

        const int lim = qpos - kbase;  // key column c is visible iff c <= lim
        if (__any_sync(0xffffffffu, lim < kPpKeys - 1)) {
#pragma unroll
          for (int c = 0; c < kPpKeys; ++c) sr[c] = c <= lim ? sr[c] : __float_as_uint(-INFINITY);
        }
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < kPpKeys; c += 2)
          mx4[(c >> 1) & 3] = fmax3(mx4[(c >> 1) & 3], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        const float mx = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]);
        // Raw q.k scores; the softmax scale is folded into the exponent and the subtracted
        // maximum is raised only past kPpLazyRescale (log2 units) of headroom, as in the
        // single-CTA kernel.
        const float mx_s = mx * p.qscale;
        const bool grow = mx_s > m_run + kPpLazyRescale;
        const float m_new = grow ? mx_s : m_run;
        const float alpha = grow ? ex2(m_run - m_new) : 1.f;
        const uint64_t sc2 = f2pack(p.qscale, p.qscale), mn2 = f2pack(-m_new, -m_new);
        uint64_t rs2[2] = {0ull, 0ull};
        uint32_t pk[kPpKeys / 2];
#pragma unroll
        for (int c = 0; c < kPpKeys; c += 2) {
          float x0, x1;
          f2unpack(fma2(f2pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sc2, mn2), x0, x1);
          const float e0 = ex2(x0), e1 = ex2(x1);
          rs2[(c >> 1) & 1] = add2(rs2[(c >> 1) & 1], f2pack(e0, e1));
          pk[c / 2] = pack2<T>(e0, e1);
        }
        float r0, r1, r2, r3;
        f2unpack(rs2[0], r0, r1);
        f2unpack(rs2[1], r2, r3);
        l_run = l_run * alpha + ((r0 + r1) + (r2 + r3));
        m_run = m_new;

        const int pb = g & 1;
        if (g >= 2) {  // the P.V that read this buffer two tiles ago has retired
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_free[pb], ((g - 2) >> 1) & 1));
          if (!ok) break;
          tc_fence_after();
        }
        tmem_st32(tP + lane_base + pb * (kPpKeys / 2), *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
        if (j > 0 && __any_sync(0xffffffffu, grow)) {  // O *= alpha once the previous P.V retired
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_free[pb ^ 1], ((g - 1) >> 1) & 1));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[64];
            tmem_ld32_at<0>(tO + lane_base + 64 * c, o);
            tmem_ld32_at<32>(tO + lane_base + 64 * c + 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 64; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + lane_base + 64 * c, *reinterpret_cast<const uint32_t(*)[32]>(&o[0]));
            tmem_st32(tO + lane_base + 64 * c + 32, *reinterpret_cast<const uint32_t(*)[32]>(&o[32]));
          }
        }
        tmem_wait_st();
        if (zero_v) fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->p_full[pb]);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> out, once the item's last P.V retired
      const int h = g - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_free[h & 1], (h >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool row_valid = t_row < d.ntok;
      T* dst = static_cast<T*>(p.out) + int64_t(d.tokbase + d.t0 + t_eff) * p.o_st +
               int64_t(d.kvh * G + g_row) * p.o_sh;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
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
      // The next item's first P.V overwrites O only after p_full, which these threads
      // arrive on after the loads above completed (tcgen05.wait::ld).
    }
    if (!ok && lane == 0) set_error(p.err, kErrWaitTimeout);
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
static cudaError_t launch_pp_one(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tq,
                                 const PrefillParams& p, cudaStream_t stream) {
  using C = PpCfg<D>;
  auto kern = paged_prefill_persist_kernel<T, D, G>;
  int dev = 0;
  cudaGetDevice(&dev);
  static int sms[64] = {};
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!sms[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  // Two CTAs per SM by design (registers, shared memory and TMEM each allow two; the
  // occupancy API does not count the shared-memory carveout preference and reports one).
  // CTAs never wait on one another, so a CTA without a free slot simply starts later.
  const int items = p.num_tiles * p.num_kv_heads;
  const int grid = min(items, 2 * sms[dev]);
  kern<<<grid, kPpThreads, C::SMEM, stream>>>(tk, tv, tq, p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t pp_by_group(int group, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tq,
                               const PrefillParams& p, cudaStream_t s) {
  switch (group) {
    case 1: return launch_pp_one<T, D, 1>(tk, tv, tq, p, s);
    case 2: return launch_pp_one<T, D, 2>(tk, tv, tq, p, s);
    case 4: return launch_pp_one<T, D, 4>(tk, tv, tq, p, s);
    case 8: return launch_pp_one<T, D, 8>(tk, tv, tq, p, s);
    default: return cudaErrorInvalidValue;
  }
}

bool prefill_persist_supported(int dtype, int head_dim, int group, int block_size) {
  return prefill_tc_supported(dtype, head_dim, group, block_size);
}

cudaError_t launch_prefill_persist(int dtype, int head_dim, int group, const CUtensorMap& tk, const CUtensorMap& tv,
                                   const CUtensorMap& tq, const PrefillParams& p, cudaStream_t stream) {
  if (p.num_tiles == 0) return cudaSuccess;
  if (dtype == PA_DTYPE_BF16)
    return head_dim == 64 ? pp_by_group<__nv_bfloat16, 64>(group, tk, tv, tq, p, stream)
                          : pp_by_group<__nv_bfloat16, 128>(group, tk, tv, tq, p, stream);
  if (dtype == PA_DTYPE_F16)
    return head_dim == 64 ? pp_by_group<__half, 64>(group, tk, tv, tq, p, stream)
                          : pp_by_group<__half, 128>(group, tk, tv, tq, p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
