// Per-step planning on the host: validate the ragged batch once, then pack every
// per-step array the kernels read into one int32 buffer that is uploaded with a single
// copy and shared by all layers of the step.
//
// Reference behaviour restated here:
//   validation      inference_server/core/attention.py:202-219 (_check), same messages
//   seq_idx / q_pos inference_server/core/attention_triton.py:129-150 (_token_map)
//   slot_mapping    inference_server/core/block_table.py:143-159 (slots), restricted to
//                   the new tokens as inference_server/core/paged_executor.py:245 does
//   0-padded tables inference_server/core/paged_executor.py:250-251
// The split-K work list and the combine list have no reference counterpart: the
// reference walks each sequence's whole context in one program.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "paged_attention_b200.h"
#include "pa_host.h"

namespace pa {

static thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

const char* last_error() { return g_last_error.c_str(); }

// Decode split size: the largest power of two (in blocks, at most kMaxSplitBlocks) that
// still gives the grid at least kCtasPerSmTarget CTAs per SM, so long and short contexts
// balance while each CTA streams enough blocks to amortise its setup and its partial.
constexpr int kMaxSplitBlocks = 256;
constexpr int kCtasPerSmTarget = 4;

static int choose_split(const std::vector<int>& decode_nblk, int num_kv_heads, int sm_count) {
  const int64_t target = int64_t(std::max(sm_count, 1)) * kCtasPerSmTarget;
  for (int sb = kMaxSplitBlocks; sb > 1; sb >>= 1) {
    int64_t items = 0;
    for (int n : decode_nblk) items += (n + sb - 1) / sb;
    if (items * std::max(num_kv_heads, 1) >= target) return sb;
  }
  return 1;
}

}  // namespace pa

extern "C" {

int32_t pa_abi_version(void) { return 7; }

const char* pa_last_error(void) { return pa::last_error(); }

int64_t pa_plan_words_bound(int32_t num_seqs, int32_t num_tokens, int32_t max_blocks_per_seq) {
  const int64_t B = std::max(num_seqs, 0), T = std::max(num_tokens, 0);
  const int64_t W = std::max(max_blocks_per_seq, 1);
  // tables + lens + cu + per-token arrays + decode items (<= one per block) + combine
  // + prefill tiles (<= one per token) + alignment slack.
  return B * W + 3 * B + 1 + 3 * T + 4 * B * W + 4 * B + 2 * T + 64;
}

}  // extern "C"

namespace pa {

// Fixed shape of a padded decode plan (a CUDA-graph bucket): split size, table width and
// the capacities the decode-item and combine lists are padded to.
struct PlanCaps {
  int32_t split_blocks, width, items, combine;
};

static int32_t plan_impl(const int64_t* context_lens, const int64_t* query_lens, int32_t num_seqs,
                         const int64_t* block_tables, int64_t table_row_stride, int32_t table_cols,
                         int32_t num_tokens, int64_t pool_num_blocks, int32_t block_size, int32_t num_kv_heads,
                         int32_t sm_count, int32_t prefill_tile_tokens, int32_t* meta_out, int64_t meta_capacity,
                         pa_step_plan* plan, const PlanCaps* caps) {
  using pa::fail;
  if (!plan) return fail(PA_ERR_INVALID_ARGUMENT, "plan must not be NULL");
  std::memset(plan, 0, sizeof(*plan));
  if (num_seqs < 0 || num_tokens < 0) return fail(PA_ERR_INVALID_ARGUMENT, "negative batch or token count");
  if (block_size <= 0) return fail(PA_ERR_INVALID_ARGUMENT, "block_size must be positive");
  if (num_seqs > 0 && (!context_lens || !query_lens || !block_tables))
    return fail(PA_ERR_INVALID_ARGUMENT, "context_lens, query_lens and block_tables must not be NULL");
  if (table_cols < 0) return fail(PA_ERR_INVALID_ARGUMENT, "negative block_tables width");

  // ---- _check (attention.py:202-219), same messages
  int64_t qsum = 0;
  for (int i = 0; i < num_seqs; ++i) qsum += query_lens[i];
  if (qsum != num_tokens)
    return fail(PA_ERR_INVALID_ARGUMENT, "query_lens sum to %lld but query has %d tokens", (long long)qsum,
                num_tokens);
  for (int i = 0; i < num_seqs; ++i)
    if (query_lens[i] > context_lens[i])
      return fail(PA_ERR_INVALID_ARGUMENT,
                  "query_len exceeds context_len — the query tokens must be counted in the context");
  int64_t max_ctx = 0, total_ctx = 0;
  int32_t max_q = 0, width = 1;
  for (int i = 0; i < num_seqs; ++i) {
    if (query_lens[i] < 0 || context_lens[i] < 0)
      return fail(PA_ERR_INVALID_ARGUMENT, "context_lens and query_lens must be non-negative");
    if (context_lens[i] > (int64_t(1) << 30))
      return fail(PA_ERR_UNSUPPORTED, "context_len %lld exceeds 2^30", (long long)context_lens[i]);
    const int64_t need = (context_lens[i] + block_size - 1) / block_size;
    if (need > table_cols)
      return fail(PA_ERR_INVALID_ARGUMENT, "a sequence's context needs more blocks than its block_tables row holds");
    max_ctx = std::max(max_ctx, context_lens[i]);
    total_ctx += context_lens[i];
    max_q = std::max<int32_t>(max_q, int32_t(query_lens[i]));
    width = std::max<int32_t>(width, int32_t(need));
  }
  // Every block a sequence reads must exist: an out-of-range id would read another
  // allocation (the reference raises IndexError from its gather).
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t need = (context_lens[i] + block_size - 1) / block_size;
    const int64_t* row = block_tables + int64_t(i) * table_row_stride;
    for (int64_t b = 0; b < need; ++b)
      if (row[b] < 0 || row[b] >= pool_num_blocks)
        return fail(PA_ERR_INVALID_ARGUMENT, "block_tables[%d, %lld] = %lld is outside the pool of %lld blocks", i,
                    (long long)b, (long long)row[b], (long long)pool_num_blocks);
  }
  if (pool_num_blocks * int64_t(block_size) > (int64_t(1) << 31) - 1)
    return fail(PA_ERR_UNSUPPORTED, "pool has more than 2^31 slots");
  if (caps) {
    if (num_tokens != num_seqs)
      return fail(PA_ERR_UNSUPPORTED, "a padded plan is for decode steps (every query_len 1)");
    for (int i = 0; i < num_seqs; ++i)
      if (query_lens[i] != 1) return fail(PA_ERR_UNSUPPORTED, "a padded plan is for decode steps (every query_len 1)");
    if (caps->split_blocks <= 0 || caps->width <= 0 || caps->items < 0 || caps->combine < 0)
      return fail(PA_ERR_INVALID_ARGUMENT, "bad padded-plan capacities");
    if (width > caps->width)
      return fail(PA_ERR_BUFFER_TOO_SMALL, "bucket: a context needs %d blocks, the bucket's tables hold %d", width,
                  caps->width);
    width = caps->width;
  }

  // ---- split-K decode work list
  std::vector<int> decode_seqs, decode_nblk;
  int n_prefill = 0, n_prefill_tok = 0;
  for (int i = 0; i < num_seqs; ++i) {
    if (query_lens[i] == 1) {
      decode_seqs.push_back(i);
      decode_nblk.push_back(int((context_lens[i] + block_size - 1) / block_size));
    } else if (query_lens[i] > 1) {
      ++n_prefill;
      n_prefill_tok += int(query_lens[i]);
    }
  }
  const int sb = caps ? caps->split_blocks : pa::choose_split(decode_nblk, num_kv_heads, sm_count);
  int64_t n_items = 0, n_combine = 0;
  for (int n : decode_nblk) {
    const int ns = (n + sb - 1) / sb;
    n_items += ns;
    if (ns > 1) ++n_combine;
  }
  const int64_t real_items = n_items, real_combine = n_combine;
  if (caps) {
    if (n_items > caps->items || n_combine > caps->combine)
      return fail(PA_ERR_BUFFER_TOO_SMALL, "bucket: %lld work items / %lld combines, the bucket holds %d / %d",
                  (long long)n_items, (long long)n_combine, caps->items, caps->combine);
    n_items = caps->items;
    n_combine = caps->combine;
  }
  int64_t n_tiles = 0;
  if (prefill_tile_tokens > 0)
    for (int i = 0; i < num_seqs; ++i)
      if (query_lens[i] > 1) n_tiles += (query_lens[i] + prefill_tile_tokens - 1) / prefill_tile_tokens;

  // ---- layout (each array starts on a 4-word boundary)
  int64_t off = 0;
  auto take = [&](int64_t words) {
    const int64_t o = off;
    off += (words + 3) & ~int64_t(3);
    return o;
  };
  const int64_t B = num_seqs, T = num_tokens;
  plan->off_block_tables = take(B * width);
  plan->off_context_lens = take(B);
  plan->off_query_lens = take(B);
  plan->off_cu_query_lens = take(B + 1);
  plan->off_seq_idx = take(T);
  plan->off_q_pos = take(T);
  plan->off_slot_mapping = take(T);
  plan->off_decode_items = take(4 * n_items);
  plan->off_combine = take(4 * n_combine);
  plan->off_prefill_tiles = take(2 * n_tiles);
  plan->words = off;

  plan->num_seqs = num_seqs;
  plan->num_tokens = num_tokens;
  plan->table_width = width;
  plan->block_size = block_size;
  plan->num_decode_seqs = int32_t(decode_seqs.size());
  plan->num_prefill_seqs = n_prefill;
  plan->num_prefill_tokens = n_prefill_tok;
  plan->split_blocks = sb;
  plan->num_decode_items = int32_t(n_items);
  plan->num_combine_seqs = int32_t(n_combine);
  plan->max_context = int32_t(max_ctx);
  plan->max_query_len = max_q;
  plan->prefill_tile_tokens = prefill_tile_tokens > 0 ? prefill_tile_tokens : 0;
  plan->num_prefill_tiles = int32_t(n_tiles);
  plan->total_context = total_ctx;

  if (!meta_out) return PA_OK;  // size query only
  if (meta_capacity < plan->words)
    return fail(PA_ERR_BUFFER_TOO_SMALL, "metadata buffer holds %lld words, plan needs %lld",
                (long long)meta_capacity, (long long)plan->words);
  std::memset(meta_out, 0, sizeof(int32_t) * size_t(plan->words));

  int32_t* tables = meta_out + plan->off_block_tables;
  int32_t* ctx_out = meta_out + plan->off_context_lens;
  int32_t* q_out = meta_out + plan->off_query_lens;
  int32_t* cu = meta_out + plan->off_cu_query_lens;
  int32_t* seq_idx = meta_out + plan->off_seq_idx;
  int32_t* q_pos = meta_out + plan->off_q_pos;
  int32_t* slots = meta_out + plan->off_slot_mapping;
  cu[0] = 0;
  for (int i = 0; i < num_seqs; ++i) {
    const int64_t ctx = context_lens[i], q = query_lens[i];
    const int64_t need = (ctx + block_size - 1) / block_size;
    const int64_t* row = block_tables + int64_t(i) * table_row_stride;
    for (int64_t b = 0; b < need; ++b) tables[int64_t(i) * width + b] = int32_t(row[b]);
    ctx_out[i] = int32_t(ctx);
    q_out[i] = int32_t(q);
    cu[i + 1] = cu[i] + int32_t(q);
    for (int64_t t = 0; t < q; ++t) {
      const int64_t tok = cu[i] + t, pos = ctx - q + t;
      seq_idx[tok] = i;
      q_pos[tok] = int32_t(pos);
      slots[tok] = int32_t(row[pos / block_size] * block_size + pos % block_size);
    }
  }

  // Decode items in launch order: all full-length splits first, then the shorter last
  // splits longest first, so the tail of the grid is made of the smallest pieces.
  // Partial-result slots ("parts") are numbered sequence-major so a sequence's splits
  // are contiguous for the combine pass.
  int32_t* items = meta_out + plan->off_decode_items;
  int32_t* comb = meta_out + plan->off_combine;
  struct Item { int seq, split, part, nsplit, nblk; };
  std::vector<Item> full, tail;
  int part = 0, ci = 0;
  for (size_t k = 0; k < decode_seqs.size(); ++k) {
    const int i = decode_seqs[k], n = decode_nblk[k];
    const int ns = (n + sb - 1) / sb;
    if (ns > 1) {
      comb[4 * ci + 0] = i;
      comb[4 * ci + 1] = cu[i];
      comb[4 * ci + 2] = part;
      comb[4 * ci + 3] = ns;
      ++ci;
    }
    for (int s = 0; s < ns; ++s) {
      const int nb = std::min(sb, n - s * sb);
      Item it{i, s, part + s, ns, nb};
      (nb == sb ? full : tail).push_back(it);
    }
    part += ns;
  }
  std::stable_sort(tail.begin(), tail.end(), [](const Item& a, const Item& b) { return a.nblk > b.nblk; });
  int64_t w = 0;
  for (const auto* list : {&full, &tail})
    for (const Item& it : *list) {
      items[4 * w + 0] = it.seq;
      items[4 * w + 1] = it.split;
      items[4 * w + 2] = it.part;
      items[4 * w + 3] = it.nsplit;
      ++w;
    }
  // Padding of a bucketed plan: null items and combines (sequence -1) the kernels skip.
  for (; w < n_items; ++w) {
    items[4 * w + 0] = -1;
    items[4 * w + 2] = -1;
  }
  for (int64_t c = real_combine; c < n_combine; ++c) comb[4 * c + 0] = -1;
  (void)real_items;

  // Prefill tiles in launch order, heaviest first: a tile's work is the causal key range
  // of its last token, so the grid's tail is made of the tiles with the fewest keys
  // (longest-processing-time-first list scheduling over the SMs).
  if (n_tiles > 0) {
    int32_t* tiles = meta_out + plan->off_prefill_tiles;
    struct Tile { int seq, row; int64_t keys; };
    std::vector<Tile> list;
    list.reserve(size_t(n_tiles));
    for (int i = 0; i < num_seqs; ++i)
      if (query_lens[i] > 1)
        for (int64_t r = 0; r < query_lens[i]; r += prefill_tile_tokens) {
          const int64_t last = std::min<int64_t>(r + prefill_tile_tokens, query_lens[i]);
          list.push_back({i, int32_t(r), context_lens[i] - query_lens[i] + last});
        }
    std::stable_sort(list.begin(), list.end(), [](const Tile& a, const Tile& b) { return a.keys > b.keys; });
    for (size_t k = 0; k < list.size(); ++k) {
      tiles[2 * k + 0] = list[k].seq;
      tiles[2 * k + 1] = list[k].row;
    }
  }
  return PA_OK;
}

}  // namespace pa

extern "C" {

int32_t pa_plan_step(const int64_t* context_lens, const int64_t* query_lens, int32_t num_seqs,
                     const int64_t* block_tables, int64_t table_row_stride, int32_t table_cols,
                     int32_t num_tokens, int64_t pool_num_blocks, int32_t block_size,
                     int32_t num_kv_heads, int32_t sm_count, int32_t prefill_tile_tokens,
                     int32_t* meta_out, int64_t meta_capacity, pa_step_plan* plan) {
  return pa::plan_impl(context_lens, query_lens, num_seqs, block_tables, table_row_stride, table_cols, num_tokens,
                       pool_num_blocks, block_size, num_kv_heads, sm_count, prefill_tile_tokens, meta_out,
                       meta_capacity, plan, nullptr);
}

int32_t pa_plan_decode_padded(const int64_t* context_lens, int32_t num_seqs, const int64_t* block_tables,
                              int64_t table_row_stride, int32_t table_cols, int64_t pool_num_blocks,
                              int32_t block_size, int32_t num_kv_heads, int32_t split_blocks, int32_t width_cap,
                              int32_t items_cap, int32_t combine_cap, int32_t* meta_out, int64_t meta_capacity,
                              pa_step_plan* plan) {
  std::vector<int64_t> ones(size_t(std::max(num_seqs, 0)), 1);
  const pa::PlanCaps caps{split_blocks, width_cap, items_cap, combine_cap};
  return pa::plan_impl(context_lens, ones.data(), num_seqs, block_tables, table_row_stride, table_cols, num_seqs,
                       pool_num_blocks, block_size, num_kv_heads, 0, 0, meta_out, meta_capacity, plan, &caps);
}

}  // extern "C"
