// Host-side step planner: the index arrays of one paged step, built once per
// step and shared by every layer (as the reference builds them once,
// tokquay/kv_cache.py:170-172, :174-226).
//
// Differences from the reference's PagedBatch, all by design:
//   * rows are ragged (N = sum of q_len), never padded to B x T, so there is
//     no mask tensor and no padded query row is ever computed;
//   * the scatter targets are one int32 slot per new token
//     (block_table[p // bs] * bs + p % bs) instead of four int64 index lists;
//   * attention work items (query-row groups x key chunks, split-K where the
//     grid would otherwise be too small) are planned here too.
// Validation keeps the reference's conditions and messages
// (kv_cache.py:182-191) and adds pool / vocabulary range checks.
#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/tokquay_b200.h"
#include "host_error.h"

namespace {

// Must match the attention kernel's pipeline shape (paged_attention.cuh).
#ifndef TQ_ATTN_CHUNK
#define TQ_ATTN_CHUNK 32
#endif
#ifndef TQ_ATTN_MAX_ROWS
#define TQ_ATTN_MAX_ROWS 2
#endif
constexpr int kChunk = TQ_ATTN_CHUNK;      // keys per attention chunk
constexpr int kMaxRows = TQ_ATTN_MAX_ROWS; // query rows per work item
constexpr int kUnitBlocks = 64;            // most blocks one work item may span

inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t align4(int64_t n) { return (n + 3) & ~int64_t(3); }

}  // namespace

extern "C" int tq_plan_step(int32_t num_seqs, const int32_t* start, const int32_t* q_len,
                            const int32_t* table_offsets, const int32_t* table_data,
                            const int32_t* token_ids, int32_t block_size, int64_t num_blocks,
                            int32_t n_head, int32_t vocab_size, int32_t target_units,
                            int32_t min_split_chunks, const int32_t* caps, int32_t* out,
                            int64_t out_capacity, int32_t* layout) {
  using tq::set_error;
  if (layout == nullptr) return set_error(TQ_ERR_INVALID, "layout must not be NULL");
  std::memset(layout, 0, sizeof(int32_t) * TQ_PLAN_LAYOUT_LEN);
  if (num_seqs < 1)
    return set_error(TQ_ERR_INVALID,
                     "block_tables, start and new_lens must be non-empty and the same length");
  if (!start || !q_len || !table_offsets || (!table_data && table_offsets[num_seqs] > 0))
    return set_error(TQ_ERR_INVALID, "start, q_len and the block tables must not be NULL");
  if (block_size < 1 || (block_size & (block_size - 1)) != 0 || block_size > 256)
    return set_error(TQ_ERR_UNSUPPORTED, "block_size must be a power of two in [1, 256], got %d",
                     block_size);
  if (num_blocks < 1 || num_blocks * (int64_t)block_size > INT32_MAX)
    return set_error(TQ_ERR_UNSUPPORTED, "num_blocks * block_size must be in [1, 2^31), got %lld",
                     (long long)num_blocks * block_size);
  if (n_head < 1) return set_error(TQ_ERR_INVALID, "n_head must be positive");
  if (min_split_chunks < 1) min_split_chunks = 1;
  if (target_units < 1) target_units = 1;

  // ---- pass 1: validate, size everything -----------------------------------
  int64_t N = 0, max_nb = 0, max_ctx = 0, n_groups = 0, total_chunks = 0;
  for (int b = 0; b < num_seqs; ++b) {
    if (q_len[b] < 1) return set_error(TQ_ERR_INVALID, "every sequence must feed at least one token");
    if (start[b] < 0) return set_error(TQ_ERR_INVALID, "sequence %d: negative start %d", b, start[b]);
    const int64_t ctx = (int64_t)start[b] + q_len[b];
    const int64_t have = (int64_t)table_offsets[b + 1] - table_offsets[b];
    const int64_t need = cdiv64(ctx, block_size);
    if (have < need)
      return set_error(TQ_ERR_INVALID, "sequence %d: %lld blocks cannot hold %lld tokens", b,
                       (long long)have, (long long)ctx);
    for (int64_t i = 0; i < need; ++i) {
      const int32_t blk = table_data[table_offsets[b] + i];
      if (blk < 0 || blk >= num_blocks)
        return set_error(TQ_ERR_INVALID, "sequence %d: block id %d outside the pool of %lld blocks",
                         b, blk, (long long)num_blocks);
    }
    N += q_len[b];
    max_nb = std::max(max_nb, need);
    max_ctx = std::max(max_ctx, ctx);
    for (int64_t g0 = 0; g0 < q_len[b]; g0 += kMaxRows) {
      const int64_t nrows = std::min<int64_t>(kMaxRows, q_len[b] - g0);
      total_chunks += cdiv64(start[b] + g0 + nrows, kChunk);
      ++n_groups;
    }
  }
  if (N > INT32_MAX / 4) return set_error(TQ_ERR_UNSUPPORTED, "too many tokens in one step");
  if (token_ids && vocab_size > 0) {
    for (int64_t n = 0; n < N; ++n)
      if (token_ids[n] < 0 || token_ids[n] >= vocab_size)
        return set_error(TQ_ERR_INVALID, "token id %d outside the vocabulary of %d", token_ids[n],
                         vocab_size);
  }

  // Split-K size: split only when the unsplit grid would have fewer
  // (item, head) units than target_units.
  int64_t split_chunks = INT32_MAX;
  if (n_groups * n_head < target_units)
    split_chunks = std::max<int64_t>(min_split_chunks, cdiv64(total_chunks * n_head, target_units));
  // A work item stores its split index and count in 16 bits each.
  split_chunks = std::max<int64_t>(split_chunks, cdiv64(cdiv64(max_ctx, kChunk), 0x7fff));
  // The kernel keeps one item's block ids in two registers per lane, so an
  // item spans at most kUnitBlocks blocks: (split_chunks * kChunk) keys can
  // straddle one extra block boundary.
  split_chunks = std::min<int64_t>(split_chunks, std::max<int64_t>(1, (int64_t)(kUnitBlocks - 1) * block_size / kChunk));

  int64_t n_items = 0, n_combine = 0, n_partials = 0;
  auto count_items = [&]() {
    n_items = n_combine = n_partials = 0;
    for (int b = 0; b < num_seqs; ++b) {
      for (int64_t g0 = 0; g0 < q_len[b]; g0 += kMaxRows) {
        const int64_t nrows = std::min<int64_t>(kMaxRows, q_len[b] - g0);
        const int64_t nc = cdiv64(start[b] + g0 + nrows, kChunk);
        const int64_t nsplit = cdiv64(nc, split_chunks);
        n_items += nsplit;
        if (nsplit > 1) {
          n_combine += nrows;
          n_partials += nrows * n_head * nsplit;
        }
      }
    }
  };
  count_items();
  // With fixed capacities, coarsen the split until the items and partials fit.
  while (caps && split_chunks < INT32_MAX && (n_items > caps[3] || n_partials > caps[5])) {
    split_chunks = split_chunks >= (INT32_MAX / 2) ? INT32_MAX : split_chunks * 2;
    count_items();
  }
  if (n_partials > INT32_MAX || n_items > INT32_MAX / n_head)
    return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");

  const int64_t B = num_seqs;
  // Region sizes: this step's own, or the fixed capacities (caps) so that the
  // offsets -- and every pointer a captured CUDA graph holds -- stay put.
  int64_t dim_B = B, dim_N = N, dim_nb = max_nb, dim_items = n_items, dim_comb = n_combine;
  if (caps) {
    if (B > caps[0] || N > caps[1] || max_nb > caps[2] || n_items > caps[3] ||
        n_combine > caps[4] || n_partials > caps[5])
      return set_error(TQ_ERR_CAPACITY,
                       "step (seqs %lld, tokens %lld, blocks/seq %lld, items %lld, combine %lld, "
                       "partials %lld) exceeds the fixed plan capacities (%d, %d, %d, %d, %d, %d)",
                       (long long)B, (long long)N, (long long)max_nb, (long long)n_items,
                       (long long)n_combine, (long long)n_partials, caps[0], caps[1], caps[2],
                       caps[3], caps[4], caps[5]);
    dim_B = caps[0];
    dim_N = caps[1];
    dim_nb = caps[2];
    dim_items = caps[3];
    dim_comb = caps[4];
  }
  int64_t off = 0;
  auto take = [&](int64_t n) {
    const int64_t o = off;
    off = align4(off + n);
    return o;
  };
  const int64_t o_counts = take(4);
  const int64_t o_seq = take(dim_B * 4);
  const int64_t o_tab = take(dim_B * dim_nb);
  const int64_t o_slot = take(dim_N);
  const int64_t o_pos = take(dim_N);
  const int64_t o_ids = take(dim_N);
  const int64_t o_last = take(dim_B);
  const int64_t o_items = take(dim_items * 8);
  const int64_t o_comb = take(dim_comb * 4);
  const int64_t total = off;
  if (total > INT32_MAX) return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");
  max_nb = dim_nb;  // row stride of the packed tables

  layout[TQ_PLAN_NUM_TOKENS] = (int32_t)N;
  layout[TQ_PLAN_NUM_SEQS] = (int32_t)B;
  layout[TQ_PLAN_NUM_ITEMS] = (int32_t)n_items;
  layout[TQ_PLAN_NUM_COMBINE] = (int32_t)n_combine;
  layout[TQ_PLAN_NUM_PARTIALS] = (int32_t)n_partials;
  layout[TQ_PLAN_TABLE_STRIDE] = (int32_t)max_nb;
  layout[TQ_PLAN_MAX_CTX] = (int32_t)max_ctx;
  layout[TQ_PLAN_SPLIT_CHUNKS] = (int32_t)std::min<int64_t>(split_chunks, INT32_MAX);
  layout[TQ_PLAN_TOTAL_INTS] = (int32_t)total;
  layout[TQ_PLAN_OFF_COUNTS] = (int32_t)o_counts;
  layout[TQ_PLAN_OFF_SEQ_INFO] = (int32_t)o_seq;
  layout[TQ_PLAN_OFF_TABLES] = (int32_t)o_tab;
  layout[TQ_PLAN_OFF_SLOTS] = (int32_t)o_slot;
  layout[TQ_PLAN_OFF_POSITIONS] = (int32_t)o_pos;
  layout[TQ_PLAN_OFF_TOKEN_IDS] = (int32_t)o_ids;
  layout[TQ_PLAN_OFF_LAST_ROWS] = (int32_t)o_last;
  layout[TQ_PLAN_OFF_ITEMS] = (int32_t)o_items;
  layout[TQ_PLAN_OFF_COMBINE] = (int32_t)o_comb;
  if (out == nullptr || out_capacity < total)
    return set_error(TQ_ERR_CAPACITY, "plan needs %lld int32, buffer holds %lld", (long long)total,
                     (long long)out_capacity);

  // ---- pass 2: write --------------------------------------------------------
  std::memset(out, 0, sizeof(int32_t) * total);
  std::vector<int32_t> items((size_t)n_items * 8);
  out[o_counts + 0] = (int32_t)N;
  out[o_counts + 1] = (int32_t)n_items;
  out[o_counts + 2] = (int32_t)n_combine;
  out[o_counts + 3] = (int32_t)B;
  int64_t row = 0, item = 0, comb = 0, part = 0;
  for (int b = 0; b < num_seqs; ++b) {
    const int32_t* tbl = table_data + table_offsets[b];
    const int64_t s0 = start[b], n = q_len[b], ctx = s0 + n;
    const int64_t need = cdiv64(ctx, block_size);
    int32_t* seq = out + o_seq + 4 * b;
    seq[0] = (int32_t)row;
    seq[1] = (int32_t)n;
    seq[2] = (int32_t)s0;
    seq[3] = (int32_t)ctx;
    std::memcpy(out + o_tab + b * max_nb, tbl, sizeof(int32_t) * need);  // rest stays 0
    for (int64_t t = 0; t < n; ++t) {
      const int64_t p = s0 + t;
      out[o_slot + row + t] = (int32_t)((int64_t)tbl[p / block_size] * block_size + p % block_size);
      out[o_pos + row + t] = (int32_t)p;
      out[o_ids + row + t] = token_ids ? token_ids[row + t] : 0;
    }
    out[o_last + b] = (int32_t)(row + n - 1);
    for (int64_t g0 = 0; g0 < n; g0 += kMaxRows) {
      const int64_t nrows = std::min<int64_t>(kMaxRows, n - g0);
      const int64_t nc = cdiv64(s0 + g0 + nrows, kChunk);
      const int64_t nsplit = cdiv64(nc, split_chunks);
      for (int64_t s = 0; s < nsplit; ++s) {
        int32_t* it = items.data() + 8 * item++;
        it[0] = b;
        it[1] = (int32_t)(row + g0);
        it[2] = (int32_t)nrows;
        it[3] = (int32_t)(s0 + g0);
        it[4] = (int32_t)(s * split_chunks);
        it[5] = (int32_t)std::min(nc, (s + 1) * split_chunks);
        it[6] = nsplit > 1 ? (int32_t)part : -1;
        it[7] = (int32_t)(s | (nsplit << 16));
      }
      if (nsplit > 1) {
        for (int64_t r = 0; r < nrows; ++r) {
          int32_t* e = out + o_comb + 4 * comb++;
          e[0] = (int32_t)(row + g0 + r);
          e[1] = (int32_t)(part + r * n_head * nsplit);
          e[2] = (int32_t)nsplit;
          e[3] = 0;
        }
        part += nrows * n_head * nsplit;
      }
    }
    row += n;
  }
  // Longest items first: the kernel hands unit u to warp u % (warps in the
  // grid), so every warp then gets one item of each length class and all
  // warps finish within about one item of each other.
  std::vector<int32_t> order((size_t)n_items);
  for (int64_t i = 0; i < n_items; ++i) order[i] = (int32_t)i;
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
    return items[8 * a + 5] - items[8 * a + 4] > items[8 * b + 5] - items[8 * b + 4];
  });
  for (int64_t i = 0; i < n_items; ++i)
    std::memcpy(out + o_items + 8 * i, items.data() + 8 * (size_t)order[i], 8 * sizeof(int32_t));
  return TQ_OK;
}
