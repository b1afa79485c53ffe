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

#include "../../include/tokquay_b200.h"
#include "host_error.h"

namespace {

constexpr int kChunk = 32;    // keys per attention chunk (paged_attention.cuh)
constexpr int kMaxRows = 4;   // query rows per work item

inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t align4(int64_t n) { return (n + 3) & ~int64_t(3); }

}  // namespace

extern "C" int tq_plan_step(int32_t num_seqs, const int32_t* start, const int32_t* q_len,
                            const int32_t* table_offsets, const int32_t* table_data,
                            const int32_t* token_ids, int32_t block_size, int64_t num_blocks,
                            int32_t n_head, int32_t vocab_size, int32_t target_units,
                            int32_t min_split_chunks, int32_t* out, int64_t out_capacity,
                            int32_t* layout) {
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

  int64_t n_items = 0, n_combine = 0, n_partials = 0;
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
  if (n_partials > INT32_MAX || n_items > INT32_MAX / n_head)
    return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");

  const int64_t B = num_seqs;
  int64_t off = 0;
  auto take = [&](int64_t n) {
    const int64_t o = off;
    off = align4(off + n);
    return o;
  };
  const int64_t o_counts = take(4);
  const int64_t o_seq = take(B * 4);
  const int64_t o_tab = take(B * max_nb);
  const int64_t o_slot = take(N);
  const int64_t o_pos = take(N);
  const int64_t o_ids = take(N);
  const int64_t o_last = take(B);
  const int64_t o_items = take(n_items * 8);
  const int64_t o_comb = take(n_combine * 4);
  const int64_t total = off;
  if (total > INT32_MAX) return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");

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
        int32_t* it = out + o_items + 8 * item++;
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
  return TQ_OK;
}
