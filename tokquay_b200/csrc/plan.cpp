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
#include <array>
#include <atomic>
#include <cmath>
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
#ifndef TQ_ATTN_WARPS
#define TQ_ATTN_WARPS 6
#endif
constexpr int kChunk = TQ_ATTN_CHUNK;      // keys per attention chunk
constexpr int kMaxRows = TQ_ATTN_MAX_ROWS; // query rows per work item
constexpr int kWarps = TQ_ATTN_WARPS;      // computing warps per attention CTA
constexpr int kUnitBlocks = 64;            // most blocks one work item may span
constexpr int kMaxChunkIndex = 0xffff;     // chunk indices are stored in 16 bits
// Work item flags (word 2, bits 24..31).
constexpr int kFlagLocal = 1;   // keys cut between warps of one CTA: merged in shared memory
constexpr int kFlagGlobal = 2;  // keys split across CTAs: merged through the split-K scratch
constexpr int kFlagDecode = 4;  // the sequence feeds one token: pos0 is its only new key
// Shared-memory partial slots one CTA holds (each warp boundary cuts at most
// one pair, so a CTA needs at most 2 * (kWarps - 1) * kMaxRows).
constexpr int kLocalSlots = 2 * (kWarps - 1) * kMaxRows;
// A warp's first work item (at a fixed place in the plan) carries the block
// ids of its first chunk, so the kernel's first copies need no table lookup.
constexpr int kFirstWords = 16;   // 8 item words + up to kFirstBlocks block ids
constexpr int kFirstBlocks = kFirstWords - 8;
// Prompt tiles: a sequence that feeds many rows this step goes to whole-CTA
// tiles of up to kTileRows rows x one head, run on the tensor cores
// (paged_attention.cuh, prompt-tile CTAs) instead of 2-row warp items.
constexpr int kFlagTile = 8;       // item of a prompt-tile CTA (word 2, bits 24..31)
constexpr int kTileRows = 128;     // query rows of one tile (the MMA's M)
constexpr int kTileMaxItems = 96;  // tile items one CTA holds (its shared-memory list)

// Tile planning knobs (tq_plan_prompt_tiles): the least q_len that is tiled
// (0: never), and a tile item's cost against a warp-path chunk, in percent:
// chunk_cost per 32-key chunk plus item_cost per item.
std::atomic<int> g_tile_min_rows{16};
std::atomic<int> g_tile_chunk_cost{1500};
std::atomic<int> g_tile_item_cost{200};
std::atomic<int> g_tile_max_pieces{1};  // most pieces a tile is cut into (1: never cut)

inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t align4(int64_t n) { return (n + 3) & ~int64_t(3); }
inline int64_t align8(int64_t n) { return (n + 7) & ~int64_t(7); }

struct Group {  // one query-row group of a sequence
  int32_t seq, row0, nrows, pos0, nc;  // nc: 32-key chunks it attends to
};

struct Tile {  // a run of one sequence's query rows, run as one MMA tile per head
  int32_t seq, row0, nrows, pos0, nc;  // nc: 32-key chunks its last row attends to
};

struct TilePiece {  // a run of a tile's chunks, bound for one CTA (per head)
  int32_t tile, cbeg, cend, gsplit, gnsplit;
  int64_t gbase;  // split-K partial of (head 0, row 0, split 0), or -1; head h adds h * nrows * gnsplit
};

struct Piece {  // a run of chunks of a group's pairs (one per head), each bound for one CTA
  int32_t group, cbeg, cend, gsplit, gnsplit;
  int64_t gbase;  // split-K partial of (head 0, row 0, split 0), or -1; head h adds h * nrows * gnsplit
};

}  // namespace

extern "C" int tq_plan_prompt_tiles(int32_t min_rows, int32_t chunk_cost_pct, int32_t item_cost_pct,
                                    int32_t max_pieces) {
  const int prev = g_tile_min_rows.load();
  if (min_rows >= 0) g_tile_min_rows.store(min_rows);
  if (chunk_cost_pct > 0) g_tile_chunk_cost.store(chunk_cost_pct);
  if (item_cost_pct >= 0) g_tile_item_cost.store(item_cost_pct);
  if (max_pieces > 0) g_tile_max_pieces.store(max_pieces);
  return prev;
}

extern "C" int tq_plan_step(int32_t num_seqs, const int32_t* start, const int32_t* q_len,
                            const int32_t* table_offsets, const int32_t* table_data,
                            const int32_t* token_ids, int32_t block_size, int64_t num_blocks,
                            int32_t n_head, int32_t vocab_size, int32_t n_ctas,
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
  if (n_head < 1 || n_head > 0xffff) return set_error(TQ_ERR_INVALID, "n_head must be in [1, 65535]");
  if (n_ctas < 1 || n_ctas > 0xffff) return set_error(TQ_ERR_INVALID, "n_ctas must be in [1, 65535]");
  if (min_split_chunks < 1) min_split_chunks = 1;

  // ---- pass 1: validate, size everything -----------------------------------
  int64_t N = 0, max_nb = 0, max_ctx = 0, n_groups = 0, total_chunks = 0;
  const int tile_min = g_tile_min_rows.load(std::memory_order_relaxed);
  const int64_t tile_chunk_cost = g_tile_chunk_cost.load(std::memory_order_relaxed);
  const int64_t tile_item_cost = g_tile_item_cost.load(std::memory_order_relaxed);
  const int64_t tile_max_pieces = g_tile_max_pieces.load(std::memory_order_relaxed);
  std::vector<Tile> tiles;
  std::vector<char> tiled((size_t)num_seqs, 0);
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
    if (tile_min > 0 && q_len[b] >= tile_min) {
      tiled[b] = 1;
      // Rows cut evenly into the fewest tiles of at most kTileRows.
      const int64_t nt = cdiv64(q_len[b], kTileRows), per = cdiv64(q_len[b], nt);
      for (int64_t t0 = 0; t0 < q_len[b]; t0 += per) {
        const int64_t nrows = std::min<int64_t>(per, q_len[b] - t0);
        tiles.push_back({b, (int32_t)(N - q_len[b] + t0), (int32_t)nrows, (int32_t)(start[b] + t0),
                         (int32_t)cdiv64(start[b] + t0 + nrows, kChunk)});
      }
      continue;
    }
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

  if (cdiv64(max_ctx, kChunk) > kMaxChunkIndex)
    return set_error(TQ_ERR_UNSUPPORTED, "a context of %lld tokens exceeds %d chunks of %d keys",
                     (long long)max_ctx, kMaxChunkIndex, kChunk);

  // ---- prompt tiles -> tile CTAs ---------------------------------------------
  // Tile items (one per tile piece and head) run on CTAs of their own, the
  // last n_tctas of the grid; the warp path below gets the first n_wctas.
  // The split follows the estimated loads -- a warp-path CTA's load is its
  // chunks (x 100); a tile item costs tile_chunk_cost per chunk plus
  // tile_item_cost.  With max_pieces > 1, a tile whose item would cost more
  // than the balanced load of a CTA is cut over its keys into up to
  // max_pieces pieces of at least two chunks (never in plans of fixed
  // capacity).  Each piece leaves its partials in the split-K scratch, and
  // the merge kernel after the attention grid combines them (the entries of
  // the tile-merge trailer).
  // The items go longest first to the least loaded tile
  // CTA.  A step whose tiles do not fit (a one-CTA grid beside warp work, or
  // more than kTileMaxItems on a CTA) runs every row on the warp path.
  int32_t n_tctas = 0;
  std::vector<TilePiece> tpieces;
  std::vector<std::vector<int32_t>> tile_lists;  // per tile CTA: items (piece * n_head + head)
  int64_t tile_partials = 0, tile_combine = 0;
  if (!tiles.empty()) {
    const int64_t warp_load = total_chunks * n_head * 100;
    const int64_t max_tctas0 = n_groups == 0 ? n_ctas : n_ctas - 1;
    // Tile CTAs for a given tile load: the grid's share of the estimated work.
    auto tile_ctas_for = [&](int64_t tile_load) {
      if (n_groups == 0) return max_tctas0;
      return std::min<int64_t>(max_tctas0, std::max<int64_t>(1, (int64_t)((double)n_ctas * tile_load /
                                                                            (double)(tile_load + warp_load) + 0.5)));
    };
    // Pieces per tile: one, then (plans without fixed capacities) one more for
    // the tile with the costliest piece, while that piece costs more than a
    // CTA's balanced load and every tile item still gets a CTA of its own.
    std::vector<int64_t> gns(tiles.size(), 1);
    for (;;) {
      int64_t tile_load = 0, n_pieces = 0;
      for (size_t i = 0; i < tiles.size(); ++i) {
        tile_load += (tiles[i].nc * tile_chunk_cost + gns[i] * tile_item_cost) * n_head;
        n_pieces += gns[i];
      }
      if (caps || tile_max_pieces < 2) break;
      const double balanced = (double)(tile_load + warp_load) / n_ctas;
      int64_t best = -1;
      double best_cost = 0.0;
      for (size_t i = 0; i < tiles.size(); ++i) {
        const double c = (double)cdiv64(tiles[i].nc, gns[i]) * tile_chunk_cost + tile_item_cost;
        if (gns[i] < std::min<int64_t>(tile_max_pieces, tiles[i].nc / 2) && c > best_cost) {
          best = (int64_t)i;
          best_cost = c;
        }
      }
      if (best < 0 || best_cost <= balanced) break;
      const int64_t more = tile_load + (tile_item_cost * n_head);
      if ((n_pieces + 1) * n_head > tile_ctas_for(more)) break;
      ++gns[(size_t)best];
    }
    for (size_t i = 0; i < tiles.size(); ++i) {
      const Tile& t = tiles[i];
      const int64_t gn = gns[i];
      for (int64_t sp = 0; sp < gn; ++sp)
        tpieces.push_back({(int32_t)i, (int32_t)(sp * t.nc / gn), (int32_t)((sp + 1) * t.nc / gn), (int32_t)sp,
                           (int32_t)gn, gn > 1 ? tile_partials : -1});
      if (gn > 1) {
        tile_partials += (int64_t)n_head * t.nrows * gn;
        tile_combine += t.nrows;
      }
    }
    std::vector<int64_t> cost(tpieces.size());
    int64_t tile_load = 0;
    for (size_t i = 0; i < tpieces.size(); ++i) {
      cost[i] = (tpieces[i].cend - tpieces[i].cbeg) * tile_chunk_cost + tile_item_cost;
      tile_load += cost[i] * n_head;
    }
    const int64_t n_titems = (int64_t)tpieces.size() * n_head;
    const int64_t max_tctas = max_tctas0;
    int64_t nt = std::min<int64_t>({max_tctas, n_titems, tile_ctas_for(tile_load)});
    nt = std::max(nt, cdiv64(n_titems, kTileMaxItems));
    bool fits = nt >= 1 && nt <= max_tctas;
    if (fits) {
      std::vector<int32_t> ord(tpieces.size());
      for (size_t i = 0; i < ord.size(); ++i) ord[i] = (int32_t)i;
      std::stable_sort(ord.begin(), ord.end(), [&](int32_t a, int32_t b) { return cost[a] > cost[b]; });
      std::vector<int64_t> load((size_t)nt, 0);
      tile_lists.assign((size_t)nt, {});
      for (int32_t i : ord)
        for (int h = 0; h < n_head && fits; ++h) {
          size_t c = 0;
          for (size_t j = 1; j < load.size(); ++j)
            if (load[j] < load[c]) c = j;
          tile_lists[c].push_back(i * n_head + h);
          load[c] += cost[i];
          fits = tile_lists[c].size() <= (size_t)kTileMaxItems;
        }
    }
    if (fits) {
      n_tctas = (int32_t)nt;
    } else {  // back to the warp path
      tile_lists.clear();
      tiles.clear();
      tpieces.clear();
      tile_partials = tile_combine = 0;
      for (int b = 0; b < num_seqs; ++b) {
        if (!tiled[b]) continue;
        tiled[b] = 0;
        for (int64_t g0 = 0; g0 < q_len[b]; g0 += kMaxRows) {
          const int64_t nrows = std::min<int64_t>(kMaxRows, q_len[b] - g0);
          total_chunks += cdiv64(start[b] + g0 + nrows, kChunk);
          ++n_groups;
        }
      }
    }
  }
  const int32_t n_wctas = n_ctas - n_tctas;  // CTAs of the warp path: 0 .. n_wctas-1
  int64_t n_tile_items = 0;
  for (const auto& l : tile_lists) n_tile_items += (int64_t)l.size();

  // ---- attention work: (group, head) pairs -> pieces -> CTAs -> warps ----------
  std::vector<Group> groups;
  groups.reserve((size_t)n_groups);
  {
    int64_t row = 0;
    for (int b = 0; b < num_seqs; ++b) {
      if (tiled[b]) {
        row += q_len[b];
        continue;
      }
      for (int64_t g0 = 0; g0 < q_len[b]; g0 += kMaxRows) {
        const int64_t nrows = std::min<int64_t>(kMaxRows, q_len[b] - g0);
        groups.push_back({b, (int32_t)(row + g0), (int32_t)nrows, (int32_t)(start[b] + g0),
                          (int32_t)cdiv64(start[b] + g0 + nrows, kChunk)});
      }
      row += q_len[b];
    }
  }
  // The kernel keeps one item's block ids in two registers per lane, so an
  // item spans at most kUnitBlocks blocks: (chunks * kChunk) keys can
  // straddle one extra block boundary.
  const int64_t max_piece = std::max<int64_t>(1, (int64_t)(kUnitBlocks - 1) * block_size / kChunk);
  const int64_t n_warps = (int64_t)n_ctas * kWarps;
  // A CTA's fair share of chunks: a pair longer than that (and than twice
  // the smallest cross-CTA piece) is split across CTAs.
  const int64_t share = std::max<int64_t>(1, cdiv64(total_chunks * n_head, std::max<int32_t>(n_wctas, 1)));
  int64_t split_min = min_split_chunks;

  // Pieces: a group's keys, cut across CTAs when longer than a CTA's share.
  // All heads of a group are alike, so a piece stands for its n_head (group,
  // head) pairs: pair p of the step is piece p / n_head, head p % n_head.
  std::vector<Piece> pieces;
  int64_t n_partials = 0, n_combine = 0, max_items = 0, n_pairs = 0;
  pieces.reserve((size_t)n_groups);
  auto make_pieces = [&]() {
    pieces.clear();
    n_partials = n_combine = 0;
    for (size_t gi = 0; gi < groups.size(); ++gi) {
      const Group& g = groups[gi];
      int64_t gn = 1;
      if (g.nc > share && g.nc >= 2 * split_min) gn = std::min(cdiv64(g.nc, share), g.nc / split_min);
      gn = std::min<int64_t>(std::max(gn, cdiv64(g.nc, max_piece)), g.nc);
      const int64_t gbase = gn > 1 ? n_partials : -1;
      for (int64_t sp = 0; sp < gn; ++sp)
        pieces.push_back({(int32_t)gi, (int32_t)(sp * g.nc / gn), (int32_t)((sp + 1) * g.nc / gn), (int32_t)sp,
                          (int32_t)gn, gbase});
      if (gn > 1) {
        n_combine += g.nrows;
        n_partials += (int64_t)n_head * g.nrows * gn;
      }
    }
    n_pairs = (int64_t)pieces.size() * n_head;
    // Each warp boundary cuts at most one pair in two; tile items are one each.
    max_items = n_pairs + (int64_t)n_wctas * (kWarps - 1) + n_tile_items;
  };
  make_pieces();
  // With fixed capacities, coarsen the cross-CTA split until items and partials fit.
  while (caps && (max_items > caps[3] || n_partials > caps[5]) && split_min < kMaxChunkIndex) {
    split_min *= 2;
    make_pieces();
  }
  // Split tiles' partials follow the warp path's.
  for (TilePiece& tp : tpieces)
    if (tp.gbase >= 0) tp.gbase += n_partials;
  n_partials += tile_partials;
  n_combine += tile_combine;
  if (n_partials > INT32_MAX || max_items > INT32_MAX / 8)
    return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");

  // CTAs: longest pair first (a stable counting sort of the pieces on
  // length), each to the least loaded CTA.  Loads are whole chunks and only
  // grow, so the least loaded CTA comes from a bucket queue (one intrusive
  // list per load value, scanned upward from the lowest non-empty one):
  // O(pairs + largest load).  A CTA that receives a pair had at most the mean
  // load, so no load exceeds the mean plus the longest pair.
  int64_t longest_piece = 1, sum_len = 0;
  for (const Piece& pc : pieces) {
    longest_piece = std::max<int64_t>(longest_piece, pc.cend - pc.cbeg);
    sum_len += (int64_t)(pc.cend - pc.cbeg) * n_head;
  }
  std::vector<int32_t> order(pieces.size());
  {
    std::vector<int32_t> start_of((size_t)longest_piece + 2, 0);
    for (const Piece& pc : pieces) ++start_of[(size_t)(longest_piece - (pc.cend - pc.cbeg)) + 1];
    for (size_t i = 1; i < start_of.size(); ++i) start_of[i] += start_of[i - 1];
    for (size_t i = 0; i < pieces.size(); ++i)
      order[start_of[(size_t)(longest_piece - (pieces[i].cend - pieces[i].cbeg))]++] = (int32_t)i;
  }
  std::vector<int64_t> cta_load((size_t)n_wctas, 0);
  std::vector<int32_t> cta_count((size_t)n_wctas + 1, 0), cta_of((size_t)n_pairs);
  if (n_pairs > 0) {
    const int64_t max_load = sum_len / n_wctas + longest_piece + 1;
    std::vector<int32_t> head((size_t)max_load + 1, -1), next((size_t)n_wctas, -1);
    for (int32_t c = n_wctas - 1; c >= 0; --c) {  // bucket 0 lists CTA 0 first
      next[c] = head[0];
      head[0] = c;
    }
    int64_t lo = 0;
    for (int32_t i : order) {
      const int64_t len = pieces[i].cend - pieces[i].cbeg;
      for (int h = 0; h < n_head; ++h) {
        while (head[(size_t)lo] < 0) ++lo;
        const int32_t c = head[(size_t)lo];
        head[(size_t)lo] = next[c];
        cta_of[(size_t)i * n_head + h] = c;
        ++cta_count[(size_t)c + 1];
        const int64_t l = cta_load[c] += len;
        if (l > max_load)
          return set_error(TQ_ERR_UNSUPPORTED, "internal: CTA load %lld above the bound %lld",
                           (long long)l, (long long)max_load);
        next[c] = head[(size_t)l];
        head[(size_t)l] = c;
      }
    }
  }
  for (int32_t c = 0; c < n_wctas; ++c) cta_count[c + 1] += cta_count[c];
  std::vector<int32_t> by_cta((size_t)n_pairs);  // pairs grouped by CTA, in assignment order
  {
    std::vector<int32_t> fill(cta_count.begin(), cta_count.end() - 1);
    for (int32_t i : order)
      for (int h = 0; h < n_head; ++h) {
        const int32_t pr = i * n_head + h;
        by_cta[fill[cta_of[pr]]++] = pr;
      }
  }

  const int64_t B = num_seqs;
  // Region sizes: this step's own, or the fixed capacities (caps) so that the
  // offsets -- and every pointer a captured CUDA graph holds -- stay put.
  // Without caps the other-items region is sized for the most items the cuts
  // can make (max_items); the step uses, and copies, only its used prefix.
  int64_t dim_B = B, dim_N = N, dim_nb = max_nb, dim_rest = max_items, dim_comb = n_combine;
  if (caps) {
    if (B > caps[0] || N > caps[1] || max_nb > caps[2] || max_items > caps[3] ||
        n_combine > caps[4] || n_partials > caps[5])
      return set_error(TQ_ERR_CAPACITY,
                       "step (seqs %lld, tokens %lld, blocks/seq %lld, items %lld, combine %lld, "
                       "partials %lld) exceeds the fixed plan capacities (%d, %d, %d, %d, %d, %d)",
                       (long long)B, (long long)N, (long long)max_nb, (long long)max_items,
                       (long long)n_combine, (long long)n_partials, caps[0], caps[1], caps[2],
                       caps[3], caps[4], caps[5]);
    dim_B = caps[0];
    dim_N = caps[1];
    dim_nb = caps[2];
    dim_rest = caps[3];
    dim_comb = caps[4];
  }
  int64_t off = 0;
  auto take = [&](int64_t n) {
    const int64_t o = off;
    off = align8(off + n);
    return o;
  };
  const int64_t o_counts = take(4);
  const int64_t o_seq = take(dim_B * 4);
  const int64_t o_tab = take(dim_B * dim_nb);
  const int64_t o_slot = take(dim_N);
  const int64_t o_pos = take(dim_N);
  const int64_t o_ids = take(dim_N);
  const int64_t o_last = take(dim_B);
  const int64_t o_comb = take(dim_comb * 4);
  // The attention plan goes last, so a step copies only its used prefix.
  const int64_t o_items = off;
  const int64_t o_ranges = o_items + kFirstWords * n_warps;
  const int64_t o_rest = o_ranges + align8(n_warps + 1);
  // The tile-merge trailer follows the items actually written: a count word
  // (padded to 8) and one entry of 4 per row of a split tile.
  const int64_t n_tile_merges = tile_combine;
  const int64_t trailer_ints = 8 + align8(4 * n_tile_merges);
  const int64_t total = o_rest + 8 * dim_rest + trailer_ints;
  if (total > INT32_MAX) return set_error(TQ_ERR_UNSUPPORTED, "step too large to plan");
  max_nb = dim_nb;  // row stride of the packed tables
  std::memset(layout, 0, sizeof(int32_t) * TQ_PLAN_LAYOUT_LEN);
  layout[TQ_PLAN_TOTAL_INTS] = (int32_t)total;
  if (out == nullptr || out_capacity < total)
    return set_error(TQ_ERR_CAPACITY, "plan needs %lld int32, buffer holds %lld", (long long)total,
                     (long long)out_capacity);

  // ---- pass 2: write --------------------------------------------------------
  // Attention items.  Each CTA's chunks, in assignment order, are cut into
  // kWarps runs of equal length; a piece a cut falls in is shared by the
  // warps on both sides and merged in the CTA's shared memory.  Items come out
  // warp by warp: a warp's first item to its fixed place, the others to the
  // list after the offsets.
  int64_t rest = 0, n_items = 0, longest = 0;
  int32_t* const first_items = out + o_items;
  int32_t* const ranges = out + o_ranges;
  int32_t* const rest_items = out + o_rest;
  for (int32_t c = 0; c < n_wctas; ++c) {
    const int64_t L = cta_load[c];
    int64_t bnd[kWarps + 1];
    for (int w = 0; w <= kWarps; ++w) bnd[w] = (int64_t)w * L / kWarps;
    const int64_t wbase = (int64_t)c * kWarps;
    bool has[kWarps] = {};  // warp has its first item
    int cur = 0;            // warp of this CTA whose items are being written
    ranges[wbase] = (int32_t)rest;
    int32_t slot = 0;
    int64_t x = 0;
    int w0 = 0;  // the warp whose run holds chunk position x (x only grows)
    for (int32_t k = cta_count[c]; k < cta_count[c + 1]; ++k) {
      const int32_t pair = by_cta[k];
      const Piece& pc = pieces[pair / n_head];
      const int head = pair - (pair / n_head) * n_head;
      const Group& g = groups[pc.group];
      const int64_t len = pc.cend - pc.cbeg;
      while (w0 + 1 < kWarps && bnd[w0 + 1] <= x) ++w0;
      int w1 = w0;  // the warp whose run holds the piece's last chunk
      while (w1 + 1 < kWarps && bnd[w1 + 1] <= x + len - 1) ++w1;
      int lcount = 0;  // warps with a non-empty share of this piece (runs can be empty)
      for (int w = w0; w <= w1; ++w) lcount += std::min(x + len, bnd[w + 1]) > std::max(x, bnd[w]);
      if (lcount > 1 && slot + lcount * g.nrows > kLocalSlots)
        return set_error(TQ_ERR_UNSUPPORTED, "internal: CTA %d needs more than %d merge slots", c,
                         kLocalSlots);
      const int32_t w2 = g.nrows | (head << 8) |
                         (((lcount > 1 ? kFlagLocal : 0) | (pc.gnsplit > 1 ? kFlagGlobal : 0) |
                           (q_len[g.seq] == 1 ? kFlagDecode : 0)) << 24);
      const int32_t w6 =
          pc.gnsplit > 1 ? (int32_t)(pc.gbase + (int64_t)head * g.nrows * pc.gnsplit) : -1;
      const int32_t w7 = pc.gsplit | (pc.gnsplit << 16);
      int lsplit = 0;
      for (int w = w0; w <= w1; ++w) {
        const int64_t lo = std::max(x, bnd[w]) - x, hi = std::min(x + len, bnd[w + 1]) - x;
        if (hi <= lo) continue;
        while (cur < w) ranges[wbase + (++cur)] = (int32_t)rest;  // entering warp w
        int32_t* const it = has[w] ? rest_items + 8 * rest++ : first_items + kFirstWords * (wbase + w);
        if (!has[w]) {  // block ids of the first chunk, -1 past them
          const int64_t key0 = (pc.cbeg + lo) * kChunk;
          const int64_t key_end = std::min<int64_t>(key0 + kChunk, g.pos0 + g.nrows);
          const int64_t kb0 = key0 / block_size, kb_end = (key_end - 1) / block_size + 1;
          const int32_t* tbl = table_data + table_offsets[g.seq];
          for (int j = 0; j < kFirstBlocks; ++j) it[8 + j] = kb0 + j < kb_end ? tbl[kb0 + j] : -1;
        }
        has[w] = true;
        it[0] = g.seq;
        it[1] = g.row0;
        it[2] = w2;
        it[3] = g.pos0;
        it[4] = (int32_t)(pc.cbeg + lo) | ((int32_t)(pc.cbeg + hi) << 16);
        it[5] = lcount > 1 ? (lsplit++ | (lcount << 8) | (slot << 16)) : 0;
        it[6] = w6;
        it[7] = w7;
        ++n_items;
        longest = std::max(longest, hi - lo);
      }
      if (lcount > 1) slot += lcount * g.nrows;
      x += len;
    }
    while (cur < kWarps - 1) ranges[wbase + (++cur)] = (int32_t)rest;
    for (int w = 0; w < kWarps; ++w)  // a warp without work: an all-zero first item
      if (!has[w]) std::memset(first_items + kFirstWords * (wbase + w), 0, kFirstWords * sizeof(int32_t));
  }
  // Tile CTAs: warp 0 holds the CTA's tile items (the first at its fixed
  // place, the others in its list); warps 1.. hold a marker (the tile flag
  // alone) that sends them to the CTA's tile code too.
  for (int32_t t = 0; t < n_tctas; ++t) {
    const int64_t wbase = (int64_t)(n_wctas + t) * kWarps;
    const std::vector<int32_t>& list = tile_lists[(size_t)t];
    ranges[wbase] = (int32_t)rest;
    for (size_t k = 0; k < list.size(); ++k) {
      const TilePiece& tp = tpieces[(size_t)(list[k] / n_head)];
      const Tile& tl = tiles[(size_t)tp.tile];
      const int head = list[k] % n_head;
      int32_t* const it = k == 0 ? first_items + kFirstWords * wbase : rest_items + 8 * rest++;
      if (k == 0) {  // the block ids of the first chunk ride along (-1 past them), as for warp items
        const int64_t key0 = (int64_t)tp.cbeg * kChunk;
        const int64_t key_end = std::min<int64_t>(key0 + kChunk, (int64_t)tl.pos0 + tl.nrows);
        const int64_t kb0 = key0 / block_size, kb_end = (key_end - 1) / block_size + 1;
        const int32_t* tbl = table_data + table_offsets[tl.seq];
        for (int j = 0; j < kFirstBlocks; ++j) it[8 + j] = kb0 + j < kb_end ? tbl[kb0 + j] : -1;
      }
      it[0] = tl.seq;
      it[1] = tl.row0;
      it[2] = tl.nrows | (head << 8) | ((kFlagTile | (tp.gnsplit > 1 ? kFlagGlobal : 0)) << 24);
      it[3] = tl.pos0;
      it[4] = tp.cbeg | (tp.cend << 16);
      it[5] = 0;
      it[6] = tp.gnsplit > 1 ? (int32_t)(tp.gbase + (int64_t)head * tl.nrows * tp.gnsplit) : -1;
      it[7] = tp.gsplit | (tp.gnsplit << 16);
      ++n_items;
      longest = std::max<int64_t>(longest, tp.cend - tp.cbeg);
    }
    for (int w = 1; w < kWarps; ++w) {
      ranges[wbase + w] = (int32_t)rest;
      int32_t* const it = first_items + kFirstWords * (wbase + w);
      std::memset(it, 0, kFirstWords * sizeof(int32_t));
      it[2] = kFlagTile << 24;
    }
  }
  ranges[n_warps] = (int32_t)rest;
  std::memset(ranges + n_warps + 1, 0, sizeof(int32_t) * (align8(n_warps + 1) - (n_warps + 1)));
  {  // the tile-merge trailer
    int32_t* const trailer = rest_items + 8 * rest;
    std::memset(trailer, 0, sizeof(int32_t) * trailer_ints);
    trailer[0] = (int32_t)n_tile_merges;
    int32_t* e = trailer + 8;
    for (const TilePiece& tp : tpieces) {
      if (tp.gsplit != 0 || tp.gnsplit < 2) continue;
      const Tile& tl = tiles[(size_t)tp.tile];
      for (int r = 0; r < tl.nrows; ++r, e += 4) {
        e[0] = tl.row0 + r;
        e[1] = (int32_t)(tp.gbase + (int64_t)r * tp.gnsplit);
        e[2] = tp.gnsplit;
        e[3] = tl.nrows * tp.gnsplit;
      }
    }
  }
  const int64_t used = o_rest + 8 * rest + trailer_ints;

  layout[TQ_PLAN_NUM_TOKENS] = (int32_t)N;
  layout[TQ_PLAN_NUM_SEQS] = (int32_t)B;
  layout[TQ_PLAN_NUM_ITEMS] = (int32_t)n_items;
  layout[TQ_PLAN_NUM_COMBINE] = (int32_t)n_combine;
  layout[TQ_PLAN_NUM_PARTIALS] = (int32_t)n_partials;
  layout[TQ_PLAN_TABLE_STRIDE] = (int32_t)max_nb;
  layout[TQ_PLAN_MAX_CTX] = (int32_t)max_ctx;
  layout[TQ_PLAN_SPLIT_CHUNKS] = (int32_t)longest;
  layout[TQ_PLAN_OFF_COUNTS] = (int32_t)o_counts;
  layout[TQ_PLAN_OFF_SEQ_INFO] = (int32_t)o_seq;
  layout[TQ_PLAN_OFF_TABLES] = (int32_t)o_tab;
  layout[TQ_PLAN_OFF_SLOTS] = (int32_t)o_slot;
  layout[TQ_PLAN_OFF_POSITIONS] = (int32_t)o_pos;
  layout[TQ_PLAN_OFF_TOKEN_IDS] = (int32_t)o_ids;
  layout[TQ_PLAN_OFF_LAST_ROWS] = (int32_t)o_last;
  layout[TQ_PLAN_OFF_ITEMS] = (int32_t)o_items;
  layout[TQ_PLAN_OFF_COMBINE] = (int32_t)o_comb;
  layout[TQ_PLAN_NUM_CTAS] = n_ctas;
  layout[TQ_PLAN_USED_INTS] = (int32_t)used;
  layout[TQ_PLAN_NUM_TILE_CTAS] = n_tctas;
  layout[TQ_PLAN_NUM_TILE_MERGES] = (int32_t)n_tile_merges;

  // Everything before the attention plan: zeros first (padding, table tails).
  std::memset(out, 0, sizeof(int32_t) * o_items);
  out[o_counts + 0] = (int32_t)N;
  out[o_counts + 1] = (int32_t)n_items;
  out[o_counts + 2] = (int32_t)n_combine;
  out[o_counts + 3] = (int32_t)B;
  int64_t row = 0, comb = 0;
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
    row += n;
  }
  for (const TilePiece& tp : tpieces) {  // split tiles' rows, likewise
    if (tp.gsplit != 0 || tp.gnsplit < 2) continue;
    const Tile& tl = tiles[(size_t)tp.tile];
    for (int r = 0; r < tl.nrows; ++r) {
      int32_t* e = out + o_comb + 4 * comb++;
      e[0] = tl.row0 + r;
      e[1] = (int32_t)(tp.gbase + (int64_t)r * tp.gnsplit);
      e[2] = tp.gnsplit;
      e[3] = 0;
    }
  }
  for (const Piece& pc : pieces) {  // one combine entry per row whose keys are split across CTAs
    if (pc.gsplit != 0 || pc.gnsplit < 2) continue;
    const Group& g = groups[pc.group];
    for (int r = 0; r < g.nrows; ++r) {
      int32_t* e = out + o_comb + 4 * comb++;
      e[0] = g.row0 + r;
      e[1] = (int32_t)(pc.gbase + (int64_t)r * pc.gnsplit);
      e[2] = pc.gnsplit;
      e[3] = 0;
    }
  }
  return TQ_OK;
}
