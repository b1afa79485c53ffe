// Paged attention over the Tokquay block pool, decode and causal prefill rows
// in one launch, plus the split-K combine.
//
// Replaces the dense gather + masked softmax of the reference
// (tokquay/kv_cache.py:234-242 and tokquay/model.py:94-96): K/V blocks are
// read in place, straight from the pool
//     pool[num_blocks][n_layer][2][n_head][block_size][64]   (fp32)
// and never copied into a dense [B, H, S, d] tensor.
//
// Work decomposition.  The host planner (plan.cpp) cuts every sequence's new
// query rows into groups of up to kMaxRows consecutive rows and the keys each
// group may see (positions 0 .. last row's position, the causal rule of
// kv_cache.py:213-214) into chunks of kChunk keys; a group with many chunks is
// split into several work items (split-K).  One *unit* = (work item, head)
// is processed by one warp.  Decode rows are simply groups of one row.
//
// Pipeline.  Each warp is an independent persistent worker with its own ring
// of kStages shared-memory stages.  Lane 0 issues TMA bulk copies
// (cp.async.bulk, global -> shared, mbarrier completion) for the K and V rows
// of upcoming chunks -- across unit boundaries, so short decode units keep the
// ring full -- while the warp computes on the oldest stage:
//   * QK^T: lane j owns key j of the chunk and reads its 256-byte row with a
//     lane-rotated float4 order (conflict-free), q rows come from shared memory;
//   * online softmax in the log2 domain, state in registers;
//   * PV: lane l owns output dims 2l, 2l+1; probabilities are broadcast by
//     warp shuffles.
// Finished units write either the normalised output row or (split items) an
// un-normalised partial (m, l, acc[64]) that attn_combine_kernel merges.
#pragma once

#include "common.cuh"

namespace tq {

constexpr int kHeadDim = 64;
constexpr int kChunk = 32;    // keys per pipeline stage
constexpr int kMaxRows = 4;   // query rows per work item
constexpr int kStages = 3;    // stages per warp
constexpr int kAttnWarps = 4; // independent warps per CTA

constexpr int kRowBytes = kHeadDim * 4;                        // 256
constexpr int kKBytes = kChunk * kRowBytes;                    // 8 KiB
constexpr int kQBytes = kMaxRows * kRowBytes;                  // 1 KiB
constexpr int kStageBytes = 2 * kKBytes + kQBytes;             // K | V | Q
constexpr int kWarpSmemBytes = kStages * kStageBytes + kQBytes + 64;  // + current q + barriers
constexpr int kAttnSmemBytes = kAttnWarps * kWarpSmemBytes;

// One work item: rows [row0, row0+nrows) of sequence `seq` (absolute
// positions pos0 ..), keys of chunks [cbeg, cend).  Split items (nsplit > 1)
// write partials at part + (r*n_head + h)*nsplit + split.
struct __align__(16) WorkItem {
  int seq, row0, nrows, pos0;
  int cbeg, cend, part, split_nsplit;  // split | nsplit << 16
};
static_assert(sizeof(WorkItem) == 32, "WorkItem is 8 int32");

struct AttnParams {
  float* out;
  long long out_stride;  // floats between output rows; head h at h*64
  const float* q;
  long long q_stride;    // floats between query rows; head h at h*64
  const float* pool;
  long long num_blocks;
  int n_layer, n_head, block_size, log2_bs, layer;
  const int* tables;     // [num_seqs][table_stride] block ids
  int table_stride;
  const WorkItem* items;
  const int* n_items;    // device-resident count
  float* part_ml;        // [P][2]  (m in log2 units, l)
  float* part_acc;       // [P][64]
  float scale_log2;      // log2(e) / sqrt(head_dim)
};

__device__ __forceinline__ size_t pool_tile_offset(const AttnParams& p, long long blk, int kv,
                                                   int h) {
  // Float offset of pool[blk][layer][kv][h][0][0].
  return ((((size_t)blk * p.n_layer + p.layer) * 2 + kv) * p.n_head + h) *
         (size_t)p.block_size * kHeadDim;
}

// Lane 0 only: arm `bar` and issue the bulk copies of chunk c of unit (it, h)
// into `stage`.  The q rows ride along with the unit's first chunk.
__device__ __forceinline__ void issue_chunk(const AttnParams& p, const WorkItem& it, int h, int c,
                                            unsigned char* stage, uint32_t bar) {
  const int kend = min(it.pos0 + it.nrows, it.cend * kChunk);  // this item's last key + 1
  const int key0 = c * kChunk;
  const int nkeys = min(kChunk, kend - key0);
  const bool first = (c == it.cbeg);
  const int* tbl = p.tables + (size_t)it.seq * p.table_stride;
  const int bs = p.block_size;

  // Pass 1: count the bytes that will really be copied (a block id outside
  // the pool is flagged and skipped, so expect_tx always matches).
  uint32_t bytes = first ? (uint32_t)it.nrows * kRowBytes : 0u;
  if (bs <= kChunk) {
    for (int kb = key0 >> p.log2_bs; kb * bs < key0 + nkeys; ++kb) {
      const long long blk = tbl[kb];
      if (blk < 0 || blk >= p.num_blocks) continue;
      const int rows = min(bs, key0 + nkeys - kb * bs);
      bytes += 2u * rows * kRowBytes;
    }
  } else {
    const long long blk = tbl[key0 >> p.log2_bs];
    if (blk >= 0 && blk < p.num_blocks) bytes += 2u * nkeys * kRowBytes;
  }
  mbar_arrive_expect_tx(bar, bytes);

  const uint32_t sK = smem_addr(stage);
  const uint32_t sV = sK + kKBytes;
  const uint32_t sQ = sK + 2 * kKBytes;
  if (first) {
    for (int r = 0; r < it.nrows; ++r)
      bulk_copy_g2s(sQ + r * kRowBytes, p.q + (size_t)(it.row0 + r) * p.q_stride + h * kHeadDim,
                    kRowBytes, bar);
  }
  const size_t kv_stride = (size_t)p.n_head * bs * kHeadDim;  // K tile -> V tile
  if (bs <= kChunk) {
    for (int kb = key0 >> p.log2_bs; kb * bs < key0 + nkeys; ++kb) {
      const long long blk = tbl[kb];
      if (blk < 0 || blk >= p.num_blocks) {
        raise_device_error(TQ_DEVERR_BAD_BLOCK);
        continue;
      }
      const int rows = min(bs, key0 + nkeys - kb * bs);
      const float* src = p.pool + pool_tile_offset(p, blk, 0, h);
      const uint32_t dst_off = (uint32_t)(kb * bs - key0) * kRowBytes;
      bulk_copy_g2s(sK + dst_off, src, rows * kRowBytes, bar);
      bulk_copy_g2s(sV + dst_off, src + kv_stride, rows * kRowBytes, bar);
    }
  } else {
    const long long blk = tbl[key0 >> p.log2_bs];
    if (blk < 0 || blk >= p.num_blocks) {
      raise_device_error(TQ_DEVERR_BAD_BLOCK);
    } else {
      const float* src =
          p.pool + pool_tile_offset(p, blk, 0, h) + (size_t)(key0 & (bs - 1)) * kHeadDim;
      bulk_copy_g2s(sK, src, nkeys * kRowBytes, bar);
      bulk_copy_g2s(sV, src + kv_stride, nkeys * kRowBytes, bar);
    }
  }
}

__global__ void __launch_bounds__(kAttnWarps * 32, 1) paged_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char* wsm = smem + warp * kWarpSmemBytes;
  float* qcur = reinterpret_cast<float*>(wsm + kStages * kStageBytes);
  const uint32_t bar0 = smem_addr(wsm + kStages * kStageBytes + kQBytes);

  const int H = p.n_head;
  const int n_units = *p.n_items * H;
  const int TW = gridDim.x * kAttnWarps;
  int unit = blockIdx.x * kAttnWarps + warp;
  if (unit >= n_units) return;  // warp-uniform; warps never synchronise with each other

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(bar0 + 8 * s, 1);
    mbar_init_fence();
  }
  __syncwarp();

  // Producer cursor (meaningful in lane 0 only).
  int p_unit = unit;
  WorkItem p_it = p.items[p_unit / H];
  int p_chunk = p_it.cbeg;
  bool p_live = true;
  int issued = 0, consumed = 0;

  auto refill = [&]() {
    while (p_live && issued < consumed + kStages) {
      const int s = issued % kStages;
      if (issued >= kStages) fence_proxy_async_smem();  // stage was read by the warp before
      issue_chunk(p, p_it, p_unit % H, p_chunk, wsm + s * kStageBytes, bar0 + 8 * s);
      ++issued;
      if (++p_chunk == p_it.cend) {
        p_unit += TW;
        if (p_unit < n_units) {
          p_it = p.items[p_unit / H];
          p_chunk = p_it.cbeg;
        } else {
          p_live = false;
        }
      }
    }
  };

  WorkItem it = p.items[unit / H];
  int h = unit % H;
  int c = it.cbeg;
  float m[kMaxRows], lsum[kMaxRows];
  float2 acc[kMaxRows];
  bool failed = false;

  if (lane == 0) refill();
  while (true) {
    const int s = consumed % kStages;
    const uint32_t parity = (uint32_t)(consumed / kStages) & 1u;
    const bool ok = mbar_wait_bounded(bar0 + 8 * s, parity);
    if (!__all_sync(kFullMask, ok)) {
      failed = true;
      break;
    }
    unsigned char* stage = wsm + s * kStageBytes;
    const float* K = reinterpret_cast<const float*>(stage);
    const float2* V2 = reinterpret_cast<const float2*>(stage + kKBytes);

    if (c == it.cbeg) {  // first chunk of a unit: take its q rows, reset state
      const float4* qsrc = reinterpret_cast<const float4*>(stage + 2 * kKBytes);
      float4* qdst = reinterpret_cast<float4*>(qcur);
      for (int i = lane; i < it.nrows * (kHeadDim / 4); i += 32) qdst[i] = qsrc[i];
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        m[r] = -INFINITY;
        lsum[r] = 0.f;
        acc[r] = make_float2(0.f, 0.f);
      }
      __syncwarp();
    }

    const int key0 = c * kChunk;
    const int kend = min(it.pos0 + it.nrows, it.cend * kChunk);
    const int nkeys = min(kChunk, kend - key0);

    // ---- scores: lane j <-> key key0 + j ------------------------------------
    float sc[kMaxRows];
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) sc[r] = 0.f;
    const float4* krow = reinterpret_cast<const float4*>(K) + lane * (kHeadDim / 4);
    const float4* q4 = reinterpret_cast<const float4*>(qcur);
#pragma unroll
    for (int i = 0; i < kHeadDim / 4; ++i) {
      const int ch = (i + lane) & (kHeadDim / 4 - 1);
      const float4 k = krow[ch];
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r < it.nrows) {
          const float4 q = q4[r * (kHeadDim / 4) + ch];
          sc[r] = fmaf(q.x, k.x, sc[r]);
          sc[r] = fmaf(q.y, k.y, sc[r]);
          sc[r] = fmaf(q.z, k.z, sc[r]);
          sc[r] = fmaf(q.w, k.w, sc[r]);
        }
      }
    }

    // ---- online softmax update per row --------------------------------------
    float pr[kMaxRows];
#pragma unroll
    for (int r = 0; r < kMaxRows; ++r) {
      pr[r] = 0.f;
      if (r < it.nrows) {
        const int nvalid = min(kChunk, it.pos0 + r + 1 - key0);  // causal: keys <= position
        if (nvalid > 0) {
          const float x = (lane < nvalid) ? sc[r] * p.scale_log2 : -INFINITY;
          const float mn = fmaxf(m[r], warp_max(x));
          const float alpha = exp2f(m[r] - mn);
          pr[r] = exp2f(x - mn);
          lsum[r] = fmaf(lsum[r], alpha, pr[r]);
          acc[r].x *= alpha;
          acc[r].y *= alpha;
          m[r] = mn;
        }
      }
    }

    // ---- PV: lane l owns dims 2l, 2l+1 --------------------------------------
#pragma unroll 4
    for (int j = 0; j < nkeys; ++j) {
      const float2 v = V2[j * (kHeadDim / 2) + lane];
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r < it.nrows) {
          const float pj = __shfl_sync(kFullMask, pr[r], j);
          acc[r].x = fmaf(pj, v.x, acc[r].x);
          acc[r].y = fmaf(pj, v.y, acc[r].y);
        }
      }
    }
    __syncwarp();
    ++consumed;

    if (++c == it.cend) {  // unit finished: write its rows
      const int split = it.split_nsplit & 0xffff;
      const int nsplit = it.split_nsplit >> 16;
#pragma unroll
      for (int r = 0; r < kMaxRows; ++r) {
        if (r < it.nrows) {
          const float l = warp_sum(lsum[r]);
          if (nsplit == 1) {
            const float inv = 1.f / l;
            float2* o = reinterpret_cast<float2*>(p.out + (size_t)(it.row0 + r) * p.out_stride +
                                                  h * kHeadDim);
            o[lane] = make_float2(acc[r].x * inv, acc[r].y * inv);
          } else {
            const size_t idx = (size_t)it.part + ((size_t)r * H + h) * nsplit + split;
            reinterpret_cast<float2*>(p.part_acc + idx * kHeadDim)[lane] = acc[r];
            if (lane == 0) {
              p.part_ml[2 * idx] = m[r];
              p.part_ml[2 * idx + 1] = l;
            }
          }
        }
      }
      unit += TW;
      if (unit >= n_units) break;
      it = p.items[unit / H];
      h = unit % H;
      c = it.cbeg;
    }
    if (lane == 0) refill();
  }

  if (failed) {
    // Drain: give every copy this warp issued a bounded chance to land before
    // the CTA exits, so no bulk copy targets the shared memory of a dead CTA.
    for (int k = consumed; k < issued; ++k) {
      if (!mbar_wait_bounded(bar0 + 8 * (k % kStages), (uint32_t)(k / kStages) & 1u)) break;
    }
  }
}

// Merge split-K partials: one warp per (combine entry, head).
struct CombineParams {
  float* out;
  long long out_stride;
  const float* part_ml;
  const float* part_acc;
  const int4* entries;    // {row, partial base of (row, head 0), nsplit, unused}
  const int* n_entries;   // device-resident count
  int n_head;
};

__global__ void __launch_bounds__(256) attn_combine_kernel(const CombineParams p) {
  const int lane = threadIdx.x & 31;
  const int TW = gridDim.x * (blockDim.x >> 5);
  const int n_units = *p.n_entries * p.n_head;
  for (int u = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units; u += TW) {
    const int4 e = p.entries[u / p.n_head];
    const int h = u % p.n_head;
    const size_t base = (size_t)e.y + (size_t)h * e.z;
    float mmax = -INFINITY;
    for (int s = lane; s < e.z; s += 32) mmax = fmaxf(mmax, p.part_ml[2 * (base + s)]);
    mmax = warp_max(mmax);
    float l = 0.f;
    float2 o = make_float2(0.f, 0.f);
    for (int s = 0; s < e.z; ++s) {
      const float ms = p.part_ml[2 * (base + s)];
      const float w = exp2f(ms - mmax);  // 0 for a split that saw no key of this row
      l = fmaf(p.part_ml[2 * (base + s) + 1], w, l);
      const float2 a = reinterpret_cast<const float2*>(p.part_acc + (base + s) * kHeadDim)[lane];
      o.x = fmaf(a.x, w, o.x);
      o.y = fmaf(a.y, w, o.y);
    }
    const float inv = 1.f / l;
    reinterpret_cast<float2*>(p.out + (size_t)e.x * p.out_stride + h * kHeadDim)[lane] =
        make_float2(o.x * inv, o.y * inv);
  }
}

}  // namespace tq
