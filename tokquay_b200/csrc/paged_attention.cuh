// Paged attention over the Tokquay block pool, decode and causal prefill rows
// in one launch, every merge of split keys included.
//
// Replaces the dense gather + masked softmax of the reference
// (tokquay/kv_cache.py:234-242 and tokquay/model.py:94-96): K/V blocks are
// read in place, straight from the pool
//     pool[num_blocks][n_layer][2][n_head][block_size][64]   (fp32)
// and never copied into a dense [B, H, S, d] tensor.
//
// Work decomposition.  The host planner (plan.cpp) cuts every sequence's new
// query rows into groups of up to kMaxRows consecutive rows; a (row group,
// head) pair attends to keys 0 .. its last row's position (the causal rule of
// kv_cache.py:213-214), a run of kChunk-key chunks.  Pairs go to the grid's
// CTAs longest first (each to the least loaded CTA), and each CTA's chunks are
// cut evenly over its kAttnWarps computing warps, so a pair may be shared by
// neighbouring warps.  Those cuts are merged through shared memory once the
// CTA's warps are done -- no global fence, no atomic.  Only a pair longer than
// a CTA's share is split across CTAs; those pieces are merged through split-K
// scratch by the last one to finish (acq_rel counter).  A work item is one
// warp's share of one pair: rows, head, chunk range, merge target.
//
// Pipeline.  Each computing (consumer) warp has a producer warp and a ring of
// kStages shared-memory stages.  The producer walks the same work items,
// prefetches item metadata two items ahead and block ids one item ahead, and
// issues TMA bulk copies (cp.async.bulk, global -> shared, mbarrier
// completion) for the K and V rows of upcoming chunks -- one copy per lane,
// one warp instruction per chunk -- as soon as the consumer releases a stage.
// Each stage carries a header with the item, so the consumer never reads
// work metadata from global memory.  Per chunk the consumer does:
//   * QK^T and PV with lane = (key group, quarter of the head dims): q rows
//     and output accumulators live in registers, 4 passes of 8 keys cover
//     the chunk, shared loads are conflict-free (see attend_chunk);
//   * online softmax in the log2 domain, state in registers.
// A finished item writes the normalised output row, or an unnormalised
// partial (m, l, acc[64]) to its shared slot or split-K slot.
#pragma once

#include "common.cuh"

namespace tq {

// Pipeline shape (overridable at build time for tuning sweeps).
#ifndef TQ_ATTN_CHUNK
#define TQ_ATTN_CHUNK 32
#endif
#ifndef TQ_ATTN_MAX_ROWS
#define TQ_ATTN_MAX_ROWS 2
#endif
#ifndef TQ_ATTN_STAGES
#define TQ_ATTN_STAGES 2
#endif
#ifndef TQ_ATTN_WARPS
#define TQ_ATTN_WARPS 6
#endif
constexpr int kHeadDim = 64;
constexpr int kChunk = TQ_ATTN_CHUNK;        // keys per pipeline stage (16 or 32)
constexpr int kMaxRows = TQ_ATTN_MAX_ROWS;   // query rows per work item
constexpr int kStages = TQ_ATTN_STAGES;      // stages per warp
constexpr int kAttnWarps = TQ_ATTN_WARPS;    // independent warps per CTA
constexpr int kPasses = kChunk / 8;          // 8 keys per pass (lane = key group x dim quarter)
constexpr int kUnitBlocks = 64;              // most blocks one work item's key range may span
static_assert(kChunk == 16 || kChunk == 32, "chunk of 16 or 32 keys");

#ifdef TQ_ATTN_TRACE
// Tuning builds only: per-warp timeline of the last launch, [warp][16] =
// {start ns, first data ns, end ns, wait, compute, finish, SM id, chunks,
//  issue:block-id wait, issue:copies, advance, finish:reduce+store,
//  finish:fence+atomic, finish:merge, producer entry ns, producer end ns}
// (cycles unless noted).
// Read back with tq_debug_attention_trace.
constexpr int kTraceWarps = 8192;
// Per layer: the first CTA entry (ns) of the latest launches (reset by the host).
__device__ unsigned long long g_attn_entry[64];
constexpr int kTraceSlots = 16;
__device__ unsigned long long g_attn_trace[kTraceWarps * kTraceSlots];
// Per warp, per chunk (first kTraceChunks): {issue ns, data-ready ns, bytes}.
constexpr int kTraceChunks = 32;
__device__ unsigned long long g_attn_chunks[kTraceWarps * kTraceChunks * 3];
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define TQ_TRACE(...) __VA_ARGS__
#define TQ_TRACE_ARG(x) x
#else
#define TQ_TRACE(...)
#define TQ_TRACE_ARG(x) nullptr
#endif

constexpr int kRowBytes = kHeadDim * 4;                        // 256
constexpr int kKBytes = kChunk * kRowBytes;                    // 8 KiB
constexpr int kQBytes = kMaxRows * kRowBytes;                  // 1 KiB
constexpr int kHeaderBytes = 64;                               // StageHeader, padded
constexpr int kStageBytes = 2 * kKBytes + kQBytes + kHeaderBytes;  // K | V | Q | header
constexpr int kWarpSmemBytes = kStages * kStageBytes + 64;  // + barriers

// Shared-memory partials of keys cut between warps of one CTA: one slot per
// (piece, row) = {m, l, -, -, acc[64]} floats.  Each warp boundary cuts at
// most one (row group, head) pair, so 2 * (warps - 1) * max_rows slots hold
// every cut (the planner's bound).
constexpr int kLocalSlots = 2 * (kAttnWarps - 1) * kMaxRows;
constexpr int kSlotFloats = 4 + kHeadDim;
constexpr int kLocalBytes = kLocalSlots * kSlotFloats * 4;
constexpr int kAttnSmemBytes = kAttnWarps * kWarpSmemBytes + kLocalBytes;

// One work item (8 int32, written by the planner): query rows
// [row0, row0+nrows) of sequence seq (absolute positions pos0 ..), head, the
// keys of chunks [cbeg, cend).  Keys of one (row group, head) pair cut between
// warps of a CTA (flag kLocal) go to shared-memory slots lslot + r*lcount +
// lsplit and are merged by the warp holding lsplit 0 once the CTA's warps are
// done; pairs split across CTAs (flag kGlobal) go to split-K partials
// gbase + r*gnsplit + gsplit, merged by the last split to finish.
//   w[0] seq   w[1] row0   w[2] nrows | head << 8 | flags << 24   w[3] pos0
//   w[4] cbeg | cend << 16   w[5] lsplit | lcount << 8 | lslot << 16
//   w[6] gbase   w[7] gsplit | gnsplit << 16
// An all-zero item (cend == 0) marks a warp without work.
constexpr int kFlagLocal = 1, kFlagGlobal = 2;
// The item's sequence feeds one token this step: pos0 is its only new key.
constexpr int kFlagDecode = 4;
constexpr int kMergeFlags = kFlagLocal | kFlagGlobal;
struct __align__(16) WorkItem {
  int w[8];
  __device__ __forceinline__ int seq() const { return w[0]; }
  __device__ __forceinline__ int row0() const { return w[1]; }
  __device__ __forceinline__ int nrows() const { return w[2] & 0xff; }
  __device__ __forceinline__ int head() const { return (w[2] >> 8) & 0xffff; }
  __device__ __forceinline__ int flags() const { return (int)((unsigned)w[2] >> 24); }
  __device__ __forceinline__ int pos0() const { return w[3]; }
  __device__ __forceinline__ int cbeg() const { return w[4] & 0xffff; }
  __device__ __forceinline__ int cend() const { return (int)((unsigned)w[4] >> 16); }
  __device__ __forceinline__ int lsplit() const { return w[5] & 0xff; }
  __device__ __forceinline__ int lcount() const { return (w[5] >> 8) & 0xff; }
  __device__ __forceinline__ int lslot() const { return (int)((unsigned)w[5] >> 16); }
  __device__ __forceinline__ int gbase() const { return w[6]; }
  __device__ __forceinline__ int gsplit() const { return w[7] & 0xffff; }
  __device__ __forceinline__ int gnsplit() const { return (int)((unsigned)w[7] >> 16); }
};
static_assert(sizeof(WorkItem) == 32, "WorkItem is 8 int32");

// Written into each stage by the producer together with the copies, so the
// consumer never reads work metadata from global memory.
struct StageHeader {
  WorkItem it;
  int c, pad0, pad1, pad2;
};
static_assert(sizeof(StageHeader) <= kHeaderBytes, "header fits its slot");

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
  const int* attn;       // attention plan: [W][8] first items, [W+1] offsets (padded to 8), other items
  int n_warps;           // W = grid * kAttnWarps
  float* part_ml;        // [P][2]  (m in log2 units, l)
  float* part_acc;       // [P][64]
  int* part_cnt;         // [P] split counters (zero between launches)
  int max_partials;      // P
  float scale_log2;      // log2(e) / sqrt(head_dim)
};

// A work item's merge targets lie inside the shared slots and the split-K
// scratch; one that does not (a corrupted plan) is flagged and not written.
__device__ __forceinline__ bool merge_targets_ok(const AttnParams& p, const WorkItem& it) {
  const int f = it.flags() & kMergeFlags;
  bool ok = true;
  if (f & kFlagLocal)
    ok = it.lcount() >= 2 && it.lsplit() < it.lcount() && it.lslot() + it.nrows() * it.lcount() <= kLocalSlots;
  if (f & kFlagGlobal)
    ok = ok && it.gbase() >= 0 && it.gsplit() < it.gnsplit() &&
         (long long)it.gbase() + (long long)it.nrows() * it.gnsplit() <= p.max_partials;
  if (!ok && (threadIdx.x & 31) == 0) raise_device_error(TQ_DEVERR_BAD_PLAN);
  return ok;
}

__device__ __forceinline__ size_t pool_tile_offset(const AttnParams& p, long long blk, int kv,
                                                   int h) {
  // Float offset of pool[blk][layer][kv][h][0][0].
  return ((((size_t)blk * p.n_layer + p.layer) * 2 + kv) * p.n_head + h) *
         (size_t)p.block_size * kHeadDim;
}

// Lanes 0..7 hold the 8 ints of a work item; every lane gets them all.
__device__ __forceinline__ WorkItem item_from_lanes(int v) {
  WorkItem it;
#pragma unroll
  for (int i = 0; i < 8; ++i) it.w[i] = __shfl_sync(kFullMask, v, i);
  return it;
}

// Word `lane` (lanes 0..7) of item k of warp slot `ws`: k == 0 is the warp's
// first item, at a fixed place (kFirstWords words: the item, then the block
// ids of its first chunk), so its load needs no offset; items k >= 1 follow
// the warp's offset r0 in the list of the others.
constexpr int kFirstWords = 16;
constexpr int kFirstBlocks = kFirstWords - 8;
__device__ __forceinline__ const int* warp_offsets(const AttnParams& p) { return p.attn + kFirstWords * p.n_warps; }
__device__ __forceinline__ const int* other_items(const AttnParams& p) {
  return p.attn + kFirstWords * p.n_warps + ((p.n_warps + 1 + 7) & ~7);
}
__device__ __forceinline__ int item_lane_load(const AttnParams& p, int ws, int r0, int k, int count, int lane) {
  if (k >= count || lane >= 8) return 0;
  const int* src = k == 0 ? p.attn + kFirstWords * (size_t)ws : other_items(p) + 8 * (size_t)(r0 + k - 1);
  return __ldg(src + lane);
}

// Keys [key0, key0+nkeys) of chunk c, and the blocks [kb0, kb0+nblk) they live in.
struct ChunkSpan {
  int key0, nkeys, kb0, nblk;
};

__device__ __forceinline__ ChunkSpan chunk_span(const AttnParams& p, const WorkItem& it, int c) {
  ChunkSpan sp;
  const int kend = min(it.pos0() + it.nrows(), it.cend() * kChunk);  // this item's last key + 1
  sp.key0 = c * kChunk;
  sp.nkeys = min(kChunk, kend - sp.key0);
  sp.kb0 = sp.key0 >> p.log2_bs;
  sp.nblk = p.block_size <= kChunk ? ((sp.key0 + sp.nkeys - 1) >> p.log2_bs) - sp.kb0 + 1 : 1;
  return sp;
}

// Lane layout inside a chunk of kChunk keys: lane = g*4 + qq, with g (0..7)
// a key group and qq (0..3) a quarter of the 64 head dims.  Pass t
// (0..kPasses-1) covers key t*8 + g.  A lane keeps its quarter of each q row and of each
// output accumulator in registers, as 4 float4 "slots": slot i holds float4
// (i + rot) & 3 of the quarter, rot = (qq >> 1) + 2*(g & 1).  With that
// rotation the 8 lanes of every quarter-warp read 8 different 16-byte bank
// groups of a 256-byte K or V row, so the shared loads are conflict-free.
// Scores need 2 shuffles per pass (sum over quarters); PV needs none (a lane
// already holds the probabilities of its own keys); the reductions over key
// groups happen once per unit, in finish_rows().
__device__ __forceinline__ int lane_rot(int lane) { return ((lane & 3) >> 1) + 2 * ((lane >> 2) & 1); }

template <int NR>
__device__ __forceinline__ void attend_chunk(const float* __restrict__ K, const float* __restrict__ V,
                                             const float4 (&q)[kMaxRows][4], int nrows, int pos0,
                                             int key0, int nkeys, float scale_log2, int lane,
                                             float (&m)[kMaxRows], float (&lsum)[kMaxRows],
                                             float4 (&acc)[kMaxRows][4]) {
  const int g = lane >> 2, qq = lane & 3, rot = lane_rot(lane);
  // ---- scores: sc[r][t] = q_r . k_{t*8+g} ------------------------------------
  float sc[NR][kPasses];
#pragma unroll
  for (int t = 0; t < kPasses; ++t) {
    const float4* krow = reinterpret_cast<const float4*>(K + (t * 8 + g) * kHeadDim + qq * 16);
    float4 k[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) k[i] = krow[(i + rot) & 3];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float a = q[r][0].x * k[0].x, b = q[r][0].y * k[0].y;
      a = fmaf(q[r][0].z, k[0].z, a);
      b = fmaf(q[r][0].w, k[0].w, b);
#pragma unroll
      for (int i = 1; i < 4; ++i) {
        a = fmaf(q[r][i].x, k[i].x, a);
        b = fmaf(q[r][i].y, k[i].y, b);
        a = fmaf(q[r][i].z, k[i].z, a);
        b = fmaf(q[r][i].w, k[i].w, b);
      }
      sc[r][t] = a + b;
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int t = 0; t < kPasses; ++t) {
      sc[r][t] += __shfl_xor_sync(kFullMask, sc[r][t], 1);
      sc[r][t] += __shfl_xor_sync(kFullMask, sc[r][t], 2);
    }

  // ---- online softmax update per row (causal: keys <= the row's position) ----
  float pr[NR][kPasses];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
#pragma unroll
    for (int t = 0; t < kPasses; ++t) pr[r][t] = 0.f;
    if (NR == 1 || r < nrows) {
      const int nvalid = min(kChunk, pos0 + r + 1 - key0);
      if (nvalid > 0) {
        float x[kPasses];
#pragma unroll
        for (int t = 0; t < kPasses; ++t) x[t] = (t * 8 + g < nvalid) ? sc[r][t] * scale_log2 : -INFINITY;
        float mx = x[0];
#pragma unroll
        for (int t = 1; t < kPasses; ++t) mx = fmaxf(mx, x[t]);
        mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(kFullMask, mx, 16));
        const float mn = fmaxf(m[r], mx);
        const float alpha = exp2f(m[r] - mn);  // 0 while m is still -inf
        float psum = 0.f;
#pragma unroll
        for (int t = 0; t < kPasses; ++t) {
          pr[r][t] = exp2f(x[t] - mn);
          psum += pr[r][t];
        }
        lsum[r] = fmaf(lsum[r], alpha, psum);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[r][i].x *= alpha;
          acc[r][i].y *= alpha;
          acc[r][i].z *= alpha;
          acc[r][i].w *= alpha;
        }
        m[r] = mn;
      }
    }
  }

  // ---- PV over this lane's keys (rows past nkeys were not copied: skip them) --
#pragma unroll
  for (int t = 0; t < kPasses; ++t) {
    if (t * 8 + g < nkeys) {
      const float4* vrow = reinterpret_cast<const float4*>(V + (t * 8 + g) * kHeadDim + qq * 16);
      float4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = vrow[(i + rot) & 3];
#pragma unroll
      for (int r = 0; r < NR; ++r) {
        const float pp = pr[r][t];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[r][i].x = fmaf(pp, v[i].x, acc[r][i].x);
          acc[r][i].y = fmaf(pp, v[i].y, acc[r][i].y);
          acc[r][i].z = fmaf(pp, v[i].z, acc[r][i].z);
          acc[r][i].w = fmaf(pp, v[i].w, acc[r][i].w);
        }
      }
    }
  }
}

// Split-K merge across CTAs: the warp that writes the last partial of a (row,
// head) merges all of them into the output row.  Each (row, head) has a
// counter in part_cnt (at the index of its split 0 partial); every split
// publishes its partial, then bumps the counter (release: the partial is
// visible before the count says so; acquire: the last split sees every other
// split's partial).  The one that sees nsplit - 1 reads the partials back
// through L2 and resets the counter to 0, so the scratch is ready for the next
// launch without a memset.
__device__ __forceinline__ void merge_global_if_last(const AttnParams& p, size_t idx0, int nsplit, int out_row,
                                                     int h, int lane, long long* tr_sub) {
  __syncwarp();  // the lanes' partial stores are ordered before lane 0's release
  TQ_TRACE(long long tm0 = clock64();)
  int last = 0;
  if (lane == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(p.part_cnt + idx0) : "memory");
    last = old == nsplit - 1;
  }
  last = __shfl_sync(kFullMask, last, 0);
  TQ_TRACE(if (lane == 0) tr_sub[4] += clock64() - tm0; tm0 = clock64();)
  if (!last) return;
  __syncwarp();  // lane 0's acquire orders the other lanes' reads of the partials below
  float mmax = -INFINITY;
  for (int s = lane; s < nsplit; s += 32) mmax = fmaxf(mmax, __ldcg(p.part_ml + 2 * (idx0 + s)));
  mmax = warp_max(mmax);
  float l = 0.f;
  float2 o = make_float2(0.f, 0.f);
  for (int s = 0; s < nsplit; ++s) {
    const float ms = __ldcg(p.part_ml + 2 * (idx0 + s));
    const float w = ms == -INFINITY ? 0.f : exp2f(ms - mmax);  // 0 for a split without keys
    l = fmaf(__ldcg(p.part_ml + 2 * (idx0 + s) + 1), w, l);
    const float2 a = __ldcg(reinterpret_cast<const float2*>(p.part_acc + (idx0 + s) * kHeadDim) + lane);
    o.x = fmaf(a.x, w, o.x);
    o.y = fmaf(a.y, w, o.y);
  }
  const float inv = 1.f / l;
  reinterpret_cast<float2*>(p.out + (size_t)out_row * p.out_stride + h * kHeadDim)[lane] =
      make_float2(o.x * inv, o.y * inv);
  if (lane == 0) p.part_cnt[idx0] = 0;
  TQ_TRACE(if (lane == 0) tr_sub[5] += clock64() - tm0;)
}

// End of a work item: sum l and the accumulators over the 8 key groups (lanes
// xor 4, 8, 16; partners across xor 4 hold their slots rotated by 2) and write
// each row: the normalised output, a shared-memory partial (keys cut between
// this CTA's warps) or a split-K partial (keys split across CTAs).
__device__ __forceinline__ void finish_rows(const AttnParams& p, const WorkItem& it, int lane,
                                            const float (&m)[kMaxRows], float (&lsum)[kMaxRows],
                                            float4 (&acc)[kMaxRows][4], float* local, long long* tr_sub) {
  TQ_TRACE(const long long tf0 = clock64(); if (lane == 0) tr_sub[6] += 1;)
  const int qq = lane & 3, rot = lane_rot(lane);
  const int flags = it.flags() & kMergeFlags, h = it.head();
  if (flags != 0 && !merge_targets_ok(p, it)) return;
#pragma unroll
  for (int r = 0; r < kMaxRows; ++r) {
    if (r < it.nrows()) {
      float l = lsum[r];
      l += __shfl_xor_sync(kFullMask, l, 4);
      l += __shfl_xor_sync(kFullMask, l, 8);
      l += __shfl_xor_sync(kFullMask, l, 16);
      float4 other[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 a = acc[r][(i + 2) & 3];
        other[i] = make_float4(__shfl_xor_sync(kFullMask, a.x, 4), __shfl_xor_sync(kFullMask, a.y, 4),
                               __shfl_xor_sync(kFullMask, a.z, 4), __shfl_xor_sync(kFullMask, a.w, 4));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 a = acc[r][i];
        a.x += other[i].x;
        a.y += other[i].y;
        a.z += other[i].z;
        a.w += other[i].w;
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1) {
          a.x += __shfl_xor_sync(kFullMask, a.x, o);
          a.y += __shfl_xor_sync(kFullMask, a.y, o);
          a.z += __shfl_xor_sync(kFullMask, a.z, o);
          a.w += __shfl_xor_sync(kFullMask, a.w, o);
        }
        acc[r][i] = a;
      }
      if (lane < 4) {  // key group 0 writes the row: 4 lanes x 64 bytes
        if (flags == 0) {
          const float inv = 1.f / l;
          float4* o = reinterpret_cast<float4*>(p.out + (size_t)(it.row0() + r) * p.out_stride +
                                                h * kHeadDim + qq * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[(i + rot) & 3] = make_float4(acc[r][i].x * inv, acc[r][i].y * inv, acc[r][i].z * inv,
                                           acc[r][i].w * inv);
        } else {
          float* ml;
          float4* o;
          if (flags & kFlagLocal) {
            float* sl = local + (size_t)(it.lslot() + r * it.lcount() + it.lsplit()) * kSlotFloats;
            ml = sl;
            o = reinterpret_cast<float4*>(sl + 4 + qq * 16);
          } else {
            const size_t idx = (size_t)it.gbase() + (size_t)r * it.gnsplit() + it.gsplit();
            ml = p.part_ml + 2 * idx;
            o = reinterpret_cast<float4*>(p.part_acc + idx * kHeadDim + qq * 16);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) o[(i + rot) & 3] = acc[r][i];
          if (lane == 0) {
            ml[0] = m[r];
            ml[1] = l;
          }
        }
      }
      TQ_TRACE(if (lane == 0) tr_sub[3] += clock64() - tf0;)
      if (flags == kFlagGlobal)
        merge_global_if_last(p, (size_t)it.gbase() + (size_t)r * it.gnsplit(), it.gnsplit(), it.row0() + r, h,
                             lane, tr_sub);
    }
  }
}

// After every warp of the CTA is done: merge the shared-memory partials of
// the pair whose lsplit-0 piece this warp ran, into the output row or (keys
// also split across CTAs) into this CTA's split-K partial.
__device__ __forceinline__ void merge_local(const AttnParams& p, const WorkItem& it, const float* local,
                                            int lane, long long* tr_sub) {
  const int k = it.lcount(), h = it.head();
  for (int r = 0; r < it.nrows(); ++r) {
    const float* s0 = local + (size_t)(it.lslot() + r * k) * kSlotFloats;
    float mmax = -INFINITY;
    for (int s = 0; s < k; ++s) mmax = fmaxf(mmax, s0[s * kSlotFloats]);
    float l = 0.f;
    float2 o = make_float2(0.f, 0.f);
    for (int s = 0; s < k; ++s) {
      const float* sl = s0 + s * kSlotFloats;
      const float w = sl[0] == -INFINITY ? 0.f : exp2f(sl[0] - mmax);  // 0 for a piece without keys
      l = fmaf(sl[1], w, l);
      const float2 a = reinterpret_cast<const float2*>(sl + 4)[lane];
      o.x = fmaf(a.x, w, o.x);
      o.y = fmaf(a.y, w, o.y);
    }
    if (it.flags() & kFlagGlobal) {
      const size_t idx0 = (size_t)it.gbase() + (size_t)r * it.gnsplit();
      const size_t idx = idx0 + it.gsplit();
      reinterpret_cast<float2*>(p.part_acc + idx * kHeadDim)[lane] = o;
      if (lane == 0) {
        p.part_ml[2 * idx] = mmax;
        p.part_ml[2 * idx + 1] = l;
      }
      merge_global_if_last(p, idx0, it.gnsplit(), it.row0() + r, h, lane, tr_sub);
    } else {
      const float inv = 1.f / l;
      reinterpret_cast<float2*>(p.out + (size_t)(it.row0() + r) * p.out_stride + h * kHeadDim)[lane] =
          make_float2(o.x * inv, o.y * inv);
    }
  }
}

}  // namespace tq

#include "prompt_tile.cuh"

namespace tq {

// Block layout: warps 0..kAttnWarps-1 are consumers, warps kAttnWarps.. their
// producers; consumer w and producer kAttnWarps+w share ring w and walk the
// same work items (the planner's list for warp slot blockIdx.x*kAttnWarps+w).
constexpr int kAttnThreads = 2 * kAttnWarps * 32;

// kTiles: the kernel also carries the prompt-tile role (prompt_tile.cuh).
// The variant without it serves plans without tile CTAs (every decode step):
// the tile code's register and call overhead would cost its launches ~1.5 %
// (measured on config 2: 21.9 vs 21.6 us).
template <bool kTiles>
__global__ void __launch_bounds__(kAttnThreads, 1) paged_attention_kernel(const AttnParams p) {
  TQ_TRACE(const unsigned long long tr_entry = global_ns();
           if (threadIdx.x == 0 && p.layer < 64) atomicMin(&g_attn_entry[p.layer], tr_entry);)
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool producer = warp >= kAttnWarps;
  const int pair = producer ? warp - kAttnWarps : warp;
  unsigned char* wsm = smem + pair * kWarpSmemBytes;
  float* local = reinterpret_cast<float*>(smem + kAttnWarps * kWarpSmemBytes);
  const uint32_t full0 = smem_addr(wsm + kStages * kStageBytes);  // TMA bytes landed
  const uint32_t empty0 = full0 + 8 * kStages;                    // consumer done reading

  const int H = p.n_head;
  const int ws = blockIdx.x * kAttnWarps + pair;
  // The first item sits at a fixed place: its load and the offsets' load go out together.
  const int first_word = lane < kFirstWords ? __ldg(p.attn + kFirstWords * (size_t)ws + lane) : 0;
  const int r0 = __ldg(warp_offsets(p) + ws), r1 = __ldg(warp_offsets(p) + ws + 1);
  const bool has_work = ((unsigned)__shfl_sync(kFullMask, first_word, 4) >> 16) != 0;  // cend != 0
  const int count = has_work ? 1 + r1 - r0 : 0;
  TQ_TRACE(const int gw = ws; unsigned long long* trec = g_attn_trace + (size_t)gw * kTraceSlots;
           long long tr_sub[8] = {0, 0, 0, 0, 0, 0, 0, 0};)

  pdl_launch_dependents();  // a following dependent launch may stage its own prologue
  // Every warp slot of a prompt-tile CTA carries the tile flag: the whole CTA
  // runs its tile items on the tensor cores (prompt_tile.cuh).
  const bool tile_cta = ((unsigned)__shfl_sync(kFullMask, first_word, 2) >> 24) & kFlagTile;
#ifdef TQ_TILE_DEBUG
  if (threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_cta_time[3 * blockIdx.x] = t;
    g_cta_time[3 * blockIdx.x + 2] = tile_cta ? 1 : 0;
  }
#define TQ_CTA_END()                                               \
  do {                                                             \
    unsigned long long t_;                                         \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));         \
    if ((threadIdx.x & 31) == 0) atomicMax(&g_cta_time[3 * blockIdx.x + 1], t_); \
  } while (0)
#else
#define TQ_CTA_END() do { } while (0)
#endif
  if constexpr (!kTiles) {
    if (tile_cta) {  // a plan with tile CTAs, launched on the variant without them
      if (threadIdx.x == 0) raise_device_error(TQ_DEVERR_BAD_PLAN);
      return;
    }
  } else if (tile_cta) {
    // The tile code reads the parameters from shared memory: passed by
    // reference, the kernel's would be copied to (slow, under load) local memory.
    AttnParams* const sp = reinterpret_cast<AttnParams*>(smem + kTileOffParams);
    if (threadIdx.x == 0) *sp = p;
    __syncthreads();
    prompt_tile_cta(*sp, smem);
    TQ_CTA_END();
    return;
  }

  if (!producer && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);   // the producer's arrive_expect_tx + the copies' bytes
      mbar_init(empty0 + 8 * s, 1);  // the consumer's arrive
    }
    mbar_init_fence();
  }
  __syncthreads();  // every ring's barriers are initialised before either warp of a pair uses them

  if (producer) {
    if (count == 0) return;
    // ---- producer: work metadata and TMA issue, up to kStages chunks ahead ----
    // Block ids of the current item's key range (at most kUnitBlocks; the
    // planner keeps items that short) live in two registers per lane: lane i
    // holds blocks kb0+i and kb0+32+i.  They are loaded one item ahead, and
    // the item itself two ahead, so neither load sits between two issues.
    int p_k = 0;
    WorkItem p_it = item_from_lanes(first_word);
    int p_chunk = p_it.cbeg();
    int pf_a = 0, pf_b = 0;  // current item's block ids
    int nx_a = 0, nx_b = 0;  // next item's block ids (in flight)
    // The first chunk's block ids came with the item (lane j: block j), so
    // its copies go out now; the item's whole list loads meanwhile.
    const int first_ids = __shfl_sync(kFullMask, first_word, 8 + (lane & (kFirstBlocks - 1)));
    int full_a = 0, full_b = 0;
    auto load_item_blocks = [&](const WorkItem& w, bool valid, int& a, int& b) {
      if (!valid) return;
      const int kb0 = (w.cbeg() * kChunk) >> p.log2_bs;
      const int kend = min(w.pos0() + w.nrows(), w.cend() * kChunk);
      const int n = ((kend - 1) >> p.log2_bs) - kb0 + 1;
      const int* tbl = p.tables + (size_t)w.seq() * p.table_stride + kb0;
      a = lane < n ? __ldg(tbl + lane) : 0;
      b = lane + 32 < n ? __ldg(tbl + 32 + lane) : 0;
    };
    load_item_blocks(p_it, true, full_a, full_b);
    const bool inline_first = chunk_span(p, p_it, p_chunk).nblk <= kFirstBlocks;  // warp-uniform
    if (inline_first) {
      pf_a = lane < kFirstBlocks ? first_ids : 0;
    } else {
      pf_a = full_a;
      pf_b = full_b;
    }
    WorkItem nx_it = item_from_lanes(item_lane_load(p, ws, r0, 1, count, lane));
    load_item_blocks(nx_it, 1 < count, nx_a, nx_b);
    int nx2_word = item_lane_load(p, ws, r0, 2, count, lane);
    int issued = 0;
    bool ok = true;
    bool more = true;  // the cursor still holds a chunk to issue
    // Issue chunk p_chunk of the current item into the next stage (waiting
    // for the consumer to release it), then advance the cursor.  defer_q
    // leaves the item's q rows out: their bytes are in the stage's count, and
    // their copies go out later.
    auto issue_next = [&](bool defer_q) {
      const int s = issued % kStages;
      if (issued >= kStages) {  // wait for the consumer to release the stage
        ok = mbar_wait_bounded(empty0 + 8 * s, (uint32_t)(issued / kStages - 1) & 1u);
        if (!__all_sync(kFullMask, ok)) {
          ok = false;
          return;
        }
      }
      // Issue chunk p_chunk of the current item into stage s.  Each lane
      // describes one copy (K or V rows of one block, or a q row), and the
      // copies go out as one warp-wide cp.async.bulk.
      unsigned char* stage = wsm + s * kStageBytes;
      const uint32_t bar = full0 + 8 * s;
      const ChunkSpan sp = chunk_span(p, p_it, p_chunk);
      const bool first = (p_chunk == p_it.cbeg());
      const int bs = p.block_size;
      const int h = p_it.head();
      const int item_kb0 = (p_it.cbeg() * kChunk) >> p.log2_bs;
      const int n_kv = 2 * sp.nblk;
      const int n_desc = n_kv + (first ? p_it.nrows() : 0);
      const uint32_t sK = smem_addr(stage);
      const size_t kv_stride = (size_t)H * bs * kHeadDim;  // K tile -> V tile
      TQ_TRACE(long long ti0 = clock64();)
      auto describe = [&](int d, const float*& src, uint32_t& dst, uint32_t& bytes) {
        // Every lane shuffles (the source lane varies per lane).
        const int rel = (sp.kb0 - item_kb0) + min(d, max(n_kv - 1, 0)) / 2;
        const int a = __shfl_sync(kFullMask, pf_a, rel & 31);
        const int b = __shfl_sync(kFullMask, pf_b, rel & 31);
        bytes = 0;
        if (d < n_kv) {
          const long long blk = rel < 32 ? a : b;
          if (blk < 0 || blk >= p.num_blocks) {
            raise_device_error(TQ_DEVERR_BAD_BLOCK);
            return;
          }
          const int kv = d & 1;
          if (bs <= kChunk) {
            const int kb = sp.kb0 + (d >> 1);
            const int rows = min(bs, sp.key0 + sp.nkeys - kb * bs);
            src = p.pool + pool_tile_offset(p, blk, 0, h) + kv * kv_stride;
            dst = sK + kv * kKBytes + (uint32_t)(kb * bs - sp.key0) * kRowBytes;
            bytes = rows * kRowBytes;
          } else {
            src = p.pool + pool_tile_offset(p, blk, 0, h) + kv * kv_stride +
                  (size_t)(sp.key0 & (bs - 1)) * kHeadDim;
            dst = sK + kv * kKBytes;
            bytes = sp.nkeys * kRowBytes;
          }
        } else if (d < n_desc) {
          const int r = d - n_kv;
          src = p.q + (size_t)(p_it.row0() + r) * p.q_stride + h * kHeadDim;
          dst = sK + 2 * kKBytes + r * kRowBytes;
          bytes = kRowBytes;
        }
      };
      // Descriptors 0..31 stay in registers between the byte count and the
      // issue; more than 32 (block_size < 16) are described twice.
      const float* src0 = nullptr;
      uint32_t dst0 = 0, bytes0 = 0;
      describe(lane, src0, dst0, bytes0);
      uint32_t total = __reduce_add_sync(kFullMask, bytes0);
      for (int base = 32; base < n_desc; base += 32) {
        const float* src = nullptr;
        uint32_t dst = 0, bytes = 0;
        describe(base + lane, src, dst, bytes);
        total += __reduce_add_sync(kFullMask, bytes);
      }
      TQ_TRACE(if (lane == 0) tr_sub[0] += clock64() - ti0; ti0 = clock64();)
      if (lane == 0) {
        if (first) {  // the consumer picks the item up from here
          StageHeader* hd = reinterpret_cast<StageHeader*>(stage + 2 * kKBytes + kQBytes);
          hd->it = p_it;
          hd->c = p_chunk;
        }
        // Releases the header store to the consumer's acquiring wait.  A
        // reused stage needs no proxy fence: the consumer's reads of it fed
        // arithmetic that completed before its arrive on the empty barrier.
        mbar_arrive_expect_tx(bar, total);
        TQ_TRACE(if (gw < kTraceWarps && issued < kTraceChunks) {
          g_attn_chunks[((size_t)gw * kTraceChunks + issued) * 3] = global_ns();
          g_attn_chunks[((size_t)gw * kTraceChunks + issued) * 3 + 2] = total;
        })
      }
      __syncwarp();
      // With defer_q the q rows (descriptors n_kv ..) stay out; their bytes are counted above.
      if (bytes0 && !(defer_q && lane >= n_kv)) bulk_copy_g2s(dst0, src0, bytes0, bar);
      for (int base = 32; base < n_desc; base += 32) {
        const float* src = nullptr;
        uint32_t dst = 0, bytes = 0;
        describe(base + lane, src, dst, bytes);
        if (bytes && !(defer_q && base + lane >= n_kv)) bulk_copy_g2s(dst, src, bytes, bar);
      }
      TQ_TRACE(if (lane == 0) tr_sub[1] += clock64() - ti0; ti0 = clock64();)
      if (++issued == 1 && inline_first) {  // from the second chunk on: the loaded list
        pf_a = full_a;
        pf_b = full_b;
      }

      // Advance the cursor.
      if (++p_chunk == p_it.cend()) {
        if (++p_k == count) {
          more = false;
          return;
        }
        p_it = nx_it;
        pf_a = nx_a;
        pf_b = nx_b;
        p_chunk = p_it.cbeg();
        nx_it = item_from_lanes(nx2_word);
        load_item_blocks(nx_it, p_k + 1 < count, nx_a, nx_b);
        nx2_word = item_lane_load(p, ws, r0, p_k + 2, count, lane);
      }
      TQ_TRACE(if (lane == 0) tr_sub[2] += clock64() - ti0;)
    };
    // Early copies.  This launch is a programmatic dependent of the kernel
    // before it (this step's KV write), which may still be running: only the
    // K/V rows it cannot be writing are read before the wait -- for a decode
    // item (the sequence's one new key is at pos0), the chunks of the first
    // item whose keys all lie before pos0 -- at most the ring's kStages
    // chunks, and never the q rows.  The consumer computes nothing before the
    // stage's q rows land, and those go out after the wait, so every store of
    // this launch still follows the preceding kernel.
    const WorkItem first_it = p_it;
    int early = 0;
    if (first_it.flags() & kFlagDecode) {
      while (ok && more && p_k == 0 && early < kStages) {
        const ChunkSpan sp = chunk_span(p, p_it, p_chunk);
        if (sp.key0 + sp.nkeys > p_it.pos0()) break;  // holds the new key
        issue_next(true);
        ++early;
      }
    }
    pdl_wait();
    if (early > 0 && lane < first_it.nrows())  // the first chunk's q rows, into stage 0
      bulk_copy_g2s(smem_addr(wsm) + 2 * kKBytes + lane * kRowBytes,
                    p.q + (size_t)(first_it.row0() + lane) * p.q_stride + first_it.head() * kHeadDim, kRowBytes,
                    full0);
    while (ok && more) issue_next(false);
    if (!ok) {
      // The consumer stopped releasing stages.  Give every copy still in
      // flight a bounded chance to land before the CTA exits, so no bulk copy
      // targets the shared memory of a finished CTA.
      for (int k = max(issued - kStages, 0); k < issued; ++k)
        if (!mbar_wait_bounded(full0 + 8 * (k % kStages), (uint32_t)(k / kStages) & 1u)) break;
    }
    TQ_TRACE(if (lane == 0 && gw < kTraceWarps) {
      unsigned smid_;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid_));
      trec[6] = smid_; trec[8] = tr_sub[0]; trec[9] = tr_sub[1]; trec[10] = tr_sub[2]; trec[14] = tr_entry;
      trec[15] = global_ns();
    })
    return;
  }

  // ---- consumer: wait, compute, release; everything it needs is in the stage --
  TQ_TRACE(unsigned long long tr_start = global_ns(), tr_first = 0;
           long long tr_wait = 0, tr_comp = 0, tr_fin = 0, tr_chunks = 0;)
  float m[kMaxRows], lsum[kMaxRows];
  float4 acc[kMaxRows][4];
  float4 qr[kMaxRows][4];
  const int rot = lane_rot(lane);
  int consumed = 0;
  bool failed = false;
  WorkItem owned;  // the cut pair whose shared-memory partials this warp merges
  bool has_owned = false;
  for (int k = 0; k < count; ++k) {
    WorkItem it;
    int c = 0;
    bool at_item_start = true;
    do {
      const int s = consumed % kStages;
      const uint32_t parity = (uint32_t)(consumed / kStages) & 1u;
      TQ_TRACE(long long tr0 = clock64();)
      const bool ok = mbar_wait_bounded(full0 + 8 * s, parity);
      TQ_TRACE(tr_wait += clock64() - tr0; if (tr_first == 0) tr_first = global_ns(); ++tr_chunks;
               if (lane == 0 && gw < kTraceWarps && consumed < kTraceChunks)
                 g_attn_chunks[((size_t)gw * kTraceChunks + consumed) * 3 + 1] = global_ns();)
      if (!__all_sync(kFullMask, ok)) {
        failed = true;
        break;
      }
      const unsigned char* stage = wsm + s * kStageBytes;
      if (at_item_start) {  // take the item and its q rows, reset state
        const StageHeader* hd = reinterpret_cast<const StageHeader*>(stage + 2 * kKBytes + kQBytes);
        it = hd->it;
        c = it.cbeg();
        const float4* qsrc = reinterpret_cast<const float4*>(stage + 2 * kKBytes);
#pragma unroll
        for (int r = 0; r < kMaxRows; ++r) {
          m[r] = -INFINITY;
          lsum[r] = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[r][i] = make_float4(0.f, 0.f, 0.f, 0.f);
            qr[r][i] = r < it.nrows() ? qsrc[r * (kHeadDim / 4) + (lane & 3) * 4 + ((i + rot) & 3)]
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        at_item_start = false;
      }
      const ChunkSpan sp = chunk_span(p, it, c);
      const float* K = reinterpret_cast<const float*>(stage);
      const float* V = reinterpret_cast<const float*>(stage + kKBytes);
      TQ_TRACE(tr0 = clock64();)
      if (it.nrows() == 1)
        attend_chunk<1>(K, V, qr, 1, it.pos0(), sp.key0, sp.nkeys, p.scale_log2, lane, m, lsum, acc);
      else
        attend_chunk<kMaxRows>(K, V, qr, it.nrows(), it.pos0(), sp.key0, sp.nkeys, p.scale_log2, lane, m,
                               lsum, acc);
      __syncwarp();  // every lane's reads of the stage are done
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
      TQ_TRACE(tr_comp += clock64() - tr0;)
      ++consumed;
    } while (++c < it.cend());
    if (failed) break;
    TQ_TRACE(long long tf0 = clock64();)
    finish_rows(p, it, lane, m, lsum, acc, local, TQ_TRACE_ARG(tr_sub));
    if ((it.flags() & kFlagLocal) && it.lsplit() == 0 && merge_targets_ok(p, it)) {
      owned = it;
      has_owned = true;
    }
    TQ_TRACE(tr_fin += clock64() - tf0;)
  }
  if (failed) {
    // Give the copies the producer may still have in flight (at most the
    // ring's depth) a bounded chance to land before this warp moves on; the
    // producer, no longer released, times out on its empty barrier and exits.
    for (int k = consumed; k < consumed + kStages; ++k)
      if (!mbar_wait_bounded(full0 + 8 * (k % kStages), (uint32_t)(k / kStages) & 1u)) break;
  }
  // Every consumer warp of the CTA (with or without work, failed or not)
  // meets here, so the shared-memory partials are complete and visible.
  asm volatile("bar.sync 1, %0;" ::"r"(kAttnWarps * 32) : "memory");
  if (has_owned && !failed) {
    TQ_TRACE(long long tf0 = clock64();)
    merge_local(p, owned, local, lane, TQ_TRACE_ARG(tr_sub));
    TQ_TRACE(tr_fin += clock64() - tf0;)
  }
  TQ_TRACE(if (lane == 0 && gw < kTraceWarps) {
    trec[0] = tr_start; trec[1] = tr_first; trec[2] = global_ns(); trec[3] = tr_wait; trec[4] = tr_comp;
    trec[5] = tr_fin; trec[7] = tr_chunks;
    for (int k = 3; k < 6; ++k) trec[8 + k] = tr_sub[k];  // slot 14: the producer's entry stamp
  })
  TQ_CTA_END();
}

}  // namespace tq
