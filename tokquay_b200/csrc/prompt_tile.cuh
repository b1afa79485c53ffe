// Prompt tiles on the tensor cores: the causal-prefill part of the mixed
// paged-attention launch for sequences that feed many rows in one step.
//
// Replaces, for those rows, the dense gather + masked softmax of the
// reference (tokquay/kv_cache.py:234-242, tokquay/model.py:94-96), with the
// causal rule key <= position of tokquay/kv_cache.py:213-214.
//
// A prompt-tile CTA runs a list of tile items (written by the planner into
// warp slot 0 of the CTA; every other warp slot holds a marker).  One item is
// up to 128 consecutive query rows of one sequence and one head, attending to
// keys [0, last row's position] in 32-key chunks.  Per chunk:
//   S = Q K^T      (M = 128 rows, N = 32 keys, K = 64 dims)
//   P = exp2(S * scale_log2 - m)  (online softmax, one row per thread)
//   O += P V       (M = 128 rows, N = 64 dims, K = 32 keys, accumulated in TMEM)
// Both products run as tcgen05.mma kind::tf32 with fp32 accumulation in
// tensor memory.  fp32 accuracy comes from splitting every operand x into
// hi = x with its low 13 mantissa bits cleared (exact in TF32) and lo = x - hi,
// and summing hi*hi + hi*lo + lo*hi (the dropped lo*lo term is ~2^-22 of the
// product).
//
// Roles (12 warps):
//   warps 0-3   row threads: thread t owns query row t = TMEM lane t.  They
//               write Q (hi | lo) into TMEM, read S back, run the softmax,
//               write P (hi | lo) into TMEM over S, rescale the item's PV
//               accumulator when a row's maximum jumps, and store the
//               normalised output rows.
//   warp 4      QK^T issuer and warp 11 PV issuer (each: the whole warp walks
//               the loop, one elected lane issues); two issuing threads keep
//               the tensor core busy while the softmax runs (one thread's
//               tcgen05.mma stream is issue-bound, measured on B200).
//   warp 5      producer: TMA bulk copies of each chunk's K and V rows from the
//               pool (through the block table) into a raw ring, one per block.
//   warps 6-10  converters: the hi/lo split of each raw chunk into the MMA
//               operand layouts (V transposed), up to kTileKVBufs chunks ahead
//               of the MMAs.
//
// Tensor memory (512 columns): Q (hi 64 | lo 64) at 0 (the next item's Q is
// written once the current item's last S is out); three S/P buffers at 128,
// 192 and 256 (S in 32 columns, then P hi over them, P lo at +32); PV
// accumulators at 320 and 384, one per item parity.
//
// Shared-memory operand layout (K-major, no swizzle): element (r, k) of an
// operand with R rows and k along the reduction dimension sits at
//   (k / 4) * (R / 8) * 128 + (r / 8) * 128 + (r % 8) * 16 + (k % 4) * 4
// bytes: core matrices of 8 rows x 16 bytes.  K is the B operand of QK^T as
// it is (rows = keys, k = dims); V is the B operand of PV transposed (rows =
// dims, k = keys).  (The MN-major form of a TF32 B operand, which would take
// V untransposed, gave all-zero products on B200 in this no-swizzle layout.)
//
// Every mbarrier wait is bounded; a wait that runs out sets the device error
// word and a CTA-wide abort flag, every role leaves its loop, the MMA issuer
// drains the tensor core, and the tensor memory is freed before the CTA exits.
#pragma once

namespace tq {

constexpr int kFlagTile = 8;          // work-item flag: a prompt-tile item / CTA marker
constexpr int kTileRows = 128;        // query rows per tile (the MMA's M)
constexpr int kTileMaxItems = 96;     // tile items one CTA holds
#ifndef TQ_TILE_KV_BUFS
#define TQ_TILE_KV_BUFS 3
#endif
#ifndef TQ_TILE_RAW_STAGES
#define TQ_TILE_RAW_STAGES 4
#endif
constexpr int kTileKVBufs = TQ_TILE_KV_BUFS;        // converted K/V chunks (hi | lo) in shared memory
constexpr int kTileRawStages = TQ_TILE_RAW_STAGES;  // raw K/V chunks in flight (the producer's ring)
constexpr int kTileRowWarps = 4;
constexpr int kTileMmaWarp = 4;
constexpr int kTileProducerWarp = 5;  // TMA copies of the K/V rows
constexpr int kTileCvtWarp0 = 6;      // converters: hi/lo split into the MMA layout
constexpr int kTilePvWarp = 2 * kAttnWarps - 1;  // PV issuer (warp 11)
constexpr int kTileCvtWarps = kTilePvWarp - kTileCvtWarp0;  // 5
constexpr int kTileUnits = 32;  // per chunk: {K, V} x 4 groups of 8 keys x 4 blocks of 16 dims
constexpr int kTileUnitsPerThread = (kTileUnits + kTileCvtWarps - 1) / kTileCvtWarps;
constexpr int kTileOpBytes = 32 * kHeadDim * 4;  // one hi or lo half of a K chunk
// V^T halves (64 dim rows x 32 keys): 4-key groups 1040 bytes apart (LBO),
// 8-row groups 128 bytes apart (SBO); the 16-byte gap after each 4-key group
// keeps the converters' scalar stores at most 2-way bank-conflicted.
constexpr int kTileVtSbo = 128, kTileVtLbo = 1040;
constexpr int kTileVtBytes = 8320;  // >= 7 * LBO + 7 * SBO + 128, a multiple of 128
constexpr int kTileOffVt = 2 * kTileOpBytes;  // V hi within a buffer; V lo at + kTileVtBytes
constexpr int kTileBufBytes = 2 * kTileOpBytes + 2 * kTileVtBytes;  // K hi | K lo | V hi | V lo
constexpr int kTileOffRaw = kTileKVBufs * kTileBufBytes;
// Raw ring stage: the chunk's 32 K rows, then its 32 V rows, as the pool
// holds them (256 bytes per row), copied block by block.
constexpr int kTileRawStageBytes = 2 * kTileOpBytes;
constexpr int kTileQStride = kHeadDim * 4 + 16;  // padded q rows: thread t's row reads are conflict-free
constexpr int kTileOffQStage = kTileOffRaw + kTileRawStages * kTileRawStageBytes;
constexpr int kTileOffItems = kTileOffQStage + kTileRows * kTileQStride;
constexpr int kTileOffBars = kTileOffItems + kTileMaxItems * 32;
// kv_ready[B] kv_free[B] s_full[SP] p_full[SP] o_full[SP] q_ready done raw_full[R] raw_empty[R]
#ifndef TQ_TILE_SP
#define TQ_TILE_SP 3
#endif
constexpr int kTileSP = TQ_TILE_SP;  // S/P buffers in TMEM (chunk g uses g % kTileSP)
constexpr int kTileBarKvReady = 0, kTileBarKvFree = kTileKVBufs, kTileBarSFull = 2 * kTileKVBufs,
              kTileBarPFull = kTileBarSFull + kTileSP, kTileBarOFull = kTileBarPFull + kTileSP,
              kTileBarQReady = kTileBarOFull + kTileSP, kTileBarDone = kTileBarQReady + 1,
              kTileBarRawFull = kTileBarDone + 1,
              kTileBarRawEmpty = kTileBarRawFull + kTileRawStages, kTileNumBars = kTileBarRawEmpty + kTileRawStages;
// [0] TMEM base, [1] abort flag
static_assert(kTileBarRawFull == kTileBarDone + 1 && kTileBarDone == kTileBarQReady + 1 &&
                  kTileBarQReady == kTileBarOFull + kTileSP && kTileBarOFull == kTileBarPFull + kTileSP &&
                  kTileBarPFull == kTileBarSFull + kTileSP && kTileBarSFull == kTileBarKvFree + kTileKVBufs &&
                  kTileBarKvFree == kTileBarKvReady + kTileKVBufs,
              "tile barriers do not overlap");
constexpr int kTileOffMisc = kTileOffBars + kTileNumBars * 8;
constexpr int kTileOffParams = kTileOffMisc + 16;  // the launch's AttnParams, copied here
constexpr int kTileSmemBytes = kTileOffParams + (int)((sizeof(AttnParams) + 15) / 16 * 16);
static_assert(kChunk == 32, "prompt tiles take 32-key chunks");
// A launch that may hold tile CTAs asks for the larger of the two layouts.
constexpr int kTileLaunchSmemBytes = kTileSmemBytes > kAttnSmemBytes ? kTileSmemBytes : kAttnSmemBytes;
static_assert(kTileLaunchSmemBytes <= 232448, "a tile CTA fits an SM's shared memory");
static_assert(2 * kAttnWarps * 32 == 384, "tile roles assume 12 warps");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemQ = 0, kTmemS = 128, kTmemO = kTmemS + 64 * kTileSP;
static_assert(kTmemO + 128 <= kTmemCols, "Q, the S/P buffers and two PV accumulators fit the tensor memory");
constexpr uint32_t kTmemP = kTmemS;  // P hi (+32: P lo) over S of the same buffer
constexpr float kTileRescale = 8.f;
#ifndef TQ_TILE_FAST_WAIT_SLEEP
#define TQ_TILE_FAST_WAIT_SLEEP 0
#endif
constexpr bool kTileFastWaitSleep = TQ_TILE_FAST_WAIT_SLEEP;  // row threads' and MMA issuers' waits  // log2 units a row's maximum may pass its reference by

// Instruction descriptors (kind::tf32, fp32 accumulator, M = 128, both
// operands K-major): bits 4-5 D format (1 = f32), 7-9 A format (2 = tf32),
// 10-12 B format, 17-22 N >> 3, 24-28 M >> 4.
constexpr uint32_t kIdescQK = (1u << 4) | (2u << 7) | (2u << 10) | ((32u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (2u << 7) | (2u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);

// Shared-memory matrix descriptor, K-major, no swizzle: start address,
// leading-byte offset (between core matrices along the reduction dimension),
// stride-byte offset (between 8-row core groups), all >> 4; bit 46: the sm_100
// descriptor version.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// D[tmem] (+)= A[tmem] x B[smem].  The whole (converged) warp calls it with
// the same, warp-uniform operands; one elected lane issues the MMA.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d, uint32_t a, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d),
      "r"(a), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// The barrier's next phase completes once every tcgen05 operation the
// elected lane issued so far has completed (whole warp, as umma_tf32_ts).
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// Tensor-memory allocation (one warp, .sync.aligned): the base address is
// written to shared memory at dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive columns of this thread's TMEM lane, loaded and waited for in
// one asm statement (so no use of the registers can move above the wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 consecutive columns of this thread's TMEM lane, stored and waited for.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// TMA bulk store of `bytes` from this CTA's shared memory to global memory,
// in this thread's bulk group; wait_read: until the sources have been read.
__device__ __forceinline__ void bulk_store_s2g(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// 16-byte global -> shared copy; src_bytes 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t tf32_hi(float x) { return __float_as_uint(x) & 0xffffe000u; }

// try_wait that lets the thread sleep until the phase completes (or the
// hint, in ns, runs out), so waiting warps leave the issue slots to the
// working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(100000u)
      : "memory");
  return done != 0;
}

// tile_wait for a whole (converged) warp: the outcome is the same in every
// lane, so the warp leaves its loops together.
__device__ __forceinline__ bool tile_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                               bool sleep = true);

// One arrival for the whole warp, once every lane's earlier tcgen05 stores
// (waited for) are ordered before it.
__device__ __forceinline__ void warp_arrive_after_tmem_st(uint32_t bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ float fast_exp2(float x) {  // ex2.approx.ftz: exp2(-inf) = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded wait that also gives up once another role has aborted the CTA.
// sleep: let the thread sleep until the phase completes (warps whose wake-up
// latency does not sit on the chunk's critical path: producer, converters);
// otherwise poll (row threads, MMA issuers).
__device__ __forceinline__ bool tile_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          bool sleep = true) {
  auto probe = [&]() { return sleep ? mbar_try_wait_sleep(bar, parity) : mbar_try_wait(bar, parity); };
  if (probe()) return true;
  const long long t0 = clock64();
  while (!probe()) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      raise_device_error(TQ_DEVERR_WAIT_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool tile_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                               bool sleep) {
  return __all_sync(kFullMask, tile_wait(bar, parity, abort_flag, sleep));
}

// Row t's q row of head h (zeros for rows past the item), copied into the
// q staging area at qrow (cp.async: one commit group).
__device__ __forceinline__ void tile_issue_q(const AttnParams& p, const WorkItem& it, int t, uint32_t qrow) {
  const bool real = t < it.nrows();
  const float* src = p.q + (size_t)(it.row0() + (real ? t : 0)) * p.q_stride + it.head() * kHeadDim;
#pragma unroll
  for (int i = 0; i < 16; ++i) cp_async16(qrow + 16 * i, src + 4 * i, real ? 16u : 0u);
  cp_async_commit();
}

// The staged q row, split into hi | lo, into this thread's TMEM lane: hi at
// columns taddr .. +63, lo at taddr + 64 .. +127.
__device__ __forceinline__ void tile_q_to_tmem(uint32_t taddr, uint32_t qrow) {
  uint32_t r[32];
  float4 v[8];
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // dims 0-31, then 32-63
#pragma unroll
    for (int i = 0; i < 8; ++i)
      asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(v[i].x), "=f"(v[i].y), "=f"(v[i].z), "=f"(v[i].w)
                   : "r"(qrow + 16 * (8 * half + i)));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r[4 * i + 0] = tf32_hi(v[i].x);
      r[4 * i + 1] = tf32_hi(v[i].y);
      r[4 * i + 2] = tf32_hi(v[i].z);
      r[4 * i + 3] = tf32_hi(v[i].w);
    }
    tmem_st32(taddr + 32 * half, r);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      r[4 * i + 0] = __float_as_uint(v[i].x - __uint_as_float(tf32_hi(v[i].x)));
      r[4 * i + 1] = __float_as_uint(v[i].y - __uint_as_float(tf32_hi(v[i].y)));
      r[4 * i + 2] = __float_as_uint(v[i].z - __uint_as_float(tf32_hi(v[i].z)));
      r[4 * i + 3] = __float_as_uint(v[i].w - __uint_as_float(tf32_hi(v[i].w)));
    }
    tmem_st32(taddr + 64 + 32 * half, r);
  }
}

// The 64 accumulator columns of this thread's TMEM lane at taddr, times
// factor (whole warp: the loads and stores are .sync.aligned).
__device__ __forceinline__ void tile_scale_o(uint32_t taddr, float factor) {
  uint32_t v[32];
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    tmem_ld32(taddr + 32 * half, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * factor);
    tmem_st32(taddr + 32 * half, v);
  }
}

// S of chunk g (buffer g % kTileSP) = Q x K^T (shared-memory
// buffer g % kTileKVBufs): 8 k-steps of 8 dims, hi*hi + hi*lo + lo*hi each.
__device__ __forceinline__ void tile_issue_qk(uint32_t tmem, uint32_t kv0, int g) {
  const uint32_t d = tmem + kTmemS + 64 * (g % kTileSP);
  const uint32_t a = tmem + kTmemQ;
  const uint32_t kb = kv0 + (uint32_t)((g % kTileKVBufs) * kTileBufBytes);
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint64_t bhi = umma_smem_desc(kb + 1024 * s, 512, 128);
    const uint64_t blo = umma_smem_desc(kb + kTileOpBytes + 1024 * s, 512, 128);
    umma_tf32_ts(d, a + 8 * s, bhi, kIdescQK, s > 0);
    umma_tf32_ts(d, a + 8 * s, blo, kIdescQK, 1);
    umma_tf32_ts(d, a + 64 + 8 * s, bhi, kIdescQK, 1);
  }
}

// Item k's accumulator (+)= P of chunk g x V (transposed in the shared-memory
// buffer g % kTileKVBufs): 4 k-steps of 8 keys; `first` starts the sum.
__device__ __forceinline__ void tile_issue_pv(uint32_t tmem, uint32_t kv0, int g, int k, bool first) {
  const uint32_t d = tmem + kTmemO + 64 * (k & 1);
  const uint32_t a = tmem + kTmemP + 64 * (g % kTileSP);
  const uint32_t vb = kv0 + (uint32_t)((g % kTileKVBufs) * kTileBufBytes + kTileOffVt);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint64_t bhi = umma_smem_desc(vb + 2 * kTileVtLbo * s, kTileVtLbo, kTileVtSbo);
    const uint64_t blo = umma_smem_desc(vb + kTileVtBytes + 2 * kTileVtLbo * s, kTileVtLbo, kTileVtSbo);
    umma_tf32_ts(d, a + 8 * s, bhi, kIdescPV, !first || s > 0);
    umma_tf32_ts(d, a + 8 * s, blo, kIdescPV, 1);
    umma_tf32_ts(d, a + 32 + 8 * s, bhi, kIdescPV, 1);
  }
}

// The K/V role's cursor over (item, chunk) of the CTA's list.
struct TileCursor {
  int k, c;  // item index (== count when past the end), chunk
};
__device__ __forceinline__ void tile_advance(TileCursor& cur, const WorkItem* items, int count) {
  if (cur.k >= count) return;
  if (++cur.c >= items[cur.k].cend()) {
    if (++cur.k < count) cur.c = items[cur.k].cbeg();
  }
}

#ifdef TQ_TILE_DEBUG
// Per-chunk event clocks (SM cycles since the role started) of the last 4
// CTAs: [cta][event][chunk], events: 0 K/V data landed, 1 K/V buffer free,
// 2 K/V ready, 3 MMA saw kv_ready, 4 MMA saw p_full, 5 PV issued, 6 row saw
// S, 7 row P written, 8 row saw O (fold).
constexpr int kTrEv = 20, kTrCh = 48;
// Per CTA of the last launch: globaltimer at entry, latest warp exit, tile CTA (1) or not.
__device__ unsigned long long g_cta_time[3 * 1024];
__device__ long long g_tile_trace[160 * kTrEv * kTrCh];
#define TQ_TILE_TR(ev, ch) \
  do { if (blockIdx.x < 160 && (ch) < kTrCh) \
    g_tile_trace[(blockIdx.x * kTrEv + (ev)) * kTrCh + (ch)] = clock64() - tr_t0; } while (0)
#else
#define TQ_TILE_TR(ev, ch) do { } while (0)
#endif

__device__ __noinline__ void prompt_tile_cta(const AttnParams& p, unsigned char* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef TQ_TILE_DEBUG
  const long long tr_t0 = clock64();
#endif
  WorkItem* items = reinterpret_cast<WorkItem*>(smem + kTileOffItems);
  const uint32_t bars = smem_addr(smem + kTileOffBars);
  auto bar = [&](int i) { return bars + 8u * (uint32_t)i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + kTileOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);

  // ---- the CTA's items (warp slot 0's list) and set-up ----------------------
  const int ws0 = blockIdx.x * kAttnWarps;
  // The producer's first copies use the block ids that ride with the first item.
  const int first_blk = warp == kTileProducerWarp ? __ldg(p.attn + kFirstWords * (size_t)ws0 + 8 + ((lane >> 1) & 7)) : -1;
  const int r0 = __ldg(warp_offsets(p) + ws0), r1 = __ldg(warp_offsets(p) + ws0 + 1);
  const int count = 1 + r1 - r0;
  if (count > kTileMaxItems) {  // the planner never writes such a list
    if (threadIdx.x == 0) raise_device_error(TQ_DEVERR_BAD_PLAN);
    return;
  }
  for (int i = threadIdx.x; i < 8 * count; i += blockDim.x) {
    const int* src = i < 8 ? p.attn + kFirstWords * (size_t)ws0 + i : other_items(p) + 8 * (size_t)r0 + (i - 8);
    reinterpret_cast<int*>(items)[i] = __ldg(src);
  }
  if (threadIdx.x == 0) {
    // Threads arrive one per warp (after a warp sync): an mbarrier arrival by
    // every thread of a role serialises on the barrier's shared-memory word.
    for (int i = 0; i < kTileRawStages; ++i) {
      mbar_init(bar(kTileBarRawFull + i), 1);                 // the producer's expect_tx + the bytes
      mbar_init(bar(kTileBarRawEmpty + i), kTileCvtWarps);    // every converter warp has read it
    }
    for (int i = 0; i < kTileKVBufs; ++i) {
      mbar_init(bar(kTileBarKvReady + i), kTileCvtWarps);
      mbar_init(bar(kTileBarKvFree + i), 1);
    }
    for (int i = 0; i < kTileSP; ++i) {
      mbar_init(bar(kTileBarSFull + i), 1);
      mbar_init(bar(kTileBarPFull + i), kTileRowWarps);
      mbar_init(bar(kTileBarOFull + i), 1);
    }
    mbar_init(bar(kTileBarQReady), kTileRowWarps);
    mbar_init(bar(kTileBarDone), 2);  // both MMA issuers' work has completed
    misc[1] = 0;
    mbar_init_fence();
  }
  if (warp == 0) {
    tmem_alloc(smem_addr(misc), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  if (threadIdx.x == 0) TQ_TILE_TR(18, 0);
  // Items are checked once, here: rows within a tile, keys within the sequence's
  // table (the K/V role also checks each block id against the pool).
  bool bad = false;
  for (int k = 0; k < count; ++k) {
    const WorkItem& it = items[k];
    const int f = it.flags() & ~kFlagTile;
    bad |= it.nrows() < 1 || it.nrows() > kTileRows || it.head() >= p.n_head || it.cbeg() >= it.cend() ||
           it.cend() > (it.pos0() + it.nrows() + kChunk - 1) / kChunk || (f != 0 && f != kFlagGlobal) ||
           (f == kFlagGlobal && (it.gbase() < 0 || it.gsplit() >= it.gnsplit() ||
                                 (long long)it.gbase() + (long long)it.nrows() * it.gnsplit() > p.max_partials));
  }
  if (bad && threadIdx.x == 0) raise_device_error(TQ_DEVERR_BAD_PLAN);
  pdl_wait();  // q rows and this step's K/V rows come from the kernels before this one

  if (!bad && warp < kTileRowWarps) {
    // ---- row threads ----------------------------------------------------------
    const int t = threadIdx.x;  // query row in the tile = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const uint32_t qrow = smem_addr(smem + kTileOffQStage) + (uint32_t)(t * kTileQStride);
    tile_issue_q(p, items[0], t, qrow);
    cp_async_wait<0>();
    tile_q_to_tmem(lane_base + kTmemQ, qrow);
    warp_arrive_after_tmem_st(bar(kTileBarQReady));
    int g = 0;
    bool ok = true;
    for (int k = 0; k < count && ok; ++k) {
      const WorkItem it = items[k];
      const bool has_next = k + 1 < count;
      if (has_next) {  // lands while the first chunk's S is computed
        bulk_store_wait_read();  // the previous item's output has left the staging row
        tile_issue_q(p, items[k + 1], t, qrow);
      }
      const int kend = it.pos0() + it.nrows();
      const int lim_abs = min(it.pos0() + t, kend - 1);  // this row's last key
      const uint32_t o_col = lane_base + kTmemO + 64 * (k & 1);  // this item's PV accumulator
      // m: the reference the item's P is taken against (log2 units); l: the
      // sum of P.  The PVs of the item accumulate in TMEM against m, which
      // moves only when a chunk's maximum passes it by more than
      // kTileRescale (P stays below 2^kTileRescale); then the accumulator is
      // rescaled in place before that chunk's PV is issued.
      float m = -INFINITY, l = 0.f;
      for (int c = it.cbeg(); c < it.cend() && ok; ++c, ++g) {
        const int b = g % kTileSP;
        ok = tile_wait_warp(bar(kTileBarSFull + b), (uint32_t)(g / kTileSP) & 1u, abort_flag, kTileFastWaitSleep);
        if (!ok) break;
        if (t == 0) TQ_TILE_TR(6, g);
        tc_fence_after();
        if (c + 1 == it.cend() && has_next) {  // every QK^T of this item is done: the next item's Q
          cp_async_wait<0>();
          tile_q_to_tmem(lane_base + kTmemQ, qrow);
          warp_arrive_after_tmem_st(bar(kTileBarQReady));
        }
        uint32_t s[32];
        tmem_ld32(lane_base + kTmemS + 64 * b, s);
        const int lim = lim_abs - c * kChunk;  // keys j <= lim of this chunk are valid
        float mx = -INFINITY;
        if (lim < kChunk - 1) {  // the causal diagonal: keys past the row's position
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j > lim) s[j] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(s[j]));
        // Scores are finite (fp32 products of finite q and k): mx is -inf only
        // for a row without a key in this chunk, whose P is all zero.
        const float mxs = mx * p.scale_log2;
        const bool bump = mxs > m + kTileRescale;  // always at the item's first chunk
        const float mnew = bump ? mxs : m;
        const float mref = mnew == -INFINITY ? 0.f : mnew;
        float psum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float pj = fast_exp2(fmaf(__uint_as_float(s[j]), p.scale_log2, -mref));  // exp2(-inf) = 0
          psum += pj;
          s[j] = __float_as_uint(pj);
        }
        const float factor = bump ? fast_exp2(m - mnew) : 1.f;  // 0 while m is -inf
        l = fmaf(l, factor, psum);
        m = mnew;
        uint32_t hi[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          hi[j] = tf32_hi(__uint_as_float(s[j]));
          s[j] = __float_as_uint(__uint_as_float(s[j]) - __uint_as_float(hi[j]));
        }
        tmem_st32(lane_base + kTmemP + 64 * b, hi);
        tmem_st32(lane_base + kTmemP + 64 * b + 32, s);
        bool waited = c == it.cbeg();  // the item's first PV overwrites the accumulator
        if (!waited && __any_sync(kFullMask, bump)) {
          // Rescale the accumulator (every PV issued so far has completed)
          // before this chunk's PV adds to it.
          const int pg = g - 1;
          if (!(ok = tile_wait_warp(bar(kTileBarOFull + pg % kTileSP), (uint32_t)(pg / kTileSP) & 1u, abort_flag, kTileFastWaitSleep))) break;
          tc_fence_after();
          tile_scale_o(o_col, factor);
          waited = true;
        }
        warp_arrive_after_tmem_st(bar(kTileBarPFull + b));
        if (t == 0) TQ_TILE_TR(7, g);
        if (!waited) {  // chunk g-1's PV: consumed, so the barrier's phases stay in step
          const int pg = g - 1;
          if (!(ok = tile_wait_warp(bar(kTileBarOFull + pg % kTileSP), (uint32_t)(pg / kTileSP) & 1u, abort_flag, kTileFastWaitSleep))) break;
          if (t == 0) TQ_TILE_TR(8, pg);
        }
      }
      if (!ok) break;
      {  // the last chunk's PV completes the accumulator
        const int pg = g - 1;
        if (!(ok = tile_wait_warp(bar(kTileBarOFull + pg % kTileSP), (uint32_t)(pg / kTileSP) & 1u, abort_flag, kTileFastWaitSleep))) break;
        if (t == 0) TQ_TILE_TR(13, k);
        tc_fence_after();
      }
      float* const orow = p.out + (size_t)(it.row0() + t) * p.out_stride + it.head() * kHeadDim;
      if (!(it.flags() & kFlagGlobal)) {
        // The whole key range: the normalised row, staged in this thread's q
        // row (its q has been consumed; the next q copy waits for this store
        // to have read it) and written by one 256-byte bulk store.
        const float inv = 1.f / l;
        uint32_t v[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(o_col + 32 * half, v);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(qrow + 128 * half + 16 * i),
                         "f"(__uint_as_float(v[4 * i]) * inv), "f"(__uint_as_float(v[4 * i + 1]) * inv),
                         "f"(__uint_as_float(v[4 * i + 2]) * inv), "f"(__uint_as_float(v[4 * i + 3]) * inv)
                         : "memory");
        }
        if (t < it.nrows()) {
          fence_proxy_async_smem();
          bulk_store_s2g(orow, qrow, kRowBytes);
        }
        if (t == 0) TQ_TILE_TR(14, k);
        continue;
      }
      // A piece of a split tile: this piece's partial (m, l, unnormalised
      // accumulator) per row into the split-K scratch, and on to the next
      // item.  tile_merge_kernel, the launch's programmatic dependent, merges
      // the pieces of every row (rows without a key in a piece carry m = -inf
      // and weigh nothing): no fence, counter or round trip on this CTA's path.
      const size_t idx = (size_t)it.gbase() + (size_t)t * it.gnsplit() + it.gsplit();
      uint32_t v[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld32(o_col + 32 * half, v);
        if (t < it.nrows()) {
          float4* dst = reinterpret_cast<float4*>(p.part_acc + idx * kHeadDim + 32 * half);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                 __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        }
      }
      if (t < it.nrows()) *reinterpret_cast<float2*>(p.part_ml + 2 * idx) = make_float2(m, l);
      if (t == 0) TQ_TILE_TR(14, k);
    }
    cp_async_wait<0>();     // no copy of a q row may land after the CTA is gone
    bulk_store_wait_read();  // nor an output store read its shared memory
  } else if (!bad && warp == kTileMmaWarp) {
    // ---- QK^T issuer: the whole warp walks the loop, one lane issues ------
    // S buffer g % kTileSP last held chunk g-kTileSP's P: QK^T of chunk g
    // waits for that chunk's PV (issued by the PV warp) to complete.
    const uint32_t kv0 = smem_addr(smem);
    int g = 0;
    bool ok = true;
    for (int k = 0; k < count && ok; ++k) {
      const WorkItem& it = items[k];
      if (!(ok = tile_wait_warp(bar(kTileBarQReady), (uint32_t)k & 1u, abort_flag, kTileFastWaitSleep))) break;
      for (int c = it.cbeg(); c < it.cend(); ++c, ++g) {
        if (!(ok = tile_wait_warp(bar(kTileBarKvReady + g % kTileKVBufs), (uint32_t)(g / kTileKVBufs) & 1u,
                                  abort_flag)))
          break;
        TQ_TILE_TR(3, g);
        if (g >= kTileSP &&
            !(ok = tile_wait_warp(bar(kTileBarOFull + g % kTileSP), (uint32_t)(g / kTileSP - 1) & 1u, abort_flag, kTileFastWaitSleep)))
          break;
        tc_fence_after();
        TQ_TILE_TR(9, g);
        tile_issue_qk(tmem, kv0, g);
        umma_commit(bar(kTileBarSFull + g % kTileSP));
        TQ_TILE_TR(10, g);
      }
    }
    // Every MMA issued has completed before the CTA may free TMEM or exit.
    umma_commit(bar(kTileBarDone));
    mbar_wait_bounded(bar(kTileBarDone), 0);
    if (lane == 0) TQ_TILE_TR(16, 0);
  } else if (!bad && warp == kTilePvWarp) {
    // ---- PV issuer ------------------------------------------------------------
    const uint32_t kv0 = smem_addr(smem);
    int g = 0;
    bool ok = true;
    for (int k = 0; k < count && ok; ++k) {
      const WorkItem& it = items[k];
      for (int c = it.cbeg(); c < it.cend(); ++c, ++g) {
        if (!(ok = tile_wait_warp(bar(kTileBarPFull + g % kTileSP), (uint32_t)(g / kTileSP) & 1u, abort_flag, kTileFastWaitSleep))) break;
        TQ_TILE_TR(4, g);
        tc_fence_after();
        tile_issue_pv(tmem, kv0, g, k, c == it.cbeg());
        umma_commit(bar(kTileBarOFull + g % kTileSP));
        umma_commit(bar(kTileBarKvFree + g % kTileKVBufs));
        TQ_TILE_TR(5, g);
      }
    }
    umma_commit(bar(kTileBarDone));
    mbar_wait_bounded(bar(kTileBarDone), 0);
  } else if (!bad && warp == kTileProducerWarp) {
    // ---- producer: each chunk's K and V rows, a bulk copy per block --------
    // Copy d of a chunk (d < 2 * its blocks) is the K (d even) or V (d odd)
    // rows of its block d / 2, into raw stage g % kTileRawStages; lane i
    // describes copies i and i + 32 (block size 1 needs 64).  Rows past the
    // item's end are not copied (the converters write zeros for them).  Block
    // ids are loaded two chunks ahead of their copies.
    const uint32_t raw0 = smem_addr(smem + kTileOffRaw);
    const size_t kv_stride = (size_t)p.n_head * p.block_size * kHeadDim;  // K tile -> V tile
    const int bs = p.block_size;
    int total = 0;
    for (int k = 0; k < count; ++k) total += items[k].cend() - items[k].cbeg();
    auto nblocks = [&](const TileCursor& cur) {  // blocks of chunk cur.c of item cur.k
      const WorkItem& it = items[cur.k];
      const int key0 = cur.c * kChunk, nkeys = min(kChunk, it.pos0() + it.nrows() - key0);
      return bs <= kChunk ? ((key0 + nkeys - 1) >> p.log2_bs) - (key0 >> p.log2_bs) + 1 : 1;
    };
    auto load_blocks = [&](const TileCursor& cur, int& b0, int& b1) {
      b0 = b1 = -1;
      if (cur.k >= count) return;
      const WorkItem& it = items[cur.k];
      const int nb = nblocks(cur);
      const int* tbl = p.tables + (size_t)it.seq() * p.table_stride + ((cur.c * kChunk) >> p.log2_bs);
      if (lane < 2 * nb) b0 = __ldg(tbl + (lane >> 1));
      if (lane + 32 < 2 * nb) b1 = __ldg(tbl + ((lane + 32) >> 1));
    };
    TileCursor cur{0, items[0].cbeg()}, nxt = cur;
    tile_advance(nxt, items, count);
    int ba, bb, na, nb2;
    if (bs >= kChunk / kFirstBlocks) {  // the first chunk spans at most kFirstBlocks blocks
      ba = lane < 2 * nblocks(cur) ? first_blk : -1;
      bb = -1;
    } else {
      load_blocks(cur, ba, bb);
    }
    load_blocks(nxt, na, nb2);
    for (int g = 0; g < total; ++g) {
      const int st = g % kTileRawStages;
      if (g >= kTileRawStages &&
          !tile_wait_warp(bar(kTileBarRawEmpty + st), (uint32_t)(g / kTileRawStages - 1) & 1u, abort_flag))
        break;
      const WorkItem& it = items[cur.k];
      const int key0 = cur.c * kChunk, nkeys = min(kChunk, it.pos0() + it.nrows() - key0);
      const int kb0 = key0 >> p.log2_bs;
      const uint32_t stage = raw0 + (uint32_t)(st * kTileRawStageBytes);
      // Copy d: source, destination and bytes (0: no copy).
      auto describe = [&](int d, int blk, const float*& src, uint32_t& dst) -> uint32_t {
        if (blk < 0) return 0u;
        if (blk >= p.num_blocks) {
          raise_device_error(TQ_DEVERR_BAD_BLOCK);
          return 0u;
        }
        const int kv = d & 1;
        if (bs <= kChunk) {
          const int kb = kb0 + (d >> 1);
          src = p.pool + pool_tile_offset(p, blk, 0, it.head()) + kv * kv_stride;
          dst = stage + (uint32_t)(kv * kTileOpBytes + (kb * bs - key0) * kRowBytes);
          return (uint32_t)(min(bs, key0 + nkeys - kb * bs) * kRowBytes);
        }
        src = p.pool + pool_tile_offset(p, blk, 0, it.head()) + kv * kv_stride + (size_t)(key0 & (bs - 1)) * kHeadDim;
        dst = stage + (uint32_t)(kv * kTileOpBytes);
        return (uint32_t)(nkeys * kRowBytes);
      };
      const float *src0 = p.pool, *src1 = p.pool;
      uint32_t dst0 = 0, dst1 = 0;
      const uint32_t bytes0 = describe(lane, ba, src0, dst0), bytes1 = describe(lane + 32, bb, src1, dst1);
      const uint32_t bytes = __reduce_add_sync(kFullMask, bytes0 + bytes1);
      if (lane == 0) mbar_arrive_expect_tx(bar(kTileBarRawFull + st), bytes);
      __syncwarp();
      if (bytes0) bulk_copy_g2s(dst0, src0, bytes0, bar(kTileBarRawFull + st));
      if (bytes1) bulk_copy_g2s(dst1, src1, bytes1, bar(kTileBarRawFull + st));
      cur = nxt;
      ba = na;
      bb = nb2;
      tile_advance(nxt, items, count);
      load_blocks(nxt, na, nb2);
    }
    if (lane == 0) TQ_TILE_TR(17, 0);
    // Copies still in flight land before the CTA may exit (bounded).
    for (int g = max(total - kTileRawStages, 0); g < total; ++g)
      if (!mbar_wait_bounded(bar(kTileBarRawFull + g % kTileRawStages), (uint32_t)(g / kTileRawStages) & 1u)) break;
  } else if (!bad && warp >= kTileCvtWarp0 && warp < kTilePvWarp) {
    // ---- converters: raw rows -> hi/lo halves in the MMA layout ------------
    const int cw = warp - kTileCvtWarp0;
    const int f4 = lane >> 3, kk = lane & 7;
    const uint32_t raw0 = smem_addr(smem + kTileOffRaw);
    const uint32_t kv0 = smem_addr(smem);
    TileCursor cur{0, items[0].cbeg()};
    int total = 0;
    for (int k = 0; k < count; ++k) total += items[k].cend() - items[k].cbeg();
    for (int g = 0; g < total; ++g) {
      const int st = g % kTileRawStages, b = g % kTileKVBufs;
      if (!tile_wait_warp(bar(kTileBarRawFull + st), (uint32_t)(g / kTileRawStages) & 1u, abort_flag)) break;
      if (kk == 0 && f4 == 0 && cw == 0) TQ_TILE_TR(0, g);
      if (g >= kTileKVBufs &&
          !tile_wait_warp(bar(kTileBarKvFree + b), (uint32_t)(g / kTileKVBufs - 1) & 1u, abort_flag))
        break;
      if (kk == 0 && f4 == 0 && cw == 0) TQ_TILE_TR(1, g);
      const WorkItem& it = items[cur.k];
      const int nvalid = it.pos0() + it.nrows() - cur.c * kChunk;  // keys of this chunk in the item
      const uint32_t rs = raw0 + (uint32_t)(st * kTileRawStageBytes);
      // Unit u covers keys 8*kg .. +7 (kg = (u >> 2) & 3) of K (u < 16) or V;
      // lane (f4, kk) takes key 8*kg + kk and dims 4m .. 4m+3 with the column
      // m = (4*(u & 3) + f4 + kk) mod 16 rotated by kk, so a quarter-warp's
      // 16-byte accesses to 256-byte rows (and to the K layout) hit 8
      // different bank groups.  Every unit's raw float4 first (independent
      // loads), then the splits.
      float4 x[kTileUnitsPerThread];
#pragma unroll
      for (int i = 0; i < kTileUnitsPerThread; ++i) {
        const int u = cw + kTileCvtWarps * i;
        const int j = 8 * ((u >> 2) & 3) + kk;  // key in the chunk
        const int m = (4 * (u & 3) + f4 + kk) & 15;
        x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (u < kTileUnits && j < nvalid)
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(x[i].x), "=f"(x[i].y), "=f"(x[i].z), "=f"(x[i].w)
                       : "r"(rs + (uint32_t)((u >> 4) * kTileOpBytes + j * kRowBytes + m * 16)));
      }
      // The raw stage is read (the arrive's release orders the loads before
      // it): the producer may refill it while this chunk is split.
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kTileBarRawEmpty + st));
#pragma unroll
      for (int i = 0; i < kTileUnitsPerThread; ++i) {
        const int u = cw + kTileCvtWarps * i;
        if (u >= kTileUnits) continue;
        const int j = 8 * ((u >> 2) & 3) + kk;
        const int m = (4 * (u & 3) + f4 + kk) & 15;
        const float4 hi = make_float4(__uint_as_float(tf32_hi(x[i].x)), __uint_as_float(tf32_hi(x[i].y)),
                                      __uint_as_float(tf32_hi(x[i].z)), __uint_as_float(tf32_hi(x[i].w)));
        const float4 lo = make_float4(x[i].x - hi.x, x[i].y - hi.y, x[i].z - hi.z, x[i].w - hi.w);
        if (u >= 16) {
          // V^T: element (dim n, key j) at (j/4)*LBO + (n/8)*SBO + (n%8)*16 + (j%4)*4.
          const int n0 = 4 * m;
          const uint32_t vt = kv0 + (uint32_t)(b * kTileBufBytes + kTileOffVt) +
                              (uint32_t)((j >> 2) * kTileVtLbo + (j & 3) * 4 + (n0 >> 3) * kTileVtSbo + (n0 & 7) * 16);
          const float hv[4] = {hi.x, hi.y, hi.z, hi.w}, lv[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {  // n0 % 4 == 0: dims n0 .. n0+3 share the 8-row group
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(vt + 16 * e), "f"(hv[e]) : "memory");
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(vt + 16 * e + kTileVtBytes), "f"(lv[e]) : "memory");
          }
        } else {
          // element (key j, dims 4m ..) of K: (d/4)*512 + (j/8)*128 + (j%8)*16
          const uint32_t dst = kv0 + (uint32_t)(b * kTileBufBytes) + (uint32_t)(m * 512 + ((u >> 2) & 3) * 128 + kk * 16);
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(hi.x), "f"(hi.y), "f"(hi.z),
                       "f"(hi.w)
                       : "memory");
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + kTileOpBytes), "f"(lo.x),
                       "f"(lo.y), "f"(lo.z), "f"(lo.w)
                       : "memory");
        }
      }
      if (kk == 0 && f4 == 0 && cw == 0) TQ_TILE_TR(11, g);
      fence_proxy_async_smem();  // the split halves are read by the tensor core
      if (kk == 0 && f4 == 0 && cw == 0) TQ_TILE_TR(12, g);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kTileBarKvReady + b));
      if (kk == 0 && f4 == 0 && cw == 0) TQ_TILE_TR(2, g);
      tile_advance(cur, items, count);
    }
  }

  // ---- every role done: free the tensor memory --------------------------------
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) TQ_TILE_TR(15, 0);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- merge of split prompt tiles ---------------------------------------------
// The plan's attention region ends with a trailer after the other items: word
// 0 the number E of rows of split tiles, then (after 8 words) E entries
// {output row, partial of (head 0, split 0), splits, partials between heads}.
// One warp per (entry, head) merges that row's per-piece partials
//   O = sum_s exp2(m_s - M) acc_s / sum_s exp2(m_s - M) l_s,  M = max_s m_s,
// lane i holding dims 2i and 2i+1.  Launched as a programmatic dependent of
// the attention launch that wrote the partials: it waits for that grid.
constexpr int kMergeThreads = 256;
__device__ __forceinline__ const int* tile_merge_trailer(const AttnParams& p) {
  return other_items(p) + 8 * (size_t)__ldg(warp_offsets(p) + p.n_warps);
}
__global__ void __launch_bounds__(kMergeThreads) tile_merge_kernel(const AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int* trailer = tile_merge_trailer(p);
  const int E = __ldg(trailer);
  const int* ent = trailer + 8;
  const int lane = threadIdx.x & 31;
  const long long tasks = (long long)E * p.n_head;
  const long long step = (long long)gridDim.x * (kMergeThreads / 32);
  for (long long task = (long long)blockIdx.x * (kMergeThreads / 32) + (threadIdx.x >> 5); task < tasks;
       task += step) {
    const int e = (int)(task / p.n_head), h = (int)(task - (long long)e * p.n_head);
    const int row = __ldg(ent + 4 * e), base = __ldg(ent + 4 * e + 1), ns = __ldg(ent + 4 * e + 2),
              hstride = __ldg(ent + 4 * e + 3);
    const long long idx0 = (long long)base + (long long)h * hstride;
    if (row < 0 || ns < 2 || hstride < 0 || idx0 < 0 || idx0 + ns > p.max_partials) {  // a corrupted plan
      if (lane == 0) raise_device_error(TQ_DEVERR_BAD_PLAN);
      continue;
    }
    float mmax = -INFINITY;
    for (int sp = 0; sp < ns; ++sp) mmax = fmaxf(mmax, __ldg(p.part_ml + 2 * (idx0 + sp)));
    float lt = 0.f;
    float2 acc = make_float2(0.f, 0.f);
    for (int sp = 0; sp < ns; ++sp) {
      const float2 ml = __ldg(reinterpret_cast<const float2*>(p.part_ml + 2 * (idx0 + sp)));
      const float w = ml.x == -INFINITY ? 0.f : fast_exp2(ml.x - mmax);
      lt = fmaf(ml.y, w, lt);
      const float2 a = __ldg(reinterpret_cast<const float2*>(p.part_acc + (idx0 + sp) * kHeadDim) + lane);
      acc = make_float2(fmaf(a.x, w, acc.x), fmaf(a.y, w, acc.y));
    }
    const float inv = 1.f / lt;
    reinterpret_cast<float2*>(p.out + (size_t)row * p.out_stride + h * kHeadDim)[lane] =
        make_float2(acc.x * inv, acc.y * inv);
  }
}

}  // namespace tq
