// Greedy decoding's last step fused into one kernel: ln_f of each sequence's
// last row, the tied LM head (logits = h . wte^T) and argmax over the vocabulary,
// with no [rows, vocab] logits tensor written or read back.
//
// Replaces tokquay/model.py:179-181 (last-row select, ln_f, x @ wte.T) and the
// greedy argmax of tokquay/engine.py:189-194 for steps whose every row samples
// greedily.  fp32 throughout on the CUDA cores (the reference's linears are
// fp32; tensor cores would change the products' rounding): only the order of
// the fp32 sums differs from a matmul library's.
//
// Work: CTA c owns vocabulary columns [c * kLmWidth, (c+1) * kLmWidth) (one
// slice per CTA for GPT-2: 143 CTAs of 352 columns).  Every CTA normalises all
// rows into shared memory (h: rows x C floats, at most 64 x 768 = 192 KiB),
// then streams its slice of the transposed, padded embedding matrix
// (wt[C][vstride]) through a kLmStages-deep ring of TMA bulk copies, kLmKTile
// rows of C per stage.  Thread layout: warp w holds rows 4w .. 4w+3, lane l
// the columns v0 + l + 32 j (j < kLmPerLane): 44 fp32 accumulators per thread;
// per 4 k, 4 broadcast float4 loads of h and 44 conflict-free loads of wt feed
// 176 FMAs, 16 warps per SM.
//
// Argmax across CTAs: each warp reduces its rows over its columns (torch's
// rules: NaN wins, the first index among equals), then one 64-bit atomicMax
// per row on (order-preserving value key << 32 | ~column).  The last CTA to
// finish (acq_rel counter) turns the winners into int64 tokens (and the max
// logits) and zeroes the scratch, so a replayed CUDA graph finds it clean.
#pragma once

#include "common.cuh"
#include "elementwise.cuh"  // argmax_take / argmax_warp: torch.argmax's rules

namespace tq {

constexpr int kLmMaxRows = 64;                // rows per launch (decode batch of up to 64)
constexpr int kLmThreads = 512;               // 16 warps x 4 rows
constexpr int kLmRowsPerWarp = kLmMaxRows / (kLmThreads / 32);
constexpr int kLmPerLane = 11;                // columns per lane
constexpr int kLmWidth = 32 * kLmPerLane;     // 352 vocabulary columns per CTA slice
constexpr int kLmKTile = 8;                   // rows of wt per stage
constexpr int kLmStages = 3;
constexpr int kLmMaxEmbd = 768;
constexpr int kLmStageBytes = kLmKTile * kLmWidth * 4;  // 11,264
constexpr int kLmHBytes = kLmMaxRows * kLmMaxEmbd * 4;  // 192 KiB: every row, every dim
constexpr int kLmSmemBytes = kLmHBytes + kLmStages * kLmStageBytes + 16 * kLmStages;

struct LmHeadParams {
  const float* x;          // residual stream rows
  long long x_stride;
  const int* sel;          // row of x for output row r (NULL: r)
  const float* ln_w;       // [C]
  const float* ln_b;       // [C]
  float eps;
  int C;                   // n_embd: a multiple of kLmKTile and of 32, <= kLmMaxEmbd
  const float* wt;         // [C][vstride]: wte transposed, columns >= V zero
  long long vstride;       // >= number of slices x kLmWidth
  int V;                   // vocabulary size
  long long* tokens;       // [max_rows] out
  float* max_logit;        // [max_rows] out, or NULL
  unsigned long long* best;  // [kLmMaxRows] scratch, zero between launches
  unsigned int* done;        // [1] scratch counter, zero between launches
  const int* n_rows;       // rows this launch (device), <= max_rows
  int max_rows;
};

// Order-preserving key of a float: larger values give larger keys; every NaN
// gives the largest key (torch.argmax counts NaN as the maximum); -0 == +0.
__device__ __forceinline__ unsigned int lm_key(float v) {
  if (v != v) return 0xffffffffu;
  unsigned int b = __float_as_uint(v == 0.f ? 0.f : v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float lm_unkey(unsigned int k) {
  if (k == 0xffffffffu) return __uint_as_float(0x7fc00000u);
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void __launch_bounds__(kLmThreads, 1) lm_head_argmax_kernel(const LmHeadParams p) {
  extern __shared__ __align__(128) unsigned char lm_smem[];
  float* hs = reinterpret_cast<float*>(lm_smem);                            // [rows][C]
  unsigned char* stages = lm_smem + kLmHBytes;                              // [kLmStages][kKTile][kLmWidth]
  const uint32_t full0 = smem_addr(stages + kLmStages * kLmStageBytes);    // one mbarrier per stage
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = p.C;
  const int n_ktiles = C / kLmKTile;
  const int v0 = blockIdx.x * kLmWidth;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLmStages; ++s) mbar_init(full0 + 8 * s, 1);
    mbar_init_fence();
  }
  __syncthreads();
  // The embedding matrix does not depend on the kernel before this one: the
  // ring's first stages go out before griddepcontrol.wait.
  auto issue = [&](int kt) {  // warp 0, lanes 0 .. kLmKTile-1: one row of wt each
    const int s = kt % kLmStages;
    const uint32_t bar = full0 + 8 * s;
    if (lane == 0) mbar_arrive_expect_tx(bar, kLmStageBytes);
    __syncwarp();
    if (lane < kLmKTile)
      bulk_copy_g2s(smem_addr(stages + s * kLmStageBytes) + lane * kLmWidth * 4,
                    p.wt + (size_t)(kt * kLmKTile + lane) * p.vstride + v0, kLmWidth * 4, bar);
  };
  if (warp == 0)
    for (int kt = 0; kt < kLmStages - 1 && kt < n_ktiles; ++kt) issue(kt);
  pdl_launch_dependents();
  pdl_wait();

  // ---- ln_f of every row into shared memory (warp w: rows w, w + 16, ...) ---------
  const int n = min(*p.n_rows, p.max_rows);
  for (int r = warp; r < n; r += kLmThreads / 32) {
    const float* xr = p.x + (size_t)(p.sel ? p.sel[r] : r) * p.x_stride;
    float v[kLmMaxEmbd / 32];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kLmMaxEmbd / 32; ++i) {
      v[i] = 32 * i + lane < C ? xr[32 * i + lane] : 0.f;
      sum += v[i];
    }
    const float mean = warp_sum(sum) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < kLmMaxEmbd / 32; ++i) {
      const float d = 32 * i + lane < C ? v[i] - mean : 0.f;
      q += d * d;
    }
    const float rstd = rsqrtf(warp_sum(q) / (float)C + p.eps);
#pragma unroll
    for (int i = 0; i < kLmMaxEmbd / 32; ++i) {
      const int c = 32 * i + lane;
      if (c < C) hs[r * C + c] = (v[i] - mean) * rstd * p.ln_w[c] + p.ln_b[c];
    }
  }
  __syncthreads();

  // ---- logits of rows r0 .. r0+3 x columns v0 + lane + 32 j --------------------------
  constexpr int R = kLmRowsPerWarp;
  float acc[R][kLmPerLane];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < kLmPerLane; ++j) acc[i][j] = 0.f;
  const int r0 = R * warp;
  const bool rows_live = r0 < n;  // warp-uniform: a warp past the rows only keeps the ring going
  bool ok = true;
  int kt = 0;
  for (; kt < n_ktiles; ++kt) {
    if (warp == 0 && kt + kLmStages - 1 < n_ktiles) issue(kt + kLmStages - 1);
    const int s = kt % kLmStages;
    ok = mbar_wait_bounded(full0 + 8 * s, (uint32_t)(kt / kLmStages) & 1u);
    if (rows_live) {
      const float* w = reinterpret_cast<const float*>(stages + s * kLmStageBytes);
#pragma unroll
      for (int k4 = 0; k4 < kLmKTile; k4 += 4) {
        const int c = kt * kLmKTile + k4;
        float4 h4[R];  // rows past n hold stale values, never read out
#pragma unroll
        for (int i = 0; i < R; ++i) h4[i] = *reinterpret_cast<const float4*>(hs + (r0 + i) * C + c);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (int j = 0; j < kLmPerLane; ++j) {
            const float wv = w[(k4 + kk) * kLmWidth + lane + 32 * j];
#pragma unroll
            for (int i = 0; i < R; ++i) {
              const float hv = kk == 0 ? h4[i].x : kk == 1 ? h4[i].y : kk == 2 ? h4[i].z : h4[i].w;
              acc[i][j] = fmaf(hv, wv, acc[i][j]);
            }
          }
        }
      }
    }
    // Every warp is done with stage s before warp 0 refills it (next iteration's
    // issue); a wait that ran out of time anywhere ends the loop for the whole CTA.
    ok = __syncthreads_and(ok);
    if (!ok) break;
  }
  if (!ok && warp == 0) {
    // Give the copies still in flight (issued for the stages after kt) a
    // bounded chance to land before the CTA exits.
    for (int k = kt + 1; k < min(n_ktiles, kt + kLmStages); ++k)
      if (!mbar_wait_bounded(full0 + 8 * (k % kLmStages), (uint32_t)(k / kLmStages) & 1u)) break;
  }

  // ---- argmax: per row over this lane's columns, the warp, then across CTAs ------
  if (ok && rows_live) {
#pragma unroll
    for (int i = 0; i < R; ++i) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < kLmPerLane; ++j) {
        const int col = v0 + lane + 32 * j;
        if (col < p.V) argmax_take(bv, bi, acc[i][j], col);
      }
      argmax_warp(bv, bi);
      if (lane == 0 && r0 + i < n && bi != 0x7fffffff)
        atomicMax(p.best + r0 + i,
                  ((unsigned long long)lm_key(bv) << 32) | (unsigned long long)(0xffffffffu - (unsigned)bi));
    }
  }
  __threadfence();  // this CTA's maxima are visible before its count below
  __syncthreads();
  // ---- the last CTA to finish writes the tokens and clears the scratch --------
  __shared__ unsigned int last;
  if (threadIdx.x == 0) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.done) : "memory");
    last = old == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  for (int r = threadIdx.x; r < kLmMaxRows; r += kLmThreads) {
    const unsigned long long b = atomicExch(p.best + r, 0ull);
    if (r < n) {
      p.tokens[r] = (long long)(0xffffffffu - (unsigned)(b & 0xffffffffu));
      if (p.max_logit) p.max_logit[r] = lm_unkey((unsigned)(b >> 32));
    }
  }
  if (threadIdx.x == 0) atomicExch(p.done, 0u);
}

}  // namespace tq
