// Fused LayerNorm / bias / GELU / residual kernels around the fp32 linears.
//
// The reference runs these as separate torch ops per layer
// (tokquay/model.py:116-124 for Block, :108-110 for MLP, :172 embeddings,
// :179-180 last-row select + ln_f).  Here each fusion reads its row once and
// writes its results once:
//   embed_ln           x = wte[id] + wpe[pos];  xa = LN(x)             (model.py:172 + ln_1 of layer 0)
//   bias_residual_ln   x += y + bias;           xa = LN(x) (optional)  (model.py:122-123 + next LN)
//   layernorm_rows     out[i] = LN(x[rows[i]])                         (model.py:179-180)
//   bias_gelu          out = gelu_tanh(sum of h parts + bias), or the biased
//                      sum alone                                         (model.py:110, :69)
// Linear outputs may arrive as split-K partial sums (K-slices computed by one
// batched fp32 matmul); the kernels add the parts up as they read them.
// LayerNorm follows nn.LayerNorm: biased variance, eps inside the square root.
// Row kernels use one block per row of C floats, one float4 per thread
// (two-pass mean / variance over the values held in registers, no re-read).
// Every kernel here is launched as a programmatic dependent of the kernel
// before it (its CTAs may be placed while that kernel drains) and waits for
// that kernel (griddepcontrol.wait) before its first load.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace tq {

// Sum over the block (one value per thread, blockDim = C/4 <= 256).
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // red may still be read by the previous reduction
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// LayerNorm of one row held one float4 per thread: biased variance, eps
// inside the root, then * w + b (nn.LayerNorm).
__device__ __forceinline__ float4 ln_value(const float4 v, const float4* __restrict__ w,
                                           const float4* __restrict__ b, int C, float eps, float* red) {
  const int k = threadIdx.x;
  const float mean = block_sum((v.x + v.y) + (v.z + v.w), red) / (float)C;
  const float a = v.x - mean, bb = v.y - mean, c = v.z - mean, d = v.w - mean;
  const float rstd = rsqrtf(block_sum((a * a + bb * bb) + (c * c + d * d), red) / (float)C + eps);
  const float4 ww = w[k], bv = b[k];
  return make_float4(a * rstd * ww.x + bv.x, bb * rstd * ww.y + bv.y, c * rstd * ww.z + bv.z,
                     d * rstd * ww.w + bv.w);
}

struct RowParams {
  float* x;            // residual stream [rows][C] (in/out)
  float* xa;           // LayerNorm output [rows][C] (may be null where noted)
  const float* y;      // linear output [rows][C] (bias_residual_ln), n_parts K-slices of it
  int n_parts;         // split-K partial sums of the linear output to add up (>= 1)
  long long part_stride;  // floats between consecutive partial sums
  const float* bias;   // [C]
  const float* ln_w;   // [C] (may be null: skip the LayerNorm)
  const float* ln_b;
  const int* ids;      // embed_ln: token ids
  const int* pos;      // embed_ln: absolute positions
  const float* wte;    // [vocab][C]
  const float* wpe;    // [n_positions][C]
  const int* rows;     // layernorm_rows: source row of each output row
  const int* n_rows;   // device-resident row count
  int C, vocab, n_positions;
  float eps;
};

// The row kernels run one block per row, one float4 of the row per thread
// (blockDim = C/4), so every load of a row is in flight at once; rows beyond
// the grid are taken in a grid-stride loop.

__global__ void __launch_bounds__(256) embed_ln_kernel(const RowParams p) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const int n = *p.n_rows;
  const int k = threadIdx.x;
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    int id = p.ids[r];
    int ps = p.pos[r];
    if (id < 0 || id >= p.vocab) {
      if (k == 0) raise_device_error(TQ_DEVERR_BAD_TOKEN);
      id = 0;
    }
    ps = min(max(ps, 0), p.n_positions - 1);  // real rows are always in range (model.py:163)
    const float4 a = reinterpret_cast<const float4*>(p.wte + (size_t)id * p.C)[k];
    const float4 b = reinterpret_cast<const float4*>(p.wpe + (size_t)ps * p.C)[k];
    const float4 v = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    reinterpret_cast<float4*>(p.x + (size_t)r * p.C)[k] = v;
    reinterpret_cast<float4*>(p.xa + (size_t)r * p.C)[k] =
        ln_value(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b), p.C,
                 p.eps, red);
  }
}

// NP > 0: exactly NP partial sums, loads unrolled; NP == 0: p.n_parts, looped.
template <int NP>
__global__ void __launch_bounds__(256) bias_residual_ln_kernel(const RowParams p) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const int n = *p.n_rows;
  const int k = threadIdx.x;
  const float4 b = reinterpret_cast<const float4*>(p.bias)[k];
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    const float4* yr = reinterpret_cast<const float4*>(p.y + (size_t)r * p.C) + k;
    const long long ps4 = p.part_stride >> 2;
    float4 y = yr[0];
    if (NP > 0) {
      float4 t[NP > 1 ? NP - 1 : 1];
#pragma unroll
      for (int s = 1; s < NP; ++s) t[s - 1] = yr[s * ps4];
#pragma unroll
      for (int s = 1; s < NP; ++s) {  // same order as the looped form: ((y0 + y1) + y2) + ...
        y.x += t[s - 1].x;
        y.y += t[s - 1].y;
        y.z += t[s - 1].z;
        y.w += t[s - 1].w;
      }
    } else {
      for (int s = 1; s < p.n_parts; ++s) {
        const float4 t = yr[s * ps4];
        y.x += t.x;
        y.y += t.y;
        y.z += t.z;
        y.w += t.w;
      }
    }
    float4* xr = reinterpret_cast<float4*>(p.x + (size_t)r * p.C) + k;
    const float4 a = *xr;
    // x + (y + b): the linear's bias first, as addmm produces it.
    const float4 v = make_float4(a.x + (y.x + b.x), a.y + (y.y + b.y), a.z + (y.z + b.z), a.w + (y.w + b.w));
    *xr = v;
    if (p.ln_w != nullptr)
      reinterpret_cast<float4*>(p.xa + (size_t)r * p.C)[k] =
          ln_value(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b), p.C,
                   p.eps, red);
  }
}

__global__ void __launch_bounds__(256) layernorm_rows_kernel(const RowParams p) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const int n = *p.n_rows;
  const int k = threadIdx.x;
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    const int src = p.rows ? p.rows[r] : r;
    const float4 v = reinterpret_cast<const float4*>(p.x + (size_t)src * p.C)[k];
    reinterpret_cast<float4*>(p.xa + (size_t)r * p.C)[k] =
        ln_value(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b), p.C,
                 p.eps, red);
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), F.gelu(approximate="tanh").
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

struct GeluParams {
  float* out;           // [rows][F]
  const float* h;       // [rows][F], n_parts split-K partial sums part_stride floats apart (may be out)
  int n_parts;
  long long part_stride;
  const float* bias;    // [F]
  const int* n_rows;    // device-resident row count
  int F;                // multiple of 4
  int gelu;             // 1: gelu_tanh(sum + bias); 0: sum + bias
};

// out = gelu_tanh(sum_s h_s + bias)  (or just the biased sum).  NP > 0:
// exactly NP partial sums, loads unrolled; NP == 0: p.n_parts, looped.
template <int NP>
__global__ void __launch_bounds__(256) bias_gelu_kernel(const GeluParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const long long f4 = p.F >> 2;
  const long long total = (long long)(*p.n_rows) * f4;
  const float4* h = reinterpret_cast<const float4*>(p.h);
  float4* out = reinterpret_cast<float4*>(p.out);
  const float4* bias = reinterpret_cast<const float4*>(p.bias);
  const long long ps4 = p.part_stride >> 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 b = bias[i % f4];
    float4 v = h[i];
    if (NP > 0) {
      float4 t[NP > 1 ? NP - 1 : 1];
#pragma unroll
      for (int s = 1; s < NP; ++s) t[s - 1] = h[s * ps4 + i];
#pragma unroll
      for (int s = 1; s < NP; ++s) {
        v.x += t[s - 1].x;
        v.y += t[s - 1].y;
        v.z += t[s - 1].z;
        v.w += t[s - 1].w;
      }
    } else {
      for (int s = 1; s < p.n_parts; ++s) {
        const float4 t = h[s * ps4 + i];
        v.x += t.x;
        v.y += t.y;
        v.z += t.z;
        v.w += t.w;
      }
    }
    if (p.gelu) {
      v.x = gelu_tanh(v.x + b.x);
      v.y = gelu_tanh(v.y + b.y);
      v.z = gelu_tanh(v.z + b.z);
      v.w = gelu_tanh(v.w + b.w);
    } else {
      v.x += b.x;
      v.y += b.y;
      v.z += b.z;
      v.w += b.w;
    }
    out[i] = v;
  }
}

// Greedy sampling: out[r] = argmax_c x[r][c], as torch.argmax(-1) picks it
// (tokquay/engine.py:189-194 samples greedy rows this way): NaN counts as the
// largest value, and among equal values the first index wins.
__device__ __forceinline__ void argmax_take(float& v, int& i, float v2, int i2) {
  const bool nan1 = v != v, nan2 = v2 != v2;
  const bool take = (nan1 || nan2) ? (nan2 && (!nan1 || i2 < i)) : (v2 > v || (v2 == v && i2 < i));
  if (take) {
    v = v2;
    i = i2;
  }
}

// A cluster of kArgmaxSlices CTAs per row: CTA k scans slice k of the
// columns (coalesced loads, kArgmaxUnroll in flight per thread; rows of odd
// length are not 16-byte aligned), reduces it over its warps, and CTA 0 of the
// cluster combines the slices' results through distributed shared memory.
// Slices are in column order and every reduction keeps the first of equal
// values, so ties resolve as a left-to-right scan would.
#ifndef TQ_ARGMAX_THREADS
#define TQ_ARGMAX_THREADS 512
#endif
#ifndef TQ_ARGMAX_UNROLL
#define TQ_ARGMAX_UNROLL 8
#endif
constexpr int kArgmaxSlices = 8;
constexpr int kArgmaxThreads = TQ_ARGMAX_THREADS;
constexpr int kArgmaxUnroll = TQ_ARGMAX_UNROLL;

__device__ __forceinline__ void argmax_warp(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(kFullMask, v, o);
    const int i2 = __shfl_xor_sync(kFullMask, i, o);
    argmax_take(v, i, v2, i2);
  }
}

__global__ void __cluster_dims__(kArgmaxSlices, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_rows_kernel(const float* __restrict__ x, long long stride, int n_cols, long long* __restrict__ out,
                       const int* n_rows) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  __shared__ float slice_v;
  __shared__ int slice_i;
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int r = blockIdx.x / kArgmaxSlices;  // cluster-uniform
  const int k = (int)cluster.block_rank();
  const bool live = r < *n_rows;
  if (live) {
    const int per = (n_cols + kArgmaxSlices - 1) / kArgmaxSlices;
    const int c_lo = k * per, c_hi = min(n_cols, c_lo + per);
    const float* row = x + (size_t)r * stride;
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int c0 = c_lo + (int)threadIdx.x; c0 < c_hi; c0 += kArgmaxUnroll * kArgmaxThreads) {
      float u[kArgmaxUnroll];
#pragma unroll
      for (int j = 0; j < kArgmaxUnroll; ++j) {
        const int c = c0 + j * kArgmaxThreads;
        u[j] = c < c_hi ? __ldg(row + c) : -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < kArgmaxUnroll; ++j) {
        const int c = c0 + j * kArgmaxThreads;
        if (c < c_hi) argmax_take(v, i, u[j], c);
      }
    }
    argmax_warp(v, i);
    if (lane == 0) {
      sv[w] = v;
      si[w] = i;
    }
    __syncthreads();
    if (w == 0) {
      v = lane < kArgmaxThreads / 32 ? sv[lane] : -INFINITY;
      i = lane < kArgmaxThreads / 32 ? si[lane] : 0x7fffffff;
      argmax_warp(v, i);
      if (lane == 0) {
        slice_v = v;
        slice_i = i;
      }
    }
  }
  cluster.sync();  // every slice's result is in its CTA's shared memory
  if (live && k == 0 && w == 0) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    if (lane < kArgmaxSlices) {
      v = *cluster.map_shared_rank(&slice_v, lane);
      i = *cluster.map_shared_rank(&slice_i, lane);
    }
    argmax_warp(v, i);
    if (lane == 0) out[r] = i;
  }
  cluster.sync();  // no CTA leaves while CTA 0 may still read its shared memory
}

}  // namespace tq
