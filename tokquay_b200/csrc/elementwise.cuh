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
// Row kernels use one warp per row of C = 128*VPL floats held in registers
// (two-pass mean / variance, no re-read).
#pragma once

#include "common.cuh"

namespace tq {

template <int VPL>
__device__ __forceinline__ void ln_row(const float4 (&v)[VPL], const float4* __restrict__ w,
                                       const float4* __restrict__ b, float4* __restrict__ out,
                                       int lane, int C, float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) / (float)C;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + bb * bb) + (c * c + d * d);
  }
  const float rstd = rsqrtf(warp_sum(q) / (float)C + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int k = lane + 32 * i;
    const float4 ww = w[k], bv = b[k];
    float4 o;
    o.x = (v[i].x - mean) * rstd * ww.x + bv.x;
    o.y = (v[i].y - mean) * rstd * ww.y + bv.y;
    o.z = (v[i].z - mean) * rstd * ww.z + bv.z;
    o.w = (v[i].w - mean) * rstd * ww.w + bv.w;
    out[k] = o;
  }
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

template <int VPL>
__global__ void __launch_bounds__(256) embed_ln_kernel(const RowParams p) {
  const int lane = threadIdx.x & 31;
  const int TW = gridDim.x * (blockDim.x >> 5);
  const int n = *p.n_rows;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += TW) {
    int id = p.ids[r];
    int ps = p.pos[r];
    if (id < 0 || id >= p.vocab) {
      if (lane == 0) raise_device_error(TQ_DEVERR_BAD_TOKEN);
      id = 0;
    }
    ps = min(max(ps, 0), p.n_positions - 1);  // real rows are always in range (model.py:163)
    const float4* te = reinterpret_cast<const float4*>(p.wte + (size_t)id * p.C);
    const float4* pe = reinterpret_cast<const float4*>(p.wpe + (size_t)ps * p.C);
    float4* xo = reinterpret_cast<float4*>(p.x + (size_t)r * p.C);
    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float4 a = te[lane + 32 * i], b = pe[lane + 32 * i];
      v[i] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
      xo[lane + 32 * i] = v[i];
    }
    ln_row<VPL>(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b),
                reinterpret_cast<float4*>(p.xa + (size_t)r * p.C), lane, p.C, p.eps);
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) bias_residual_ln_kernel(const RowParams p) {
  const int lane = threadIdx.x & 31;
  const int TW = gridDim.x * (blockDim.x >> 5);
  const int n = *p.n_rows;
  const float4* bias = reinterpret_cast<const float4*>(p.bias);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += TW) {
    float4* xr = reinterpret_cast<float4*>(p.x + (size_t)r * p.C);
    const float4* yr = reinterpret_cast<const float4*>(p.y + (size_t)r * p.C);
    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int k = lane + 32 * i;
      float4 y = yr[k];
      for (int s = 1; s < p.n_parts; ++s) {  // split-K partial sums of the linear
        const float4 t = reinterpret_cast<const float4*>(p.y + s * p.part_stride + (size_t)r * p.C)[k];
        y.x += t.x;
        y.y += t.y;
        y.z += t.z;
        y.w += t.w;
      }
      const float4 a = xr[k], b = bias[k];
      // x + (y + b): the linear's bias first, as addmm produces it.
      v[i] = make_float4(a.x + (y.x + b.x), a.y + (y.y + b.y), a.z + (y.z + b.z), a.w + (y.w + b.w));
      xr[k] = v[i];
    }
    if (p.ln_w != nullptr)
      ln_row<VPL>(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b),
                  reinterpret_cast<float4*>(p.xa + (size_t)r * p.C), lane, p.C, p.eps);
  }
}

template <int VPL>
__global__ void __launch_bounds__(256) layernorm_rows_kernel(const RowParams p) {
  const int lane = threadIdx.x & 31;
  const int TW = gridDim.x * (blockDim.x >> 5);
  const int n = *p.n_rows;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n; r += TW) {
    const int src = p.rows ? p.rows[r] : r;
    const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)src * p.C);
    float4 v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = xr[lane + 32 * i];
    ln_row<VPL>(v, reinterpret_cast<const float4*>(p.ln_w), reinterpret_cast<const float4*>(p.ln_b),
                reinterpret_cast<float4*>(p.xa + (size_t)r * p.C), lane, p.C, p.eps);
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

// out = gelu_tanh(sum_s h_s + bias)  (or just the biased sum).
__global__ void __launch_bounds__(256) bias_gelu_kernel(const GeluParams p) {
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
    for (int s = 1; s < p.n_parts; ++s) {
      const float4 t = h[s * ps4 + i];
      v.x += t.x;
      v.y += t.y;
      v.z += t.z;
      v.w += t.w;
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

}  // namespace tq
