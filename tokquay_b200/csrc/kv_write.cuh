// KV-write: scatter each step's new K/V rows straight into their pool slots.
//
// Replaces the advanced-index scatter of the reference
// (tokquay/kv_cache.py:228-232): pool[blk, layer, kv, :, off] = k/v[b, :, t].
// The source is the c_attn output, one row of [q | k | v] (3*C floats) per new
// token; slot_mapping[n] = block_table[p // bs] * bs + p % bs for the token's
// absolute position p.  Padded query slots of the reference never exist here:
// only real tokens have rows, so nothing outside a sequence's blocks is written.
#pragma once

#include "common.cuh"

namespace tq {

struct KvWriteParams {
  float* pool;
  long long num_blocks;
  int n_layer, n_head, block_size, log2_bs, layer;
  const float* qkv;
  long long qkv_stride;  // floats between token rows
  long long k_col, v_col;  // float column of K head 0 and V head 0 in a row
  const int* slots;
  const int* n_tokens;   // device-resident count
};

// One block per token: thread t copies float4 t of the token's K and V rows
// (2 * n_head * 16 float4), 16-byte loads of contiguous source floats and
// 16-byte stores into 2 * n_head pool rows of 256 bytes each.
__global__ void __launch_bounds__(1024) kv_write_kernel(const KvWriteParams p) {
  pdl_launch_dependents();  // the attention that follows may start its prologue now
  pdl_wait();               // the kernel that wrote the K/V rows is complete
  const int n_tok = *p.n_tokens;
  const int per_kv4 = p.n_head * 16;  // float4 per K (or V) row of one token
  const long long pool_slots = p.num_blocks << p.log2_bs;
  const size_t head_stride4 = (size_t)p.block_size * 16;
  auto valid = [&](long long slot) {
    if (slot >= 0 && slot < pool_slots) return true;
    if (threadIdx.x == 0) raise_device_error(TQ_DEVERR_BAD_SLOT);
    return false;
  };
  auto dst_of = [&](long long slot, int kv, int g) {
    const long long blk = slot >> p.log2_bs;
    const int off = (int)(slot & (p.block_size - 1));
    return reinterpret_cast<float4*>(
               p.pool + ((((size_t)blk * p.n_layer + p.layer) * 2 + kv) * p.n_head) * (size_t)p.block_size * 64 +
               (size_t)off * 64) +
           (g >> 4) * head_stride4 + (g & 15);
  };
  // Two tokens per iteration: both slots, then both tokens' loads, are in
  // flight before anything is stored.
  for (int n = blockIdx.x; n < n_tok; n += 2 * gridDim.x) {
    const int n2 = n + gridDim.x;
    const bool has2 = n2 < n_tok;
    const long long slot = p.slots[n];
    const long long slot2 = has2 ? p.slots[n2] : 0;
    const bool ok = valid(slot), ok2 = has2 && valid(slot2);
    for (int f = threadIdx.x; f < 2 * per_kv4; f += blockDim.x) {
      const int kv = f >= per_kv4;
      const int g = f - kv * per_kv4;
      const long long col = kv ? p.v_col : p.k_col;
      float4 v, v2;
      if (ok) v = reinterpret_cast<const float4*>(p.qkv + (size_t)n * p.qkv_stride + col)[g];
      if (ok2) v2 = reinterpret_cast<const float4*>(p.qkv + (size_t)n2 * p.qkv_stride + col)[g];
      if (ok) *dst_of(slot, kv, g) = v;
      if (ok2) *dst_of(slot2, kv, g) = v2;
    }
  }
}

// Fused c_attn epilogue: the qkv row is the sum of the split-K partial sums
// of the c_attn matmul plus its bias (tokquay/model.py:69); q goes to q_out,
// K and V straight into their pool slot (tokquay/kv_cache.py:228-232), so the
// K/V columns are never written anywhere else.
struct QkvWriteParams {
  float* q_out;
  long long q_stride;      // floats between q rows
  const float* parts;      // [n_parts][rows][3C]
  int n_parts;
  long long part_stride;   // floats between partial sums
  const float* bias;       // [3C]
  float* pool;
  long long num_blocks;
  int n_layer, n_head, block_size, log2_bs, layer;
  const int* slots;
  const int* n_rows;       // device-resident count
};

// One block per row, thread t owns float4 t of the 3C columns (blockDim =
// 3C/4).  NP > 0: exactly NP partial sums, loads unrolled; NP == 0: looped.
// Summation order matches the unfused path (bias_gelu_kernel): ((p0 + p1) + ...) + bias.
#ifdef TQ_ATTN_TRACE
__device__ unsigned long long g_qkv_write_end;
// Per layer: {first CTA entry, first return from the wait, last CTA end} (ns).
__device__ unsigned long long g_qkv_times[64][3];
#endif
template <int NP>
__global__ void __launch_bounds__(1024) qkv_bias_kv_write_kernel(const QkvWriteParams p) {
#ifdef TQ_ATTN_TRACE
  unsigned long long tq_t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tq_t0));
#endif
  pdl_launch_dependents();  // the attention that follows may start its prologue now
  pdl_wait();               // the c_attn matmul before it is complete
#ifdef TQ_ATTN_TRACE
  if (threadIdx.x == 0 && p.layer < 64) {
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    atomicMin(&g_qkv_times[p.layer][0], tq_t0);
    atomicMin(&g_qkv_times[p.layer][1], t1);
  }
#endif
  const int n = *p.n_rows;
  const int C4 = p.n_head * 16;  // float4 per q (or K, or V) row
  const int t = threadIdx.x;
  const long long pool_slots = p.num_blocks << p.log2_bs;
  const float4 b = reinterpret_cast<const float4*>(p.bias)[t];
  const long long ps4 = p.part_stride >> 2;
  // Row r: the sum of its partial sums plus the bias, and (K/V threads) its slot.
  auto load_row = [&](int r, float4& v, long long& slot) {
    const float4* src = reinterpret_cast<const float4*>(p.parts) + (size_t)r * 3 * C4 + t;
    slot = t < C4 ? 0 : p.slots[r];
    v = src[0];
    if (NP > 0) {
      float4 u[NP > 1 ? NP - 1 : 1];
#pragma unroll
      for (int s = 1; s < NP; ++s) u[s - 1] = src[s * ps4];
#pragma unroll
      for (int s = 1; s < NP; ++s) {
        v.x += u[s - 1].x;
        v.y += u[s - 1].y;
        v.z += u[s - 1].z;
        v.w += u[s - 1].w;
      }
    } else {
      for (int s = 1; s < p.n_parts; ++s) {
        const float4 u = src[s * ps4];
        v.x += u.x;
        v.y += u.y;
        v.z += u.z;
        v.w += u.w;
      }
    }
    v = make_float4(v.x + b.x, v.y + b.y, v.z + b.z, v.w + b.w);
  };
  auto store_row = [&](int r, const float4& v, long long slot) {
    if (t < C4) {
      reinterpret_cast<float4*>(p.q_out + (size_t)r * p.q_stride)[t] = v;
      return;
    }
    if (slot < 0 || slot >= pool_slots) {
      if (t == C4) raise_device_error(TQ_DEVERR_BAD_SLOT);
      return;
    }
    const int kv = t >= 2 * C4;
    const int g = t - C4 - kv * C4;  // float4 within the K (or V) row: head g / 16, dims (g % 16) * 4
    const long long blk = slot >> p.log2_bs;
    const int off = (int)(slot & (p.block_size - 1));
    float4* dst = reinterpret_cast<float4*>(
        p.pool + (((((size_t)blk * p.n_layer + p.layer) * 2 + kv) * p.n_head + (g >> 4)) * (size_t)p.block_size +
                  off) * 64);
    dst[g & 15] = v;
  };
  // Two rows per iteration, both rows' loads in flight before either is stored.
  for (int r = blockIdx.x; r < n; r += 2 * gridDim.x) {
    const int r2 = r + gridDim.x;
    float4 v, v2;
    long long slot = 0, slot2 = 0;
    load_row(r, v, slot);
    if (r2 < n) load_row(r2, v2, slot2);
    store_row(r, v, slot);
    if (r2 < n) store_row(r2, v2, slot2);
  }
#ifdef TQ_ATTN_TRACE
  if (threadIdx.x == 0) {  // tuning builds: the latest end of any CTA of this kernel
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    atomicMax(&g_qkv_write_end, t);
    if (p.layer < 64) atomicMax(&g_qkv_times[p.layer][2], t);
  }
#endif
}

}  // namespace tq
