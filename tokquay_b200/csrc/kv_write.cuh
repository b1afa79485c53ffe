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
  const int n_tok = *p.n_tokens;
  const int per_kv4 = p.n_head * 16;  // float4 per K (or V) row of one token
  const long long pool_slots = p.num_blocks << p.log2_bs;
  const size_t head_stride4 = (size_t)p.block_size * 16;
  for (int n = blockIdx.x; n < n_tok; n += gridDim.x) {
    const long long slot = p.slots[n];
    if (slot < 0 || slot >= pool_slots) {
      if (threadIdx.x == 0) raise_device_error(TQ_DEVERR_BAD_SLOT);
      continue;
    }
    const long long blk = slot >> p.log2_bs;
    const int off = (int)(slot & (p.block_size - 1));
    for (int f = threadIdx.x; f < 2 * per_kv4; f += blockDim.x) {
      const int kv = f >= per_kv4;
      const int g = f - kv * per_kv4;
      const float4 v = reinterpret_cast<const float4*>(p.qkv + (size_t)n * p.qkv_stride +
                                                       (kv ? p.v_col : p.k_col))[g];
      float4* dst = reinterpret_cast<float4*>(
          p.pool + ((((size_t)blk * p.n_layer + p.layer) * 2 + kv) * p.n_head) * (size_t)p.block_size * 64 +
          (size_t)off * 64);
      dst[(g >> 4) * head_stride4 + (g & 15)] = v;
    }
  }
}

}  // namespace tq
