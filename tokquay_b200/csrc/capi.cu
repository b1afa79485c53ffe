// extern "C" entry points of libtokquay_b200.so (declared in include/tokquay_b200.h).
//
// The whole device side is this one translation unit: it includes every
// kernel header, validates arguments on the host (the kernels assume them),
// sizes persistent grids from the device's SM count and launches on the
// caller's stream.  No entry point allocates device memory.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <mutex>

#include "../../include/tokquay_b200.h"
#include "common.cuh"
#include "elementwise.cuh"
#include "host_error.h"
#include "kv_write.cuh"
#include "lm_head.cuh"
#include "paged_attention.cuh"

namespace tq {

char* error_buffer() {
  static thread_local char buf[kErrorBufferLen] = {0};
  return buf;
}

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sm_count = 0;
  bool ready = false;
};

DeviceInfo g_devices[kMaxDevices];
std::mutex g_devices_mu;

// SM count of the current device; on first use per device also raises the
// attention kernel's dynamic shared-memory limit.
int device_setup(int* sm_count) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(TQ_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_devices_mu);
  DeviceInfo& d = g_devices[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return set_error(TQ_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    e = cudaFuncSetAttribute(paged_attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kAttnSmemBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(paged_attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kTileLaunchSmemBytes);
    if (e != cudaSuccess)
      return set_error(TQ_ERR_CUDA, "cudaFuncSetAttribute(paged_attention): %s",
                       cudaGetErrorString(e));
    e = cudaFuncSetAttribute(lm_head_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kLmSmemBytes);
    if (e != cudaSuccess)
      return set_error(TQ_ERR_CUDA, "cudaFuncSetAttribute(lm_head_argmax): %s", cudaGetErrorString(e));
    d.ready = true;
  }
  *sm_count = d.sm_count;
  return TQ_OK;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return TQ_OK;
}

// Launches `kernel` as a programmatic dependent of the kernel before it on
// `s`: its CTAs may be placed while that kernel drains.  Every kernel
// launched this way calls pdl_wait() before it reads or writes anything the
// kernels before it may touch.  A launch error is left for check_launch().
template <typename... KArgs, typename... Args>
void launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  (void)cudaLaunchKernelEx(&cfg, kernel, args...);
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int log2_exact(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

int check_pool(const float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
               int32_t block_size, int32_t head_dim, int32_t layer) {
  if (pool == nullptr) return set_error(TQ_ERR_INVALID, "pool must not be NULL");
  if (!aligned(pool, 16)) return set_error(TQ_ERR_INVALID, "pool must be 16-byte aligned");
  if (head_dim != kHeadDim)
    return set_error(TQ_ERR_UNSUPPORTED, "head_dim must be %d, got %d", kHeadDim, head_dim);
  if (block_size < 1 || block_size > 256 || (block_size & (block_size - 1)) != 0)
    return set_error(TQ_ERR_UNSUPPORTED, "block_size must be a power of two in [1, 256], got %d",
                     block_size);
  if (num_blocks < 1 || num_blocks * (int64_t)block_size > INT32_MAX)
    return set_error(TQ_ERR_UNSUPPORTED, "num_blocks * block_size must be in [1, 2^31)");
  if (n_head < 1 || n_layer < 1 || layer < 0 || layer >= n_layer)
    return set_error(TQ_ERR_INVALID, "layer %d outside [0, %d) or n_head %d < 1", layer, n_layer,
                     n_head);
  return TQ_OK;
}

// Checks shared by the attention entry points; fills everything but the
// split-K scratch.  n_ctas == 0 (an empty plan) launches nothing.
int attention_params(float* out, int64_t out_row_stride, const float* q, int64_t q_row_stride,
                     const float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
                     int32_t block_size, int32_t head_dim, int32_t layer, const int32_t* block_tables,
                     int32_t table_stride, const int32_t* attn_plan, int32_t n_ctas, float scale,
                     AttnParams* p) {
  int st = check_pool(pool, num_blocks, n_layer, n_head, block_size, head_dim, layer);
  if (st) return st;
  if (n_ctas < 0 || n_ctas > 0xffff) return set_error(TQ_ERR_INVALID, "n_ctas must be in [0, 65535]");
  if (n_ctas == 0) return TQ_OK;
  if (!out || !q || !block_tables || !attn_plan)
    return set_error(TQ_ERR_INVALID, "out, q, block_tables and attn_plan must not be NULL");
  if (!aligned(q, 16) || q_row_stride % 4)
    return set_error(TQ_ERR_INVALID, "q rows must be 16-byte aligned");
  if (!aligned(out, 16) || out_row_stride % 4)
    return set_error(TQ_ERR_INVALID, "out rows must be 16-byte aligned");
  if (!aligned(attn_plan, 16)) return set_error(TQ_ERR_INVALID, "attn_plan must be 16-byte aligned");
  if (table_stride < 0) return set_error(TQ_ERR_INVALID, "table_stride must be >= 0");
  if (!(scale > 0.f) || !std::isfinite(scale)) return set_error(TQ_ERR_INVALID, "bad scale");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  p->out = out;
  p->out_stride = out_row_stride;
  p->q = q;
  p->q_stride = q_row_stride;
  p->pool = pool;
  p->num_blocks = num_blocks;
  p->n_layer = n_layer;
  p->n_head = n_head;
  p->block_size = block_size;
  p->log2_bs = log2_exact(block_size);
  p->layer = layer;
  p->tables = block_tables;
  p->table_stride = table_stride;
  p->attn = attn_plan;
  p->n_warps = n_ctas * kAttnWarps;
  p->part_ml = p->part_acc = nullptr;
  p->part_cnt = nullptr;
  p->max_partials = 0;
  p->scale_log2 = scale * 1.4426950408889634f;
  return TQ_OK;
}

// The attention launch, as a programmatic dependent of the kernel before it
// in the stream: its CTAs may start (barriers, work items, block ids, and for
// decode items the K/V rows before the new key) while that kernel finishes;
// everything else waits for it.
cudaError_t launch_attention(const AttnParams& p, int n_ctas, bool with_tiles, bool tile_merge,
                             cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_ctas);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = with_tiles ? kTileLaunchSmemBytes : kAttnSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = with_tiles ? cudaLaunchKernelEx(&cfg, paged_attention_kernel<true>, p)
                             : cudaLaunchKernelEx(&cfg, paged_attention_kernel<false>, p);
  if (e != cudaSuccess || !tile_merge) return e;
  // The pieces of split prompt tiles, merged once the attention grid is done
  // (the merge kernel's CTAs may be placed while it drains).
  int sms = 0;
  if (device_setup(&sms) != TQ_OK) return cudaErrorUnknown;
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  return cudaLaunchKernelEx(&cfg, tile_merge_kernel, p);
}

int check_embd(int32_t n_embd) {
  if (n_embd < 128 || n_embd > 1024 || n_embd % 128 != 0)
    return set_error(TQ_ERR_UNSUPPORTED, "n_embd must be a multiple of 128 in [128, 1024], got %d",
                     n_embd);
  return TQ_OK;
}

// Grid for block-per-row kernels: one block per row, capped at 16 blocks per
// SM (the kernels grid-stride beyond that).
int row_grid(int64_t rows, int sm_count) {
  return (int)std::min<int64_t>(std::max<int64_t>(rows, 1), (int64_t)sm_count * 16);
}

}  // namespace
}  // namespace tq

using namespace tq;

extern "C" {

int tq_abi_version(void) { return TQ_ABI_VERSION; }

#ifdef TQ_TILE_DEBUG
extern "C" TQ_API int tq_debug_cta_times(unsigned long long* host) {
  cudaDeviceSynchronize();
  cudaError_t e = cudaMemcpyFromSymbol(host, tq::g_cta_time, sizeof(tq::g_cta_time));
  unsigned long long zero[3 * 1024] = {};
  cudaMemcpyToSymbol(tq::g_cta_time, zero, sizeof(zero));
  return e == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}
extern "C" TQ_API int tq_debug_tile_trace(long long* host) {
  cudaDeviceSynchronize();
  cudaError_t e = cudaMemcpyFromSymbol(host, tq::g_tile_trace, sizeof(tq::g_tile_trace));
  return e == cudaSuccess ? TQ_OK : TQ_ERR_CUDA;
}
#endif

int tq_attention_chunk_keys(void) { return kChunk; }

int tq_attention_warps(void) { return kAttnWarps; }

const char* tq_last_error(void) { return error_buffer(); }

int tq_device_status(int clear, int32_t* bits) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "read device error word: %s", cudaGetErrorString(e));
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess)
      return set_error(TQ_ERR_CUDA, "clear device error word: %s", cudaGetErrorString(e));
  }
  if (bits) *bits = v;
  return TQ_OK;
}

int tq_kv_write(float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
                int32_t block_size, int32_t head_dim, int32_t layer, const float* qkv,
                int64_t qkv_row_stride, int64_t k_col, int64_t v_col,
                const int32_t* slot_mapping, const int32_t* d_num_tokens, int32_t max_tokens,
                void* stream) {
  int st = check_pool(pool, num_blocks, n_layer, n_head, block_size, head_dim, layer);
  if (st) return st;
  if (max_tokens < 0) return set_error(TQ_ERR_INVALID, "max_tokens must be >= 0");
  if (max_tokens == 0) return TQ_OK;
  if (!qkv || !slot_mapping || !d_num_tokens)
    return set_error(TQ_ERR_INVALID, "qkv, slot_mapping and d_num_tokens must not be NULL");
  if (!aligned(qkv, 16) || qkv_row_stride % 4 || k_col % 4 || v_col % 4)
    return set_error(TQ_ERR_INVALID, "qkv rows and the K/V columns must be 16-byte aligned");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  KvWriteParams p;
  p.pool = pool;
  p.num_blocks = num_blocks;
  p.n_layer = n_layer;
  p.n_head = n_head;
  p.block_size = block_size;
  p.log2_bs = log2_exact(block_size);
  p.layer = layer;
  p.qkv = qkv;
  p.qkv_stride = qkv_row_stride;
  p.k_col = k_col;
  p.v_col = v_col;
  p.slots = slot_mapping;
  p.n_tokens = d_num_tokens;
  const int threads = std::min(1024, ((2 * n_head * 16 + 31) / 32) * 32);
  launch_dependent(kv_write_kernel, row_grid(max_tokens, sms), threads, (cudaStream_t)stream, p);
  return check_launch("kv_write");
}

int tq_qkv_bias_kv_write(float* q_out, int64_t q_row_stride, const float* parts, int32_t n_parts,
                         int64_t part_stride, const float* bias, float* pool, int64_t num_blocks,
                         int32_t n_layer, int32_t n_head, int32_t block_size, int32_t head_dim,
                         int32_t layer, const int32_t* slot_mapping, const int32_t* d_num_rows,
                         int32_t max_rows, void* stream) {
  int st = check_pool(pool, num_blocks, n_layer, n_head, block_size, head_dim, layer);
  if (st) return st;
  if (max_rows < 0) return set_error(TQ_ERR_INVALID, "max_rows must be >= 0");
  if (n_head > 21) return set_error(TQ_ERR_UNSUPPORTED, "qkv_bias_kv_write: n_head must be at most 21");
  const int64_t cols = 3LL * n_head * head_dim;
  if (n_parts < 1 || (n_parts > 1 && (part_stride < (int64_t)max_rows * cols || part_stride % 4)))
    return set_error(TQ_ERR_INVALID, "qkv_bias_kv_write: bad split-K parts");
  if (max_rows == 0) return TQ_OK;
  if (!q_out || !parts || !bias || !slot_mapping || !d_num_rows)
    return set_error(TQ_ERR_INVALID, "qkv_bias_kv_write: NULL argument");
  if (!aligned(q_out, 16) || q_row_stride % 4 || !aligned(parts, 16) || !aligned(bias, 16))
    return set_error(TQ_ERR_INVALID, "qkv_bias_kv_write: arrays must be 16-byte aligned");
  if (reinterpret_cast<const char*>(q_out) < reinterpret_cast<const char*>(parts + part_stride * (n_parts - 1) +
                                                                           (int64_t)max_rows * cols) &&
      reinterpret_cast<const char*>(parts) < reinterpret_cast<const char*>(q_out + (int64_t)max_rows * q_row_stride))
    return set_error(TQ_ERR_INVALID, "qkv_bias_kv_write: q_out overlaps the partial sums");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  QkvWriteParams p;
  p.q_out = q_out;
  p.q_stride = q_row_stride;
  p.parts = parts;
  p.n_parts = n_parts;
  p.part_stride = part_stride;
  p.bias = bias;
  p.pool = pool;
  p.num_blocks = num_blocks;
  p.n_layer = n_layer;
  p.n_head = n_head;
  p.block_size = block_size;
  p.log2_bs = log2_exact(block_size);
  p.layer = layer;
  p.slots = slot_mapping;
  p.n_rows = d_num_rows;
  const int threads = (int)(cols / 4);
  const int grid = row_grid(max_rows, sms);
  const cudaStream_t s = (cudaStream_t)stream;
  switch (n_parts) {  // partial-sum loads unrolled for the split counts the model uses
    case 1: launch_dependent(qkv_bias_kv_write_kernel<1>, grid, threads, s, p); break;
    case 2: launch_dependent(qkv_bias_kv_write_kernel<2>, grid, threads, s, p); break;
    case 4: launch_dependent(qkv_bias_kv_write_kernel<4>, grid, threads, s, p); break;
    case 8: launch_dependent(qkv_bias_kv_write_kernel<8>, grid, threads, s, p); break;
    default: launch_dependent(qkv_bias_kv_write_kernel<0>, grid, threads, s, p); break;
  }
  return check_launch("qkv_bias_kv_write");
}

int tq_paged_attention(float* out, int64_t out_row_stride, const float* q, int64_t q_row_stride,
                       const float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
                       int32_t block_size, int32_t head_dim, int32_t layer,
                       const int32_t* block_tables, int32_t table_stride,
                       const int32_t* attn_plan, int32_t n_ctas, int32_t with_tiles,
                       float* partial_ml, float* partial_acc, int32_t* partial_counters,
                       int32_t max_partials, float scale, void* stream) {
  if (max_partials < 0) return set_error(TQ_ERR_INVALID, "negative capacity");
  if (max_partials > 0) {
    if (!partial_ml || !partial_acc || !partial_counters)
      return set_error(TQ_ERR_INVALID, "split-K scratch must not be NULL");
    if (!aligned(partial_acc, 16) || !aligned(partial_ml, 8) || !aligned(partial_counters, 4))
      return set_error(TQ_ERR_INVALID, "split-K scratch misaligned");
  }
  AttnParams p;
  int st = attention_params(out, out_row_stride, q, q_row_stride, pool, num_blocks, n_layer, n_head,
                            block_size, head_dim, layer, block_tables, table_stride, attn_plan, n_ctas,
                            scale, &p);
  if (st || n_ctas == 0) return st;
  p.part_ml = partial_ml;
  p.part_acc = partial_acc;
  p.part_cnt = partial_counters;
  p.max_partials = max_partials;
  if (with_tiles & ~(TQ_ATTN_TILES | TQ_ATTN_TILE_MERGE) || (with_tiles & TQ_ATTN_TILE_MERGE && !(with_tiles & TQ_ATTN_TILES)))
    return set_error(TQ_ERR_INVALID, "with_tiles must be 0, TQ_ATTN_TILES or TQ_ATTN_TILES | TQ_ATTN_TILE_MERGE");
  const cudaError_t e = launch_attention(p, n_ctas, with_tiles & TQ_ATTN_TILES,
                                         (with_tiles & TQ_ATTN_TILE_MERGE) != 0, (cudaStream_t)stream);
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "paged_attention launch: %s", cudaGetErrorString(e));
  return check_launch("paged_attention");
}

}  // extern "C"

// ---- paged attention whose split-K scratch lives inside this library -------
//
// tq_paged_attention needs caller-owned split-K scratch.  Some callers cannot
// provide it: a host runtime that gives this library only the tensors it
// already owns and forbids side allocations (a serving process working inside
// a fixed memory budget, or an embedding that has no device allocator of its
// own at the point it runs attention).  tq_paged_attention_noalloc serves
// them: the scratch is the file-scope array below, which every GPU that loads
// this library holds until the process exits (8.78 MB), so the entry
// point itself never allocates.  Host code must not pass the array's name to
// a kernel -- on the host that name is only a stand-in for the symbol -- so
// its device address is looked up once per device with cudaGetSymbolAddress.
namespace tq {
namespace {

constexpr int kNoAllocMaxPartials = TQ_NOALLOC_MAX_PARTIALS;
constexpr size_t kNoAllocCounterBytes = (size_t)kNoAllocMaxPartials * sizeof(int);        // 128 KiB
constexpr size_t kNoAllocMlBytes = (size_t)kNoAllocMaxPartials * 2 * sizeof(float);       // 256 KiB
constexpr size_t kNoAllocAccBytes = (size_t)kNoAllocMaxPartials * kHeadDim * sizeof(float);  // 8 MiB

// [counters | (m, l) pairs | accumulators]; each region starts 256-byte aligned.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocCounterBytes + kNoAllocMlBytes +
                                                                 kNoAllocAccBytes];

unsigned char* g_noalloc_base[kMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device, looked up on the
// first call per device and kept: valid for the device's primary context, so
// not across a cudaDeviceReset (the header says so).
int noalloc_scratch(unsigned char** base) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(TQ_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_base[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return set_error(TQ_ERR_CUDA, "cudaGetSymbolAddress(split-K scratch): %s", cudaGetErrorString(e));
    g_noalloc_base[dev] = static_cast<unsigned char*>(ptr);
  }
  *base = g_noalloc_base[dev];
  return TQ_OK;
}

}  // namespace
}  // namespace tq

extern "C" {

int tq_paged_attention_noalloc(float* out, int64_t out_row_stride, const float* q,
                               int64_t q_row_stride, const float* pool, int64_t num_blocks,
                               int32_t n_layer, int32_t n_head, int32_t block_size,
                               int32_t head_dim, int32_t layer, const int32_t* block_tables,
                               int32_t table_stride, const int32_t* attn_plan, int32_t n_ctas,
                               int32_t num_partials, float scale, void* stream) {
  if (num_partials < 0) return set_error(TQ_ERR_INVALID, "negative capacity");
  if (num_partials > kNoAllocMaxPartials)
    return set_error(TQ_ERR_CAPACITY,
                     "the plan needs %d split-K partials but the no-allocation entry point holds at "
                     "most %d; plan with fewer splits or use tq_paged_attention with your own scratch",
                     num_partials, kNoAllocMaxPartials);
  AttnParams p;
  int st = attention_params(out, out_row_stride, q, q_row_stride, pool, num_blocks, n_layer, n_head,
                            block_size, head_dim, layer, block_tables, table_stride, attn_plan, n_ctas,
                            scale, &p);
  if (st || n_ctas == 0) return st;
  unsigned char* base = nullptr;
  if ((st = noalloc_scratch(&base))) return st;
  const cudaStream_t s = (cudaStream_t)stream;
  // The split counters must start at zero.  A completed launch leaves them at
  // zero, but one that gave up early (a flagged device error) may not: clear
  // the ones this plan uses.  The other regions are fully written before read.
  if (num_partials > 0) {
    const cudaError_t e = cudaMemsetAsync(base, 0, (size_t)num_partials * sizeof(int), s);
    if (e != cudaSuccess)
      return set_error(TQ_ERR_CUDA, "clearing split-K counters: %s", cudaGetErrorString(e));
  }
  p.part_cnt = reinterpret_cast<int*>(base);
  p.part_ml = reinterpret_cast<float*>(base + kNoAllocCounterBytes);
  p.part_acc = reinterpret_cast<float*>(base + kNoAllocCounterBytes + kNoAllocMlBytes);
  p.max_partials = num_partials;
  // Any plan: the variant with tiles, and the merge of split tiles (a plan
  // without split tiles gives it no work).
  const cudaError_t e = launch_attention(p, n_ctas, true, true, s);
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "paged_attention launch: %s", cudaGetErrorString(e));
  return check_launch("paged_attention_noalloc");
}

#ifdef TQ_ATTN_TRACE
// Tuning builds only (not part of the ABI): the latest CTA end (globaltimer
// ns) of any qkv_bias_kv_write launch so far.
TQ_API int tq_debug_qkv_times(unsigned long long* host, int32_t reset) {  // [64][3] + [64] attention entries
  cudaError_t e = cudaMemcpyFromSymbol(host, g_qkv_times, sizeof(g_qkv_times));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(host + 192, g_attn_entry, sizeof(g_attn_entry));
  if (e == cudaSuccess && reset) {
    static unsigned long long init[64][3];
    for (int l = 0; l < 64; ++l) init[l][0] = init[l][1] = ~0ull, init[l][2] = 0;
    e = cudaMemcpyToSymbol(g_qkv_times, init, sizeof(init));
    static unsigned long long first[64];
    for (int l = 0; l < 64; ++l) first[l] = ~0ull;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_attn_entry, first, sizeof(first));
  }
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(host + 192, g_attn_entry, sizeof(g_attn_entry));
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return TQ_OK;
}

TQ_API int tq_debug_qkv_write_end(unsigned long long* host) {
  const cudaError_t e = cudaMemcpyFromSymbol(host, g_qkv_write_end, sizeof(unsigned long long));
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return TQ_OK;
}

// Tuning builds only (not part of the ABI): copy the per-warp timeline of the
// last attention launch to `host` ([n_warps][16] uint64).
TQ_API int tq_debug_attention_trace(unsigned long long* host, int32_t n_warps) {
  const int n = std::min<int>(n_warps, kTraceWarps);
  const cudaError_t e =
      cudaMemcpyFromSymbol(host, g_attn_trace, (size_t)n * kTraceSlots * sizeof(unsigned long long));
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return TQ_OK;
}

// Per-chunk timeline of the last launch: [n_warps][32][3] uint64 =
// {issue ns, data-ready ns, bytes}.
TQ_API int tq_debug_attention_chunks(unsigned long long* host, int32_t n_warps) {
  const int n = std::min<int>(n_warps, kTraceWarps);
  const cudaError_t e =
      cudaMemcpyFromSymbol(host, g_attn_chunks, (size_t)n * kTraceChunks * 3 * sizeof(unsigned long long));
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return TQ_OK;
}
#endif

int tq_embed_layernorm(float* x, float* xa, const int32_t* ids, const int32_t* pos,
                       const float* wte, const float* wpe, int32_t vocab_size,
                       int32_t n_positions, const float* ln_w, const float* ln_b, float eps,
                       int32_t n_embd, const int32_t* d_num_rows, int32_t max_rows, void* stream) {
  int st = check_embd(n_embd);
  if (st) return st;
  if (max_rows < 0) return set_error(TQ_ERR_INVALID, "max_rows must be >= 0");
  if (max_rows == 0) return TQ_OK;
  if (!x || !xa || !ids || !pos || !wte || !wpe || !ln_w || !ln_b || !d_num_rows)
    return set_error(TQ_ERR_INVALID, "embed_layernorm: NULL argument");
  if (!aligned(x, 16) || !aligned(xa, 16) || !aligned(wte, 16) || !aligned(wpe, 16) ||
      !aligned(ln_w, 16) || !aligned(ln_b, 16))
    return set_error(TQ_ERR_INVALID, "embed_layernorm: float arrays must be 16-byte aligned");
  if (vocab_size < 1 || n_positions < 1) return set_error(TQ_ERR_INVALID, "bad vocab / positions");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  RowParams p{};
  p.x = x;
  p.xa = xa;
  p.ids = ids;
  p.pos = pos;
  p.wte = wte;
  p.wpe = wpe;
  p.ln_w = ln_w;
  p.ln_b = ln_b;
  p.n_rows = d_num_rows;
  p.C = n_embd;
  p.vocab = vocab_size;
  p.n_positions = n_positions;
  p.eps = eps;
  launch_dependent(embed_ln_kernel, row_grid(max_rows, sms), n_embd / 4, (cudaStream_t)stream, p);
  return check_launch("embed_layernorm");
}

int tq_bias_residual_layernorm(float* x, float* xa, const float* y, int32_t n_parts,
                               int64_t part_stride, const float* bias, const float* ln_w,
                               const float* ln_b, float eps, int32_t n_embd,
                               const int32_t* d_num_rows, int32_t max_rows, void* stream) {
  int st = check_embd(n_embd);
  if (st) return st;
  if (max_rows < 0) return set_error(TQ_ERR_INVALID, "max_rows must be >= 0");
  if (n_parts < 1 || (n_parts > 1 && (part_stride < (int64_t)max_rows * n_embd || part_stride % 4)))
    return set_error(TQ_ERR_INVALID, "bias_residual_layernorm: bad split-K parts");
  if (max_rows == 0) return TQ_OK;
  if (!x || !y || !bias || !d_num_rows || (ln_w && (!ln_b || !xa)))
    return set_error(TQ_ERR_INVALID, "bias_residual_layernorm: NULL argument");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(bias, 16) || (xa && !aligned(xa, 16)) ||
      (ln_w && (!aligned(ln_w, 16) || !aligned(ln_b, 16))))
    return set_error(TQ_ERR_INVALID, "bias_residual_layernorm: arrays must be 16-byte aligned");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  RowParams p{};
  p.x = x;
  p.xa = xa;
  p.y = y;
  p.n_parts = n_parts;
  p.part_stride = part_stride;
  p.bias = bias;
  p.ln_w = ln_w;
  p.ln_b = ln_b;
  p.n_rows = d_num_rows;
  p.C = n_embd;
  p.eps = eps;
  const cudaStream_t s = (cudaStream_t)stream;
  const int grid = row_grid(max_rows, sms), threads = n_embd / 4;
  switch (n_parts) {  // partial-sum loads unrolled for the split counts the model uses
    case 1: launch_dependent(bias_residual_ln_kernel<1>, grid, threads, s, p); break;
    case 2: launch_dependent(bias_residual_ln_kernel<2>, grid, threads, s, p); break;
    case 4: launch_dependent(bias_residual_ln_kernel<4>, grid, threads, s, p); break;
    case 8: launch_dependent(bias_residual_ln_kernel<8>, grid, threads, s, p); break;
    case 16: launch_dependent(bias_residual_ln_kernel<16>, grid, threads, s, p); break;
    case 32: launch_dependent(bias_residual_ln_kernel<32>, grid, threads, s, p); break;
    default: launch_dependent(bias_residual_ln_kernel<0>, grid, threads, s, p); break;
  }
  return check_launch("bias_residual_layernorm");
}

int tq_layernorm_rows(float* out, const float* x, const int32_t* rows, const float* ln_w,
                      const float* ln_b, float eps, int32_t n_embd, const int32_t* d_num_rows,
                      int32_t max_rows, void* stream) {
  int st = check_embd(n_embd);
  if (st) return st;
  if (max_rows < 0) return set_error(TQ_ERR_INVALID, "max_rows must be >= 0");
  if (max_rows == 0) return TQ_OK;
  if (!out || !x || !ln_w || !ln_b || !d_num_rows)
    return set_error(TQ_ERR_INVALID, "layernorm_rows: NULL argument");
  if (!aligned(out, 16) || !aligned(x, 16) || !aligned(ln_w, 16) || !aligned(ln_b, 16))
    return set_error(TQ_ERR_INVALID, "layernorm_rows: arrays must be 16-byte aligned");
  int sms = 0;
  if ((st = device_setup(&sms))) return st;
  RowParams p{};
  p.xa = out;
  p.x = const_cast<float*>(x);
  p.rows = rows;
  p.ln_w = ln_w;
  p.ln_b = ln_b;
  p.n_rows = d_num_rows;
  p.C = n_embd;
  p.eps = eps;
  launch_dependent(layernorm_rows_kernel, row_grid(max_rows, sms), n_embd / 4, (cudaStream_t)stream, p);
  return check_launch("layernorm_rows");
}

int tq_argmax_rows(const float* x, int64_t row_stride, int32_t n_cols, int64_t* out, const int32_t* d_num_rows,
                   int32_t max_rows, void* stream) {
  if (max_rows < 0 || n_cols < 1 || row_stride < n_cols)
    return set_error(TQ_ERR_INVALID, "argmax_rows: need n_cols >= 1, row_stride >= n_cols, max_rows >= 0");
  if (max_rows == 0) return TQ_OK;
  if (!x || !out || !d_num_rows) return set_error(TQ_ERR_INVALID, "argmax_rows: NULL argument");
  int sms = 0;
  const int st = device_setup(&sms);
  if (st) return st;
  if ((int64_t)max_rows * kArgmaxSlices > INT32_MAX)
    return set_error(TQ_ERR_UNSUPPORTED, "argmax_rows: too many rows");
  launch_dependent(argmax_rows_kernel, max_rows * kArgmaxSlices, kArgmaxThreads, (cudaStream_t)stream, 
      x, row_stride, n_cols, reinterpret_cast<long long*>(out), d_num_rows);
  return check_launch("argmax_rows");
}

static_assert(TQ_LM_HEAD_MAX_ROWS == tq::kLmMaxRows && TQ_LM_HEAD_SLICE == tq::kLmWidth &&
                  TQ_LM_HEAD_SCRATCH_BYTES >= tq::kLmMaxRows * 8 + 4,
              "tq_lm_head_argmax limits in the header match the kernel");

int tq_lm_head_argmax(int64_t* tokens, float* max_logit, const float* x, int64_t x_row_stride,
                      const int32_t* rows, const float* ln_w, const float* ln_b, float eps, int32_t n_embd,
                      const float* wte_t, int64_t vocab_stride, int32_t vocab_size, void* scratch,
                      const int32_t* d_num_rows, int32_t max_rows, void* stream) {
  if (max_rows < 0 || max_rows > kLmMaxRows)
    return set_error(TQ_ERR_UNSUPPORTED, "lm_head_argmax: max_rows must be in [0, %d]", kLmMaxRows);
  if (n_embd < 32 || n_embd > kLmMaxEmbd || n_embd % 32 || n_embd % kLmKTile)
    return set_error(TQ_ERR_UNSUPPORTED, "lm_head_argmax: n_embd must be a multiple of 32 in [32, %d]",
                     kLmMaxEmbd);
  if (vocab_size < 1) return set_error(TQ_ERR_INVALID, "lm_head_argmax: vocab_size must be >= 1");
  const int64_t slices = ((int64_t)vocab_size + kLmWidth - 1) / kLmWidth;
  if (vocab_stride < slices * kLmWidth || vocab_stride % 4)
    return set_error(TQ_ERR_INVALID,
                     "lm_head_argmax: vocab_stride must be a multiple of 4 and >= %lld (slices of %d columns)",
                     (long long)(slices * kLmWidth), kLmWidth);
  if (x_row_stride < n_embd) return set_error(TQ_ERR_INVALID, "lm_head_argmax: x_row_stride < n_embd");
  if (max_rows == 0) return TQ_OK;
  if (!tokens || !x || !ln_w || !ln_b || !wte_t || !scratch || !d_num_rows)
    return set_error(TQ_ERR_INVALID, "lm_head_argmax: NULL argument");
  if (!aligned(wte_t, 16) || !aligned(scratch, 8))
    return set_error(TQ_ERR_INVALID, "lm_head_argmax: wte_t must be 16-byte and scratch 8-byte aligned");
  int sms = 0;
  const int st = device_setup(&sms);
  if (st) return st;
  LmHeadParams p;
  p.x = x;
  p.x_stride = x_row_stride;
  p.sel = rows;
  p.ln_w = ln_w;
  p.ln_b = ln_b;
  p.eps = eps;
  p.C = n_embd;
  p.wt = wte_t;
  p.vstride = vocab_stride;
  p.V = vocab_size;
  p.tokens = reinterpret_cast<long long*>(tokens);
  p.max_logit = max_logit;
  p.best = reinterpret_cast<unsigned long long*>(scratch);
  p.done = reinterpret_cast<unsigned int*>(reinterpret_cast<char*>(scratch) + kLmMaxRows * 8);
  p.n_rows = d_num_rows;
  p.max_rows = max_rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)slices);
  cfg.blockDim = dim3(kLmThreads);
  cfg.dynamicSmemBytes = kLmSmemBytes;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, lm_head_argmax_kernel, p);
  if (e != cudaSuccess) return set_error(TQ_ERR_CUDA, "lm_head_argmax launch: %s", cudaGetErrorString(e));
  return check_launch("lm_head_argmax");
}

int tq_bias_gelu(float* out, const float* h, int32_t n_parts, int64_t part_stride, const float* bias,
                 int32_t n_cols, int32_t apply_gelu, const int32_t* d_num_rows, int32_t max_rows,
                 void* stream) {
  if (max_rows < 0 || n_cols < 4 || n_cols % 4)
    return set_error(TQ_ERR_INVALID, "bias_gelu: n_cols must be a positive multiple of 4");
  if (n_parts < 1 || (n_parts > 1 && (part_stride < (int64_t)max_rows * n_cols || part_stride % 4)))
    return set_error(TQ_ERR_INVALID, "bias_gelu: bad split-K parts");
  if (max_rows == 0) return TQ_OK;
  if (!out || !h || !bias || !d_num_rows) return set_error(TQ_ERR_INVALID, "bias_gelu: NULL argument");
  if (!aligned(out, 16) || !aligned(h, 16) || !aligned(bias, 16))
    return set_error(TQ_ERR_INVALID, "bias_gelu: arrays must be 16-byte aligned");
  if (n_parts > 1 && out != h &&
      reinterpret_cast<const char*>(out) < reinterpret_cast<const char*>(h + part_stride * n_parts) &&
      reinterpret_cast<const char*>(h) < reinterpret_cast<const char*>(out + (int64_t)max_rows * n_cols))
    return set_error(TQ_ERR_INVALID, "bias_gelu: out overlaps the partial sums");
  int sms = 0;
  int st = device_setup(&sms);
  if (st) return st;
  GeluParams p;
  p.out = out;
  p.h = h;
  p.n_parts = n_parts;
  p.part_stride = part_stride;
  p.bias = bias;
  p.n_rows = d_num_rows;
  p.F = n_cols;
  p.gelu = apply_gelu ? 1 : 0;
  const int64_t total4 = (int64_t)max_rows * (n_cols / 4);
  const int grid = (int)std::min<int64_t>(std::max<int64_t>((total4 + 255) / 256, 1), (int64_t)sms * 8);
  const cudaStream_t s = (cudaStream_t)stream;
  switch (n_parts) {  // partial-sum loads unrolled for the split counts the model uses
    case 1: launch_dependent(bias_gelu_kernel<1>, grid, 256, s, p); break;
    case 2: launch_dependent(bias_gelu_kernel<2>, grid, 256, s, p); break;
    case 4: launch_dependent(bias_gelu_kernel<4>, grid, 256, s, p); break;
    case 8: launch_dependent(bias_gelu_kernel<8>, grid, 256, s, p); break;
    case 16: launch_dependent(bias_gelu_kernel<16>, grid, 256, s, p); break;
    default: launch_dependent(bias_gelu_kernel<0>, grid, 256, s, p); break;
  }
  return check_launch("bias_gelu");
}

}  // extern "C"
