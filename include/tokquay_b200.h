/*
 * tokquay_b200.h -- C ABI of the B200 (sm_100a) paged-attention hot path for
 * Tokquay's paged forward.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream handle
 * (`void* stream`, a cudaStream_t; NULL = the legacy default stream), returns
 * TQ_OK (0) or a nonzero TQ_ERR_* status, and never throws.  After a nonzero
 * status tq_last_error() holds a message for the calling thread.
 *
 * Device pointers point to fp32 / int32 device memory; "host" marks host
 * memory.  Counts that kernels read on the device (d_num_*) let a launch be
 * captured once in a CUDA graph and replayed for steps of different sizes up
 * to the capacity (max_*) the launch was sized for.
 *
 * Reference interfaces replaced (paths inside the Tokquay project):
 *   tq_plan_step               PagedBatch.__init__           tokquay/kv_cache.py:174-226
 *   tq_kv_write                PagedBatch.write              tokquay/kv_cache.py:228-232
 *   tq_qkv_bias_kv_write       c_attn bias + PagedBatch.write
 *                                                            tokquay/model.py:69,
 *                                                            tokquay/kv_cache.py:228-232
 *   tq_paged_attention         PagedBatch.gather + scores/mask/softmax/@v
 *                                                            tokquay/kv_cache.py:234-242,
 *                                                            tokquay/model.py:94-96
 *   tq_embed_layernorm         wte(ids) + wpe(pos), then ln_1 of layer 0
 *                                                            tokquay/model.py:163,172,122
 *   tq_bias_residual_layernorm x + (y + b), then the next LayerNorm
 *                                                            tokquay/model.py:99,122-123
 *   tq_argmax_rows             logits.argmax(-1) of greedy sampling
 *                                                            tokquay/engine.py:189-194
 *   tq_layernorm_rows          x[arange(B), last_idx] then ln_f
 *                                                            tokquay/model.py:179-180
 *   tq_bias_gelu               F.gelu(c_fc(x), approximate="tanh"), and the
 *                              bias of c_attn            tokquay/model.py:110, :69
 *   tq_lm_head_argmax          last-row select, ln_f, the tied LM head and the
 *                              greedy argmax in one kernel (no logits tensor)
 *                                                            tokquay/model.py:179-181,
 *                                                            tokquay/engine.py:189-194
 *
 * Pool layout (the reference's, tokquay/kv_cache.py:1-14, :51-53):
 *   pool[num_blocks][n_layer][2 (K,V)][n_head][block_size][head_dim], fp32,
 *   16-byte aligned.  head_dim must be 64; block_size a power of two <= 256.
 */
#ifndef TOKQUAY_B200_H
#define TOKQUAY_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define TQ_API __attribute__((visibility("default")))
#else
#define TQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TQ_ABI_VERSION 8

enum tq_status {
  TQ_OK = 0,
  TQ_ERR_INVALID = 1,     /* bad argument or batch (the reference raises ValueError) */
  TQ_ERR_UNSUPPORTED = 2, /* shape this build does not handle (head_dim != 64, ...) */
  TQ_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  TQ_ERR_CAPACITY = 4,    /* output buffer too small; the needed size is reported */
  TQ_ERR_DEVICE = 5       /* a kernel flagged an error (see tq_device_status) */
};

/* Layout of a plan (tq_plan_step): layout[] indices. */
enum tq_plan_layout {
  TQ_PLAN_NUM_TOKENS = 0,    /* N = sum of q_len */
  TQ_PLAN_NUM_SEQS = 1,      /* B */
  TQ_PLAN_NUM_ITEMS = 2,     /* attention work items (one query-row group, one head, a chunk range) */
  TQ_PLAN_NUM_COMBINE = 3,   /* rows whose keys were split (combine entries) */
  TQ_PLAN_NUM_PARTIALS = 4,  /* split-K partial slots needed (x head_dim floats of scratch each) */
  TQ_PLAN_TABLE_STRIDE = 5,  /* int32 per row of the packed block tables */
  TQ_PLAN_MAX_CTX = 6,       /* longest sequence after this step */
  TQ_PLAN_SPLIT_CHUNKS = 7,  /* longest work item, in 32-key chunks */
  TQ_PLAN_TOTAL_INTS = 8,    /* int32 the plan occupies */
  TQ_PLAN_OFF_COUNTS = 9,    /* [4]: N, num_items, num_combine, B (the d_num_* pointers) */
  TQ_PLAN_OFF_SEQ_INFO = 10, /* [B][4]: first row, q_len, start, ctx */
  TQ_PLAN_OFF_TABLES = 11,   /* [B][table_stride] block ids */
  TQ_PLAN_OFF_SLOTS = 12,    /* [N] slot = block * block_size + offset */
  TQ_PLAN_OFF_POSITIONS = 13,/* [N] absolute positions */
  TQ_PLAN_OFF_TOKEN_IDS = 14,/* [N] token ids (copied from token_ids, or 0) */
  TQ_PLAN_OFF_LAST_ROWS = 15,/* [B] row of each sequence's last new token */
  TQ_PLAN_OFF_ITEMS = 16,    /* the attention plan (tq_paged_attention's attn_plan), last region:
                                [W][16] each warp's first work item and the block ids of its first
                                chunk (-1 past them), [W+1] (padded to 8) offsets of the other
                                items, then those items [..][8], W = num_ctas * warps, then
                                the tile-merge trailer: [8] (word 0: TQ_PLAN_NUM_TILE_MERGES),
                                [num_tile_merges][4] {row, partial of head 0, pieces, partials
                                between heads} */
  TQ_PLAN_OFF_COMBINE = 17,  /* [num_combine][4] rows whose keys are split across CTAs */
  TQ_PLAN_NUM_CTAS = 18,     /* CTAs the attention plan is cut for (its launch grid) */
  TQ_PLAN_USED_INTS = 19,    /* leading int32 of the plan this step uses (what must be copied) */
  TQ_PLAN_NUM_TILE_CTAS = 20,/* CTAs of the grid that run prompt tiles (tq_plan_prompt_tiles) */
  TQ_PLAN_NUM_TILE_MERGES = 21,/* rows of prompt tiles cut over their keys: merged after the
                                attention grid (tq_paged_attention with TQ_ATTN_TILE_MERGE) */
  TQ_PLAN_LAYOUT_LEN = 22
};

TQ_API int tq_abi_version(void);

/* Keys per attention chunk of this build (the granularity of tq_plan_step
 * work items: TQ_PLAN_SPLIT_CHUNKS counts these). */
TQ_API int tq_attention_chunk_keys(void);

/* Computing warps per attention CTA of this build (a plan for n_ctas CTAs
 * holds n_ctas * this many per-warp work lists). */
TQ_API int tq_attention_warps(void);

/* Message for the last nonzero status returned on this thread. */
TQ_API const char* tq_last_error(void);

/* Reads (and with clear != 0 resets) the device error word of the current
 * device: bit 1 = a bounded wait timed out, 2 = a block id outside the pool,
 * 4 = a slot outside the pool, 8 = a token id outside the vocabulary,
 * 16 = an attention work item whose merge target lies outside its buffer.
 * Synchronises the device.  *bits receives the word. */
TQ_API int tq_device_status(int clear, int32_t* bits);

/* Host-side step planner (replaces PagedBatch.__init__, tokquay/kv_cache.py:174-226).
 * Validates the batch as the reference does (same conditions: non-empty,
 * every q_len >= 1, each block table long enough for start+q_len tokens) plus
 * block ids inside the pool and token ids inside the vocabulary, then writes
 * into the host buffer `out` every index array one step needs (see
 * tq_plan_layout), ready for a single host-to-device copy.  Sequence b feeds
 * q_len[b] tokens at positions start[b] .. start[b]+q_len[b]-1; its block
 * table is table_data[table_offsets[b] .. table_offsets[b+1]).
 * token_ids (host, [N], may be NULL) are copied into the plan.
 *
 * Attention work is cut for a grid of n_ctas CTAs (normally the SM count;
 * the attention launch must use the same grid): every (query-row group, head)
 * pair's keys are a run of 32-key chunks; pairs go to CTAs longest first, each
 * to the least loaded CTA, and each CTA's chunks are cut evenly over its warps.
 * A pair cut between warps of one CTA is merged through shared memory; a pair
 * longer than a CTA's share (and longer than 2 * min_split_chunks) is first
 * split across CTAs into pieces of at least min_split_chunks chunks, merged
 * through the split-K scratch.  Contexts up to 65535 chunks.
 * caps (host, may be NULL): fixed capacities {max_seqs, max_tokens,
 * table_stride, max_items, max_combine, max_partials}.  With caps every region
 * has its capacity's size, so the layout (and the table stride) is the same
 * for every step that fits -- the form a captured CUDA graph needs -- and the
 * cross-CTA split is coarsened until items and partials fit; a step that
 * still does not fit returns TQ_ERR_CAPACITY.  Without caps the plan is packed
 * to this step.  Returns TQ_ERR_CAPACITY (layout[TQ_PLAN_TOTAL_INTS] = ints
 * needed) if out_capacity is too small. */
/* Prompt tiles (no reference counterpart: a planning knob of this path).
 * tq_plan_step sends every sequence that feeds at least min_rows tokens this
 * step to tensor-core tiles: its rows are cut evenly into tiles of at most 128
 * rows, and each (tile, head) is one work item run by a whole CTA (QK^T and PV
 * as tcgen05 MMAs, fp32-accurate by splitting every operand into two TF32
 * halves).  Tile items run on the last CTAs of the grid; how many is set by
 * the estimated loads: a tile item costs chunk_cost_pct percent of a warp-path
 * 32-key chunk per chunk, plus item_cost_pct.  min_rows 0 turns tiles off.
 * max_pieces > 1 lets a plan without fixed capacities cut a tile whose item
 * would cost more than a CTA's balanced load over its keys, into up to that
 * many pieces of at least two chunks on different CTAs; each piece leaves its
 * partials in the split-K scratch and a merge kernel after the attention grid
 * combines them (TQ_PLAN_NUM_TILE_MERGES rows).  Arguments below 0
 * (chunk_cost_pct, max_pieces: <= 0) keep the current value.  The setting is
 * process-wide and read by each tq_plan_step call; defaults 16, 1500, 200, 1.
 * Returns the previous min_rows. */
TQ_API int tq_plan_prompt_tiles(int32_t min_rows, int32_t chunk_cost_pct, int32_t item_cost_pct,
                                int32_t max_pieces);

TQ_API int tq_plan_step(int32_t num_seqs, const int32_t* start, const int32_t* q_len,
                 const int32_t* table_offsets, const int32_t* table_data,
                 const int32_t* token_ids, int32_t block_size, int64_t num_blocks,
                 int32_t n_head, int32_t vocab_size, int32_t n_ctas,
                 int32_t min_split_chunks, const int32_t* caps, int32_t* out,
                 int64_t out_capacity, int32_t* layout);

/* KV write (replaces PagedBatch.write, tokquay/kv_cache.py:228-232).
 * For each of the *d_num_tokens new tokens n: pool[slot/bs][layer][0][h][slot%bs][:]
 * = qkv[n*qkv_row_stride + k_col + h*head_dim ...] and likewise V from v_col.
 * max_tokens sizes the grid (>= *d_num_tokens). */
TQ_API int tq_kv_write(float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
                int32_t block_size, int32_t head_dim, int32_t layer, const float* qkv,
                int64_t qkv_row_stride, int64_t k_col, int64_t v_col,
                const int32_t* slot_mapping, const int32_t* d_num_tokens, int32_t max_tokens,
                void* stream);

/* The c_attn epilogue fused with the KV write (replaces the c_attn bias,
 * tokquay/model.py:69, and PagedBatch.write, tokquay/kv_cache.py:228-232).
 * For each of the *d_num_rows new tokens r, with
 *   row = parts_0[r] + ... + parts_{n_parts-1}[r] + bias   (3 * n_head * head_dim floats,
 *   parts_s = parts + s * part_stride, rows of 3C floats: the split-K partial sums of c_attn):
 * q_out[r * q_row_stride + i] = row[i] for i < C; the K and V parts of row go
 * straight to pool[slot/bs][layer][0 / 1][h][slot%bs][:] (slot = slot_mapping[r]).
 * n_head <= 21 (one thread per 4 columns).  max_rows sizes the grid. */
TQ_API int tq_qkv_bias_kv_write(float* q_out, int64_t q_row_stride, const float* parts, int32_t n_parts,
                                int64_t part_stride, const float* bias, float* pool, int64_t num_blocks,
                                int32_t n_layer, int32_t n_head, int32_t block_size, int32_t head_dim,
                                int32_t layer, const int32_t* slot_mapping, const int32_t* d_num_rows,
                                int32_t max_rows, void* stream);

/* Paged attention, decode and causal prefill rows mixed in one launch
 * (replaces PagedBatch.gather + the masked softmax attention,
 * tokquay/kv_cache.py:234-242, tokquay/model.py:94-96).
 * Row r of the plan (a new token at position p of sequence b) attends to the
 * keys at positions 0..p of sequence b:
 *   out[r*out_row_stride + h*64 + i] = softmax_j(q_r.k_j * scale) v_j[i].
 * q rows: q[r*q_row_stride + h*64 ...]; q, out 16-byte aligned rows.
 * attn_plan / block_tables come from tq_plan_step.  Split-K scratch is the
 * caller's: partial_ml ([P][2] floats), partial_acc ([P][64] floats) and
 * partial_counters ([P] int32, all zero before the first launch; every launch
 * that completes leaves them zero again), P >= TQ_PLAN_NUM_PARTIALS of every
 * plan launched with it (max_partials; NULL scratch is fine when it is 0).
 * Launches that share scratch must not overlap on the GPU.  attn_plan is the
 * plan's attention region (TQ_PLAN_OFF_ITEMS) and n_ctas its TQ_PLAN_NUM_CTAS,
 * the launch grid.  with_tiles must hold TQ_ATTN_TILES when the plan may hold
 * prompt tiles (TQ_PLAN_NUM_TILE_CTAS > 0; for a launch captured once and
 * replayed over plans of fixed capacities: when any of them may) -- it selects
 * the kernel that carries the tile role; 0 selects the leaner one, which flags
 * (device error 16) and skips any tile item it is given.  TQ_ATTN_TILES |
 * TQ_ATTN_TILE_MERGE when the plan also cuts tiles over their keys
 * (TQ_PLAN_NUM_TILE_MERGES > 0): a second kernel then merges their pieces,
 * as a programmatic dependent of the first.  Otherwise one kernel launch on
 * `stream`, and every merge of split keys happens inside it.  The launch is a programmatic dependent of the kernel
 * before it on `stream`: for a sequence that feeds one token this step, the
 * pool rows of its earlier positions (0 .. position-1) may be read before
 * that kernel has finished, so that kernel may write this step's new K/V
 * rows (tq_kv_write, tq_qkv_bias_kv_write) and q, but no other pool row;
 * everything else is read, and every output written, after it completes. */
enum tq_attn_tiles { TQ_ATTN_TILES = 1, TQ_ATTN_TILE_MERGE = 2 };
TQ_API int tq_paged_attention(float* out, int64_t out_row_stride, const float* q, int64_t q_row_stride,
                       const float* pool, int64_t num_blocks, int32_t n_layer, int32_t n_head,
                       int32_t block_size, int32_t head_dim, int32_t layer,
                       const int32_t* block_tables, int32_t table_stride,
                       const int32_t* attn_plan, int32_t n_ctas, int32_t with_tiles,
                       float* partial_ml, float* partial_acc, int32_t* partial_counters,
                       int32_t max_partials, float scale, void* stream);

/* Split-K partials tq_paged_attention_noalloc can hold.  Its scratch,
 * TQ_NOALLOC_MAX_PARTIALS * (1 + 2 + 64) * 4 bytes (8,781,824 bytes: 8.78 MB,
 * 8.4 MiB), is a fixed
 * array inside the library on every GPU that loads it, kept until exit. */
#define TQ_NOALLOC_MAX_PARTIALS 32768

/* No counterpart in the reference (Tokquay allocates freely through torch).
 * tq_paged_attention for callers that cannot allocate device memory or hand
 * over scratch: a host runtime that passes this library only the tensors it
 * already owns (a serving process held to a fixed memory budget, an embedding
 * without its own device allocator).  Same arguments and result as
 * tq_paged_attention, minus the scratch pointers and with_tiles (it launches
 * the tile-capable kernel and the tile merge for any plan); num_partials is
 * the plan's TQ_PLAN_NUM_PARTIALS.  The split-K scratch is a library-owned array, so the
 * call allocates nothing; a plan needing more than TQ_NOALLOC_MAX_PARTIALS
 * partials is rejected with TQ_ERR_CAPACITY before anything is launched.
 * The first call on a device looks the array's address up
 * (cudaGetSymbolAddress) and keeps it for the life of the process: make that
 * first call before any stream capture, and do not use this entry point on a
 * device after cudaDeviceReset (the kept address belongs to the context the
 * reset destroyed).
 * Every call on a device shares the one array and clears the split counters
 * it uses before its kernel runs, so calls that overlap on the GPU (other
 * streams, other threads) race: issue them one after another. */
TQ_API int tq_paged_attention_noalloc(float* out, int64_t out_row_stride, const float* q,
                                      int64_t q_row_stride, const float* pool, int64_t num_blocks,
                                      int32_t n_layer, int32_t n_head, int32_t block_size,
                                      int32_t head_dim, int32_t layer, const int32_t* block_tables,
                                      int32_t table_stride, const int32_t* attn_plan,
                                      int32_t n_ctas, int32_t num_partials, float scale,
                                      void* stream);

/* x[r] = wte[ids[r]] + wpe[pos[r]];  xa[r] = LayerNorm(x[r]; ln_w, ln_b, eps).
 * n_embd must be a multiple of 128 and at most 1024. */
TQ_API int tq_embed_layernorm(float* x, float* xa, const int32_t* ids, const int32_t* pos,
                       const float* wte, const float* wpe, int32_t vocab_size,
                       int32_t n_positions, const float* ln_w, const float* ln_b, float eps,
                       int32_t n_embd, const int32_t* d_num_rows, int32_t max_rows, void* stream);

/* x[r] += (y_0[r] + ... + y_{n_parts-1}[r]) + bias;  then, if ln_w != NULL,
 * xa[r] = LayerNorm(x[r]).  y_s = y + s*part_stride: the split-K partial sums
 * of the linear (n_parts = 1: y is the whole output). */
TQ_API int tq_bias_residual_layernorm(float* x, float* xa, const float* y, int32_t n_parts,
                               int64_t part_stride, const float* bias, const float* ln_w,
                               const float* ln_b, float eps, int32_t n_embd,
                               const int32_t* d_num_rows, int32_t max_rows, void* stream);

/* Greedy sampling (the greedy rows of Engine._sample, tokquay/engine.py:189-194):
 * out[r] = argmax over c < n_cols of x[r * row_stride + c] for each of the
 * *d_num_rows rows, as torch.argmax(-1) picks it: NaN counts as the largest
 * value, the first of equal values wins.  max_rows sizes the grid. */
TQ_API int tq_argmax_rows(const float* x, int64_t row_stride, int32_t n_cols, int64_t* out,
                          const int32_t* d_num_rows, int32_t max_rows, void* stream);

/* out[i] = LayerNorm(x[rows[i]]) (rows == NULL: x[i]). */
TQ_API int tq_layernorm_rows(float* out, const float* x, const int32_t* rows, const float* ln_w,
                      const float* ln_b, float eps, int32_t n_embd, const int32_t* d_num_rows,
                      int32_t max_rows, void* stream);

/* out[r][c] = gelu_tanh(sum_s h_s[r][c] + bias[c]) (apply_gelu != 0) or the
 * biased sum alone; h_s = h + s*part_stride are split-K partial sums
 * (n_parts = 1, out == h: in place).  n_cols a multiple of 4. */
TQ_API int tq_bias_gelu(float* out, const float* h, int32_t n_parts, int64_t part_stride,
                 const float* bias, int32_t n_cols, int32_t apply_gelu,
                 const int32_t* d_num_rows, int32_t max_rows, void* stream);

/* tq_lm_head_argmax: rows per launch, vocabulary columns per CTA slice, and the
 * bytes of its scratch (per-row maxima and a counter).  Zero the scratch once;
 * every launch that completes leaves it zero again. */
#define TQ_LM_HEAD_MAX_ROWS 64
#define TQ_LM_HEAD_SLICE 352
#define TQ_LM_HEAD_SCRATCH_BYTES 520

/* Greedy tokens of a step's last rows in one kernel, without a logits tensor:
 *   h[r]      = LayerNorm(x[rows[r]]; ln_w, ln_b, eps)      (rows == NULL: x[r])
 *   tokens[r] = argmax_v sum_c h[r][c] * wte_t[c][v]       (the tied LM head)
 * with torch.argmax's rules (NaN counts as the largest value, the first index
 * among equals); max_logit[r] (may be NULL) gets that logit.  fp32 on the CUDA
 * cores.  wte_t is the embedding matrix transposed, [n_embd][vocab_stride],
 * 16-byte aligned, with vocab_stride a multiple of 4 and at least
 * ceil(vocab_size / TQ_LM_HEAD_SLICE) * TQ_LM_HEAD_SLICE, columns past
 * vocab_size zero.  n_embd a multiple of 32 and at most 768; max_rows at most
 * TQ_LM_HEAD_MAX_ROWS.  Calls that share `scratch` must not overlap on the GPU. */
TQ_API int tq_lm_head_argmax(int64_t* tokens, float* max_logit, const float* x, int64_t x_row_stride,
                             const int32_t* rows, const float* ln_w, const float* ln_b, float eps,
                             int32_t n_embd, const float* wte_t, int64_t vocab_stride,
                             int32_t vocab_size, void* scratch, const int32_t* d_num_rows,
                             int32_t max_rows, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TOKQUAY_B200_H */
