/*
 * flour_attn.h — C ABI of the B200 (sm_100a) paged KV pool + paged attention backend for flour.
 *
 * The reference (lltsdyp/flour, Rust, CPU-only) has no FFI for this path; its boundary is the
 * trio called from src/models/common/attention.rs:104-109:
 *
 *     Cache::write_kv(layer, k (1,Hkv,n,d), v)                 src/models/common/cache.rs:451
 *     Cache::kv_blocks(layer) -> Vec<(K,V) block views>          src/models/common/cache.rs:456
 *     backend::cpu::paged_attention(q, blocks, n_rep, scale)     src/backend/cpu.rs:57
 *
 * Each entry point below names the reference function it replaces. Everything here uses plain
 * pointers, sizes and a CUDA stream handle: no Rust, torch or candle types cross the boundary.
 *
 * Conventions
 *   - Device memory (pools, queries, outputs, tables, workspace) is owned by the caller. No
 *     entry point allocates device memory except fa_ipc_alloc (head-sharded group buffers).
 *   - Every call is ordered on `stream` and returns before the GPU work finishes.
 *   - Host-side argument checks return FA_EINVAL / FA_ERANGE / FA_EUNSUPPORTED without
 *     launching anything; fa_last_error_message() then describes the rejection (thread-local).
 *   - Values that live in device memory (block ids, slots, context lengths) are bounds-checked
 *     inside the kernels. A bad value is never dereferenced: the kernel skips the access and
 *     sets a bit in a per-device status word that fa_device_status() reads back.
 *   - KV layout per layer (north star): K and V slabs of shape
 *         [num_blocks, num_kv_heads, block_size, head_dim]
 *     so one (block, kv_head) page is one contiguous run of block_size*head_dim elements.
 *     The reference slab is (kv_heads, num_slots, head_dim) with slot = block*bs + offset
 *     (src/models/common/paged.rs:124-160); element (blk,h,t,:) here is element
 *     (h, blk*bs+t, :) there.
 *   - Queries and outputs are packed token-major: [total_tokens, num_heads, head_dim].
 *   - Query head h reads KV head h / n_rep (src/backend/cpu.rs:5-13).
 *   - Causal rule (src/backend/cpu.rs:66-68,87-94): a sequence with context length L (all KV
 *     tokens, cached prefix included) and q_len new query tokens lets query i see KV position j
 *     iff j <= L - q_len + i.
 *   - The output dtype equals the query dtype, which must equal the pool dtype
 *     (src/backend/cpu.rs:109-111).
 */
#ifndef FLOUR_ATTN_H
#define FLOUR_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st *fa_stream_t;

typedef enum fa_status {
  FA_OK = 0,
  FA_EINVAL = -1,        /* bad argument (null pointer, shape mismatch, n_rep mismatch ...) */
  FA_ERANGE = -2,        /* a size or index is out of range (block id, workspace too small) */
  FA_ECUDA = -3,         /* a CUDA runtime call or kernel launch failed */
  FA_ETIMEOUT = -4,      /* a bounded device-side wait gave up (see FA_DEVERR_TIMEOUT) */
  FA_EUNSUPPORTED = -5,  /* valid request this build has no kernel for */
  FA_EDEVICE = -6        /* a kernel reported bad device-resident data (see FA_DEVERR_*) */
} fa_status;

typedef enum fa_dtype { FA_F32 = 0, FA_BF16 = 1, FA_F16 = 2 } fa_dtype;

/* Bits of the per-device status word written by the kernels. */
#define FA_DEVERR_BLOCK_ID 0x1   /* block table entry outside [0, num_blocks) */
#define FA_DEVERR_CONTEXT 0x2    /* context_len < q_len, or > max_blocks_per_seq*block_size */
#define FA_DEVERR_SLOT 0x4       /* slot_mapping entry outside [-1, num_blocks*block_size) */
#define FA_DEVERR_TIMEOUT 0x8    /* a bounded wait (mbarrier, head-sharded flags) gave up */
#define FA_DEVERR_SEQLEN 0x10    /* cu_seqlens_q not non-decreasing or past total_q */
#define FA_DEVERR_PAIR 0x20      /* copy_blocks pair entry outside [0, num_blocks) */
#define FA_DEVERR_POSITION 0x40  /* RoPE position outside [0, max_position) */
#define FA_DEVERR_LAUNCH 0x80    /* a kernel refused a launch shape it does not support */

/* How attention scores are formed before the softmax (the `score_flow` argument).
 *   FA_SCORES_F32        q.k accumulated in f32 and multiplied by scale in f32 (the default:
 *                        the most accurate, and the fastest prefill).
 *   FA_SCORES_REFERENCE  the reference's dtype flow for bf16/f16 pools, src/backend/cpu.rs:84-85
 *                        `(q.matmul(k^T) * scale).to_dtype(F32)`: q.k (f32 accumulation) rounded
 *                        to the pool dtype, multiplied by scale rounded to the pool dtype, the
 *                        product rounded again, then used in f32. Outputs then track the
 *                        reference CPU backend's own rounding; for f32 pools both flows are
 *                        identical. The softmax, the f32 accumulation of P.V and the output
 *                        rounding are the same in both flows. */
typedef enum fa_score_flow { FA_SCORES_F32 = 0, FA_SCORES_REFERENCE = 1 } fa_score_flow;

/* One layer of the paged KV pool. */
typedef struct fa_kv_layer {
  void *k_cache;          /* device, [num_blocks, num_kv_heads, block_size, head_dim] */
  void *v_cache;          /* device, same shape as k_cache */
  int32_t num_blocks;
  int32_t num_kv_heads;
  int32_t block_size;     /* the reference uses 16 (src/models/common/cache.rs:10) */
  int32_t head_dim;
  int32_t dtype;          /* fa_dtype */
} fa_kv_layer;

/* ---- version / errors ---------------------------------------------------------------- */

FA_API int32_t fa_abi_version(void);
FA_API const char *fa_status_string(int32_t status);
/* Text of the last host-side rejection on the calling thread ("" if none). */
FA_API const char *fa_last_error_message(void);

/* Wait for `stream`, then copy the current device's status word (FA_DEVERR_* bits) into
 * *status_out; clear it when `clear` is non-zero. Returns FA_EDEVICE when any bit is set. */
FA_API fa_status fa_device_status(int32_t *status_out, int32_t clear, fa_stream_t stream);

/* ---- block writes: PagedKvPool::write (src/models/common/paged.rs:186-204) ------------ */

/* reshape_and_cache: scatter num_tokens new K/V rows into their pool slots.
 *   key[t*key_stride_token + h*key_stride_head + x]   (same for value; strides in elements)
 *   slot_mapping[t] (device int32): slot = block*block_size + offset, or -1 to skip the token.
 * Replaces PagedKvPool::write + KvCache::write_current (src/models/common/cache.rs:71-77) and
 * BlockTable::slots (src/models/common/paged.rs:114-121): slot ids are the reference's.
 * The reference's (1,Hkv,n,d) tensor is key_stride_token=d, key_stride_head=n*d.
 * Tokens that map to the same slot: the last one in token order is not guaranteed to win;
 * callers (like the reference) never map two live tokens to one slot. */
FA_API fa_status fa_reshape_and_cache(const fa_kv_layer *layer, const void *key, const void *value,
                               int64_t key_stride_token, int64_t key_stride_head,
                               int64_t value_stride_token, int64_t value_stride_head,
                               const int32_t *slot_mapping, int32_t num_tokens,
                               fa_stream_t stream);

/* ---- block copies: write_block / block_view (src/models/common/paged.rs:211-240,266-279) */

/* Copy whole blocks src -> dst in every layer, K and V (prefix-cache copy-on-write).
 *   block_mapping: device int32 [num_pairs][2] = (src, dst).
 * Pairs run concurrently: a dst must not appear twice nor be the src of another pair.
 * At most FA_MAX_COPY_LAYERS layers per call; all layers must share one shape and dtype. */
#define FA_MAX_COPY_LAYERS 128
FA_API fa_status fa_copy_blocks(const fa_kv_layer *layers, int32_t num_layers,
                         const int32_t *block_mapping, int32_t num_pairs, fa_stream_t stream);

/* PagedKvPool::write_block (paged.rs:211-240): overwrite physical block `block_id` of one layer
 * with key/value of shape (num_kv_heads, block_size, head_dim) — host or device memory.
 * Rejects block_id outside [0, num_blocks) with FA_ERANGE. */
FA_API fa_status fa_write_block(const fa_kv_layer *layer, int32_t block_id, const void *key,
                         const void *value, fa_stream_t stream);

/* PagedKvPool::block_view (paged.rs:266-279) materialised: copy physical block `block_id` of one
 * layer into key/value (host or device), shape (num_kv_heads, block_size, head_dim). This is the
 * per-layer piece of KvCache::export_prefix_bundle (src/models/common/cache.rs:196-213). */
FA_API fa_status fa_read_block(const fa_kv_layer *layer, int32_t block_id, void *key, void *value,
                        fa_stream_t stream);

/* ---- FLKV bundle payload: KvCache::export/import_prefix_bundle (src/models/common/cache.rs:
 * 166-349), payload order of src/kv_cache/bundle.rs:15-22 ---------------------------------- */

/* Bytes of the payload of `num_blocks` logical blocks over `num_layers` layers shaped like
 * `layer`: num_blocks * num_layers * 2 * (num_kv_heads * block_size * head_dim * dtype size). */
FA_API size_t fa_bundle_payload_bytes(const fa_kv_layer *layer, int32_t num_layers,
                                      int32_t num_blocks);

/* Export: gather, in one launch, the K and V of every layer of the physical blocks
 * block_ids[0..num_blocks) (device int32, the sequence's logical order) into `payload` (device,
 * fa_bundle_payload_bytes bytes) in the FLKV payload order:
 *     for block in 0..num_blocks: for layer in 0..num_layers: K then V, (kv_heads, bs, head_dim)
 * The caller then moves the payload to the host with one copy (the reference's export writes the
 * same bytes, block by block, from its CPU pool). All layers must share one shape and dtype; at
 * most FA_MAX_COPY_LAYERS layers. A block id outside [0, num_blocks of the pool) zero-fills its
 * pieces and sets FA_DEVERR_BLOCK_ID. Payload and pools must not overlap. */
FA_API fa_status fa_export_bundle_payload(const fa_kv_layer *layers, int32_t num_layers,
                                          const int32_t *block_ids, int32_t num_blocks,
                                          void *payload, fa_stream_t stream);

/* Import: the mirror scatter, payload (device, same order) -> physical blocks block_ids[b] of
 * every layer, as KvCache::import_prefix_bundle's write_block loop does (cache.rs:304-321). Ids
 * must be distinct; a bad id is skipped and sets FA_DEVERR_BLOCK_ID. */
FA_API fa_status fa_import_bundle_payload(const fa_kv_layer *layers, int32_t num_layers,
                                          const int32_t *block_ids, int32_t num_blocks,
                                          const void *payload, fa_stream_t stream);

/* ---- paged attention: backend::cpu::paged_attention (src/backend/cpu.rs:57-112) ------- */

/* Bytes of workspace the attention entry points need for these sizes (split-K partials and
 * merge counters). 0 means no workspace is needed. The workspace must be zero-filled once
 * before its first use; the kernels leave the counters at zero when they finish. One workspace
 * may serve calls of different sizes (the library zeroes counters that land on an earlier
 * call's partials) when it is always passed by the same base pointer. Calls that run
 * concurrently on different streams need separate workspaces. */
FA_API size_t fa_paged_attention_workspace_size(int32_t num_seqs, int32_t num_heads,
                                         int32_t num_kv_heads, int32_t head_dim,
                                         int32_t max_context_len, int32_t max_seqlen_q);

/* The library remembers, per workspace base pointer, which merge tickets are known to be zero
 * (and which smaller calls were recorded into CUDA graphs, whose replays leave partials behind),
 * so that a workspace reused across shapes is zeroed only where needed. Call this when a
 * workspace at `workspace` is freshly zero-filled, for example a new allocation that may reuse
 * the address of an earlier workspace, once no CUDA graph that recorded calls with the earlier
 * buffer will be replayed: the earlier buffer's bookkeeping no longer applies. No counterpart in
 * the reference. */
FA_API fa_status fa_workspace_reset(const void *workspace);

/* General entry, same contract as paged_attention(q, blocks, n_rep, scale) for a batch of
 * sequences with varying query counts (decode when every sequence has one query token).
 *   query/out       device [total_q, num_heads, head_dim], pool dtype
 *   cu_seqlens_q    device int32 [num_seqs+1], cu_seqlens_q[0]=0, cu_seqlens_q[S]=total_q
 *   context_lens    device int32 [num_seqs]: KV length L including the new tokens
 *   block_tables    device int32 [num_seqs, max_blocks_per_seq]: logical -> physical block
 *                   (the reference's KvCache::gather_blocks, cache.rs:83-96, one table per seq)
 *   num_heads == n_rep * layer->num_kv_heads, else FA_EINVAL (cpu.rs:78-79 repeat_kv)
 *   max_seqlen_q / max_context_len: host-side upper bounds used for launch sizing. */
FA_API fa_status fa_paged_attention(const fa_kv_layer *layer, const void *query, void *out,
                             const int32_t *cu_seqlens_q, const int32_t *context_lens,
                             const int32_t *block_tables, int32_t max_blocks_per_seq,
                             int32_t num_seqs, int32_t num_heads, int32_t n_rep,
                             int32_t total_q, int32_t max_seqlen_q, int32_t max_context_len,
                             float scale, int32_t score_flow, void *workspace, size_t workspace_bytes,
                             fa_stream_t stream);

/* Decode specialisation (one query token per sequence): query/out [num_seqs, num_heads, d].
 * Split-K over the context with a log-sum-exp merge of the partial results. */
FA_API fa_status fa_paged_decode(const fa_kv_layer *layer, const void *query, void *out,
                          const int32_t *context_lens, const int32_t *block_tables,
                          int32_t max_blocks_per_seq, int32_t num_seqs, int32_t num_heads,
                          int32_t n_rep, int32_t max_context_len, float scale, int32_t score_flow, void *workspace,
                          size_t workspace_bytes, fa_stream_t stream);

/* One decode step of the reference's attention in one launch: Cache::write_kv of the new token
 * (src/models/common/cache.rs:451 -> PagedKvPool::write, paged.rs:186-204) followed by
 * paged_attention over the whole context (cpu.rs:57-112), the order of attention.rs:104-109.
 * For each sequence b the new token is position L-1 of its context (L = context_lens[b] >= 1);
 * key[b*key_stride_token + h*key_stride_head + x] (and value alike, strides in elements) is
 * written to that position's slot, block_tables[b][(L-1)/16]*16 + (L-1)%16, for every KV head h,
 * and query[b] then attends to positions 0..L-1, the new one included. Same result, bit for
 * bit, as fa_reshape_and_cache with those slots followed by fa_paged_decode (same kernel, same
 * split plan), minus one launch. The new token's slot must not lie inside another sequence's
 * context in the same call (a shared prefix block is copied before it is written, as the
 * reference's copy-on-write does). Sequences with an invalid length are not written (zero
 * output, FA_DEVERR_CONTEXT). Requires the fast decode path (16-bit pool, block_size 16,
 * head_dim 64/128, n_rep <= 8, 16-byte aligned query/out); other shapes: FA_EUNSUPPORTED. */
FA_API fa_status fa_paged_decode_append(const fa_kv_layer *layer, const void *query,
                                        const void *key, const void *value,
                                        int64_t key_stride_token, int64_t key_stride_head,
                                        int64_t value_stride_token, int64_t value_stride_head,
                                        void *out, const int32_t *context_lens,
                                        const int32_t *block_tables, int32_t max_blocks_per_seq,
                                        int32_t num_seqs, int32_t num_heads, int32_t n_rep,
                                        int32_t max_context_len, float scale, int32_t score_flow, void *workspace,
                                        size_t workspace_bytes, fa_stream_t stream);

/* Decode without a caller-provided workspace. No counterpart in the reference: the reference's
 * CPU path never needs scratch memory. Some callers of this library cannot allocate device
 * memory at the point where they run attention — for example an engine whose KV pool was sized
 * to fill the GPU's memory and that forbids allocations while serving, or a host runtime that
 * reaches the GPU only through these raw-pointer entry points and has no device allocator of
 * its own. For them this variant takes its split-K scratch from a fixed buffer inside the
 * library (FA_NOALLOC_DECODE_SCRATCH_BYTES; every GPU that loads the library holds it until the
 * process exits) and calls no allocating routine. Same arguments and results as
 * fa_paged_decode with score_flow FA_SCORES_F32, minus the workspace.
 *   - Requests whose split-K scratch would exceed FA_NOALLOC_DECODE_SCRATCH_BYTES are rejected
 *     with FA_ERANGE (use fa_paged_decode with a workspace for those). The test is exact: a call
 *     is accepted when fa_paged_attention_workspace_size(num_seqs, num_heads, num_kv_heads,
 *     head_dim, max_context_len, 1) <= FA_NOALLOC_DECODE_SCRATCH_BYTES, so a caller can ask in
 *     advance. Shapes outside the fast decode path run the generic kernel, which needs no
 *     scratch, and are never rejected for size.
 *   - The first call on each device looks up the buffer's device address (with that device
 *     current); make that first call before any stream capture. The address is kept for the
 *     life of the process: a device reset (cudaDeviceReset, or a primary-context reset) after
 *     that first call is not supported by this entry point.
 *   - All calls share the one buffer per device, so calls whose GPU work overlaps (different
 *     streams, or threads without ordering) race; order them on one stream. */
#define FA_NOALLOC_DECODE_SCRATCH_BYTES (8u * 1024u * 1024u)
FA_API fa_status fa_paged_decode_noalloc(const fa_kv_layer *layer, const void *query, void *out,
                                         const int32_t *context_lens, const int32_t *block_tables,
                                         int32_t max_blocks_per_seq, int32_t num_seqs,
                                         int32_t num_heads, int32_t n_rep, int32_t max_context_len,
                                         float scale, fa_stream_t stream);

/* Varlen causal prefill over prefix-cached blocks: the suffix tokens' K/V must already be in
 * the pool (fa_reshape_and_cache); queries are the suffix tokens only. */
FA_API fa_status fa_paged_prefill(const fa_kv_layer *layer, const void *query, void *out,
                           const int32_t *cu_seqlens_q, const int32_t *context_lens,
                           const int32_t *block_tables, int32_t max_blocks_per_seq,
                           int32_t num_seqs, int32_t num_heads, int32_t n_rep, int32_t total_q,
                           int32_t max_seqlen_q, int32_t max_context_len, float scale, int32_t score_flow,
                           void *workspace, size_t workspace_bytes, fa_stream_t stream);

/* ---- the steps either side of attention (CausalSelfAttention::forward) ----------------- */

/* Weights of one layer's q/k/v projections, as candle's Linear stores them (out, in). */
typedef struct fa_qkv_weights {
  const void *weight;         /* device [(num_heads + 2*num_kv_heads) * head_dim, hidden]: the
                                 q_proj, k_proj, v_proj weights stacked in that order; pool dtype */
  const void *bias;           /* device [(num_heads + 2*num_kv_heads) * head_dim] or NULL
                                 (use_qkv_bias, attention.rs:28-33) */
  const void *q_norm_weight;  /* device [head_dim] or NULL: RMSNorm per query head (use_qk_norm) */
  const void *k_norm_weight;  /* device [head_dim] or NULL: RMSNorm per key head */
  float rms_eps;
  int32_t hidden;
  int32_t num_heads;
  const float *rope_cos;      /* device f32 [max_position, head_dim/2]: Cache::new's cos table */
  const float *rope_sin;      /* (src/models/common/cache.rs:378-392), 16-byte aligned */
  int32_t max_position;
} fa_qkv_weights;

/* Fused QKV projection + RoPE + reshape_and_cache. For each token t of x [num_tokens, hidden]:
 *   q|k|v = x[t] W^T (+ bias); q, k -> RMSNorm per head when a norm weight is given;
 *   q, k  -> rotate-half RoPE at positions[t] (candle_nn::rotary_emb::rope with the tables above);
 *   q     -> q_out[t] ([num_tokens, num_heads, head_dim]);
 *   k, v  -> the pool slot slot_mapping[t] (-1 skips the token), like fa_reshape_and_cache.
 * Replaces q/k/v_proj, q/k_norm, rope and Cache::write_kv of CausalSelfAttention::forward
 * (src/models/common/attention.rs:75-104). Computes in f32 and rounds each output once.
 * Requires a 16-bit pool, head_dim 64 or 128, hidden % 8 == 0, 16-byte aligned x and weight,
 * 32-byte aligned q_out. Bad positions / slots in device memory set FA_DEVERR_POSITION /
 * FA_DEVERR_SLOT and skip the row. */
FA_API fa_status fa_qkv_rope_cache(const fa_kv_layer *layer, const fa_qkv_weights *weights,
                                   const void *x, const int32_t *positions,
                                   const int32_t *slot_mapping, int32_t num_tokens, void *q_out,
                                   fa_stream_t stream);

/* Fused output projection + residual: out[t] = residual[t] + attn[t] W_o^T, with attn
 * [num_tokens, in_features] (the attention output, heads concatenated), weight
 * [out_features, in_features] and residual / out [num_tokens, out_features]; residual may be
 * NULL (plain projection) and may alias out. Replaces o_proj (attention.rs:116) and the residual
 * add of DecoderLayer::forward (src/models/common/transformer.rs:37-38).
 * Requires dtype FA_BF16 or FA_F16, in_features % 8 == 0, out_features % 32 == 0, 16-byte
 * aligned attn / weight / residual and 32-byte aligned out. */
FA_API fa_status fa_o_proj_residual(const void *attn, const void *weight, const void *residual,
                                    void *out, int32_t num_tokens, int32_t in_features,
                                    int32_t out_features, int32_t dtype, fa_stream_t stream);

/* The logits the engine reads after a forward: the final RMSNorm (CausalLM::forward,
 * src/models/common/model.rs:56) and lm_head (model.rs:58) applied to the last token of each
 * sequence, as f32 (engine.rs:220-222 takes logits[seq_len-1] and converts it to f32). The
 * reference projects every position and keeps the last; rows are independent, so only the
 * last rows are computed.
 *   hidden      [total_tokens, hidden_size] packed tokens (sequence s = rows
 *               cu_seqlens[s] .. cu_seqlens[s+1]-1), 16-bit
 *   norm_weight [hidden_size] or NULL (no scale), rms_eps its epsilon
 *   lm_head     [vocab, hidden_size] (candle Linear layout; a tied embedding works the same)
 *   normed_out  [num_seqs, hidden_size] scratch that receives the normalised last rows
 *   logits_out  [num_seqs, vocab] f32, device; copy it to the host (pinned memory,
 *               cudaMemcpyAsync on the same stream) for the sampler.
 * The norm is computed in f32 and rounded once to the model dtype (the GEMM operand); the
 * logits are accumulated in f32 and not rounded (the reference rounds them to the model dtype
 * before converting to f32). Requires dtype FA_BF16 or FA_F16, hidden_size % 8 == 0,
 * vocab % 32 == 0, 16-byte aligned hidden / lm_head / normed_out / logits_out. A sequence with
 * an empty or out-of-range token range gets zero logits and FA_DEVERR_SEQLEN. */
FA_API fa_status fa_last_token_logits(const void *hidden, const int32_t *cu_seqlens,
                                      int32_t num_seqs, int32_t total_tokens,
                                      const void *norm_weight, float rms_eps, const void *lm_head,
                                      int32_t hidden_size, int32_t vocab, int32_t dtype,
                                      void *normed_out, float *logits_out, fa_stream_t stream);

/* Width in output columns of the tiles the projection GEMMs above use for an M x N x K problem
 * (128 or 256; 128 when K is split over a thread-block cluster), as chosen on the current device.
 * A reporting aid: the choice depends only on the shape and the device's SM count. No
 * counterpart in the reference. */
FA_API int32_t fa_gemm_tile_width(int32_t M, int32_t N, int32_t K);

/* The projection GEMMs (fa_qkv_rope_cache, fa_o_proj_residual, fa_last_token_logits) are
 * launched with programmatic stream serialization: each may start its prologue and request its
 * first weight tiles while the preceding kernel on the stream finishes, and waits for that
 * kernel's completion before it reads activations or writes outputs. So are the decode kernels,
 * fa_tp_sync, fa_reshape_and_cache and fa_paged_prefill, which set up only on-chip state before
 * that wait. For a caller this changes nothing: stream order holds for every call. */

/* ---- head-sharded decode (tensor parallel over KV heads, one process per GPU) ----------
 * The reference runs attention on one CPU and has no sharding (its plan shards sequences,
 * which needs no exchange). This optional mode splits a layer's KV heads over `tp` GPUs: rank r
 * holds KV heads [r*kv/tp, (r+1)*kv/tp) of every block and the matching query heads. The decode
 * kernel writes each finished (sequence, kv head) output into EVERY rank's output buffer at the
 * rank's head offset (stores into peer memory over NVLink, mapped with CUDA IPC), so the
 * all-gather of the head outputs is part of the attention kernel, with no separate collective.
 * fa_tp_sync then publishes an epoch into slot [rank] of every rank's flag array (system-scope
 * release; stream order has completed the decode's stores) and waits, bounded, until every rank
 * published it into this rank's flags.
 *
 * Protocol: every rank makes the same calls, each fa_paged_decode_tp followed on the same
 * stream by fa_tp_sync(FA_TP_PUBLISH | FA_TP_WAIT) before the rank's next fa_paged_decode_tp
 * and before anything reads the output. Buffers: every rank allocates two output buffers, a flag
 * array of FA_MAX_TP u32 and an epoch counter with fa_ipc_alloc (zero-filled), exchanges the
 * handles and opens its peers' handles with fa_ipc_open. Consecutive decodes alternate the two
 * output buffers (two fa_tp_group values): a rank can be one decode ahead of a slower peer, and
 * the buffer of decode k is rewritten by decode k+2 only after every peer's sync k+1, i.e. after
 * each peer enqueued its reads of decode k's output ahead of its decode k+1. */
#define FA_MAX_TP 8
typedef struct fa_ipc_handle {
  unsigned char bytes[64]; /* cudaIpcMemHandle_t */
} fa_ipc_handle;

/* cudaMalloc + zero fill + cudaIpcGetMemHandle on the current device. */
FA_API fa_status fa_ipc_alloc(size_t bytes, void **ptr_out, fa_ipc_handle *handle_out);
FA_API fa_status fa_ipc_free(void *ptr);
/* Map a peer process's allocation into this process (peer access enabled lazily). */
FA_API fa_status fa_ipc_open(const fa_ipc_handle *handle, void **ptr_out);
FA_API fa_status fa_ipc_close(void *ptr);

typedef struct fa_tp_group {
  int32_t tp;                  /* ranks, 1..FA_MAX_TP */
  int32_t rank;                /* this process's rank */
  void *out[FA_MAX_TP];        /* rank r's output buffer [num_seqs, tp*num_heads, head_dim] for
                                  this call, as mapped in this process; 16-byte aligned */
  uint32_t *flags[FA_MAX_TP];  /* rank r's flag array (FA_MAX_TP u32), as mapped here */
  uint32_t *epoch_counter;     /* this rank's device epoch (4 bytes, zero): used when epoch == 0 */
} fa_tp_group;

/* fa_paged_decode over this rank's head shard (layer = the rank's KV heads, query [num_seqs,
 * num_heads, head_dim] = its query heads), writing the rows into every rank's group->out at
 * head offset rank*num_heads. Requires the fast decode path (16-bit pool, block_size 16,
 * head_dim 64/128, n_rep <= 8). Signals nothing: fa_tp_sync follows it. */
FA_API fa_status fa_paged_decode_tp(const fa_tp_group *group, const fa_kv_layer *layer,
                                    const void *query, const int32_t *context_lens,
                                    const int32_t *block_tables, int32_t max_blocks_per_seq,
                                    int32_t num_seqs, int32_t num_heads, int32_t n_rep,
                                    int32_t max_context_len, float scale, int32_t score_flow, void *workspace,
                                    size_t workspace_bytes, fa_stream_t stream);

/* FA_TP_PUBLISH: store the epoch into every rank's flag slot [group->rank]; FA_TP_WAIT: make
 * `stream` wait until every rank's slot in this rank's flags holds the epoch (or a later one).
 * epoch >= 1: that value (the host counts epochs). epoch == 0: device-counted, so the calls can
 * be captured in a CUDA graph and replayed: a publish first adds one to *group->epoch_counter,
 * and the epoch is the counter's value. Use one kind of epoch per group. The wait gives up
 * after timeout_ns (1 us .. 10 s) of device time, sets FA_DEVERR_TIMEOUT (fa_device_status)
 * and returns, leaving the context usable. */
#define FA_TP_PUBLISH 1
#define FA_TP_WAIT 2
FA_API fa_status fa_tp_sync(const fa_tp_group *group, uint32_t epoch, int32_t mode,
                            int64_t timeout_ns, fa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLOUR_ATTN_H */
