// flour_host.h — C++ host side of the B200 paged KV path, above the C ABI (flour_attn.h).
//
// The reference (lltsdyp/flour) is Rust; its host-side types on this path are mirrored here
// with the same names, argument meaning and error behaviour, so a C++ caller (or a Rust caller
// through a thin binding) drives the GPU pool exactly as the reference drives its CPU pool:
//
//   BlockAllocator    src/models/common/paged.rs:7-53     refcounted free list (host only)
//   BlockTable        src/models/common/paged.rs:57-122   logical position -> physical slot
//   block_hash,
//   PrefixRegistry    src/models/common/prefix.rs         chained prefix hashes -> block ids
//   PagedKvPool       src/models/common/paged.rs:129-280  per-layer K/V slabs, now in HBM with
//                                                         layout [num_blocks, kv_heads, bs, d]
//   KvCache           src/models/common/cache.rs:12-165   one sequence: allocator, table,
//                                                         registry, pool
//   Cache             src/models/common/cache.rs:367-500  RoPE tables + KvCache (allocate_kv,
//                                                         write_kv, kv_blocks, prefix reuse)
//   paged_attention   src/backend/cpu.rs:57-112           one sequence's attention on the GPU
//   build_batch       (new)                               many sequences' tables packed into the
//                                                         int32 arrays the batched kernels take
//
// Reference errors (candle_core::bail!) are thrown as flour::Error with the reference's text;
// C ABI failures are thrown as flour::Error carrying the library's message and status.
// Device memory of the pool is allocated once, when the pool is built; nothing on the per-step
// path allocates except the growth of reusable staging buffers.
#pragma once

#include <cstddef>
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "flour_attn.h"

// Exported from libflour_attn.so (built with hidden visibility by default).
namespace flour __attribute__((visibility("default"))) {

struct Error : std::runtime_error {
  explicit Error(const std::string &msg, int32_t status = FA_EINVAL)
      : std::runtime_error(msg), status(status) {}
  int32_t status;
};

// Throws flour::Error for a non-OK fa_status, with the library's message.
void check(int32_t status, const char *what);

enum class DType : int32_t { F32 = FA_F32, BF16 = FA_BF16, F16 = FA_F16 };
size_t dtype_size(DType t);

// Device memory helpers for callers that do not link a CUDA runtime of their own (bindings,
// tests): allocation, synchronous copies and the device count, through this library's runtime.
int device_count();
void *device_alloc(size_t bytes);
void device_free(void *p);
void copy_to_device(void *dst, const void *src, size_t bytes);
void copy_to_host(void *dst, const void *src, size_t bytes);
void device_synchronize();

// A view of device memory with a shape (the stand-in for the reference's candle Tensor at the
// boundary). Contiguous, row-major.
struct DeviceTensor {
  void *data = nullptr;
  DType dtype = DType::BF16;
  std::vector<int64_t> shape;
  size_t rank() const { return shape.size(); }
  int64_t numel() const;
  std::string dims() const;  // "[a, b, c]" like candle's {:?} of dims()
};

// ---- paged.rs:7-53 ---------------------------------------------------------------------------
class BlockAllocator {
 public:
  explicit BlockAllocator(size_t num_blocks);
  std::optional<size_t> allocate();  // the first call returns block 0
  void incref(size_t block_id);
  bool decref(size_t block_id);      // true when the block returned to the free list
  size_t ref_count(size_t block_id) const;
  size_t num_free() const { return free_.size(); }

 private:
  std::vector<size_t> free_;
  std::vector<size_t> ref_counts_;
};

// ---- paged.rs:57-122 -------------------------------------------------------------------------
class BlockTable {
 public:
  explicit BlockTable(size_t block_size) : block_size_(block_size) {}
  size_t len() const { return len_; }
  bool is_empty() const { return len_ == 0; }
  size_t block_size() const { return block_size_; }
  size_t capacity() const { return blocks_.size() * block_size_; }
  void push_block(size_t block_id) { blocks_.push_back(block_id); }
  const std::vector<size_t> &blocks() const { return blocks_; }
  size_t block_at(size_t logical_block) const { return blocks_.at(logical_block); }
  void clear();
  void advance(size_t n) { len_ += n; }
  size_t slot(size_t pos) const;                          // blocks[pos/bs]*bs + pos%bs
  std::vector<uint32_t> slots(size_t start, size_t end) const;

 private:
  std::vector<size_t> blocks_;
  size_t block_size_;
  size_t len_ = 0;
};

// ---- prefix.rs -------------------------------------------------------------------------------
constexpr uint64_t PREFIX_HASH_SEED = 0;
// Chained content hash of one full block: SipHash-1-3 with zero keys (what Rust's DefaultHasher
// computes) over parent (u64 LE) || token count (u64 LE) || tokens (u32 LE each).
uint64_t block_hash(uint64_t parent, const uint32_t *tokens, size_t n);

class PrefixRegistry {
 public:
  std::optional<size_t> get(uint64_t hash, const uint32_t *tokens, size_t n) const;
  bool contains(uint64_t hash) const { return entries_.count(hash) != 0; }
  void insert(uint64_t hash, std::vector<uint32_t> tokens, size_t block_id);
  void clear() { entries_.clear(); }
  std::vector<size_t> drain_block_ids();
  size_t size() const { return entries_.size(); }

 private:
  std::unordered_map<uint64_t, std::pair<std::vector<uint32_t>, size_t>> entries_;
};

// ---- paged.rs:129-280 ------------------------------------------------------------------------
struct BlockView {     // (1, kv_heads, n, head_dim) slots of one physical block, zero-copy
  void *k = nullptr;   // device address of (head 0, first slot)
  void *v = nullptr;
  int64_t head_stride; // elements between heads (block_size * head_dim)
  int64_t n;
};

class PagedKvPool {
 public:
  // Zero-filled device slabs [num_blocks, kv_heads, block_size, head_dim] per layer for K and
  // V. with_device=false keeps only the bookkeeping (host-only tests of the logic above it).
  PagedKvPool(size_t num_layers, size_t num_blocks, size_t kv_heads, size_t head_dim, DType dtype,
              size_t block_size = 16, bool with_device = true);
  ~PagedKvPool();
  PagedKvPool(const PagedKvPool &) = delete;
  PagedKvPool &operator=(const PagedKvPool &) = delete;

  size_t num_layers() const { return num_layers_; }
  size_t num_blocks() const { return num_blocks_; }
  size_t kv_heads() const { return kv_heads_; }
  size_t head_dim() const { return head_dim_; }
  size_t block_size() const { return block_size_; }
  DType dtype() const { return dtype_; }
  bool has_device() const { return with_device_; }
  fa_kv_layer layer(size_t layer_idx) const;

  // k, v: device (1, kv_heads, n, head_dim) or (kv_heads, n, head_dim), pool dtype; token i goes
  // to slots[i] (one fa_reshape_and_cache launch).
  void write(size_t layer_idx, const std::vector<uint32_t> &slots, const DeviceTensor &k,
             const DeviceTensor &v, fa_stream_t stream = nullptr);
  // Overwrite physical block `block_id` with (1, kv_heads, bs, d) or (kv_heads, bs, d) K/V
  // (device or host memory).
  void write_block(size_t layer_idx, size_t block_id, const DeviceTensor &k, const DeviceTensor &v,
                   fa_stream_t stream = nullptr);
  // Copy the slots into host buffers as (kv_heads, n, head_dim) (test / export helper).
  void gather(size_t layer_idx, const std::vector<uint32_t> &slots, void *k_host, void *v_host) const;
  BlockView block_view(size_t layer_idx, size_t start_slot, size_t n) const;

 private:
  size_t num_layers_, num_blocks_, kv_heads_, head_dim_, block_size_;
  DType dtype_;
  bool with_device_;
  std::vector<void *> k_, v_;
  int32_t *slot_buf_ = nullptr;  // device staging for slot ids, grown on demand
  size_t slot_cap_ = 0;
};

// What kv_blocks hands to paged_attention: the layer's slabs, this sequence's logical ->
// physical blocks and its live length (cache.rs:83-96 returns one view per logical block).
struct SequenceBlocks {
  fa_kv_layer layer;
  std::vector<int32_t> block_table;
  int32_t kv_len;
};

// ---- cache.rs:12-165 -------------------------------------------------------------------------
class KvCache {
 public:
  KvCache(size_t num_layers, size_t max_seq_len, size_t kv_heads, size_t head_dim, DType dtype,
          size_t block_size = 16, bool with_device = true);
  std::optional<size_t> allocate();
  size_t len() const { return table_.len(); }
  bool is_empty() const { return table_.is_empty(); }
  size_t capacity() const { return table_.capacity(); }
  std::vector<uint32_t> slots(size_t start, size_t end) const { return table_.slots(start, end); }
  void advance(size_t seq_len) { table_.advance(seq_len); }
  // The trailing k.shape[-2] tokens of the sequence go to their slots (cache.rs:71-77).
  void write_current(size_t layer_idx, const DeviceTensor &k, const DeviceTensor &v,
                     fa_stream_t stream = nullptr);
  SequenceBlocks gather_blocks(size_t layer_idx) const;
  void reset_sequence();
  size_t match_prefix(const std::vector<uint32_t> &token_ids);
  void register_prefix(const std::vector<uint32_t> &token_ids);
  void clear_prefix_cache();
  size_t free_blocks() const { return allocator_.num_free(); }
  const BlockTable &table() const { return table_; }
  PagedKvPool &pool() { return pool_; }
  const BlockAllocator &allocator() const { return allocator_; }

 private:
  BlockAllocator allocator_;
  BlockTable table_;
  PrefixRegistry registry_;
  PagedKvPool pool_;
};

// The Config fields Cache::new reads (src/models/common/mod.rs).
struct Config {
  size_t num_hidden_layers;
  size_t num_attention_heads;
  size_t num_key_value_heads;
  size_t head_dim;
  double rope_theta;
  size_t max_seq_len;
};

// ---- cache.rs:367-500 ------------------------------------------------------------------------
class Cache {
 public:
  Cache(const Config &cfg, DType dtype, bool with_device = true);
  ~Cache();
  Cache(const Cache &) = delete;
  Cache &operator=(const Cache &) = delete;
  // f32 tables [max_seq_len, head_dim/2] holding cos/sin rounded to the model dtype (cache.rs:
  // 378-392); host copies and, with a device, device copies the fused QKV kernel reads.
  const std::vector<float> &cos_host() const { return cos_; }
  const std::vector<float> &sin_host() const { return sin_; }
  const float *rope_cos_device() const { return cos_dev_; }
  const float *rope_sin_device() const { return sin_dev_; }
  void allocate_kv(size_t seq_len);
  void write_kv(size_t layer_idx, const DeviceTensor &k, const DeviceTensor &v,
                fa_stream_t stream = nullptr) { kvs_.write_current(layer_idx, k, v, stream); }
  SequenceBlocks kv_blocks(size_t layer_idx) const { return kvs_.gather_blocks(layer_idx); }
  void reset_sequence() { kvs_.reset_sequence(); }
  size_t match_prefix(const std::vector<uint32_t> &ids) { return kvs_.match_prefix(ids); }
  void register_prefix(const std::vector<uint32_t> &ids) { kvs_.register_prefix(ids); }
  void clear_prefix_cache() { kvs_.clear_prefix_cache(); }
  size_t free_blocks() const { return kvs_.free_blocks(); }
  KvCache &kvs() { return kvs_; }
  size_t max_seq_len() const { return max_seq_len_; }

 private:
  std::vector<float> cos_, sin_;
  float *cos_dev_ = nullptr, *sin_dev_ = nullptr;
  KvCache kvs_;
  size_t max_seq_len_;
};

// cpu.rs:57-112 on the GPU for one sequence (the reference's b is 1): q and out are device
// [q_len, num_heads, head_dim] (token-major) in the pool dtype; the last q_len tokens of the
// sequence are the queries. Uses the workspace and device table buffers of `scratch`.
struct AttentionScratch {
  AttentionScratch() = default;
  ~AttentionScratch();
  AttentionScratch(const AttentionScratch &) = delete;
  AttentionScratch &operator=(const AttentionScratch &) = delete;
  void *workspace = nullptr;
  size_t workspace_bytes = 0;
  int32_t *tables = nullptr;   // [2 + 1 + max_blocks]: cu_seqlens, context_len, block table
  size_t tables_cap = 0;
};
// score_flow: FA_SCORES_F32 (default) or FA_SCORES_REFERENCE (the reference's bf16/f16 score
// rounding of cpu.rs:84-85).
void paged_attention(const DeviceTensor &q, const SequenceBlocks &blocks, int32_t n_rep,
                     double scale, DeviceTensor &out, AttentionScratch &scratch,
                     fa_stream_t stream = nullptr, int32_t score_flow = FA_SCORES_F32);

// ---- batched metadata (new) ------------------------------------------------------------------
// Sequence i contributes q_lens[i] new tokens (its last q_lens[i] positions) and its table's
// blocks; the result is what fa_paged_attention / fa_reshape_and_cache take.
struct BatchMetadata {
  std::vector<int32_t> block_tables;   // [num_seqs, max_blocks_per_seq], unused entries 0
  std::vector<int32_t> context_lens;   // [num_seqs]
  std::vector<int32_t> cu_seqlens_q;   // [num_seqs + 1]
  std::vector<int32_t> slot_mapping;   // [total_q]
  int32_t num_seqs = 0, max_blocks_per_seq = 1, max_context_len = 0, max_seqlen_q = 0,
          total_q = 0;
};
BatchMetadata build_batch(const std::vector<const BlockTable *> &tables,
                          const std::vector<size_t> &q_lens);

}  // namespace flour
