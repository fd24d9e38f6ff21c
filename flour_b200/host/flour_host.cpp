// Implementation of the C++ host side (flour_host.h). Each type cites the reference lines it
// mirrors; the GPU work goes through the C ABI entry points of flour_attn.h.
#include "flour_host.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <sstream>

namespace flour {

namespace {

void cuda_check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e), FA_ECUDA);
}

// bf16 / f16 rounding of an f32 value, returned as f32 (the reference casts its f32 RoPE
// tables to the model dtype, cache.rs:388-392).
float round_to(float x, DType t) {
  if (t == DType::F32) return x;
  if (t == DType::F16) {
    // IEEE binary16 round-to-nearest-even through the hardware-independent bit route.
    uint32_t u;
    std::memcpy(&u, &x, 4);
    const uint32_t sign = u & 0x80000000u;
    float a = std::fabs(x);
    if (!(a < 65520.0f)) {  // overflow (or NaN) -> inf / NaN
      const float r = std::isnan(x) ? x : (sign ? -INFINITY : INFINITY);
      return r;
    }
    // Scale so that the f16 quantum becomes 1, round to nearest even, scale back.
    int e;
    std::frexp(a, &e);               // a = m * 2^e, m in [0.5, 1)
    const int q = std::max(e - 11, -24);  // f16 has 11 significant bits; subnormals at 2^-24
    const float scaled = std::ldexp(a, -q);
    const float r = std::nearbyint(scaled);  // default rounding mode: to nearest even
    const float out = std::ldexp(r, q);
    return sign ? -out : out;
  }
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;  // inf / NaN unchanged
  u = (u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

// ---- SipHash-1-3 (Aumasson & Bernstein, "SipHash: a fast short-input PRF", 2012), zero key ----
inline uint64_t rotl(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }

struct Sip13 {
  uint64_t v0 = 0x736f6d6570736575ull, v1 = 0x646f72616e646f6dull, v2 = 0x6c7967656e657261ull,
           v3 = 0x7465646279746573ull;
  uint64_t tail = 0;
  int ntail = 0;
  uint64_t length = 0;
  void round() {
    v0 += v1; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32);
    v2 += v3; v3 = rotl(v3, 16); v3 ^= v2;
    v0 += v3; v3 = rotl(v3, 21); v3 ^= v0;
    v2 += v1; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32);
  }
  void block(uint64_t m) {
    v3 ^= m;
    round();
    v0 ^= m;
  }
  void write(const uint8_t *p, size_t n) {
    length += n;
    for (size_t i = 0; i < n; ++i) {
      tail |= uint64_t(p[i]) << (8 * ntail);
      if (++ntail == 8) {
        block(tail);
        tail = 0;
        ntail = 0;
      }
    }
  }
  uint64_t finish() {
    block(tail | ((length & 0xff) << 56));
    v2 ^= 0xff;
    round();
    round();
    round();
    return v0 ^ v1 ^ v2 ^ v3;
  }
};

void put_u64(Sip13 &h, uint64_t x) {
  uint8_t b[8];
  for (int i = 0; i < 8; ++i) b[i] = uint8_t(x >> (8 * i));
  h.write(b, 8);
}

}  // namespace

void check(int32_t status, const char *what) {
  if (status == FA_OK) return;
  throw Error(std::string(what) + ": " + fa_last_error_message() + " (status " +
                  std::to_string(status) + ")",
              status);
}

size_t dtype_size(DType t) { return t == DType::F32 ? 4 : 2; }

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

void *device_alloc(size_t bytes) {
  void *p = nullptr;
  cuda_check(cudaMalloc(&p, bytes), "device_alloc");
  return p;
}

void device_free(void *p) {
  if (p) cudaFree(p);
}

void copy_to_device(void *dst, const void *src, size_t bytes) {
  cuda_check(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "copy_to_device");
}

void copy_to_host(void *dst, const void *src, size_t bytes) {
  cuda_check(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "copy_to_host");
}

void device_synchronize() { cuda_check(cudaDeviceSynchronize(), "device_synchronize"); }

int64_t DeviceTensor::numel() const {
  int64_t n = 1;
  for (int64_t s : shape) n *= s;
  return n;
}

std::string DeviceTensor::dims() const {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < shape.size(); ++i) o << (i ? ", " : "") << shape[i];
  o << "]";
  return o.str();
}

// ---- BlockAllocator (paged.rs:7-53) -----------------------------------------------------------

BlockAllocator::BlockAllocator(size_t num_blocks) : ref_counts_(num_blocks, 0) {
  free_.reserve(num_blocks);
  for (size_t i = num_blocks; i-- > 0;) free_.push_back(i);  // the first allocate returns 0
}

std::optional<size_t> BlockAllocator::allocate() {
  if (free_.empty()) return std::nullopt;
  const size_t id = free_.back();
  free_.pop_back();
  ref_counts_[id] = 1;
  return id;
}

void BlockAllocator::incref(size_t block_id) { ref_counts_.at(block_id) += 1; }

bool BlockAllocator::decref(size_t block_id) {
  size_t &rc = ref_counts_.at(block_id);
  if (rc == 0) throw Error("decref of unreferenced block");
  if (--rc == 0) {
    free_.push_back(block_id);
    return true;
  }
  return false;
}

size_t BlockAllocator::ref_count(size_t block_id) const { return ref_counts_.at(block_id); }

// ---- BlockTable (paged.rs:57-122) -----------------------------------------------------------------

void BlockTable::clear() {
  blocks_.clear();
  len_ = 0;
}

size_t BlockTable::slot(size_t pos) const {
  return blocks_.at(pos / block_size_) * block_size_ + pos % block_size_;
}

std::vector<uint32_t> BlockTable::slots(size_t start, size_t end) const {
  std::vector<uint32_t> s;
  s.reserve(end > start ? end - start : 0);
  for (size_t p = start; p < end; ++p) s.push_back(uint32_t(slot(p)));
  return s;
}

// ---- prefix.rs --------------------------------------------------------------------------------------

uint64_t block_hash(uint64_t parent, const uint32_t *tokens, size_t n) {
  Sip13 h;
  put_u64(h, parent);               // u64::hash -> write_u64
  put_u64(h, uint64_t(n));          // [u32]::hash -> length prefix (usize) ...
  for (size_t i = 0; i < n; ++i) {  // ... then the elements' bytes
    uint8_t b[4] = {uint8_t(tokens[i]), uint8_t(tokens[i] >> 8), uint8_t(tokens[i] >> 16),
                    uint8_t(tokens[i] >> 24)};
    h.write(b, 4);
  }
  return h.finish();
}

std::optional<size_t> PrefixRegistry::get(uint64_t hash, const uint32_t *tokens,
                                                 size_t n) const {
  auto it = entries_.find(hash);
  if (it == entries_.end()) return std::nullopt;
  const auto &stored = it->second.first;
  if (stored.size() != n || !std::equal(stored.begin(), stored.end(), tokens)) return std::nullopt;
  return it->second.second;
}

void PrefixRegistry::insert(uint64_t hash, std::vector<uint32_t> tokens, size_t block_id) {
  entries_[hash] = {std::move(tokens), block_id};
}

std::vector<size_t> PrefixRegistry::drain_block_ids() {
  std::vector<size_t> ids;
  ids.reserve(entries_.size());
  for (auto &e : entries_) ids.push_back(e.second.second);
  entries_.clear();
  return ids;
}

// ---- PagedKvPool (paged.rs:129-280) --------------------------------------------------------------

PagedKvPool::PagedKvPool(size_t num_layers, size_t num_blocks, size_t kv_heads,
                                size_t head_dim, DType dtype, size_t block_size, bool with_device)
    : num_layers_(num_layers), num_blocks_(num_blocks), kv_heads_(kv_heads), head_dim_(head_dim),
      block_size_(block_size), dtype_(dtype), with_device_(with_device) {
  if (!with_device_) return;
  const size_t bytes = num_blocks * kv_heads * block_size * head_dim * dtype_size(dtype);
  try {
    for (size_t l = 0; l < num_layers; ++l) {
      void *k = nullptr, *v = nullptr;
      cuda_check(cudaMalloc(&k, bytes), "PagedKvPool: cudaMalloc");
      k_.push_back(k);
      cuda_check(cudaMalloc(&v, bytes), "PagedKvPool: cudaMalloc");
      v_.push_back(v);
      cuda_check(cudaMemset(k, 0, bytes), "PagedKvPool: cudaMemset");  // Tensor::zeros
      cuda_check(cudaMemset(v, 0, bytes), "PagedKvPool: cudaMemset");
    }
  } catch (...) {
    for (void *p : k_) cudaFree(p);
    for (void *p : v_) cudaFree(p);
    throw;
  }
}

PagedKvPool::~PagedKvPool() {
  for (void *p : k_) cudaFree(p);
  for (void *p : v_) cudaFree(p);
  if (slot_buf_) cudaFree(slot_buf_);
}

fa_kv_layer PagedKvPool::layer(size_t layer_idx) const {
  if (!with_device_) throw Error("PagedKvPool has no device slabs");
  fa_kv_layer L{};
  L.k_cache = k_.at(layer_idx);
  L.v_cache = v_.at(layer_idx);
  L.num_blocks = int32_t(num_blocks_);
  L.num_kv_heads = int32_t(kv_heads_);
  L.block_size = int32_t(block_size_);
  L.head_dim = int32_t(head_dim_);
  L.dtype = int32_t(dtype_);
  return L;
}

namespace {
// (1, kv_heads, n, d) -> squeezed dims, or (kv_heads, n, d) as is; else the reference's error.
std::vector<int64_t> normalize(const DeviceTensor &t, const char *who) {
  if (t.rank() == 4) {
    if (t.shape[0] != 1)
      throw Error(std::string(who) + ": cannot squeeze dim 0 of size " + std::to_string(t.shape[0]));
    return {t.shape[1], t.shape[2], t.shape[3]};
  }
  if (t.rank() == 3) return t.shape;
  throw Error(std::string(who) + " expects rank 3 or 4 tensor, got rank " + std::to_string(t.rank()));
}
}  // namespace

void PagedKvPool::write(size_t layer_idx, const std::vector<uint32_t> &slots,
                               const DeviceTensor &k, const DeviceTensor &v, fa_stream_t stream) {
  const auto kd = normalize(k, "write"), vd = normalize(v, "write");
  if (kd != vd) throw Error("write k/v shape mismatch: k=" + k.dims() + " v=" + v.dims());
  const int64_t n = kd[1];
  if (size_t(kd[0]) != kv_heads_ || size_t(kd[2]) != head_dim_ || size_t(n) != slots.size())
    throw Error("write expects (1, kv_heads, slots.len(), head_dim), got " + k.dims());
  if (k.dtype != dtype_ || v.dtype != dtype_) throw Error("write: k/v dtype differs from the pool");
  if (n == 0) return;
  if (slots.size() > slot_cap_) {
    if (slot_buf_) cudaFree(slot_buf_);
    slot_buf_ = nullptr;
    slot_cap_ = 0;
    cuda_check(cudaMalloc(&slot_buf_, slots.size() * sizeof(int32_t)), "PagedKvPool::write");
    slot_cap_ = slots.size();
  }
  std::vector<int32_t> s32(slots.size());
  for (size_t i = 0; i < slots.size(); ++i) {
    if (slots[i] >= num_blocks_ * block_size_)
      throw Error("write: slot " + std::to_string(slots[i]) + " outside the pool", FA_ERANGE);
    s32[i] = int32_t(slots[i]);
  }
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Pageable source: the copy is complete before cudaMemcpyAsync returns (s32 may go away).
  cuda_check(cudaMemcpyAsync(slot_buf_, s32.data(), s32.size() * sizeof(int32_t),
                             cudaMemcpyHostToDevice, st),
             "PagedKvPool::write");
  const fa_kv_layer L = layer(layer_idx);
  // (kv_heads, n, d): token stride d, head stride n*d (paged.rs:186-204 writes token i to slots[i]).
  check(fa_reshape_and_cache(&L, k.data, v.data, int64_t(head_dim_), n * int64_t(head_dim_),
                             int64_t(head_dim_), n * int64_t(head_dim_), slot_buf_, int32_t(n),
                             stream),
        "PagedKvPool::write");
}

void PagedKvPool::write_block(size_t layer_idx, size_t block_id, const DeviceTensor &k,
                                     const DeviceTensor &v, fa_stream_t stream) {
  const auto kd = normalize(k, "write_block"), vd = normalize(v, "write_block");
  if (kd != vd) {
    auto fmt = [](const std::vector<int64_t> &d) {
      std::ostringstream o;
      o << "[" << d[0] << ", " << d[1] << ", " << d[2] << "]";
      return o.str();
    };
    throw Error("write_block k/v shape mismatch: k=" + fmt(kd) + " v=" + fmt(vd));
  }
  if (size_t(kd[0]) != kv_heads_ || size_t(kd[2]) != head_dim_)
    throw Error("write_block expects (.., kv_heads=" + std::to_string(kv_heads_) +
                ", block_size, head_dim=" + std::to_string(head_dim_) +
                "), got kv_heads=" + std::to_string(kd[0]) + " head_dim=" + std::to_string(kd[2]));
  if (size_t(kd[1]) != block_size_)
    throw Error("write_block expects block_size " + std::to_string(block_size_) + ", got " +
                std::to_string(kd[1]));
  if (k.dtype != dtype_ || v.dtype != dtype_) throw Error("write_block: k/v dtype differs from the pool");
  const fa_kv_layer L = layer(layer_idx);
  check(fa_write_block(&L, int32_t(block_id), k.data, v.data, stream), "PagedKvPool::write_block");
}

void PagedKvPool::gather(size_t layer_idx, const std::vector<uint32_t> &slots, void *k_host,
                                void *v_host) const {
  const fa_kv_layer L = layer(layer_idx);
  const size_t es = dtype_size(dtype_), row = head_dim_ * es, n = slots.size();
  for (size_t i = 0; i < n; ++i) {
    if (slots[i] >= num_blocks_ * block_size_)
      throw Error("gather: slot " + std::to_string(slots[i]) + " outside the pool", FA_ERANGE);
    const size_t blk = slots[i] / block_size_, off = slots[i] % block_size_;
    for (size_t h = 0; h < kv_heads_; ++h) {
      const size_t src = ((blk * kv_heads_ + h) * block_size_ + off) * row;
      const size_t dst = (h * n + i) * row;
      cuda_check(cudaMemcpy(static_cast<char *>(k_host) + dst, static_cast<const char *>(L.k_cache) + src,
                            row, cudaMemcpyDeviceToHost), "PagedKvPool::gather");
      cuda_check(cudaMemcpy(static_cast<char *>(v_host) + dst, static_cast<const char *>(L.v_cache) + src,
                            row, cudaMemcpyDeviceToHost), "PagedKvPool::gather");
    }
  }
}

BlockView PagedKvPool::block_view(size_t layer_idx, size_t start_slot, size_t n) const {
  const size_t blk = start_slot / block_size_, off = start_slot % block_size_;
  if (off + n > block_size_) throw Error("block_view spans more than one physical block");
  if (blk >= num_blocks_) throw Error("block_view: block outside the pool", FA_ERANGE);
  const fa_kv_layer L = layer(layer_idx);
  const size_t es = dtype_size(dtype_);
  const size_t base = (blk * kv_heads_ * block_size_ + off) * head_dim_ * es;
  BlockView bv;
  bv.k = static_cast<char *>(L.k_cache) + base;
  bv.v = static_cast<char *>(L.v_cache) + base;
  bv.head_stride = int64_t(block_size_ * head_dim_);
  bv.n = int64_t(n);
  return bv;
}

// ---- KvCache (cache.rs:12-165) --------------------------------------------------------------------

KvCache::KvCache(size_t num_layers, size_t max_seq_len, size_t kv_heads, size_t head_dim,
                        DType dtype, size_t block_size, bool with_device)
    : allocator_((max_seq_len + block_size - 1) / block_size),
      table_(block_size),
      pool_(num_layers, (max_seq_len + block_size - 1) / block_size, kv_heads, head_dim, dtype,
            block_size, with_device) {}

std::optional<size_t> KvCache::allocate() {
  auto b = allocator_.allocate();
  if (b) table_.push_block(*b);
  return b;
}

void KvCache::write_current(size_t layer_idx, const DeviceTensor &k, const DeviceTensor &v,
                                   fa_stream_t stream) {
  if (k.rank() < 2) throw Error("write_current: k must be (1, kv_heads, seq_len, head_dim)");
  const size_t seq_len = size_t(k.shape[k.rank() - 2]);
  const size_t end = table_.len();
  if (seq_len > end) throw Error("write_current: more tokens than the sequence holds");
  pool_.write(layer_idx, table_.slots(end - seq_len, end), k, v, stream);
}

SequenceBlocks KvCache::gather_blocks(size_t layer_idx) const {
  SequenceBlocks sb;
  sb.layer = pool_.layer(layer_idx);
  const size_t bs = table_.block_size();
  const size_t n = (table_.len() + bs - 1) / bs;
  for (size_t i = 0; i < n; ++i) sb.block_table.push_back(int32_t(table_.block_at(i)));
  sb.kv_len = int32_t(table_.len());
  return sb;
}

void KvCache::reset_sequence() {
  for (size_t b : table_.blocks()) allocator_.decref(b);
  table_.clear();
}

size_t KvCache::match_prefix(const std::vector<uint32_t> &ids) {
  const size_t bs = table_.block_size();
  const size_t num_full = ids.size() / bs;
  // A block-aligned prompt never reuses its final full block: a suffix must remain.
  const size_t max_reusable = ids.size() % bs == 0 ? (num_full ? num_full - 1 : 0) : num_full;
  uint64_t parent = PREFIX_HASH_SEED;
  size_t matched = 0;
  for (size_t b = 0; b < max_reusable; ++b) {
    const uint32_t *chunk = ids.data() + b * bs;
    const uint64_t h = block_hash(parent, chunk, bs);
    auto id = registry_.get(h, chunk, bs);
    if (!id) break;
    allocator_.incref(*id);
    table_.push_block(*id);
    matched += bs;
    parent = h;
  }
  table_.advance(matched);
  return matched;
}

void KvCache::register_prefix(const std::vector<uint32_t> &ids) {
  const size_t bs = table_.block_size();
  const size_t num_full = ids.size() / bs;
  uint64_t parent = PREFIX_HASH_SEED;
  for (size_t b = 0; b < num_full; ++b) {
    const uint32_t *chunk = ids.data() + b * bs;
    const uint64_t h = block_hash(parent, chunk, bs);
    if (!registry_.contains(h)) {
      const size_t block_id = table_.block_at(b);
      allocator_.incref(block_id);  // the registry holds its own reference
      registry_.insert(h, std::vector<uint32_t>(chunk, chunk + bs), block_id);
    }
    parent = h;
  }
}

void KvCache::clear_prefix_cache() {
  for (size_t id : registry_.drain_block_ids()) allocator_.decref(id);
}

// ---- Cache (cache.rs:367-500) ----------------------------------------------------------------------

Cache::Cache(const Config &cfg, DType dtype, bool with_device)
    : kvs_(cfg.num_hidden_layers, cfg.max_seq_len, cfg.num_key_value_heads, cfg.head_dim, dtype,
           16, with_device),
      max_seq_len_(cfg.max_seq_len) {
  const size_t half = cfg.head_dim / 2;
  std::vector<float> theta(half);
  for (size_t i = 0; i < half; ++i)
    theta[i] = 1.0f / std::pow(float(cfg.rope_theta), float(2 * i) / float(cfg.head_dim));
  cos_.resize(cfg.max_seq_len * half);
  sin_.resize(cfg.max_seq_len * half);
  for (size_t p = 0; p < cfg.max_seq_len; ++p)
    for (size_t i = 0; i < half; ++i) {
      const float a = float(p) * theta[i];  // f32 outer product, then cos/sin in f32
      cos_[p * half + i] = round_to(std::cos(a), dtype);
      sin_[p * half + i] = round_to(std::sin(a), dtype);
    }
  if (with_device) {
    const size_t bytes = cos_.size() * sizeof(float);
    cuda_check(cudaMalloc(&cos_dev_, bytes), "Cache: cudaMalloc");
    cuda_check(cudaMalloc(&sin_dev_, bytes), "Cache: cudaMalloc");
    cuda_check(cudaMemcpy(cos_dev_, cos_.data(), bytes, cudaMemcpyHostToDevice), "Cache: upload");
    cuda_check(cudaMemcpy(sin_dev_, sin_.data(), bytes, cudaMemcpyHostToDevice), "Cache: upload");
  }
}

Cache::~Cache() {
  if (cos_dev_) cudaFree(cos_dev_);
  if (sin_dev_) cudaFree(sin_dev_);
}

void Cache::allocate_kv(size_t seq_len) {
  const size_t end = kvs_.len() + seq_len;
  if (end > max_seq_len_)
    throw Error("paged kv cache overflow: " + std::to_string(end) +
                " tokens exceeds max_seq_len " + std::to_string(max_seq_len_));
  while (kvs_.capacity() < end)
    if (!kvs_.allocate()) throw Error("out of kv blocks");
  kvs_.advance(seq_len);
}

// ---- paged_attention (cpu.rs:57-112) ------------------------------------------------------------

AttentionScratch::~AttentionScratch() {
  if (workspace) cudaFree(workspace);
  if (tables) cudaFree(tables);
}

void paged_attention(const DeviceTensor &q, const SequenceBlocks &blocks, int32_t n_rep,
                            double scale, DeviceTensor &out, AttentionScratch &scratch,
                            fa_stream_t stream, int32_t score_flow) {
  if (q.rank() != 3 || out.shape != q.shape)
    throw Error("paged_attention: q and out must be [q_len, num_heads, head_dim], got q=" +
                q.dims() + " out=" + out.dims());
  const int32_t q_len = int32_t(q.shape[0]), num_heads = int32_t(q.shape[1]);
  const int32_t kv_len = blocks.kv_len;
  if (q_len > kv_len) throw Error("paged_attention: more queries than keys");
  const int32_t nb = int32_t(std::max<size_t>(1, blocks.block_table.size()));
  const size_t need_tables = size_t(3 + nb);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (need_tables > scratch.tables_cap) {
    cuda_check(cudaStreamSynchronize(st), "paged_attention");
    if (scratch.tables) cudaFree(scratch.tables);
    scratch.tables = nullptr;
    scratch.tables_cap = 0;
    cuda_check(cudaMalloc(&scratch.tables, need_tables * sizeof(int32_t)), "paged_attention");
    scratch.tables_cap = need_tables;
  }
  std::vector<int32_t> h(need_tables, 0);
  h[0] = 0;
  h[1] = q_len;
  h[2] = kv_len;
  std::copy(blocks.block_table.begin(), blocks.block_table.end(), h.begin() + 3);
  cuda_check(cudaMemcpyAsync(scratch.tables, h.data(), h.size() * sizeof(int32_t),
                             cudaMemcpyHostToDevice, st),
             "paged_attention");
  const size_t ws = fa_paged_attention_workspace_size(1, num_heads, blocks.layer.num_kv_heads,
                                                      blocks.layer.head_dim, kv_len, q_len);
  if (ws > scratch.workspace_bytes) {
    cuda_check(cudaStreamSynchronize(st), "paged_attention");
    if (scratch.workspace) cudaFree(scratch.workspace);
    scratch.workspace = nullptr;
    scratch.workspace_bytes = 0;
    cuda_check(cudaMalloc(&scratch.workspace, ws), "paged_attention");
    cuda_check(cudaMemset(scratch.workspace, 0, ws), "paged_attention");
    scratch.workspace_bytes = ws;
  }
  check(fa_paged_attention(&blocks.layer, q.data, out.data, scratch.tables, scratch.tables + 2,
                           scratch.tables + 3, nb, 1, num_heads, n_rep, q_len, q_len, kv_len,
                           float(scale), score_flow, scratch.workspace, scratch.workspace_bytes,
                           stream),
        "paged_attention");
}

// ---- build_batch (new) -------------------------------------------------------------------------------

BatchMetadata build_batch(const std::vector<const BlockTable *> &tables,
                                 const std::vector<size_t> &q_lens) {
  if (tables.size() != q_lens.size()) throw Error("build_batch: tables and q_lens differ in length");
  BatchMetadata m;
  m.num_seqs = int32_t(tables.size());
  size_t max_blocks = 1;
  for (const BlockTable *t : tables) max_blocks = std::max(max_blocks, t->blocks().size());
  m.max_blocks_per_seq = int32_t(max_blocks);
  m.block_tables.assign(tables.size() * max_blocks, 0);
  m.cu_seqlens_q.push_back(0);
  for (size_t i = 0; i < tables.size(); ++i) {
    const BlockTable &t = *tables[i];
    if (q_lens[i] > t.len()) throw Error("build_batch: q_len exceeds the sequence length");
    for (size_t j = 0; j < t.blocks().size(); ++j)
      m.block_tables[i * max_blocks + j] = int32_t(t.blocks()[j]);
    m.context_lens.push_back(int32_t(t.len()));
    m.max_context_len = std::max(m.max_context_len, int32_t(t.len()));
    m.max_seqlen_q = std::max(m.max_seqlen_q, int32_t(q_lens[i]));
    for (uint32_t s : t.slots(t.len() - q_lens[i], t.len())) m.slot_mapping.push_back(int32_t(s));
    m.cu_seqlens_q.push_back(m.cu_seqlens_q.back() + int32_t(q_lens[i]));
  }
  m.total_q = m.cu_seqlens_q.back();
  return m;
}

}  // namespace flour
