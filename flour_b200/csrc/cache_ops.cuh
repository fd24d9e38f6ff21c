// Block writes (reshape_and_cache) and whole-block copies (copy_blocks) on the HBM pool
// [num_blocks, kv_heads, block_size, head_dim]. Both are pure data movement: HBM-bound, no
// arithmetic, bit-exact by construction. Vector width is chosen on the host from the
// alignment of every base address and stride (16 B when possible).
#pragma once

#include "fa_common.cuh"

namespace fa {

template <int V> struct VecT;
template <> struct VecT<16> { using type = uint4; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<2> { using type = uint16_t; };

struct ReshapeParams {
  const char *key;
  const char *value;
  char *k_cache;
  char *v_cache;
  const int32_t *slot_mapping;
  int64_t key_stride_token;    // bytes
  int64_t key_stride_head;     // bytes
  int64_t value_stride_token;  // bytes
  int64_t value_stride_head;   // bytes
  int64_t num_slots;
  int32_t num_tokens;
  int32_t num_kv_heads;
  int32_t block_size;
  int32_t row_bytes;           // head_dim * element size
};

// One work item = one V-byte vector of one (token, kv_head) row; grid-stride loop.
// Restates PagedKvPool::write (src/models/common/paged.rs:186-204) as a per-slot scatter:
// token t, head h goes to (slot / bs, h, slot % bs) of the build layout.
template <int V>
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(const ReshapeParams p) {
  using VT = typename VecT<V>::type;
  // Programmatic dependent launch: the next kernel (the attention that reads these slots) may
  // be launched while this one runs; this one touches memory only after its predecessor is done.
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  const int nvec = p.row_bytes / V;
  const int64_t total = int64_t(p.num_tokens) * p.num_kv_heads * nvec;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int v = int(idx % nvec);
    const int64_t th = idx / nvec;
    const int h = int(th % p.num_kv_heads);
    const int64_t t = th / p.num_kv_heads;
    const int64_t slot = p.slot_mapping[t];
    if (slot < 0 || slot >= p.num_slots) {
      if (slot != -1 && h == 0 && v == 0) report(FA_DEVERR_SLOT);
      continue;
    }
    const int64_t blk = slot / p.block_size, off = slot % p.block_size;
    const int64_t dst = ((blk * p.num_kv_heads + h) * p.block_size + off) * p.row_bytes + int64_t(v) * V;
    const VT kv = *reinterpret_cast<const VT *>(p.key + t * p.key_stride_token +
                                                h * p.key_stride_head + int64_t(v) * V);
    const VT vv = *reinterpret_cast<const VT *>(p.value + t * p.value_stride_token +
                                                h * p.value_stride_head + int64_t(v) * V);
    *reinterpret_cast<VT *>(p.k_cache + dst) = kv;
    *reinterpret_cast<VT *>(p.v_cache + dst) = vv;
  }
}

struct CopyParams {
  char *k[FA_MAX_COPY_LAYERS];
  char *v[FA_MAX_COPY_LAYERS];
  const int32_t *pairs;  // [num_pairs][2] (src, dst)
  int64_t block_bytes;
  int32_t num_pairs;
  int32_t num_blocks;
};

// grid = (num_pairs, num_layers, 2 [K,V]). Each CTA copies one whole block (contiguous
// block_bytes) with V-byte vectors, 4 loads in flight per thread before the stores.
template <int V>
__global__ void __launch_bounds__(256) copy_blocks_kernel(const CopyParams p) {
  using VT = typename VecT<V>::type;
  const int pair = blockIdx.x, layer = blockIdx.y;
  const int32_t src = p.pairs[2 * pair], dst = p.pairs[2 * pair + 1];
  if (uint32_t(src) >= uint32_t(p.num_blocks) || uint32_t(dst) >= uint32_t(p.num_blocks)) {
    if (threadIdx.x == 0 && layer == 0 && blockIdx.z == 0) report(FA_DEVERR_PAIR);
    return;
  }
  char *base = blockIdx.z == 0 ? p.k[layer] : p.v[layer];
  const VT *s = reinterpret_cast<const VT *>(base + int64_t(src) * p.block_bytes);
  VT *d = reinterpret_cast<VT *>(base + int64_t(dst) * p.block_bytes);
  const int64_t n = p.block_bytes / V;
  constexpr int U = 4;
  int64_t i = threadIdx.x;
  for (; i + (U - 1) * blockDim.x < n; i += U * blockDim.x) {
    VT r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) r[u] = s[i + u * blockDim.x];
#pragma unroll
    for (int u = 0; u < U; ++u) d[i + u * blockDim.x] = r[u];
  }
  for (; i < n; i += blockDim.x) d[i] = s[i];
}

struct BundleParams {
  char *k[FA_MAX_COPY_LAYERS];
  char *v[FA_MAX_COPY_LAYERS];
  const int32_t *block_ids;  // [num_logical]: physical block of each logical block, in order
  char *payload;             // [num_logical][num_layers][2 (K, V)][block_bytes]
  int64_t block_bytes;
  int32_t num_logical;
  int32_t num_layers;
  int32_t num_blocks;        // pool size, for the block-id check
};

// FLKV bundle payload (src/kv_cache/bundle.rs:15-22): for each logical block, for each layer,
// the K then the V of that block, shape (kv_heads, block_size, head_dim). In the pool layout
// [num_blocks, kv_heads, block_size, head_dim] each piece is one contiguous run of block_bytes,
// so the payload is a gather of whole runs (export) or the mirror scatter (import).
// grid = (2 * num_layers, num_logical): CTA (x, b) moves piece (b, x / 2, x % 2), 4 vectors in
// flight per thread. Export of a bad block id zero-fills its pieces; import skips them; both
// set FA_DEVERR_BLOCK_ID.
template <int V, bool kImport>
__global__ void __launch_bounds__(256) bundle_payload_kernel(const BundleParams p) {
  using VT = typename VecT<V>::type;
  const int l = blockIdx.x >> 1, kv = blockIdx.x & 1, b = blockIdx.y;
  const int32_t id = p.block_ids[b];
  const bool bad = uint32_t(id) >= uint32_t(p.num_blocks);
  if (bad && threadIdx.x == 0 && blockIdx.x == 0) report(FA_DEVERR_BLOCK_ID);
  VT *piece = reinterpret_cast<VT *>(p.payload + ((int64_t(b) * p.num_layers + l) * 2 + kv) *
                                                     p.block_bytes);
  VT *pool = reinterpret_cast<VT *>((kv ? p.v[l] : p.k[l]) + int64_t(bad ? 0 : id) * p.block_bytes);
  const int64_t n = p.block_bytes / V;
  if (bad) {
    if (!kImport)
      for (int64_t i = threadIdx.x; i < n; i += blockDim.x) piece[i] = VT{};
    return;
  }
  const VT *src = kImport ? piece : pool;
  VT *dst = kImport ? pool : piece;
  constexpr int U = 4;
  int64_t i = threadIdx.x;
  for (; i + (U - 1) * blockDim.x < n; i += U * blockDim.x) {
    VT r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) r[u] = src[i + u * blockDim.x];
#pragma unroll
    for (int u = 0; u < U; ++u) dst[i + u * blockDim.x] = r[u];
  }
  for (; i < n; i += blockDim.x) dst[i] = src[i];
}

}  // namespace fa
