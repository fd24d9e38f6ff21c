// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
//
// CPU restatement of the FLKV bundle payload order used by remote prefix-cache export/import:
//   KvCache::export_prefix_bundle   src/models/common/cache.rs:166-228
//   KvBundleCodec::encode/decode    src/kv_cache/bundle.rs:108-214 (payload order :15-22)
//
//   for block in 0..num_blocks:            (logical order of the sequence's block table)
//     for layer in 0..num_layers:
//       K block bytes, shape (num_kv_heads, block_size, head_dim)
//       V block bytes, shape (num_kv_heads, block_size, head_dim)
//
// With the build layout [num_blocks, kv_heads, block_size, head_dim] each (layer, block) K or V
// piece is one contiguous run of block_bytes, so the payload is a gather of whole blocks.

#include <cstdint>
#include <cstring>

extern "C" {

// Export: payload of `n_logical` logical blocks whose physical ids are block_ids[0..n_logical).
// Returns the number of bytes written (n_logical * num_layers * 2 * block_bytes).
int64_t oracle_bundle_export(void *const *k_caches, void *const *v_caches, int32_t num_layers,
                             int64_t block_bytes, const int32_t *block_ids, int32_t n_logical,
                             void *payload) {
  char *out = static_cast<char *>(payload);
  for (int32_t b = 0; b < n_logical; ++b) {
    const int64_t off = int64_t(block_ids[b]) * block_bytes;
    for (int32_t l = 0; l < num_layers; ++l) {
      std::memcpy(out, static_cast<const char *>(k_caches[l]) + off, block_bytes);
      out += block_bytes;
      std::memcpy(out, static_cast<const char *>(v_caches[l]) + off, block_bytes);
      out += block_bytes;
    }
  }
  return int64_t(out - static_cast<char *>(payload));
}

// Import: the inverse, writing logical block b of the payload into physical block block_ids[b]
// (KvCache::import_prefix_bundle's write_block loop, cache.rs:304-321).
void oracle_bundle_import(void *const *k_caches, void *const *v_caches, int32_t num_layers,
                          int64_t block_bytes, const int32_t *block_ids, int32_t n_logical,
                          const void *payload) {
  const char *in = static_cast<const char *>(payload);
  for (int32_t b = 0; b < n_logical; ++b) {
    const int64_t off = int64_t(block_ids[b]) * block_bytes;
    for (int32_t l = 0; l < num_layers; ++l) {
      std::memcpy(static_cast<char *>(k_caches[l]) + off, in, block_bytes);
      in += block_bytes;
      std::memcpy(static_cast<char *>(v_caches[l]) + off, in, block_bytes);
      in += block_bytes;
    }
  }
}

}  // extern "C"
