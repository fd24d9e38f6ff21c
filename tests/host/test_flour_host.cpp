// Tests of the C++ host side (flour_b200/host/flour_host.h), written after the reference's own
// unit tests so they read alike:
//   src/models/common/paged.rs:288-410, src/models/common/prefix.rs (tests),
//   src/models/common/cache.rs:536-910.
// Host-only cases always run; with --gpu the pool / attention cases run on device 0 and check
// the paged attention result against the C++ oracle (oracle/ref_paged_attention.cpp).
//
//   test_flour_host [--gpu]      exit status 0 when every case passes
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "flour_host.h"

extern "C" int32_t oracle_paged_attention(int32_t dt, int32_t score_mode, const void *q, void *out,
                                          const void *k_cache, const void *v_cache,
                                          int32_t num_blocks, int32_t kv_heads, int32_t block_size,
                                          int32_t head_dim, int32_t num_heads, int32_t n_rep,
                                          const int32_t *cu_seqlens_q, const int32_t *context_lens,
                                          const int32_t *block_tables, int32_t max_blocks,
                                          int32_t num_seqs, float scale, int32_t num_threads);

using namespace flour;

namespace {

int g_failed = 0, g_run = 0;

struct Failure {
  std::string msg;
};

#define EXPECT(cond)                                                                          \
  do {                                                                                        \
    if (!(cond)) throw Failure{std::string(__FILE__ ":") + std::to_string(__LINE__) + ": " #cond}; \
  } while (0)

template <class F>
void expect_error(F &&f, const std::string &needle) {
  try {
    f();
  } catch (const Error &e) {
    if (std::string(e.what()).find(needle) == std::string::npos)
      throw Failure{std::string("error text '") + e.what() + "' lacks '" + needle + "'"};
    return;
  }
  throw Failure{"expected an error containing '" + needle + "'"};
}

void run(const char *name, const std::function<void()> &f) {
  ++g_run;
  try {
    f();
    std::printf("ok   %s\n", name);
  } catch (const Failure &e) {
    ++g_failed;
    std::printf("FAIL %s: %s\n", name, e.msg.c_str());
  } catch (const std::exception &e) {
    ++g_failed;
    std::printf("FAIL %s: exception %s\n", name, e.what());
  }
}

// The reference's test configs: cache.rs:516-534 (max_seq_len 16 -> 1 block) and prefix_config
// (cache.rs:639-645, max_seq_len 64 -> 4 blocks); kv_heads 2, head_dim 4, 2 layers.
Config test_config(size_t max_seq_len = 16) {
  return Config{2, 2, 2, 4, 10000.0, max_seq_len};
}

// f32 device tensor (1, kv_heads, n, d) filled from a host vector.
struct DevBuf {
  DeviceTensor t;
  explicit DevBuf(const std::vector<float> &h, std::vector<int64_t> shape) {
    t.dtype = DType::F32;
    t.shape = std::move(shape);
    t.data = device_alloc(h.size() * 4);
    copy_to_device(t.data, h.data(), h.size() * 4);
  }
  ~DevBuf() { device_free(t.data); }
};

std::vector<float> iota(size_t n, float start) {
  std::vector<float> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = start + float(i);
  return v;
}

// ---- paged.rs --------------------------------------------------------------------------------

void allocator_hands_out_distinct_blocks_then_exhausts() {  // paged.rs:343-354
  BlockAllocator alloc(2);
  EXPECT(alloc.num_free() == 2);
  const size_t a = *alloc.allocate(), b = *alloc.allocate();
  EXPECT(a != b);
  EXPECT(!alloc.allocate());
  EXPECT(alloc.decref(a));
  EXPECT(alloc.num_free() == 1);
  EXPECT(alloc.allocate() == std::optional<size_t>(a));
}

void allocator_refcounts_govern_when_a_block_is_freed() {  // paged.rs:356-375
  BlockAllocator alloc(2);
  EXPECT(alloc.num_free() == 2);
  const size_t a = *alloc.allocate();
  EXPECT(alloc.ref_count(a) == 1);
  alloc.incref(a);
  EXPECT(alloc.ref_count(a) == 2);
  EXPECT(!alloc.decref(a));
  EXPECT(alloc.num_free() == 1);
  EXPECT(alloc.decref(a));
  EXPECT(alloc.ref_count(a) == 0);
  EXPECT(alloc.num_free() == 2);
  EXPECT(alloc.allocate() == std::optional<size_t>(a));
  // the reference debug-asserts here; this build reports it
  BlockAllocator one(1);
  expect_error([&] { one.decref(0); }, "decref of unreferenced block");
}

void block_table_maps_logical_positions_to_physical_slots() {  // paged.rs:378-394
  BlockTable table(2);
  EXPECT(table.is_empty());
  table.push_block(5);
  table.push_block(3);
  EXPECT(table.capacity() == 4);
  EXPECT(table.slot(0) == 10 && table.slot(1) == 11 && table.slot(2) == 6 && table.slot(3) == 7);
  table.advance(3);
  EXPECT(table.len() == 3);
  EXPECT(table.slots(0, 3) == std::vector<uint32_t>({10, 11, 6}));
}

void block_table_exposes_blocks_and_clears() {  // paged.rs:397-410
  BlockTable table(2);
  table.push_block(5);
  table.push_block(3);
  table.advance(4);
  EXPECT(table.blocks() == std::vector<size_t>({5, 3}));
  EXPECT(table.block_at(0) == 5 && table.block_at(1) == 3);
  table.clear();
  EXPECT(table.is_empty() && table.len() == 0 && table.blocks().empty());
  EXPECT(table.block_size() == 2);
}

void write_block_rejects_mismatched_kv_heads() {  // paged.rs:334-340
  PagedKvPool pool(1, 2, 1, 2, DType::F32, 2, /*with_device=*/false);
  DeviceTensor k{nullptr, DType::F32, {1, 2, 2, 2}};  // kv_heads = 2, the pool has 1
  expect_error([&] { pool.write_block(0, 0, k, k); }, "write_block expects (.., kv_heads=1");
  DeviceTensor k5{nullptr, DType::F32, {1, 1, 1, 2, 2}};
  expect_error([&] { pool.write_block(0, 0, k5, k5); }, "write_block expects rank 3 or 4 tensor, got rank 5");
  DeviceTensor a{nullptr, DType::F32, {1, 2, 2}}, b{nullptr, DType::F32, {1, 1, 2}};
  expect_error([&] { pool.write_block(0, 0, a, b); }, "write_block k/v shape mismatch");
}

// ---- prefix.rs -------------------------------------------------------------------------------

void block_hash_is_deterministic_and_parent_sensitive() {
  const uint32_t toks[] = {1, 2, 3}, other[] = {1, 2, 4};
  EXPECT(block_hash(PREFIX_HASH_SEED, toks, 3) == block_hash(PREFIX_HASH_SEED, toks, 3));
  EXPECT(block_hash(PREFIX_HASH_SEED, toks, 3) != block_hash(42, toks, 3));
  EXPECT(block_hash(PREFIX_HASH_SEED, toks, 3) != block_hash(PREFIX_HASH_SEED, other, 3));
  EXPECT(block_hash(PREFIX_HASH_SEED, toks, 2) != block_hash(PREFIX_HASH_SEED, toks, 3));
}

void registry_get_verifies_tokens_against_collisions() {
  PrefixRegistry reg;
  const uint32_t t12[] = {1, 2}, t99[] = {9, 9}, t34[] = {3, 4};
  const uint64_t h = block_hash(PREFIX_HASH_SEED, t12, 2);
  reg.insert(h, {1, 2}, 7);
  EXPECT(reg.get(h, t12, 2) == std::optional<size_t>(7));
  EXPECT(reg.contains(h));
  EXPECT(!reg.get(h, t99, 2));  // same hash, other tokens: a miss, not a wrong reuse
  EXPECT(!reg.get(block_hash(PREFIX_HASH_SEED, t34, 2), t34, 2));
  reg.clear();
  EXPECT(!reg.contains(h));
}

// ---- cache.rs --------------------------------------------------------------------------------

void rope_tables_have_expected_shape() {
  Cache c(test_config(), DType::F32, false);
  EXPECT(c.cos_host().size() == 16 * 2 && c.sin_host().size() == 16 * 2);
}

void rope_tables_respect_index_pos_offset() {
  Cache c(test_config(), DType::F32, false);
  const size_t half = 2;
  // position p row: cos(p * theta_i); theta_0 = 1
  EXPECT(std::fabs(c.cos_host()[3 * half + 0] - std::cos(3.0f)) < 1e-6f);
  EXPECT(c.cos_host()[0] == 1.0f && c.sin_host()[0] == 0.0f);
  const float theta1 = 1.0f / std::pow(10000.0f, 2.0f / 4.0f);
  EXPECT(std::fabs(c.sin_host()[5 * half + 1] - std::sin(5.0f * theta1)) < 1e-6f);
}

void allocate_kv_overflow_past_max_seq_len_errors() {
  Cache c(test_config(), DType::F32, false);
  c.allocate_kv(10);
  expect_error([&] { c.allocate_kv(7); }, "paged kv cache overflow: 17 tokens exceeds max_seq_len 16");
}

std::vector<uint32_t> ids(size_t n) {
  std::vector<uint32_t> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = uint32_t(i);
  return v;
}

void match_prefix_is_empty_before_anything_is_registered() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(40)) == 0);
}

void register_then_match_reuses_full_blocks_and_leaves_a_suffix() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(40)) == 0);
  c.allocate_kv(40);
  c.register_prefix(ids(40));
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(40)) == 32);
}

void match_prefix_leaves_last_block_when_prompt_is_block_aligned() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  c.match_prefix(ids(32));
  c.allocate_kv(32);
  c.register_prefix(ids(32));
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(32)) == 16);
}

void reset_sequence_frees_unregistered_blocks_but_keeps_registered_ones() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  c.match_prefix(ids(40));
  c.allocate_kv(40);
  c.register_prefix(ids(40));
  const size_t free_after_first = c.free_blocks();
  c.reset_sequence();
  EXPECT(c.free_blocks() == free_after_first + 1);
}

void clear_prefix_cache_disables_reuse() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  c.match_prefix(ids(40));
  c.allocate_kv(40);
  c.register_prefix(ids(40));
  c.clear_prefix_cache();
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(40)) == 0);
}

void clear_prefix_cache_releases_registry_only_blocks_to_the_pool() {
  Cache c(test_config(64), DType::F32, false);
  c.reset_sequence();
  c.match_prefix(ids(40));
  c.allocate_kv(40);
  c.register_prefix(ids(40));
  c.reset_sequence();
  const size_t free_before = c.free_blocks();
  c.clear_prefix_cache();
  EXPECT(c.free_blocks() == free_before + 2);
  c.reset_sequence();
  EXPECT(c.match_prefix(ids(40)) == 0);
}

void build_batch_packs_tables_lengths_and_slots() {
  BlockTable a(16), b(16);
  a.push_block(3);
  a.push_block(7);
  a.advance(20);  // 20 tokens, the last 4 new
  b.push_block(1);
  b.advance(5);   // 5 tokens, all new
  const BatchMetadata m = build_batch({&a, &b}, {4, 5});
  EXPECT(m.num_seqs == 2 && m.max_blocks_per_seq == 2 && m.total_q == 9);
  EXPECT(m.block_tables == std::vector<int32_t>({3, 7, 1, 0}));
  EXPECT(m.context_lens == std::vector<int32_t>({20, 5}));
  EXPECT(m.cu_seqlens_q == std::vector<int32_t>({0, 4, 9}));
  EXPECT(m.slot_mapping == std::vector<int32_t>({7 * 16 + 0, 7 * 16 + 1, 7 * 16 + 2, 7 * 16 + 3,
                                                 16, 17, 18, 19, 20}));
  EXPECT(m.max_context_len == 20 && m.max_seqlen_q == 5);
  expect_error([&] { build_batch({&b}, {6}); }, "q_len exceeds the sequence length");
}

void build_batch_edge_cases() {
  const BatchMetadata e = build_batch({}, {});
  EXPECT(e.num_seqs == 0 && e.max_blocks_per_seq == 1 && e.total_q == 0);
  EXPECT(e.block_tables.empty() && e.context_lens.empty() && e.slot_mapping.empty());
  EXPECT(e.cu_seqlens_q == std::vector<int32_t>({0}));
  EXPECT(e.max_context_len == 0 && e.max_seqlen_q == 0);
  BlockTable a(16), b(16);
  a.push_block(3);
  a.advance(10);
  b.push_block(5);
  b.push_block(6);
  b.advance(17);
  const BatchMetadata m = build_batch({&a, &b}, {0, 2});  // a sequence with no new tokens
  EXPECT(m.cu_seqlens_q == std::vector<int32_t>({0, 0, 2}) && m.total_q == 2);
  EXPECT(m.slot_mapping == std::vector<int32_t>({5 * 16 + 15, 6 * 16 + 0}));
  EXPECT(m.block_tables == std::vector<int32_t>({3, 0, 5, 6}) && m.max_seqlen_q == 2);
  expect_error([&] { build_batch({&a, &b}, {1}); }, "tables and q_lens differ in length");
}

// ---- GPU cases -------------------------------------------------------------------------------

void paged_pool_write_then_gather_round_trips() {  // paged.rs:288-306
  // 1 layer, 4 slots (2 blocks of 2), 1 kv head, head_dim 2
  PagedKvPool pool(1, 2, 1, 2, DType::F32, 2);
  DevBuf k({1, 2, 3, 4}, {1, 1, 2, 2}), v({5, 6, 7, 8}, {1, 1, 2, 2});
  pool.write(0, {2, 0}, k.t, v.t);  // deliberately out of order
  device_synchronize();
  std::vector<float> gk(4), gv(4);
  pool.gather(0, {0, 2}, gk.data(), gv.data());
  EXPECT(gk == std::vector<float>({3, 4, 1, 2}));
  EXPECT(gv == std::vector<float>({7, 8, 5, 6}));
}

void paged_pool_write_block_round_trips_full_block() {  // paged.rs:309-331
  PagedKvPool pool(1, 2, 1, 2, DType::F32, 2);
  DevBuf k({1, 2, 3, 4}, {1, 1, 2, 2}), v({5, 6, 7, 8}, {1, 1, 2, 2});
  pool.write_block(0, 1, k.t, v.t);
  device_synchronize();
  const BlockView rv = pool.block_view(0, 2, 2);
  std::vector<float> rk(4), rvv(4);
  copy_to_host(rk.data(), rv.k, 16);
  copy_to_host(rvv.data(), rv.v, 16);
  EXPECT(rk == std::vector<float>({1, 2, 3, 4}));
  EXPECT(rvv == std::vector<float>({5, 6, 7, 8}));
  const BlockView zv = pool.block_view(0, 0, 2);
  std::vector<float> zk(4);
  copy_to_host(zk.data(), zv.k, 16);
  EXPECT(zk == std::vector<float>({0, 0, 0, 0}));
  expect_error([&] { pool.block_view(0, 1, 2); }, "more than one physical block");
}

void write_kv_then_blocks_spans_appended_batches_and_attention_matches_oracle() {
  // One sequence, 2 layers, appended in two batches (prefill 20 tokens, then 3), then the
  // attention of the last 3 queries over all 23 tokens against the oracle.
  Config cfg{2, 8, 2, 64, 10000.0, 64};
  Cache cache(cfg, DType::F32);
  std::mt19937 rng(7);
  std::normal_distribution<float> nd(0.f, 1.f);
  auto randv = [&](size_t n) {
    std::vector<float> v(n);
    for (auto &x : v) x = nd(rng) * 0.25f;
    return v;
  };
  for (size_t n : {20u, 3u}) {
    cache.allocate_kv(n);
    for (size_t l = 0; l < 2; ++l) {
      DevBuf k(randv(2 * n * 64), {1, 2, int64_t(n), 64}), v(randv(2 * n * 64), {1, 2, int64_t(n), 64});
      cache.write_kv(l, k.t, v.t);
      device_synchronize();
    }
  }
  const SequenceBlocks sb = cache.kv_blocks(1);
  EXPECT(sb.kv_len == 23 && sb.block_table.size() == 2);
  EXPECT(sb.block_table[0] == 0 && sb.block_table[1] == 1);
  // queries: last 3 positions, 8 heads, token-major
  const auto qh = randv(3 * 8 * 64);
  DevBuf q(qh, {3, 8, 64});
  std::vector<float> zeros(3 * 8 * 64, 0.f);
  DevBuf out(zeros, {3, 8, 64});
  AttentionScratch scratch;
  paged_attention(q.t, sb, 4, 1.0 / 8.0, out.t, scratch);
  device_synchronize();
  std::vector<float> got(3 * 8 * 64);
  copy_to_host(got.data(), out.t.data, got.size() * 4);
  // oracle on a host copy of the layer's pool
  const fa_kv_layer L = sb.layer;
  const size_t pool_elems = size_t(L.num_blocks) * L.num_kv_heads * L.block_size * L.head_dim;
  std::vector<float> kh(pool_elems), vh(pool_elems);
  copy_to_host(kh.data(), L.k_cache, pool_elems * 4);
  copy_to_host(vh.data(), L.v_cache, pool_elems * 4);
  std::vector<float> want(got.size());
  const int32_t cu[2] = {0, 3}, ctx[1] = {23};
  const int32_t bt[2] = {sb.block_table[0], sb.block_table[1]};
  const int32_t rc = oracle_paged_attention(FA_F32, 0, qh.data(), want.data(), kh.data(), vh.data(),
                                            L.num_blocks, 2, 16, 64, 8, 4, cu, ctx, bt, 2, 1,
                                            1.0f / 8.0f, 1);
  EXPECT(rc == 0);
  double worst = 0;
  for (size_t i = 0; i < got.size(); ++i) worst = std::max(worst, double(std::fabs(got[i] - want[i])));
  EXPECT(worst <= 1e-5);
}

void kv_blocks_round_trips_written_values() {
  Cache cache(test_config(), DType::F32);
  cache.allocate_kv(5);
  const auto k = iota(2 * 5 * 4, 1.0f), v = iota(2 * 5 * 4, -50.0f);
  DevBuf kd(k, {1, 2, 5, 4}), vd(v, {1, 2, 5, 4});
  cache.write_kv(0, kd.t, vd.t);
  device_synchronize();
  std::vector<float> gk(40), gv(40);
  cache.kvs().pool().gather(0, cache.kvs().slots(0, 5), gk.data(), gv.data());
  EXPECT(gk == k && gv == v);
  expect_error([&] { cache.allocate_kv(12); }, "paged kv cache overflow");
}

}  // namespace

int main(int argc, char **argv) {
  const bool gpu = argc > 1 && std::strcmp(argv[1], "--gpu") == 0;
  run("allocator_hands_out_distinct_blocks_then_exhausts", allocator_hands_out_distinct_blocks_then_exhausts);
  run("allocator_refcounts_govern_when_a_block_is_freed", allocator_refcounts_govern_when_a_block_is_freed);
  run("block_table_maps_logical_positions_to_physical_slots", block_table_maps_logical_positions_to_physical_slots);
  run("block_table_exposes_blocks_and_clears", block_table_exposes_blocks_and_clears);
  run("write_block_rejects_mismatched_kv_heads", write_block_rejects_mismatched_kv_heads);
  run("block_hash_is_deterministic_and_parent_sensitive", block_hash_is_deterministic_and_parent_sensitive);
  run("registry_get_verifies_tokens_against_collisions", registry_get_verifies_tokens_against_collisions);
  run("rope_tables_have_expected_shape", rope_tables_have_expected_shape);
  run("rope_tables_respect_index_pos_offset", rope_tables_respect_index_pos_offset);
  run("allocate_kv_overflow_past_max_seq_len_errors", allocate_kv_overflow_past_max_seq_len_errors);
  run("match_prefix_is_empty_before_anything_is_registered", match_prefix_is_empty_before_anything_is_registered);
  run("register_then_match_reuses_full_blocks_and_leaves_a_suffix", register_then_match_reuses_full_blocks_and_leaves_a_suffix);
  run("match_prefix_leaves_last_block_when_prompt_is_block_aligned", match_prefix_leaves_last_block_when_prompt_is_block_aligned);
  run("reset_sequence_frees_unregistered_blocks_but_keeps_registered_ones", reset_sequence_frees_unregistered_blocks_but_keeps_registered_ones);
  run("clear_prefix_cache_disables_reuse", clear_prefix_cache_disables_reuse);
  run("clear_prefix_cache_releases_registry_only_blocks_to_the_pool", clear_prefix_cache_releases_registry_only_blocks_to_the_pool);
  run("build_batch_packs_tables_lengths_and_slots", build_batch_packs_tables_lengths_and_slots);
  run("build_batch_edge_cases", build_batch_edge_cases);
  if (gpu) {
    if (device_count() < 1) {
      std::printf("FAIL no CUDA device for --gpu\n");
      return 1;
    }
    run("paged_pool_write_then_gather_round_trips", paged_pool_write_then_gather_round_trips);
    run("paged_pool_write_block_round_trips_full_block", paged_pool_write_block_round_trips_full_block);
    run("write_kv_then_blocks_spans_appended_batches_and_attention_matches_oracle",
        write_kv_then_blocks_spans_appended_batches_and_attention_matches_oracle);
    run("kv_blocks_round_trips_written_values", kv_blocks_round_trips_written_values);
  }
  std::printf("%d run, %d failed\n", g_run, g_failed);
  return g_failed ? 1 : 0;
}
