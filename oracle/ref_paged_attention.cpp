// TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
//
// CPU restatement of the reference hot path (lltsdyp/flour, Rust, candle-core 0.9.2 CPU):
//   - backend::cpu::paged_attention     src/backend/cpu.rs:57-112  (block-streaming online softmax)
//   - backend::cpu::causal_attention    src/backend/cpu.rs:24-42   (dense SDPA, test reference)
//   - backend::cpu::repeat_kv           src/backend/cpu.rs:5-13    (query head h -> kv head h/n_rep)
//   - BlockTable::slot / slots          src/models/common/paged.rs:114-121
//   - PagedKvPool::write                src/models/common/paged.rs:186-204
//   - PagedKvPool::write_block/block_view src/models/common/paged.rs:211-240, 266-279
//   - KvCache::gather_blocks            src/models/common/cache.rs:83-96   (logical block walk)
//
// Only tests, the smoke check and bench.py's CPU-baseline / reference arm load this library, and
// only as the checker or the timed CPU baseline. The CUDA product never calls it.
//
// The reference cannot be built in this environment (Rust, no cargo), so this restatement is
// pinned against the reference's own known-answer and integer golden tests (ported in
// tests/test_oracle.py) and against an independent float64 dense restatement of
// cpu.rs:24-42 (tests/golden/).
//
// Pool layout here is the build's [num_blocks, kv_heads, block_size, head_dim]; the literal
// PagedKvPool::write restatement below works on the reference layout (kv_heads, num_slots, d).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

enum { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };
// Device-status bit values shared with include/flour_attn.h.
enum { ERR_BLOCK_ID = 0x1, ERR_CONTEXT = 0x2, ERR_SLOT = 0x4, ERR_SEQLEN = 0x10, ERR_PAIR = 0x20 };

inline float bf16_to_f32(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// Round-to-nearest-even, the rounding `half::bf16::from_f32` performs.
inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

inline float f16_to_f32(uint16_t h) {
  _Float16 x;
  std::memcpy(&x, &h, 2);
  return float(x);
}

inline uint16_t f32_to_f16(float f) {
  _Float16 x = _Float16(f);  // IEEE round-to-nearest-even
  uint16_t h;
  std::memcpy(&h, &x, 2);
  return h;
}

inline size_t dt_size(int dt) { return dt == DT_F32 ? 4 : 2; }

inline float load(const void *p, size_t i, int dt) {
  switch (dt) {
    case DT_F32: return static_cast<const float *>(p)[i];
    case DT_BF16: return bf16_to_f32(static_cast<const uint16_t *>(p)[i]);
    default: return f16_to_f32(static_cast<const uint16_t *>(p)[i]);
  }
}

inline void store(void *p, size_t i, int dt, float v) {
  switch (dt) {
    case DT_F32: static_cast<float *>(p)[i] = v; break;
    case DT_BF16: static_cast<uint16_t *>(p)[i] = f32_to_bf16(v); break;
    default: static_cast<uint16_t *>(p)[i] = f32_to_f16(v); break;
  }
}

// Round a float to the model dtype and back (identity for f32).
inline float round_dt(float v, int dt) {
  switch (dt) {
    case DT_F32: return v;
    case DT_BF16: return bf16_to_f32(f32_to_bf16(v));
    default: return f16_to_f32(f32_to_f16(v));
  }
}

}  // namespace

extern "C" {

int32_t oracle_abi_version(void) { return 1; }

// BlockTable::slot (paged.rs:114-116): blocks[pos / bs] * bs + pos % bs.
int64_t oracle_slot(const int32_t *blocks, int32_t block_size, int64_t pos) {
  return int64_t(blocks[pos / block_size]) * block_size + pos % block_size;
}

// BlockTable::slots (paged.rs:119-121): slots for logical positions start..end as u32.
void oracle_slots(const int32_t *blocks, int32_t block_size, int64_t start, int64_t end,
                  uint32_t *out) {
  for (int64_t p = start; p < end; ++p) out[p - start] = uint32_t(oracle_slot(blocks, block_size, p));
}

// Literal restatement of PagedKvPool::write (paged.rs:186-204) on the reference layout
// pool (kv_heads, num_slots, head_dim) and k/v (kv_heads, n, head_dim), including its
// run-coalescing loop exactly as written at paged.rs:192-201:
//     while i + n < slots.len() && i + n == start_slot + n { n += 1 }
// (the condition reduces to i == start_slot). Each run copies n consecutive source rows to n
// consecutive slots starting at start_slot, as slice_set does.
// Returns ERR_SLOT (and writes nothing for that run) when a run would leave the pool, the
// case where candle's slice_set returns an error.
int32_t oracle_pool_write_literal(void *k_pool, void *v_pool, int32_t kv_heads, int64_t num_slots,
                                  int32_t head_dim, int32_t elem_size, const uint32_t *slots,
                                  int64_t n_tokens, const void *k, const void *v) {
  int32_t err = 0;
  const size_t row = size_t(head_dim) * elem_size;
  int64_t i = 0;
  while (i < n_tokens) {
    int64_t n = 1;
    const int64_t start_slot = slots[i];
    while (i + n < n_tokens && i + n == start_slot + n) ++n;
    if (start_slot + n > num_slots) {
      err |= ERR_SLOT;
    } else {
      for (int32_t h = 0; h < kv_heads; ++h) {
        const size_t src = (size_t(h) * n_tokens + i) * row;
        const size_t dst = (size_t(h) * num_slots + start_slot) * row;
        std::memcpy(static_cast<char *>(k_pool) + dst, static_cast<const char *>(k) + src, n * row);
        std::memcpy(static_cast<char *>(v_pool) + dst, static_cast<const char *>(v) + src, n * row);
      }
    }
    i += n;
  }
  return err;
}

// Per-slot scatter, the documented meaning of PagedKvPool::write ("write the tokens into their
// reserved slots", cache.rs:69-77) and the contract of the reshape_and_cache kernel, on the
// build layout [num_blocks, kv_heads, block_size, head_dim]. Source row (t, h) is read at
// key[t*stride_token + h*stride_head]. slot -1 skips the token; other out-of-range slots are
// skipped and reported as ERR_SLOT.
int32_t oracle_reshape_and_cache(void *k_cache, void *v_cache, int32_t num_blocks,
                                 int32_t kv_heads, int32_t block_size, int32_t head_dim,
                                 int32_t elem_size, const void *key, const void *value,
                                 int64_t k_stride_token, int64_t k_stride_head,
                                 int64_t v_stride_token, int64_t v_stride_head,
                                 const int32_t *slot_mapping, int64_t num_tokens) {
  int32_t err = 0;
  const int64_t num_slots = int64_t(num_blocks) * block_size;
  const size_t row = size_t(head_dim) * elem_size;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot == -1) continue;
    if (slot < 0 || slot >= num_slots) {
      err |= ERR_SLOT;
      continue;
    }
    const int64_t blk = slot / block_size, off = slot % block_size;
    for (int32_t h = 0; h < kv_heads; ++h) {
      const size_t dst = ((size_t(blk) * kv_heads + h) * block_size + off) * row;
      std::memcpy(static_cast<char *>(k_cache) + dst,
                  static_cast<const char *>(key) + (t * k_stride_token + h * k_stride_head) * elem_size, row);
      std::memcpy(static_cast<char *>(v_cache) + dst,
                  static_cast<const char *>(value) + (t * v_stride_token + h * v_stride_head) * elem_size, row);
    }
  }
  return err;
}

// Whole-block copy src -> dst in every layer for K and V: block_view(src) followed by
// write_block(dst) (paged.rs:211-240, 266-279). Pairs are applied in order.
int32_t oracle_copy_blocks(void *const *k_caches, void *const *v_caches, int32_t num_layers,
                           int32_t num_blocks, int64_t block_bytes, const int32_t *pairs,
                           int32_t num_pairs) {
  int32_t err = 0;
  for (int32_t p = 0; p < num_pairs; ++p) {
    const int32_t src = pairs[2 * p], dst = pairs[2 * p + 1];
    if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
      err |= ERR_PAIR;
      continue;
    }
    for (int32_t l = 0; l < num_layers; ++l) {
      std::memmove(static_cast<char *>(k_caches[l]) + dst * block_bytes,
                   static_cast<const char *>(k_caches[l]) + src * block_bytes, block_bytes);
      std::memmove(static_cast<char *>(v_caches[l]) + dst * block_bytes,
                   static_cast<const char *>(v_caches[l]) + src * block_bytes, block_bytes);
    }
  }
  return err;
}

// backend::cpu::causal_attention (cpu.rs:24-42) for one batch element, heads already expanded
// by repeat_kv semantics (query head h reads kv head h / n_rep, cpu.rs:5-13):
//   att = (q @ k^T) * scale           in the model dtype (f32 accumulate, one rounding each)
//   att = masked_fill(att, mask, -inf)
//   att = softmax_last_dim(att as f32) as dtype
//   out = att @ v                      in the model dtype
// q (num_heads, seq_q, d), k/v (num_heads / n_rep, kv_len, d), mask (seq_q, kv_len) u8 or NULL.
int32_t oracle_causal_attention(int32_t dt, const void *q, const void *k, const void *v, void *out,
                                int32_t num_heads, int32_t n_rep, int32_t seq_q, int32_t kv_len,
                                int32_t head_dim, float scale, const uint8_t *mask) {
  if (n_rep <= 0 || num_heads % n_rep) return -1;
  const float sc = round_dt(scale, dt);
  std::vector<float> att(kv_len);
  for (int32_t h = 0; h < num_heads; ++h) {
    const int32_t kh = h / n_rep;
    for (int32_t i = 0; i < seq_q; ++i) {
      const size_t qo = (size_t(h) * seq_q + i) * head_dim;
      for (int32_t j = 0; j < kv_len; ++j) {
        const size_t ko = (size_t(kh) * kv_len + j) * head_dim;
        float dot = 0.f;
        for (int32_t x = 0; x < head_dim; ++x) dot += load(q, qo + x, dt) * load(k, ko + x, dt);
        float s = round_dt(round_dt(dot, dt) * sc, dt);
        if (mask && mask[size_t(i) * kv_len + j]) s = -std::numeric_limits<float>::infinity();
        att[j] = s;
      }
      float mx = -std::numeric_limits<float>::infinity();
      for (int32_t j = 0; j < kv_len; ++j) mx = std::max(mx, att[j]);
      float sum = 0.f;
      for (int32_t j = 0; j < kv_len; ++j) {
        att[j] = std::exp(att[j] - mx);
        sum += att[j];
      }
      for (int32_t j = 0; j < kv_len; ++j) att[j] = round_dt(att[j] / sum, dt);
      for (int32_t x = 0; x < head_dim; ++x) {
        float acc = 0.f;
        for (int32_t j = 0; j < kv_len; ++j)
          acc += att[j] * load(v, (size_t(kh) * kv_len + j) * head_dim + x, dt);
        store(out, qo + x, dt, acc);
      }
    }
  }
  return 0;
}

// backend::cpu::paged_attention (cpu.rs:57-112) over a batch of sequences, each given the way
// KvCache::gather_blocks (cache.rs:83-96) hands blocks to it: logical block b of sequence s
// covers KV positions [b*bs, min((b+1)*bs, L)) and lives in physical block
// block_tables[s*max_blocks + b] of the build-layout pool.
//
// Per (sequence, head, query row) the fold follows cpu.rs:70-107 in order, in f32:
//   scores = (q . k) * scale, cast to f32                       cpu.rs:84-85
//   scores[j] = -inf where kv_start + j > offset + i            cpu.rs:87-94, offset = L - q_len
//   block_max = max_j scores; new_max = max(running_max, block_max)         cpu.rs:96-97
//   correction = exp(running_max - new_max); probs = exp(scores - new_max)  cpu.rs:99-100
//   running_sum = running_sum * correction + sum(probs)                      cpu.rs:102
//   acc = acc * correction + probs @ v_f32                                   cpu.rs:103-104
// then out = acc / running_sum cast to the query dtype (cpu.rs:111).
//
// score_mode 0: scores in f32 from f32-converted q and k (what the GPU kernels compute).
// score_mode 1: the candle dtype flow for bf16/f16 — the q@k^T matmul result is rounded to the
//   dtype, multiplied by scale in the dtype (rounded again), then cast to f32. candle's internal
//   accumulation for low-precision matmul is not pinned by any reference test; this mode
//   assumes an f32 accumulator with a single rounding. For f32 both modes are identical.
//
// q/out: [total_q, num_heads, head_dim] token-major, pool dtype.
// Returns 0, -1 for invalid scalar arguments, or an OR of ERR_* bits for bad table data
// (sequences with bad data are skipped and their output rows zeroed).
int32_t oracle_paged_attention(int32_t dt, int32_t score_mode, const void *q, void *out,
                               const void *k_cache, const void *v_cache, int32_t num_blocks,
                               int32_t kv_heads, int32_t block_size, int32_t head_dim,
                               int32_t num_heads, int32_t n_rep, const int32_t *cu_seqlens_q,
                               const int32_t *context_lens, const int32_t *block_tables,
                               int32_t max_blocks, int32_t num_seqs, float scale,
                               int32_t num_threads) {
  if (n_rep <= 0 || num_heads != n_rep * kv_heads || block_size <= 0 || head_dim <= 0) return -1;
  const float sc_dt = round_dt(scale, dt);
  const bool faithful = score_mode == 1 && dt != DT_F32;
  const float neg_inf = -std::numeric_limits<float>::infinity();

  // Validate tables first (host data here); bad sequences are skipped and reported.
  std::vector<int32_t> seq_err(num_seqs, 0);
  int32_t err = 0;
  for (int32_t s = 0; s < num_seqs; ++s) {
    const int32_t q0 = cu_seqlens_q[s], q1 = cu_seqlens_q[s + 1];
    const int32_t L = context_lens[s];
    if (q1 < q0 || q0 < 0) { seq_err[s] |= ERR_SEQLEN; }
    else if (L < q1 - q0 || int64_t(L) > int64_t(max_blocks) * block_size) { seq_err[s] |= ERR_CONTEXT; }
    else {
      const int32_t nb = (L + block_size - 1) / block_size;
      for (int32_t b = 0; b < nb; ++b) {
        const int32_t id = block_tables[size_t(s) * max_blocks + b];
        if (id < 0 || id >= num_blocks) { seq_err[s] |= ERR_BLOCK_ID; break; }
      }
    }
    err |= seq_err[s];
  }

  // One task per (sequence, kv head): the K/V block is converted to f32 once and reused by the
  // n_rep query heads and all query rows of the sequence.
  const int64_t ntask = int64_t(num_seqs) * kv_heads;
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#pragma omp parallel
#endif
  {
    std::vector<float> kb(size_t(block_size) * head_dim), vb(size_t(block_size) * head_dim);
    std::vector<float> qf, m, l, acc, sc(block_size);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
    for (int64_t task = 0; task < ntask; ++task) {
      const int32_t s = int32_t(task / kv_heads), kh = int32_t(task % kv_heads);
      const int32_t q0 = cu_seqlens_q[s], q1 = cu_seqlens_q[s + 1];
      const int32_t seq_q = q1 - q0;
      if (seq_err[s]) {
        for (int32_t i = 0; i < seq_q; ++i)
          for (int32_t r = 0; r < n_rep; ++r)
            for (int32_t x = 0; x < head_dim; ++x)
              store(out, (size_t(q0 + i) * num_heads + kh * n_rep + r) * head_dim + x, dt, 0.f);
        continue;
      }
      if (seq_q == 0) continue;
      const int32_t L = context_lens[s];
      const int32_t offset = L - seq_q;  // cpu.rs:68
      const int32_t rows = seq_q * n_rep;
      qf.assign(size_t(rows) * head_dim, 0.f);
      m.assign(rows, neg_inf);
      l.assign(rows, 0.f);
      acc.assign(size_t(rows) * head_dim, 0.f);
      for (int32_t i = 0; i < seq_q; ++i)
        for (int32_t r = 0; r < n_rep; ++r)
          for (int32_t x = 0; x < head_dim; ++x)
            qf[(size_t(i) * n_rep + r) * head_dim + x] =
                load(q, (size_t(q0 + i) * num_heads + kh * n_rep + r) * head_dim + x, dt);

      const int32_t nb = (L + block_size - 1) / block_size;
      for (int32_t b = 0; b < nb; ++b) {
        const int32_t kv_start = b * block_size;
        const int32_t bn = std::min(block_size, L - kv_start);
        const int64_t phys = block_tables[size_t(s) * max_blocks + b];
        const size_t base = ((size_t(phys) * kv_heads + kh) * block_size) * head_dim;
        for (int32_t j = 0; j < bn; ++j)
          for (int32_t x = 0; x < head_dim; ++x) {
            kb[size_t(j) * head_dim + x] = load(k_cache, base + size_t(j) * head_dim + x, dt);
            vb[size_t(j) * head_dim + x] = load(v_cache, base + size_t(j) * head_dim + x, dt);
          }
        for (int32_t i = 0; i < seq_q; ++i) {
          // Rows whose whole block is in their future still run the fold (probs are 0),
          // exactly as the reference does.
          for (int32_t r = 0; r < n_rep; ++r) {
            const int32_t row = i * n_rep + r;
            const float *qr = &qf[size_t(row) * head_dim];
            float bmax = neg_inf;
            for (int32_t j = 0; j < bn; ++j) {
              const float *kr = &kb[size_t(j) * head_dim];
              float dot = 0.f;
              for (int32_t x = 0; x < head_dim; ++x) dot += qr[x] * kr[x];
              float sv = faithful ? round_dt(round_dt(dot, dt) * sc_dt, dt) : dot * scale;
              if (kv_start + j > offset + i) sv = neg_inf;
              sc[j] = sv;
              bmax = std::max(bmax, sv);
            }
            const float new_max = std::max(m[row], bmax);
            const float corr = std::exp(m[row] - new_max);
            float psum = 0.f;
            for (int32_t j = 0; j < bn; ++j) {
              sc[j] = std::exp(sc[j] - new_max);
              psum += sc[j];
            }
            l[row] = l[row] * corr + psum;
            float *ar = &acc[size_t(row) * head_dim];
            for (int32_t x = 0; x < head_dim; ++x) ar[x] *= corr;
            for (int32_t j = 0; j < bn; ++j) {
              const float p = sc[j];
              const float *vr = &vb[size_t(j) * head_dim];
              for (int32_t x = 0; x < head_dim; ++x) ar[x] += p * vr[x];
            }
            m[row] = new_max;
          }
        }
      }
      for (int32_t i = 0; i < seq_q; ++i)
        for (int32_t r = 0; r < n_rep; ++r) {
          const int32_t row = i * n_rep + r;
          for (int32_t x = 0; x < head_dim; ++x)
            store(out, (size_t(q0 + i) * num_heads + kh * n_rep + r) * head_dim + x, dt,
                  acc[size_t(row) * head_dim + x] / l[row]);
        }
    }
  }
  return err;
}

int32_t oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
