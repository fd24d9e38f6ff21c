// Varlen causal prefill over a paged KV pool on the 5th-generation tensor cores (tcgen05).
//
// Semantics: backend::cpu::paged_attention (src/backend/cpu.rs:57-112) for every sequence of a
// packed batch: S new query tokens (the suffix) attend to the sequence's L = P + S KV tokens
// (P cached prefix tokens, possibly shared blocks) with query i seeing KV j iff j <= P + i
// (cpu.rs:66-68, 87-94). bf16/f16 pools, head_dim 128, block_size 16.
//
// CTA = (chunk of 2*TQ query tokens of one sequence, one KV head). GQA is packed into the MMA M
// dimension: a 128-row Q tile holds TQ = 128 / n_rep tokens x the n_rep query heads that share
// the KV head, so each K/V tile feeds every head of the group. Two Q tiles (A, B) per CTA share
// each K/V tile and alternate on the tensor core:
//
//   S_A(i) = Q_A K_i^T ... softmax_A(i) ... PV_A(i) = P_A(i) V_i      (and the same for B)
//   issue order: S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) PV_B(1) ...
//
// so each softmax warpgroup works while the tensor core runs the other tile's MMAs.
//
// Warp roles (320 threads): warps 0-3 softmax for tile A (thread = TMEM lane = Q row),
// warps 4-7 softmax for tile B, warp 8 TMA producer, warp 9 MMA issuer + TMEM owner.
//
// Memory: Q tiles and 2-stage K and V rings in shared memory, all 128-byte swizzled (K-major Q/K,
// MN-major V). K/V tiles are 128 tokens = 8 pages gathered through the block table with one
// 16 x 64 TMA box per (page, 64-wide half of head_dim). TMEM (512 columns): S_A, S_B (f32,
// 128 columns each; P overwrites the first 64 columns as packed 16-bit pairs and feeds the
// PV MMA straight from TMEM), O_A, O_B (f32 accumulators, 128 columns each).
//
// Online softmax: running max in log2 units with lazy rescaling: O and the row sum are rescaled
// only when the max grows by more than 8 (so un-rescaled P stays below 2^8); the final output is
// O / rowsum, cast to the query dtype (cpu.rs:111).
//
// Every mbarrier wait is bounded; a timeout sets FA_DEVERR_TIMEOUT, the roles stop, issued MMAs
// are drained and TMEM is released before the CTA exits.
#pragma once

#include "tcgen05.cuh"

namespace fa {

struct PrefillParams {
  void *out;                     // [total_q, num_heads, 128]
  const int32_t *cu_seqlens_q;   // [num_seqs + 1]
  const int32_t *context_lens;   // [num_seqs]
  const int32_t *block_tables;   // [num_seqs, max_blocks_per_seq]
  int32_t max_blocks_per_seq;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t n_rep;
  int32_t num_blocks;
  int32_t total_q;
  int32_t tq;                    // query tokens per Q tile (128 / n_rep)
  float scale_log2;              // scale * log2(e)
};

constexpr int kPfWarps = 10;
constexpr int kPfThreads = kPfWarps * 32;
constexpr int kPfBN = 128;                  // KV tokens per tile
constexpr int kPfPages = kPfBN / kPage;     // 8 pages per KV tile
constexpr int kPfStages = 2;
constexpr float kPfRescale = 8.0f;          // lazy-rescale threshold (log2 units)

struct PrefillSmem {
  static constexpr int kHalf = 128 * 128;                     // 128 rows x 64 values x 2 B
  static constexpr int kTile = 2 * kHalf;                     // 128 rows x 128 values
  static constexpr int kQOff = 0;                             // Q_A, Q_B
  static constexpr int kKOff = 2 * kTile;                     // K ring
  static constexpr int kVOff = kKOff + kPfStages * kTile;     // V ring
  static constexpr int kBarOff = kVOff + kPfStages * kTile;
  // barrier indices
  static constexpr int Q = 0, KFULL = 1, KEMPTY = KFULL + kPfStages, VFULL = KEMPTY + kPfStages,
                       VEMPTY = VFULL + kPfStages, SFULL = VEMPTY + kPfStages, PFULL = SFULL + 2,
                       ODONE = PFULL + 2, DRAIN = ODONE + 2, NBARS = DRAIN + 1;
  static constexpr int kMiscOff = kBarOff + NBARS * 8;
  static constexpr int kBytes = kMiscOff + 64;
  static constexpr int kAlloc = kBytes + 1024;
};

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_kernel(const __grid_constant__ PrefillParams p,
                         const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v) {
  using S = PrefillSmem;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S::kBarOff);
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + S::kMiscOff);
  int *s_work = reinterpret_cast<int *>(smem + S::kMiscOff + 16);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + S::kMiscOff + 48);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;
  const int chunk = 2 * p.tq;

  // ---- blockIdx.x -> (sequence, chunk): warp-parallel prefix sum of chunks per sequence ------
  if (warp == 0) {
    const int target = blockIdx.x;
    int base = 0, f_seq = -1, f_local = 0, f_n = 0;
    for (int s0 = 0; s0 < p.num_seqs && f_seq < 0; s0 += 32) {
      const int s = s0 + lane;
      int n = 0;
      if (s < p.num_seqs) {
        const int len = p.cu_seqlens_q[s + 1] - p.cu_seqlens_q[s];
        n = len > 0 ? (len + chunk - 1) / chunk : 0;
      }
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int excl = incl - n;
      const unsigned hit =
          __ballot_sync(0xffffffffu, n > 0 && target >= base + excl && target < base + incl);
      if (hit) {
        const int src = __ffs(hit) - 1;
        f_seq = s0 + src;
        f_local = __shfl_sync(0xffffffffu, target - base - excl, src);
        f_n = __shfl_sync(0xffffffffu, n, src);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_work[0] = f_seq;
      s_work[1] = f_local;
      s_work[2] = f_n;
    }
  }
  __syncthreads();
  const int seq = s_work[0];
  if (seq < 0) return;  // beyond the last chunk (the grid is an upper bound)

  const int q0 = p.cu_seqlens_q[seq];
  const int S_len = p.cu_seqlens_q[seq + 1] - q0;
  const int L = p.context_lens[seq];
  const int Pfx = L - S_len;
  const int t0 = (s_work[2] - 1 - s_work[1]) * chunk;  // the chunk seeing the most KV runs first
  T *out = static_cast<T *>(p.out);
  if (L < S_len || int64_t(L) > int64_t(p.max_blocks_per_seq) * kPage || q0 < 0 ||
      q0 + S_len > p.total_q) {
    if (tid == 0) report(q0 + S_len > p.total_q || q0 < 0 ? FA_DEVERR_SEQLEN : FA_DEVERR_CONTEXT);
    const int t_end = min(t0 + chunk, S_len);
    for (int idx = tid; idx < (t_end - t0) * p.n_rep * 128; idx += kPfThreads) {
      const int tk = t0 + idx / (p.n_rep * 128), rem = idx % (p.n_rep * 128);
      const int64_t row = int64_t(q0) + tk;
      if (row >= 0 && row < p.total_q)
        out[(row * p.num_heads + kvh * p.n_rep + rem / 128) * 128 + rem % 128] = Elem<T>::from_f(0.f);
    }
    return;
  }
  const int t_last = min(t0 + chunk, S_len) - 1;
  const int kv_end = Pfx + t_last + 1;  // KV tokens visible to at least one row of this CTA
  const int n_tiles = (kv_end + kPfBN - 1) / kPfBN;
  const int n_pages = (L + kPage - 1) / kPage;

  if (tid == 0) {
#pragma unroll 1
    for (int i = 0; i < S::NBARS; ++i) mbar_init(bar(i), (i == S::PFULL || i == S::PFULL + 1) ? 128 : 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tc::alloc(smem_u32(s_tmem), 512);
    tc::relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 8) {
    // ================= TMA producer =================
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar(S::Q), 2 * 2 * 64 * p.n_rep * p.tq * 2);
#pragma unroll
      for (int X = 0; X < 2; ++X)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_3d(sbase + S::kQOff + X * S::kTile + hf * S::kHalf, &tm_q, bar(S::Q), hf * 64,
                      kvh * p.n_rep, q0 + t0 + X * p.tq);
      const int32_t *table = p.block_tables + size_t(seq) * p.max_blocks_per_seq;
      bool bad = false;
      int issued = 0;
      for (int i = 0; i < n_tiles; ++i) {
        if (*s_abort) break;
        const int st = i % kPfStages;
        const uint32_t ph = ((i / kPfStages) - 1) & 1;
        int rows[kPfPages];
#pragma unroll
        for (int j = 0; j < kPfPages; ++j) {
          int id = table[min(i * kPfPages + j, n_pages - 1)];  // pages past the end: reload the last
          if (uint32_t(id) >= uint32_t(p.num_blocks)) {
            bad = true;
            id = 0;
          }
          rows[j] = (id * p.num_kv_heads + kvh) * kPage;
        }
        if (i >= kPfStages && !mbar_wait(bar(S::KEMPTY + st), ph)) { *s_abort = 1; break; }
        mbar_arrive_expect_tx(bar(S::KFULL + st), S::kTile);
        const uint32_t kb = sbase + S::kKOff + st * S::kTile;
#pragma unroll
        for (int j = 0; j < kPfPages; ++j) {
          tma_load_2d(kb + j * 2048, &tm_k, bar(S::KFULL + st), 0, rows[j]);
          tma_load_2d(kb + S::kHalf + j * 2048, &tm_k, bar(S::KFULL + st), 64, rows[j]);
        }
        if (i >= kPfStages && !mbar_wait(bar(S::VEMPTY + st), ph)) { *s_abort = 1; ++issued; break; }
        mbar_arrive_expect_tx(bar(S::VFULL + st), S::kTile);
        const uint32_t vb = sbase + S::kVOff + st * S::kTile;
#pragma unroll
        for (int j = 0; j < kPfPages; ++j) {
          tma_load_2d(vb + j * 2048, &tm_v, bar(S::VFULL + st), 0, rows[j]);
          tma_load_2d(vb + S::kHalf + j * 2048, &tm_v, bar(S::VFULL + st), 64, rows[j]);
        }
        ++issued;
      }
      if (bad) report(FA_DEVERR_BLOCK_ID);
      if (*s_abort) {
        // Let the loads already issued land before the CTA can exit (bounded waits).
        for (int i = max(0, issued - kPfStages); i < issued; ++i) {
          mbar_wait(bar(S::KFULL + i % kPfStages), (i / kPfStages) & 1);
          mbar_wait(bar(S::VFULL + i % kPfStages), (i / kPfStages) & 1);
        }
      }
    }
  } else if (warp == 9) {
    // ================= MMA issuer (one thread) =================
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_f16(kBf16, 128, 128, false, false);
      const uint32_t id_o = tc::idesc_f16(kBf16, 128, 128, false, true);
      auto issue_s = [&](int X, int st) {  // S_X = Q_X K^T, K = head_dim (8 steps of 16)
        const uint32_t qa = sbase + S::kQOff + X * S::kTile;
        const uint32_t kb = sbase + S::kKOff + st * S::kTile;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * S::kHalf + (k & 3) * 32;
          tc::mma_ss(tmem + X * 128, tc::sw128_desc(qa + off, 16, 1024),
                     tc::sw128_desc(kb + off, 16, 1024), id_s, k > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int X, int st, bool first) {  // O_X += P_X V, K = tokens (8 x 16)
        const uint32_t vb = sbase + S::kVOff + st * S::kTile;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          tc::mma_ts(tmem + 256 + X * 128, tmem + X * 128 + k * 8,
                     tc::sw128_desc(vb + k * 2048, S::kHalf, 1024), id_o,
                     (!first || k > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(bar(S::Q), 0) && mbar_wait(bar(S::KFULL), 0);
      if (ok) {
        tc::fence_after();
        issue_s(0, 0);
        tc::commit(bar(S::SFULL + 0));
        issue_s(1, 0);
        tc::commit(bar(S::SFULL + 1));
        tc::commit(bar(S::KEMPTY + 0));
      }
      for (int i = 0; ok && i < n_tiles; ++i) {
        const int st = i % kPfStages, st1 = (i + 1) % kPfStages;
        const uint32_t ph = (i / kPfStages) & 1, ph1 = ((i + 1) / kPfStages) & 1;
        const bool last = i + 1 == n_tiles;
        if (!(ok = mbar_wait(bar(S::PFULL + 0), i & 1) && mbar_wait(bar(S::VFULL + st), ph))) break;
        tc::fence_after();
        issue_pv(0, st, i == 0);
        if (last) tc::commit(bar(S::ODONE + 0));
        if (!last) {
          if (!(ok = mbar_wait(bar(S::KFULL + st1), ph1))) break;
          tc::fence_after();
          issue_s(0, st1);
          tc::commit(bar(S::SFULL + 0));
        }
        if (!(ok = mbar_wait(bar(S::PFULL + 1), i & 1))) break;
        tc::fence_after();
        issue_pv(1, st, i == 0);
        tc::commit(bar(S::VEMPTY + st));
        if (last) tc::commit(bar(S::ODONE + 1));
        if (!last) {
          issue_s(1, st1);
          tc::commit(bar(S::SFULL + 1));
          tc::commit(bar(S::KEMPTY + st1));
        }
      }
      if (!ok) {
        *s_abort = 1;
        report(FA_DEVERR_TIMEOUT);
      }
      tc::commit(bar(S::DRAIN));  // every MMA issued above has completed once this arrives
      mbar_wait(bar(S::DRAIN), 0);
    }
  } else {
    // ================= softmax warpgroups =================
    const int X = warp >> 2, wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = uint32_t(wq * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + X * 128;
    const uint32_t o_addr = tmem + lane_off + 256 + X * 128;
    const int tok = t0 + X * p.tq + r / p.n_rep;
    const bool row_valid = r < p.tq * p.n_rep && tok < S_len;
    const int limit = Pfx + tok;  // visible KV positions j <= limit
    const float sl2 = p.scale_log2;
    float m_run = neg_inf(), l = 0.f;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(bar(S::SFULL + X), i & 1)))) break;
      tc::fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::ld32(s_addr + c * 32, sr[c]);
      tc::wait_ld();
      const int j0 = i * kPfBN;
      float mt = neg_inf();
      if (j0 + kPfBN - 1 > limit) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = (j0 + c * 32 + e > limit) ? neg_inf() : __uint_as_float(sr[c][e]) * sl2;
            sr[c][e] = __float_as_uint(x);
            mt = fmaxf(mt, x);
          }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = __uint_as_float(sr[c][e]) * sl2;
            sr[c][e] = __float_as_uint(x);
            mt = fmaxf(mt, x);
          }
      }
      float factor = 1.f;
      bool rescale = false;
      if (i == 0) {
        m_run = mt;
      } else if (mt > m_run + kPfRescale) {
        factor = ex2(m_run - mt);
        m_run = mt;
        rescale = true;
      }
      const float m_use = m_run == neg_inf() ? 0.f : m_run;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = ex2(__uint_as_float(sr[c][2 * e]) - m_use);
          const float b = ex2(__uint_as_float(sr[c][2 * e + 1]) - m_use);
          rs += a + b;
          pk[e] = pack2<T>(a, b);
        }
        tc::st16(s_addr + c * 16, pk);  // P: token 2e,2e+1 of chunk c -> column c*16 + e
      }
      l = l * factor + rs;
      if (__any_sync(0xffffffffu, rescale)) {
        // O_X holds PV_X(i-1) (S_X(i) was committed after it): rescale in place.
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tc::ld32(o_addr + c * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
          tc::st32(o_addr + c * 32, o);
        }
      }
      tc::wait_st();
      tc::fence_before();
      mbar_arrive(bar(S::PFULL + X));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(S::ODONE + X), 0));
    if (ok) {
      tc::fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T *orow = out + (size_t(q0 + min(tok, S_len - 1)) * p.num_heads + kvh * p.n_rep +
                       r % p.n_rep) * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tc::ld32(o_addr + c * 32, o);
        tc::wait_ld();
        if (row_valid) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack2<T>(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
          uint4 *dst = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
    } else {
      *s_abort = 1;
      if (lane == 0) report(FA_DEVERR_TIMEOUT);
    }
    tc::fence_before();
  }

  __syncthreads();
  if (warp == 9) {
    tc::fence_after();
    tc::dealloc(tmem, 512);
  }
}

}  // namespace fa
