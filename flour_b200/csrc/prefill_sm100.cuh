// Varlen causal prefill over a paged KV pool on the 5th-generation tensor cores (tcgen05).
//
// Semantics: backend::cpu::paged_attention (src/backend/cpu.rs:57-112) for every sequence of a
// packed batch: S new query tokens (the suffix) attend to the sequence's L = P + S KV tokens
// (P cached prefix tokens, possibly shared blocks) with query i seeing KV j iff j <= P + i
// (cpu.rs:66-68, 87-94). bf16/f16 pools, head_dim 128, block_size 16.
//
// Work item = (chunk of 2*TQ query tokens of one sequence, one KV head). GQA is packed into the
// MMA M dimension: a 128-row Q tile holds TQ = 128 / n_rep tokens x the n_rep query heads that
// share the KV head, so each K/V tile feeds every head of the group. Two Q tiles (A, B) per item
// share each K/V tile and alternate on the tensor core:
//
//   S_X(i) = Q_X K_i^T ... softmax_X(i) ... PV_X(i) = P_X(i) V_i
//   issue order: S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) PV_B(1) ...
//
// so each softmax warpgroup works while the tensor core runs the other tile's MMAs.
//
// Persistent: one CTA per SM; the TMA warp takes work items from a global counter (heaviest
// chunk of each sequence first) and hands them to the other roles through a 2-slot descriptor
// ring in shared memory. K/V loads run ahead across item boundaries, and each Q tile is reloaded
// as soon as the previous item's last MMA reading it has completed.
//
// Warp roles (576 threads): warps 0-7 softmax for tile A, warps 8-15 for tile B (warp = column
// half x row quadrant: thread = TMEM lane = Q row, 64 of the row's 128 scores; the two warps of a
// quadrant exchange row maxima through shared memory), warp 16 TMA producer + scheduler, warp 17
// MMA issuer + TMEM owner.
//
// Memory: Q tiles and 2-stage K and V rings in shared memory, all 128-byte swizzled (K-major Q/K,
// MN-major V). K/V tiles are 128 tokens = 8 pages gathered through the block table with one
// 16 x 64 TMA box per (page, 64-wide half of head_dim). TMEM (512 columns): S_A, S_B (f32,
// 128 columns each; P overwrites the first 64 columns as packed 16-bit pairs and feeds the PV MMA
// straight from TMEM), O_A, O_B (f32 accumulators, 128 columns each).
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
  int32_t *counters;             // [0] next work item, [1] finished CTAs; both back to 0 at exit
  int32_t max_blocks_per_seq;
  int32_t num_seqs;              // <= kPfMaxSeqs per launch
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t n_rep;
  int32_t num_blocks;
  int32_t total_q;
  int32_t tq;                    // query tokens per Q tile (128 / n_rep)
  float scale_log2;              // scale * log2(e), > 0
  float scale;                   // scale as passed (the reference flow rounds it to the dtype)
};

constexpr int kPfSoftmaxWarps = 16;         // 2 Q tiles x 2 column halves x 4 row quadrants
constexpr int kPfProducerWarp = kPfSoftmaxWarps;
constexpr int kPfMmaWarp = kPfSoftmaxWarps + 1;
constexpr int kPfWarps = kPfSoftmaxWarps + 2;
constexpr int kPfThreads = kPfWarps * 32;
constexpr int kPfBN = 128;                  // KV tokens per tile
constexpr int kPfPages = kPfBN / kPage;     // 8 pages per KV tile
constexpr int kPfStages = 2;
constexpr float kPfRescale = 8.0f;          // lazy-rescale threshold (log2 units)
constexpr int kPfMaxSeqs = 2048;            // sequences per launch (chunk table in smem)

struct PfItem {
  int32_t kind;  // 0 work, 1 invalid sequence data (rows are zeroed), 2 no more work
  int32_t seq, kvh, t0, q0, S_len, Pfx, n_tiles, n_pages;
  int32_t pad[7];
};

struct PrefillSmem {
  static constexpr int kHalf = 128 * 128;                     // 128 rows x 64 values x 2 B
  static constexpr int kTile = 2 * kHalf;                     // 128 rows x 128 values
  static constexpr int kQOff = 0;                             // Q_A, Q_B
  static constexpr int kKOff = 2 * kTile;                     // K ring
  static constexpr int kVOff = kKOff + kPfStages * kTile;     // V ring
  static constexpr int kItemOff = kVOff + kPfStages * kTile;
  static constexpr int kXchOff = kItemOff + 2 * int(sizeof(PfItem));  // f32 [2 X][2 halves][128]
  static constexpr int kBarOff = kXchOff + 2 * 2 * 128 * 4;
  // barrier indices (pairs are indexed by Q tile X or ring stage)
  static constexpr int QFULL = 0, QEMPTY = 2, KFULL = 4, KEMPTY = KFULL + kPfStages,
                       VFULL = KEMPTY + kPfStages, VEMPTY = VFULL + kPfStages,
                       SFULL = VEMPTY + kPfStages, PFULL = SFULL + 2, ODONE = PFULL + 2,
                       IFULL = ODONE + 2, IEMPTY = IFULL + 2, DRAIN = IEMPTY + 2,
                       NBARS = DRAIN + 1;
  static constexpr int kMiscOff = kBarOff + NBARS * 8;
  // Chunk prefix sums [num_seqs + 1] last, so a launch requests only what its batch needs (the
  // rest of the SM's shared memory stays free for other kernels' CTAs).
  static constexpr int kOffsOff = kMiscOff + 64;
  static constexpr int alloc(int num_seqs) { return kOffsOff + (num_seqs + 1) * 4 + 1024; }
  static constexpr int kAllocMax = kOffsOff + (kPfMaxSeqs + 1) * 4 + 1024;
};

// Named-barrier helpers for a pair of warps (64 threads). pair_all is a barrier that also ANDs
// a predicate across both warps, so a bounded wait that times out in one warp ends both.
__device__ __forceinline__ void pair_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}
__device__ __forceinline__ bool pair_all(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %2, 0;\n\t"
      "bar.red.and.pred po, %1, 64, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// kRef: the reference's dtype rounding of the scores (ref_score, FA_SCORES_REFERENCE).
template <typename T, bool kRef>
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
  int32_t *offs = reinterpret_cast<int32_t *>(smem + S::kOffsOff);
  PfItem *items = reinterpret_cast<PfItem *>(smem + S::kItemOff);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S::kBarOff);
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + S::kMiscOff);
  volatile int *s_abort = reinterpret_cast<volatile int *>(smem + S::kMiscOff + 16);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = 2 * p.tq;
  T *out = static_cast<T *>(p.out);

  // Programmatic dependent launch: barriers and TMEM are set up while the preceding kernel (the
  // cache write of these tokens' K/V) finishes; global memory is touched only after it is done.
  if (tid == 0) {
    pdl_trigger();
#pragma unroll 1
    for (int i = 0; i < S::NBARS; ++i) {
      const int count = (i == S::PFULL || i == S::PFULL + 1) ? 256
                        : (i == S::IEMPTY || i == S::IEMPTY + 1) ? 1 + 32 * kPfSoftmaxWarps : 1;
      mbar_init(bar(i), count);
    }
    *s_abort = 0;
    offs[0] = 0;
    fence_mbar_init();
  }
  if (warp == kPfMmaWarp) {
    tc::alloc(smem_u32(s_tmem), 512);
    tc::relinquish();
  }
  pdl_wait();
  // ---- chunk table: offs[s] = number of chunks of sequences < s -----------------------------
  for (int s = tid; s < p.num_seqs; s += kPfThreads) {
    const int len = p.cu_seqlens_q[s + 1] - p.cu_seqlens_q[s];
    offs[s + 1] = len > 0 ? (len + chunk - 1) / chunk : 0;
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int s0 = 0; s0 < p.num_seqs; s0 += 32) {
      const int s = s0 + lane;
      const int n = s < p.num_seqs ? offs[s + 1] : 0;
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (s < p.num_seqs) offs[s + 1] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_items = offs[p.num_seqs] * p.num_kv_heads;

  if (warp == kPfProducerWarp) {
    // ================= scheduler + TMA producer =================
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int g = 0, v = 0;  // tiles and valid items issued so far
      bool bad = false;
      // Next work item: global ticket + the sequence's metadata. Called one item ahead, where the
      // producer would otherwise wait for a free ring stage, so its latency stays hidden.
      auto fetch = [&](PfItem &it) {
        it = PfItem{};
        const int w = *s_abort ? n_items : atomicAdd(p.counters, 1);
        if (w >= n_items) {
          it.kind = 2;
          return;
        }
        const int c = w / p.num_kv_heads;
        it.kvh = w % p.num_kv_heads;
        int lo = 0, hi = p.num_seqs;  // last s with offs[s] <= c
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (offs[mid] <= c) lo = mid; else hi = mid;
        }
        it.seq = lo;
        it.t0 = (offs[lo + 1] - 1 - c) * chunk;  // last chunk (most KV) of a sequence first
        it.q0 = p.cu_seqlens_q[lo];
        it.S_len = p.cu_seqlens_q[lo + 1] - it.q0;
        const int L = p.context_lens[lo];
        it.Pfx = L - it.S_len;
        if (L < it.S_len || int64_t(L) > int64_t(p.max_blocks_per_seq) * kPage || it.q0 < 0 ||
            it.q0 + it.S_len > p.total_q) {
          it.kind = 1;
          report(it.q0 < 0 || it.q0 + it.S_len > p.total_q ? FA_DEVERR_SEQLEN : FA_DEVERR_CONTEXT);
        } else {
          it.kind = 0;
          const int kv_end = it.Pfx + min(it.t0 + chunk, it.S_len);
          it.n_tiles = (kv_end + kPfBN - 1) / kPfBN;
          it.n_pages = (L + kPage - 1) / kPage;
        }
      };
      PfItem next;
      fetch(next);
      for (int k = 0;; ++k) {
        const int slot = k & 1;
        const PfItem it = next;
        if (k >= 2 && !mbar_wait(bar(S::IEMPTY + slot), ((k >> 1) - 1) & 1)) { *s_abort = 1; break; }
        items[slot] = it;
        mbar_arrive(bar(S::IFULL + slot));
        if (it.kind == 2) break;
        if (it.kind == 1) {
          fetch(next);
          continue;
        }
        const int32_t *table = p.block_tables + size_t(it.seq) * p.max_blocks_per_seq;
        int ids[kPfPages];  // block ids of the tile being issued (loaded one tile ahead)
#pragma unroll
        for (int j = 0; j < kPfPages; ++j) ids[j] = table[min(j, it.n_pages - 1)];
        // Q tiles of this item (each waits for the previous item's last S MMA reading it).
        const int qbytes = 2 * 64 * p.n_rep * p.tq * 2;
        bool ok = true;
#pragma unroll
        for (int X = 0; X < 2; ++X) {
          if (v >= 1 && !mbar_wait(bar(S::QEMPTY + X), (v - 1) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(bar(S::QFULL + X), qbytes);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
            tma_load_3d(sbase + S::kQOff + X * S::kTile + hf * S::kHalf, &tm_q, bar(S::QFULL + X),
                        hf * 64, it.kvh * p.n_rep, it.q0 + it.t0 + X * p.tq);
        }
        if (!ok) { *s_abort = 1; break; }
        // Take the next ticket two tiles before this item's loads end: early enough to hide the
        // ticket and metadata latency, late enough not to hold work another CTA could start.
        const int fetch_at = it.n_tiles >= 3 ? it.n_tiles - 2 : it.n_tiles;
        for (int i = 0; i < it.n_tiles && ok; ++i, ++g) {
          if (i == fetch_at) fetch(next);
          const int st = g % kPfStages;
          const uint32_t ph = ((g / kPfStages) - 1) & 1;
          int rows[kPfPages], nids[kPfPages];
#pragma unroll
          for (int j = 0; j < kPfPages; ++j) {
            int id = ids[j];
            if (uint32_t(id) >= uint32_t(p.num_blocks)) {
              bad = true;
              id = 0;
            }
            rows[j] = (id * p.num_kv_heads + it.kvh) * kPage;
            // next tile's ids: in flight while this tile waits for its ring stage
            nids[j] = table[min((i + 1) * kPfPages + j, it.n_pages - 1)];
          }
          if (g >= kPfStages && !mbar_wait(bar(S::KEMPTY + st), ph)) { ok = false; break; }
          mbar_arrive_expect_tx(bar(S::KFULL + st), S::kTile);
          const uint32_t kb = sbase + S::kKOff + st * S::kTile;
#pragma unroll
          for (int j = 0; j < kPfPages; ++j) {
            tma_load_2d(kb + j * 2048, &tm_k, bar(S::KFULL + st), 0, rows[j]);
            tma_load_2d(kb + S::kHalf + j * 2048, &tm_k, bar(S::KFULL + st), 64, rows[j]);
          }
          if (g >= kPfStages && !mbar_wait(bar(S::VEMPTY + st), ph)) { ok = false; break; }
          mbar_arrive_expect_tx(bar(S::VFULL + st), S::kTile);
          const uint32_t vb = sbase + S::kVOff + st * S::kTile;
#pragma unroll
          for (int j = 0; j < kPfPages; ++j) {
            tma_load_2d(vb + j * 2048, &tm_v, bar(S::VFULL + st), 0, rows[j]);
            tma_load_2d(vb + S::kHalf + j * 2048, &tm_v, bar(S::VFULL + st), 64, rows[j]);
          }
#pragma unroll
          for (int j = 0; j < kPfPages; ++j) ids[j] = nids[j];
        }
        if (!ok) { *s_abort = 1; break; }
        if (fetch_at == it.n_tiles) fetch(next);
        ++v;
      }
      if (bad) report(FA_DEVERR_BLOCK_ID);
      if (*s_abort) report(FA_DEVERR_TIMEOUT);
    }
  } else if (warp == kPfMmaWarp) {
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
      int g = 0, v = 0;
      bool ok = true;
      // S_X(0) of item `itm` (first KV tile g0, Q-tile phase v0).
      auto start_tile = [&](int X, const PfItem &itm, int g0, int v0) -> bool {
        const int st0 = g0 % kPfStages;
        if (X == 0) {
          if (!(mbar_wait(bar(S::QFULL + 0), v0 & 1) &&
                mbar_wait(bar(S::KFULL + st0), (g0 / kPfStages) & 1)))
            return false;
          tc::fence_after();
          issue_s(0, st0);
          tc::commit(bar(S::SFULL + 0));
          if (itm.n_tiles == 1) tc::commit(bar(S::QEMPTY + 0));
        } else {
          if (!mbar_wait(bar(S::QFULL + 1), v0 & 1)) return false;
          tc::fence_after();
          issue_s(1, st0);
          tc::commit(bar(S::SFULL + 1));
          tc::commit(bar(S::KEMPTY + st0));
          if (itm.n_tiles == 1) tc::commit(bar(S::QEMPTY + 1));
        }
        return true;
      };
      // The next item is fetched during this item's last tile, and its S_A(0) / S_B(0) follow
      // this item's last PV_A / PV_B at once: each Q tile's softmax warps find their next S ready
      // when they finish this item's epilogue, instead of waiting for the other tile.
      bool have_next = false, next_started = false;
      PfItem next{};
      for (int k = 0; ok; ++k) {
        const int slot = k & 1;
        PfItem it;
        bool started = false;
        if (have_next) {
          it = next;
          started = next_started;
          have_next = false;
        } else {
          if (!(ok = mbar_wait(bar(S::IFULL + slot), (k >> 1) & 1))) break;
          it = items[slot];
        }
        if (it.kind == 2) break;
        if (it.kind == 0) {
          const int n = it.n_tiles;
          if (!started && !(ok = start_tile(0, it, g, v) && start_tile(1, it, g, v))) break;
          for (int i = 0; ok && i < n; ++i) {
            const int gi = g + i;
            const int st = gi % kPfStages, st1 = (gi + 1) % kPfStages;
            const uint32_t ph = (gi / kPfStages) & 1, ph1 = ((gi + 1) / kPfStages) & 1;
            const bool last = i + 1 == n;
            if (!(ok = mbar_wait(bar(S::PFULL + 0), gi & 1) && mbar_wait(bar(S::VFULL + st), ph))) break;
            tc::fence_after();
            issue_pv(0, st, i == 0);
            if (last) {
              tc::commit(bar(S::ODONE + 0));
              if (!(ok = mbar_wait(bar(S::IFULL + (slot ^ 1)), ((k + 1) >> 1) & 1))) break;
              next = items[slot ^ 1];
              have_next = true;
              next_started = false;
              if (next.kind == 0 && !(ok = start_tile(0, next, g + n, v + 1))) break;
            } else {
              if (!(ok = mbar_wait(bar(S::KFULL + st1), ph1))) break;
              tc::fence_after();
              issue_s(0, st1);
              tc::commit(bar(S::SFULL + 0));
              if (i + 2 == n) tc::commit(bar(S::QEMPTY + 0));
            }
            if (!(ok = mbar_wait(bar(S::PFULL + 1), gi & 1))) break;
            tc::fence_after();
            issue_pv(1, st, i == 0);
            tc::commit(bar(S::VEMPTY + st));
            if (last) {
              tc::commit(bar(S::ODONE + 1));
              if (next.kind == 0) {
                if (!(ok = start_tile(1, next, g + n, v + 1))) break;
                next_started = true;
              }
            } else {
              issue_s(1, st1);
              tc::commit(bar(S::SFULL + 1));
              tc::commit(bar(S::KEMPTY + st1));
              if (i + 2 == n) tc::commit(bar(S::QEMPTY + 1));
            }
          }
          if (!ok) break;
          g += n;
          ++v;
        }
        mbar_arrive(bar(S::IEMPTY + slot));
      }
      if (!ok) {
        *s_abort = 1;
        report(FA_DEVERR_TIMEOUT);
      }
      tc::commit(bar(S::DRAIN));  // every MMA issued above has completed once this arrives
      mbar_wait(bar(S::DRAIN), 0);
    }
  } else {
    // ================= softmax warps =================
    // Warp (X, half, quadrant): rows 32*quadrant.. of Q tile X, S columns [64*half, 64*half+64).
    // The two warps sharing a row quadrant exchange row maxima / sums through shared memory and
    // take every wait decision together (reduction barrier), so neither can leave the other
    // stranded at a barrier.
    const int X = warp >> 3, hh = (warp >> 2) & 1, wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = uint32_t(wq * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + X * 128 + hh * 64;       // this half of S_X
    const uint32_t p_addr = tmem + lane_off + X * 128 + hh * 32;       // its P columns
    const uint32_t o_addr = tmem + lane_off + 256 + X * 128 + hh * 64; // this half of O_X
    const int pair_bar = 1 + X * 4 + wq;  // named barrier of the two warps sharing the rows
    float *xch = reinterpret_cast<float *>(smem + S::kXchOff);
    float *xch_own = xch + (X * 2 + hh) * 128 + r;
    const float *xch_mate = xch + (X * 2 + (hh ^ 1)) * 128 + r;
    const float sl2 = p.scale_log2;
    const uint32_t scale2 = pack2<T>(p.scale, p.scale);  // the scale rounded to T, twice
    const bool row_used = r < p.tq * p.n_rep;
    int g = 0, v = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!(ok = pair_all(pair_bar, mbar_wait(bar(S::IFULL + slot), (k >> 1) & 1)))) break;
      const PfItem it = items[slot];
      if (it.kind == 2) break;
      const int tok = it.t0 + X * p.tq + r / p.n_rep;
      const bool row_valid = row_used && tok < it.S_len;
      T *orow = out + (size_t(it.q0 + min(tok, max(it.S_len - 1, 0))) * p.num_heads +
                       it.kvh * p.n_rep + r % p.n_rep) * 128 + hh * 64;
      if (it.kind == 1) {
        const int64_t row = int64_t(it.q0) + tok;
        if (row_valid && row >= 0 && row < p.total_q) {
          const uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
          for (int c = 0; c < 4; ++c) st_global_v8(orow + c * 16, z);
        }
        mbar_arrive(bar(S::IEMPTY + slot));
        continue;
      }
      const int limit = it.Pfx + tok;  // visible KV positions j <= limit
      float m_run = neg_inf(), l = 0.f;
      for (int i = 0; i < it.n_tiles; ++i) {
        const int gi = g + i;
        if (!(ok = pair_all(pair_bar, mbar_wait(bar(S::SFULL + X), gi & 1)))) break;
        tc::fence_after();
        uint32_t sr[2][32];
        tc::ld32(s_addr, sr[0]);
        tc::ld32(s_addr + 32, sr[1]);
        tc::wait_ld();
        // Row max on the raw scores (scale > 0); keys past the causal limit become -inf.
        const int j0 = i * kPfBN + hh * 64;
        float mxp[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) mxp[q] = neg_inf();
        if (j0 + 63 > limit) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (j0 + c * 32 + e > limit) sr[c][e] = __float_as_uint(neg_inf());
              mxp[e & 7] = fmaxf(mxp[e & 7], __uint_as_float(sr[c][e]));
            }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) mxp[e & 7] = fmaxf(mxp[e & 7], __uint_as_float(sr[c][e]));
        }
        const float mx_half = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                    fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        *xch_own = mx_half;
        pair_sync(pair_bar);
        // Both halves: the same row max, in log2 units (the rounding of the reference flow is
        // monotone, so the max of the rounded scores is the rounded max).
        const float mx = fmaxf(mx_half, *xch_mate);
        const float mt = kRef ? ref_score<T>(mx, p.scale) * kLog2e : mx * sl2;
        float factor = 1.f;
        bool rescale = false;
        if (i == 0) {
          m_run = mt;
        } else if (mt > m_run + kPfRescale) {
          factor = ex2(m_run - mt);
          m_run = mt;
          rescale = true;
        }
        const float neg_m = m_run == neg_inf() ? 0.f : -m_run;
        float rsp[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) rsp[q] = 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float a, b;
            if constexpr (kRef) {
              const float2 t = ref_score2<T>(__uint_as_float(sr[c][2 * e]),
                                             __uint_as_float(sr[c][2 * e + 1]), scale2);
              a = ex2(fmaf(t.x, kLog2e, neg_m));
              b = ex2(fmaf(t.y, kLog2e, neg_m));
            } else {
              a = ex2(fmaf(__uint_as_float(sr[c][2 * e]), sl2, neg_m));
              b = ex2(fmaf(__uint_as_float(sr[c][2 * e + 1]), sl2, neg_m));
            }
            rsp[(2 * e) & 7] += a;
            rsp[(2 * e + 1) & 7] += b;
            pk[e] = pack2<T>(a, b);
          }
          tc::st16(p_addr + c * 16, pk);  // P: tokens 2e, 2e+1 of chunk c -> column c*16 + e
        }
        l = l * factor + (((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) +
                          ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7])));
        if (__any_sync(0xffffffffu, rescale)) {
          // O_X holds PV_X(i-1) (S_X(i) was committed after it): rescale this half in place.
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
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
      if (!ok) break;
      if (!(ok = pair_all(pair_bar, mbar_wait(bar(S::ODONE + X), v & 1)))) break;
      tc::fence_after();
      *xch_own = l;
      pair_sync(pair_bar);
      const float lt = l + *xch_mate;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tc::ld32(o_addr + c * 32, o);
        tc::wait_ld();
        if (row_valid) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack2<T>(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
          // Two full 32-byte sectors per store: each row half is written by one thread, so
          // wider stores mean fewer scattered transactions clogging the load/store pipe.
          st_global_v8(orow + c * 32, pk);
          st_global_v8(orow + c * 32 + 16, pk + 8);
        }
      }
      tc::fence_before();
      mbar_arrive(bar(S::IEMPTY + slot));
      g += it.n_tiles;
      ++v;
    }
    if (!ok) {
      *s_abort = 1;
      if (lane == 0) report(FA_DEVERR_TIMEOUT);
    }
    tc::fence_before();
  }

  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc::fence_after();
    tc::dealloc(tmem, 512);
  }
  if (tid == 0) {
    // The last CTA to finish returns the work counters to zero for the next launch.
    __threadfence();
    if (atomicAdd(&p.counters[1], 1) == int(gridDim.x) - 1) {
      atomicExch(&p.counters[0], 0);
      atomicExch(&p.counters[1], 0);
    }
  }
}

}  // namespace fa
