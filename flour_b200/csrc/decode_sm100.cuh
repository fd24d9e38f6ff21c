// Paged GQA decode attention for bf16/f16 pools, block_size 16, head_dim 64 or 128, n_rep <= 8.
//
// Semantics: backend::cpu::paged_attention (src/backend/cpu.rs:57-112) with seq_q = 1, where the
// single query sees every KV position (offset = L - 1, so no key is masked except the unused
// tail of the last page). Scores are kept in f32 (the reference's f32 online-softmax state,
// cpu.rs:70-73); the exponent is evaluated in base 2 with log2(e) folded into the scale.
//
// Work decomposition. One CTA = (split, kv_head, sequence). A split is a run of up to
// `pages_per_split` 16-token pages of one sequence; a CTA serves all n_rep query heads that read
// its KV head (GQA), so each K/V byte is read from HBM once per decode step.
//
// Data movement. A page of one KV head is 16 x head_dim contiguous elements (4 KB at d=128).
// It is fetched by TMA (2-D tensor map over the slab viewed as [rows, head_dim], box 16 x 64,
// 128-byte swizzle, so the ldmatrix reads below are bank-conflict free). Each of the 4 warps
// owns an NSTAGE-deep ring of (K page, V page) buffers with one mbarrier per stage; lane 0 of
// the warp issues the loads, so the warp streams its pages without CTA-wide synchronisation.
//
// Math per page (per warp), on the legacy warp-level tensor path (mma.sync m16n8k16, f32 acc):
//   S^T[16 tok x 8 heads]  = K[16 x d] . Q^T[d x 8]     (A = K via ldmatrix, B = Q in registers)
//   online softmax per head over the 16 tokens (shuffles across the 8 row-lanes)
//   O^T[d x 8 heads]      += V^T[d x 16] . P^T[16 x 8]   (A = V via ldmatrix.trans,
//                                                       B = P^T via movmatrix.trans)
// Heads fill the N=8 side of the MMA, so n_rep = 4..8 wastes at most half of N and no M rows.
// Decode is HBM-bound (~4 FLOP/byte), so the legacy MMA rate is far from the limit.
//
// Split-K merge. Splits write (O/l, log2-sum-exp) partials to the workspace; the last CTA of a
// (sequence, kv_head) to finish (atomic ticket, no waiting) merges them and resets the ticket.
// Sequences with a single split write the output directly.
//
// Fused append (fa_paged_decode_append): the new token of each sequence sits at position
// ctx - 1, i.e. on the sequence's last page, which exactly one CTA per (sequence, kv head) loads
// (the last split). That CTA first copies the token's K and V rows of its KV head from the
// caller's buffers into the pool slot (generic stores, each writer then fences the generic proxy
// against the async proxy), and only after the CTA barrier that precedes its first TMA load does
// any page arrive; so the write and the attention over it happen in one launch, in the order
// of the reference's write_kv followed by paged_attention.
//
// Head-sharded groups (tensor parallel over KV heads, one GPU per rank). The final write of each
// (sequence, kv head) goes to every rank's output buffer (peer memory over NVLink, mapped by
// CUDA IPC) at the rank's head offset, so the all-gather of the per-head outputs happens inside
// the kernel, overlapped with the attention of the other heads. Completion is signalled by the
// next launch on the stream (tp_sync_kernel): stream order makes every store of this kernel
// complete before it publishes an epoch flag to the other ranks, so the decode kernel itself
// carries no fences or counters.
#pragma once

#include "fa_common.cuh"

namespace fa {

constexpr int kMaxTp = 8;  // ranks of a head-sharded group

struct DecodeParams {
  const void *q;                 // [num_seqs, num_heads, HD]
  void *out;                     // [num_seqs, num_heads, HD] (single-GPU mode)
  // Head-sharded mode (n_outs > 0): outs[r] = rank r's [num_seqs, out_heads, HD] buffer; this
  // rank's heads start at out_head0. Otherwise out / num_heads / head 0.
  void *outs[kMaxTp];
  int32_t n_outs;
  int32_t out_heads;
  int32_t out_head0;
  const int32_t *context_lens;   // [num_seqs]
  const int32_t *block_tables;   // [num_seqs, max_blocks_per_seq]
  float *part_o;                 // [num_seqs, num_heads, max_splits, HD]
  float *part_lse;               // [num_seqs, num_heads, max_splits]
  int32_t *counters;             // [num_seqs, num_kv_heads]
  int32_t max_blocks_per_seq;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t n_rep;
  int32_t num_blocks;
  int32_t pages_per_split;
  int32_t max_splits;
  int32_t max_context_len;       // host bound the split plan was made for
  float scale_log2;              // scale * log2(e)
  float scale;                   // scale as passed (FA_SCORES_REFERENCE rounds it to the dtype)
  int32_t ref_scores;            // 1: the reference's dtype rounding of the scores (ref_score)
  // Fused append (new_k != nullptr): new_k[b*nk_token + h*nk_head + x] is the new token's key of
  // sequence b, KV head h (same for new_v); it goes to position ctx-1 of k_pool / v_pool.
  const void *new_k;
  const void *new_v;
  int64_t nk_token, nk_head, nv_token, nv_head;
  void *k_pool;
  void *v_pool;
};

constexpr int kDecodeWarps = 4;
constexpr int kDecodeThreads = kDecodeWarps * 32;
constexpr int kDecodeMaxPagesPerSplit = 256;
constexpr int kDecodeMaxSplits = 256;
constexpr int kPage = 16;  // tokens per page (block_size)

template <int HD, int NSTAGE>
struct DecodeSmem {
  static constexpr int kHalfBytes = kPage * 64 * 2;           // one 16 x 64 TMA box
  static constexpr int kPageBytes = kPage * HD * 2;           // K (or V) of one page
  static constexpr int kStageBytes = 2 * kPageBytes;          // K + V
  static constexpr int kRingBytes = kDecodeWarps * NSTAGE * kStageBytes;
  static constexpr int kIdsOff = kRingBytes;
  static constexpr int kBarOff = kIdsOff + kDecodeMaxPagesPerSplit * 4;
  static constexpr int kFlagOff = kBarOff + kDecodeWarps * NSTAGE * 8;
  static constexpr int kBytes = kFlagOff + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
  // Reduction scratch (reuses the ring once every page is consumed).
  static constexpr int kRedStride = HD + 4;     // padded row: conflict-free stores
  static_assert(kDecodeWarps * 8 * (kRedStride + 2) * 4 + 8 * kDecodeMaxSplits * 4 <= kRingBytes,
                "reduction scratch must fit in the ring");
};

// Store one output element of query head (b, hq) (hq counted within this launch's heads) to the
// output buffer, or to every rank's buffer of a head-sharded group.
template <typename T>
__device__ __forceinline__ void store_out(const DecodeParams &p, int b, int hq, int HD, int x,
                                          float v) {
  const T e = Elem<T>::from_f(v);
  if (p.n_outs == 0) {
    static_cast<T *>(p.out)[(size_t(b) * p.num_heads + hq) * HD + x] = e;
    return;
  }
  const size_t off = (size_t(b) * p.out_heads + p.out_head0 + hq) * HD + x;
  for (int r = 0; r < p.n_outs; ++r) static_cast<T *>(p.outs[r])[off] = e;
}

template <typename T, int HD, int NSTAGE>
__global__ void __launch_bounds__(kDecodeThreads, 3)
    paged_decode_kernel(const __grid_constant__ DecodeParams p,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v) {
  using S = DecodeSmem<HD, NSTAGE>;
  constexpr int KSTEPS = HD / 16;
  constexpr int HALVES = HD / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  int32_t *s_ids = reinterpret_cast<int32_t *>(smem + S::kIdsOff);
  uint64_t *s_bar = reinterpret_cast<uint64_t *>(smem + S::kBarOff);
  int32_t *s_flag = reinterpret_cast<int32_t *>(smem + S::kFlagOff);

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int n_rep = p.n_rep;
  // Programmatic dependent launch: a following kernel launched with programmatic serialization
  // (the next decode, the projection GEMMs) may start once every CTA of this grid has started;
  // this grid's own inputs, workspace and outputs are touched only after the preceding kernel
  // has completed (a no-op wait when this launch has no programmatic dependency).
  if (tid == 0) pdl_trigger();
  pdl_wait();

  const int ctx = p.context_lens[b];
  if (ctx < 1 || ctx > p.max_context_len || int64_t(ctx) > int64_t(p.max_blocks_per_seq) * kPage) {
    // Nothing valid to attend to: zero this CTA's heads once (split 0) and report.
    if (split == 0) {
      if (tid == 0) report(FA_DEVERR_CONTEXT);
      for (int x = tid; x < n_rep * HD; x += kDecodeThreads)
        store_out<T>(p, b, kvh * n_rep + x / HD, HD, x % HD, 0.f);
    }
    return;
  }
  const int n_pages = (ctx + kPage - 1) / kPage;
  const int n_splits = (n_pages + p.pages_per_split - 1) / p.pages_per_split;
  if (split >= n_splits) return;
  const int pg0 = split * p.pages_per_split;
  const int npg = min(n_pages, pg0 + p.pages_per_split) - pg0;

  if (tid == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
#pragma unroll
    for (int i = 0; i < kDecodeWarps * NSTAGE; ++i) mbar_init(smem_u32(&s_bar[i]), 1);
    fence_mbar_init();
  }
  // Block ids of this split, bounds-checked once (a bad id is replaced by block 0 and reported).
  const int32_t *table = p.block_tables + size_t(b) * p.max_blocks_per_seq + pg0;
  bool bad = false;
  for (int i = tid; i < npg; i += kDecodeThreads) {
    int id = table[i];
    if (uint32_t(id) >= uint32_t(p.num_blocks)) { bad = true; id = 0; }
    s_ids[i] = id;
  }
  if (bad) report(FA_DEVERR_BLOCK_ID);
  __syncthreads();

  // ---- per-warp page stream ---------------------------------------------------------------
  const int n_my = npg > warp ? (npg - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
  uint8_t *ring = smem + warp * NSTAGE * S::kStageBytes;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t bar0 = smem_u32(&s_bar[warp * NSTAGE]);
  const uint64_t policy = policy_evict_first();

  auto issue = [&](int i) {
    const int st = i % NSTAGE;
    const int row = (s_ids[warp + i * kDecodeWarps] * p.num_kv_heads + kvh) * kPage;
    const uint32_t kdst = ring_u32 + st * S::kStageBytes;
    const uint32_t vdst = kdst + S::kPageBytes;
    const uint32_t bar = bar0 + st * 8;
    mbar_arrive_expect_tx(bar, S::kStageBytes);
#pragma unroll
    for (int hf = 0; hf < HALVES; ++hf) {
      tma_load_2d_hint(kdst + hf * S::kHalfBytes, &tm_k, bar, hf * 64, row, policy);
      tma_load_2d_hint(vdst + hf * S::kHalfBytes, &tm_v, bar, hf * 64, row, policy);
    }
  };
  // Fused append: the warp that streams the last page (position ctx - 1) first writes the new
  // token's K/V row of this KV head into it; all of its lanes fence the generic proxy against
  // the async proxy before lane 0 issues that page's TMA load. When the last page is not among
  // the warp's first NSTAGE pages, those are issued first so the write overlaps their loads.
  const bool appender =
      p.new_k != nullptr && split == n_splits - 1 && warp == (npg - 1) % kDecodeWarps;
  auto append_row = [&]() {
    const int id = table[npg - 1];
    if (uint32_t(id) < uint32_t(p.num_blocks)) {
      const size_t dst = ((size_t(id) * p.num_kv_heads + kvh) * kPage + (ctx - 1) % kPage) * HD;
      const T *nk = static_cast<const T *>(p.new_k) + b * p.nk_token + kvh * p.nk_head;
      const T *nv = static_cast<const T *>(p.new_v) + b * p.nv_token + kvh * p.nv_head;
#pragma unroll
      for (int x = lane; x < HD; x += 32) {
        static_cast<T *>(p.k_pool)[dst + x] = nk[x];
        static_cast<T *>(p.v_pool)[dst + x] = nv[x];
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    __syncwarp();
  };
  if (appender && n_my <= NSTAGE) append_row();
  if (lane == 0) {
    for (int i = 0; i < NSTAGE && i < n_my; ++i) issue(i);
  }
  if (appender && n_my > NSTAGE) append_row();

  // Q^T fragments (B operand, k = head_dim, n = head), constant for the whole kernel.
  uint32_t qb[KSTEPS][2];
  {
    const int hq = kvh * n_rep + g;
    const T *qrow = static_cast<const T *>(p.q) + (size_t(b) * p.num_heads + hq) * HD;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      if (g < n_rep) {
        qb[ks][0] = *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * t);
        qb[ks][1] = *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * t + 8);
      } else {
        qb[ks][0] = 0u;
        qb[ks][1] = 0u;
      }
    }
  }

  const float sl2 = p.scale_log2;
  float m0 = neg_inf(), m1 = neg_inf(), l0 = 0.f, l1 = 0.f;  // heads 2t, 2t+1
  float o[KSTEPS][4];
#pragma unroll
  for (int mt = 0; mt < KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

  // ldmatrix row/chunk owned by this lane (swizzled: chunk ^ (row & 7) inside a 128-B line).
  const int k_tok = lane & 15, k_chunk_hi = lane >> 4;
  const int v_tok = (lane & 7) + ((lane >> 4) << 3), v_chunk_hi = (lane >> 3) & 1;

  int timed_out_at = -1;
  for (int i = 0; i < n_my; ++i) {
    const int st = i % NSTAGE;
    // Warp-uniform outcome: every lane polls (bounded), and the warp leaves together.
    if (!__all_sync(0xffffffffu, mbar_wait(bar0 + st * 8, (i / NSTAGE) & 1))) {
      timed_out_at = i;
      break;
    }
    const uint32_t kb = ring_u32 + st * S::kStageBytes;
    const uint32_t vb = kb + S::kPageBytes;
    const int page = pg0 + warp + i * kDecodeWarps;

    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      const int ch = ks * 2 + k_chunk_hi;
      uint32_t a[4];
      ldsm_x4(kb + (ch >> 3) * S::kHalfBytes + k_tok * 128 + (((ch & 7) ^ (k_tok & 7)) << 4), a);
      mma16816<T>(c, a, qb[ks][0], qb[ks][1]);
    }
    // c0:(tok g, head 2t) c1:(g, 2t+1) c2:(g+8, 2t) c3:(g+8, 2t+1)
    const int tok0 = page * kPage + g;
    if (p.ref_scores) {  // uniform over the launch
#pragma unroll
      for (int e = 0; e < 4; ++e) c[e] = ref_score<T>(c[e], p.scale) * kLog2e;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) c[e] *= sl2;
    }
    const float s0 = tok0 < ctx ? c[0] : neg_inf();
    const float s1 = tok0 < ctx ? c[1] : neg_inf();
    const float s2 = tok0 + 8 < ctx ? c[2] : neg_inf();
    const float s3 = tok0 + 8 < ctx ? c[3] : neg_inf();
    float bm0 = fmaxf(s0, s2), bm1 = fmaxf(s1, s3);
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, x));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, x));
    }
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);  // finite: token 0 of a page is valid
    const float c0 = ex2(m0 - mn0), c1 = ex2(m1 - mn1);
    const float p0 = ex2(s0 - mn0), p1 = ex2(s1 - mn1);
    const float p2 = ex2(s2 - mn0), p3 = ex2(s3 - mn1);
    l0 = l0 * c0 + (p0 + p2);
    l1 = l1 * c1 + (p1 + p3);
    m0 = mn0;
    m1 = mn1;
    const uint32_t pb0 = movmatrix_t(pack2<T>(p0, p1));
    const uint32_t pb1 = movmatrix_t(pack2<T>(p2, p3));
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt) {
      o[mt][0] *= c0;
      o[mt][1] *= c1;
      o[mt][2] *= c0;
      o[mt][3] *= c1;
      const int ch = mt * 2 + v_chunk_hi;
      uint32_t a[4];
      ldsm_x4_t(vb + (ch >> 3) * S::kHalfBytes + v_tok * 128 + (((ch & 7) ^ (v_tok & 7)) << 4), a);
      mma16816<T>(o[mt], a, pb0, pb1);
    }
    __syncwarp();
    if (lane == 0 && i + NSTAGE < n_my) issue(i + NSTAGE);
  }
  if (timed_out_at >= 0) {
    // Drain this warp's loads still in flight (each wait bounded again) before leaving.
    if (lane == 0) report(FA_DEVERR_TIMEOUT);
    for (int j = timed_out_at + 1; j < n_my && j < timed_out_at + NSTAGE; ++j)
      mbar_wait(bar0 + (j % NSTAGE) * 8, (j / NSTAGE) & 1);
  }
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, x);
    l1 += __shfl_xor_sync(0xffffffffu, l1, x);
  }
  __syncthreads();  // every warp is done with its ring: reuse it as reduction scratch

  // ---- combine the 4 warps ------------------------------------------------------------------
  float *red_o = reinterpret_cast<float *>(smem);                           // [W][8][HD+4]
  float *red_m = red_o + kDecodeWarps * 8 * S::kRedStride;                  // [W][8]
  float *red_l = red_m + kDecodeWarps * 8;                                  // [W][8]
  float *s_lse = red_l + kDecodeWarps * 8;                                  // [8][max_splits]
  {
    float *ro = red_o + warp * 8 * S::kRedStride;
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt) {
      ro[(2 * t) * S::kRedStride + mt * 16 + g] = o[mt][0];
      ro[(2 * t + 1) * S::kRedStride + mt * 16 + g] = o[mt][1];
      ro[(2 * t) * S::kRedStride + mt * 16 + g + 8] = o[mt][2];
      ro[(2 * t + 1) * S::kRedStride + mt * 16 + g + 8] = o[mt][3];
    }
    if (g == 0) {
      red_m[warp * 8 + 2 * t] = m0;
      red_m[warp * 8 + 2 * t + 1] = m1;
      red_l[warp * 8 + 2 * t] = l0;
      red_l[warp * 8 + 2 * t + 1] = l1;
    }
  }
  __syncthreads();

  const int hq0 = kvh * n_rep;
  const bool single = n_splits == 1;
  for (int idx = tid; idx < n_rep * HD; idx += kDecodeThreads) {
    const int h = idx / HD, x = idx % HD;
    float M = neg_inf();
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, red_m[w * 8 + h]);
    float O = 0.f, Lsum = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float e = ex2(red_m[w * 8 + h] - M);  // warps without pages: m = -inf -> 0
      O += e * red_o[(w * 8 + h) * S::kRedStride + x];
      Lsum += e * red_l[w * 8 + h];
    }
    const size_t ob = size_t(b) * p.num_heads + hq0 + h;
    if (single) {
      store_out<T>(p, b, hq0 + h, HD, x, O / Lsum);
    } else {
      const size_t pi = ob * p.max_splits + split;
      p.part_o[pi * HD + x] = O / Lsum;
      if (x == 0) p.part_lse[pi] = M + __log2f(Lsum);
    }
  }
  if (single) return;

  // ---- last split of this (sequence, kv_head) merges the partials ------------------------
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&p.counters[b * p.num_kv_heads + kvh], 1);
    s_flag[0] = (prev == n_splits - 1);
  }
  __syncthreads();
  if (!s_flag[0]) return;
  __threadfence();
  for (int idx = tid; idx < n_rep * n_splits; idx += kDecodeThreads) {
    const int h = idx / n_splits, sp = idx % n_splits;
    s_lse[h * kDecodeMaxSplits + sp] =
        __ldcg(&p.part_lse[(size_t(b) * p.num_heads + hq0 + h) * p.max_splits + sp]);
  }
  __syncthreads();
  for (int idx = tid; idx < n_rep * HD; idx += kDecodeThreads) {
    const int h = idx / HD, x = idx % HD;
    const float *lse = s_lse + h * kDecodeMaxSplits;
    float M = neg_inf();
    for (int sp = 0; sp < n_splits; ++sp) M = fmaxf(M, lse[sp]);
    const size_t ob = size_t(b) * p.num_heads + hq0 + h;
    const float *po = p.part_o + ob * p.max_splits * HD + x;
    float O = 0.f, W = 0.f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const float w = ex2(lse[sp] - M);
      O += w * __ldcg(po + size_t(sp) * HD);
      W += w;
    }
    store_out<T>(p, b, hq0 + h, HD, x, O / W);
  }
  if (tid == 0) p.counters[b * p.num_kv_heads + kvh] = 0;  // ready for the next launch
}

// Head-sharded groups: mark this rank's preceding launches on the stream complete and/or wait
// for the other ranks. Publish: epoch e (the host's, or with epoch 0 the next device epoch
// *counter + 1, taken by thread 0) goes into slot [rank] of every rank's flag array, thread r
// storing to rank r with a system-scope release, so the tp stores go out in parallel rather
// than one release after another. Every thread has waited for the preceding decode (its peer
// stores included) to complete, so each release covers them.
// Wait (thread s < tp): poll this rank's flags[s] until it reaches e (wrap-around order; with
// epoch 0, e = *counter), bounded by device time and an iteration cap; on expiry it reports
// FA_DEVERR_TIMEOUT and returns.
struct TpFlagSlots {
  uint32_t *slot[kMaxTp];
};
constexpr int kTpPublish = 1, kTpWait = 2;

__global__ void tp_sync_kernel(TpFlagSlots publish_to, const uint32_t *my_flags, int tp,
                               uint32_t epoch, uint32_t *counter, int mode,
                               unsigned long long timeout_ns) {
  __shared__ uint32_t s_epoch;
  const int s = threadIdx.x;
  // Launched with programmatic serialization: started early, it publishes only once the
  // preceding decode (its peer stores included) has completed.
  if (s == 0) pdl_trigger();
  pdl_wait();
  if (s == 0) {
    uint32_t e = epoch;
    if (e == 0) {
      e = *counter + ((mode & kTpPublish) ? 1u : 0u);
      if (mode & kTpPublish) *counter = e;
    }
    s_epoch = e;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  if ((mode & kTpPublish) && s < tp)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(publish_to.slot[s]), "r"(e)
                 : "memory");
  if (!(mode & kTpWait) || s >= tp) return;
  unsigned long long t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  const unsigned long long max_iters = timeout_ns / 64 + 4096;  // sleeps are >= ~100 ns
  for (unsigned long long it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(my_flags + s) : "memory");
    if (int32_t(v - e) >= 0) return;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > timeout_ns || it >= max_iters) {
      report(FA_DEVERR_TIMEOUT);
      return;
    }
    __nanosleep(128);
  }
}

}  // namespace fa
