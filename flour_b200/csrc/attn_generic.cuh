// Generic paged attention: any element type, any head_dim <= 256, any block_size <= 1024,
// any n_rep, any number of query tokens per sequence. One CTA of 16 warps per (query token,
// query head); the warps fold interleaved blocks and merge their states at the end.
//
// This is the per-row form of backend::cpu::paged_attention (src/backend/cpu.rs:57-112): the
// sequence's KV is walked block by block in logical order (KvCache::gather_blocks,
// src/models/common/cache.rs:83-96) and folded with the same online softmax, in f32, with
// accurate expf, so f32 pools match the reference to ~1e-6. The bf16/f16 fast paths live in
// decode_sm100.cuh / prefill_sm100.cuh; this kernel serves f32 pools and shapes those do not
// cover (e.g. the reference's unit-test shapes: head_dim 4, block sizes 2-4).
#pragma once

#include "fa_common.cuh"

namespace fa {

struct GenericParams {
  const void *q;
  void *out;
  const void *k_cache;
  const void *v_cache;
  const int32_t *cu_seqlens_q;  // [num_seqs+1]; nullptr means one query per sequence (decode)
  const int32_t *context_lens;
  const int32_t *block_tables;
  int32_t max_blocks_per_seq;
  int32_t num_seqs;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t n_rep;
  int32_t head_dim;
  int32_t block_size;
  int32_t num_blocks;
  int32_t total_q;
  float scale;
  int32_t ref_scores;  // 1: the reference's dtype rounding of the scores (ref_score)
};

constexpr int kGenericWarps = 16;
constexpr int kGenericThreads = kGenericWarps * 32;
constexpr int kGenericMaxDim = 256;
constexpr int kSmallRows = 16;  // register path: blocks of <= 16 rows, head_dim <= 64

// Shared memory: q [kGenericMaxDim] | per-warp probabilities [kGenericWarps][block_size] |
// per-warp partial accumulators [kGenericWarps][kGenericMaxDim] | per-warp max and sum.
__host__ __device__ constexpr size_t generic_smem_floats(int block_size) {
  return size_t(kGenericMaxDim) + size_t(kGenericWarps) * block_size +
         size_t(kGenericWarps) * kGenericMaxDim + 2 * kGenericWarps;
}

// Each warp folds its own blocks (b = warp, warp + 16, ...) with the reference's block-wise
// online softmax (scores of the block, block max, one correction, p = exp(s - max), sum, then
// acc = acc * corr + sum_j p_j v_j), lanes over the block's rows for the scores and over
// head_dim for the accumulation; the 16 partial states are merged at the end. Only blocks up to
// the last visible position are folded, so every folded block holds at least one visible key.
template <typename T>
__global__ void __launch_bounds__(kGenericThreads, 1) generic_attn_kernel(const GenericParams p) {
  extern __shared__ float gsm[];
  const int D = p.head_dim, BS = p.block_size;
  auto score = [&](float dot) { return p.ref_scores ? ref_score<T>(dot, p.scale) : dot * p.scale; };
  float *qs = gsm;                                        // [D]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *pw = gsm + kGenericMaxDim + size_t(warp) * BS;   // this warp's probabilities [BS]
  float *accs = gsm + kGenericMaxDim + size_t(kGenericWarps) * BS;  // [W][kGenericMaxDim]
  float *ms = accs + kGenericWarps * kGenericMaxDim;      // [W]
  float *ls = ms + kGenericWarps;                         // [W]
  const int qi = blockIdx.x, h = blockIdx.y;
  const size_t orow = (size_t(qi) * p.num_heads + h) * D;
  T *out = static_cast<T *>(p.out);

  // Locate the sequence of query token qi.
  int s, i, sq;
  if (p.cu_seqlens_q == nullptr) {
    s = qi; i = 0; sq = 1;
  } else {
    int lo = 0, hi = p.num_seqs;  // last s with cu[s] <= qi
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (p.cu_seqlens_q[mid] <= qi) lo = mid; else hi = mid;
    }
    s = lo;
    const int q0 = p.cu_seqlens_q[s], q1 = p.cu_seqlens_q[s + 1];
    if (q0 > qi || q1 <= qi || q1 > p.total_q) {
      if (tid == 0) report(FA_DEVERR_SEQLEN);
      for (int x = tid; x < D; x += kGenericThreads) out[orow + x] = Elem<T>::from_f(0.f);
      return;
    }
    i = qi - q0; sq = q1 - q0;
  }
  const int L = p.context_lens[s];
  if (L < sq || int64_t(L) > int64_t(p.max_blocks_per_seq) * BS) {
    if (tid == 0) report(FA_DEVERR_CONTEXT);
    for (int x = tid; x < D; x += kGenericThreads) out[orow + x] = Elem<T>::from_f(0.f);
    return;
  }
  const int offset = L - sq;     // cpu.rs:68
  const int limit = offset + i;  // this query sees keys j <= limit (cpu.rs:87-94)
  const int kh = h / p.n_rep;
  const T *qp = static_cast<const T *>(p.q) + orow;
  for (int x = tid; x < D; x += kGenericThreads) qs[x] = Elem<T>::to_f(qp[x]);
  __syncthreads();

  const T *kc = static_cast<const T *>(p.k_cache);
  const T *vc = static_cast<const T *>(p.v_cache);
  constexpr int kPerLane = kGenericMaxDim / 32;
  float acc[kPerLane];
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) acc[k] = 0.f;
  float m = neg_inf(), l = 0.f;
  const int nb = limit / BS + 1;  // blocks holding a visible key
  const int32_t *table = p.block_tables + size_t(s) * p.max_blocks_per_seq;
  bool bad_id = false;
  // This lane's query values: head_dim element lane + 32 k.
  float qv[kPerLane];
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) qv[k] = lane + 32 * k < D ? qs[lane + 32 * k] : 0.f;
  // Blocks of <= 16 rows with head_dim <= 64 (e.g. Qwen2.5-0.5B's f32 pool) take a register
  // path: the whole K and V block is loaded in one round trip, and the next block's id is
  // fetched while this one is folded.
  const bool small = BS <= kSmallRows && D <= 64;
  int next_id = warp < nb ? table[warp] : 0;
  for (int b = warp; b < nb; b += kGenericWarps) {
    int id = next_id;
    if (b + kGenericWarps < nb) next_id = table[b + kGenericWarps];
    if (uint32_t(id) >= uint32_t(p.num_blocks)) { bad_id = true; id = 0; }
    const int kv_start = b * BS;
    const int bn = min(BS, L - kv_start);
    const size_t base = (size_t(id) * p.num_kv_heads + kh) * BS * size_t(D);
    if (small) {
      float kr[kSmallRows][2], vr[kSmallRows][2];
#pragma unroll
      for (int j = 0; j < kSmallRows; ++j)
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const bool in = j < bn && lane + 32 * k < D;
          const size_t off = base + size_t(j) * D + lane + 32 * k;
          kr[j][k] = in ? Elem<T>::to_f(kc[off]) : 0.f;
          vr[j][k] = in ? Elem<T>::to_f(vc[off]) : 0.f;
        }
      float sc[kSmallRows];
#pragma unroll
      for (int j = 0; j < kSmallRows; ++j) sc[j] = fmaf(qv[0], kr[j][0], qv[1] * kr[j][1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < kSmallRows; ++j) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], o);
      // Every lane holds every score (the xor tree gives bit-identical sums), so the fold below
      // runs redundantly per lane with no shared-memory round trip.
      float bmax = neg_inf();
#pragma unroll
      for (int j = 0; j < kSmallRows; ++j) {
        sc[j] = (j < bn && kv_start + j <= limit) ? score(sc[j]) : neg_inf();
        bmax = fmaxf(bmax, sc[j]);
      }
      const float new_max = fmaxf(m, bmax);
      const float corr = expf(m - new_max);
      float psum = 0.f;
#pragma unroll
      for (int k = 0; k < 2; ++k) acc[k] *= corr;
#pragma unroll
      for (int j = 0; j < kSmallRows; ++j) {
        const float pj = j < bn ? expf(sc[j] - new_max) : 0.f;
        psum += pj;
#pragma unroll
        for (int k = 0; k < 2; ++k) acc[k] = fmaf(pj, vr[j][k], acc[k]);
      }
      l = l * corr + psum;
      m = new_max;
      continue;
    }
    // Scores of this block (cpu.rs:84-94): lanes over head_dim (coalesced row loads), four rows
    // in flight, each dot product completed by a warp all-reduce.
    float bmax = neg_inf();
    for (int j0 = 0; j0 < bn; j0 += 4) {
      float dot[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        dot[r] = 0.f;
        if (j0 + r < bn) {
          const T *kr = kc + base + size_t(j0 + r) * D;
#pragma unroll
          for (int k = 0; k < kPerLane; ++k)
            if (lane + 32 * k < D) dot[r] = fmaf(qv[k], Elem<T>::to_f(kr[lane + 32 * k]), dot[r]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < 4; ++r) dot[r] += __shfl_xor_sync(0xffffffffu, dot[r], o);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (j0 + r < bn) {
          const float sc = (kv_start + j0 + r > limit) ? neg_inf() : score(dot[r]);
          if (lane == 0) pw[j0 + r] = sc;
          bmax = fmaxf(bmax, sc);
        }
      }
    }
    __syncwarp();
    // Fold (cpu.rs:96-105): bmax is finite (row kv_start <= limit is visible).
    const float new_max = fmaxf(m, bmax);
    const float corr = expf(m - new_max);
    float psum = 0.f;
    for (int j = lane; j < bn; j += 32) {
      const float pj = expf(pw[j] - new_max);
      pw[j] = pj;
      psum += pj;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    __syncwarp();
#pragma unroll
    for (int k = 0; k < kPerLane; ++k) acc[k] *= corr;
#pragma unroll 4
    for (int j = 0; j < bn; ++j) {
      const float pj = pw[j];
      const T *vr = vc + base + size_t(j) * D;
#pragma unroll
      for (int k = 0; k < kPerLane; ++k)
        if (lane + 32 * k < D) acc[k] = fmaf(pj, Elem<T>::to_f(vr[lane + 32 * k]), acc[k]);
    }
    l = l * corr + psum;
    m = new_max;
    __syncwarp();
  }
  if (bad_id) report(FA_DEVERR_BLOCK_ID);
  // Merge the warps' states; warps without blocks hold m = -inf and contribute nothing.
#pragma unroll
  for (int k = 0; k < kPerLane; ++k)
    if (lane + 32 * k < D) accs[warp * kGenericMaxDim + lane + 32 * k] = acc[k];
  if (lane == 0) {
    ms[warp] = m;
    ls[warp] = l;
  }
  __syncthreads();
  float M = neg_inf();
#pragma unroll
  for (int w = 0; w < kGenericWarps; ++w) M = fmaxf(M, ms[w]);
  float wsum = 0.f;
#pragma unroll
  for (int w = 0; w < kGenericWarps; ++w)
    if (ms[w] != neg_inf()) wsum += expf(ms[w] - M) * ls[w];
  for (int x = tid; x < D; x += kGenericThreads) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kGenericWarps; ++w)
      if (ms[w] != neg_inf()) o += expf(ms[w] - M) * accs[w * kGenericMaxDim + x];
    out[orow + x] = Elem<T>::from_f(o / wsum);  // cpu.rs:111: acc / running_sum, cast to q's dtype
  }
}

}  // namespace fa
