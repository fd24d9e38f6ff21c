// Projection GEMMs around the attention call, on the 5th-generation tensor cores (tcgen05), with
// the work that follows each GEMM fused into its epilogue:
//
//   QKV:    [q | k | v] = x W^T (+ bias), per-head RMSNorm of q and k (optional), rotate-half
//           RoPE of q and k, q written token-major, k and v scattered straight into the paged
//           pool through slot_mapping. Replaces q/k/v_proj, q/k_norm, rope and write_kv of
//           CausalSelfAttention::forward (src/models/common/attention.rs:75-104).
//   o_proj: out = residual + attn W_o^T. Replaces o_proj (attention.rs:116) and the residual add
//           of DecoderLayer::forward (src/models/common/transformer.rs:37-38).
//
// GEMM: C[M, N] = A[M, K] B[N, K]^T, both operands K-major (row-major activations and
// (out, in) weights, as candle's Linear stores them). Persistent: one CTA per SM walks output
// tiles of 128 x BN. Warp 0 streams 128 x 64 A and BN x 64 B tiles by TMA (128-byte swizzle)
// through a kStages ring; warp 1 issues tcgen05.mma (M=128, N=BN, K=16, both operands in shared
// memory) into one of two TMEM accumulators; warps 2-5 (thread = output row) run the epilogue of
// tile i while the MMAs of tile i+1 accumulate into the other buffer.
//
// Every mbarrier wait is bounded; bad device data (slots, positions) sets a status bit and the
// affected row is skipped.
#pragma once

#include <cooperative_groups.h>

#include "tcgen05.cuh"

namespace fa {

constexpr int kGemmBK = 64;          // K per ring stage: one 128-byte swizzled row per operand row
constexpr int kGemmThreads = 192;    // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue

// AROWS = 64 (M <= 64 only: the split-K form, and the persistent form at BN = 128, e.g. the
// logits readback of a decode batch): the A stage holds 64 rows, so the ring takes 8 stages
// instead of 6 (more weight bytes in flight per SM; logits at 64 rows 187.1 -> 184.5 us). The M = 128 MMA still reads 128 A rows; rows
// 64-127 then fall on the same stage's B bytes and only feed accumulator rows >= 64, which the
// epilogue never stores. The kernel refuses (FA_DEVERR_LAUNCH, no work) a shape with M > 64.
template <int BN, int AROWS = 128>
struct GemmCfg {
  static_assert(BN == 128 || BN == 256, "BN is 128 or 256");
  static_assert(AROWS == 128 || (AROWS == 64 && BN == 128), "64-row A stages only at BN = 128");
  static constexpr int kStages = BN == 256 ? 4 : (AROWS == 64 ? 8 : 6);
  static constexpr int kABytes = AROWS * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int FULL = 0, EMPTY = kStages, AFULL = 2 * kStages, AEMPTY = AFULL + 2,
                       DRAIN = AEMPTY + 2, NBARS = DRAIN + 1;
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kMiscOff = kBarOff + NBARS * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;
};

struct GemmShape {
  int32_t M, N, K;
  int32_t tiles_m, tiles_n;
};

// ---- accumulator access (what the epilogues read) ------------------------------------------

// This thread's row of the tile's f32 accumulator in TMEM. ld32 is a warp-collective tcgen05.ld:
// every lane of the warp calls it with the same column.
struct TmemAcc {
  uint32_t taddr;  // TMEM address of (this warp's lane quadrant, column 0 of the tile)
  __device__ __forceinline__ void ld32(int col, float (&v)[32]) const {
    uint32_t r[32];
    tc::ld32(taddr + col, r);
    tc::wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
  }
};

// ---- epilogues (called by each epilogue thread for its row of one output tile) -------------

template <typename T>
__device__ __forceinline__ float to_f32(T x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(x);
  else return __half2float(x);
}

// 32 values -> 16 packed pairs -> two 256-bit stores.
template <typename T>
__device__ __forceinline__ void store32(T *dst, const float (&v)[32]) {
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) pk[e] = pack2<T>(v[2 * e], v[2 * e + 1]);
  st_global_v8(dst, pk);
  st_global_v8(dst + 16, pk + 8);
}

// 16 values -> 8 packed pairs -> one 256-bit store.
template <typename T>
__device__ __forceinline__ void store16(T *dst, const float (&v)[16]) {
  uint32_t pk[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) pk[e] = pack2<T>(v[2 * e], v[2 * e + 1]);
  st_global_v8(dst, pk);
}

template <typename T>
struct QkvEpilogue {
  T *q_out;                 // [M, num_heads, head_dim]
  T *k_cache, *v_cache;     // [num_blocks, num_kv_heads, block_size, head_dim]
  const T *bias;            // [N] or null
  const T *q_norm, *k_norm; // [head_dim] or null
  const float *rope_cos, *rope_sin;  // [max_position, head_dim / 2]
  const int32_t *positions, *slots;  // [M]
  float rms_eps;
  int32_t num_heads, num_kv_heads, head_dim, num_blocks, block_size, max_position;
  static constexpr bool kChunked = false;  // RoPE and the q/k norms need whole heads
  static constexpr bool kSplitUnits = true;  // the split-K form uses unit() below

  // Where this row's values of global head `gh` go (null: nothing to write), reporting bad
  // positions and slots; `pos` / `slot` are the row's.
  __device__ T *destination(int row, int gh, bool is_q, bool is_k, int pos, int slot,
                            const GemmShape &s) const {
    if (row >= s.M) return nullptr;
    if ((is_q || is_k) && !(pos >= 0 && pos < max_position)) {
      report(FA_DEVERR_POSITION);
      return nullptr;
    }
    if (is_q) return q_out + (size_t(row) * num_heads + gh) * head_dim;
    if (slot >= 0) {
      const int blk = slot / block_size, off = slot % block_size;
      if (blk < num_blocks) {
        const int kvh = gh - num_heads - (is_k ? 0 : num_kv_heads);
        return (is_k ? k_cache : v_cache) +
               ((size_t(blk) * num_kv_heads + kvh) * block_size + off) * head_dim;
      }
      report(FA_DEVERR_SLOT);
    } else if (slot < -1) {
      report(FA_DEVERR_SLOT);
    }
    return nullptr;
  }

  // Split-K form, for a tile whose few valid rows would leave most epilogue threads idle: one
  // unit = 16 rotate-half pairs (columns i..i+15 and i+d/2..) of one head of one row, BN / 32
  // units per row. The summed row sits in shared memory (acc.row), so a unit reads the whole
  // head for the norm itself. Same arithmetic, in the same order, as operator().
  template <int BN, class Acc>
  __device__ void unit(const Acc &acc, int row, int col0, int u, const GemmShape &s) const {
    const int half = head_dim / 2;
    const int per_head = half / 16;
    const int hl = u / per_head, i0 = (u % per_head) * 16;
    const int f0 = col0 + hl * head_dim;
    if (row >= s.M || f0 >= s.N) return;
    const int gh = f0 / head_dim;
    const bool is_q = gh < num_heads, is_k = !is_q && gh < num_heads + num_kv_heads;
    const int pos = positions[row], slot = slots[row];
    T *dst = destination(row, gh, is_q, is_k, pos, slot, s);
    if (dst == nullptr) return;
    const T *nw = is_q ? q_norm : (is_k ? k_norm : nullptr);
    const float *r = acc.row + hl * head_dim;
    float inv_rms = 1.f;
    if (nw) {
      float ss = 0.f;
      for (int c = 0; c < head_dim; c += 32)
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float x = r[c + e] + (bias ? to_f32(bias[f0 + c + e]) : 0.f);
          ss = fmaf(x, x, ss);
        }
      inv_rms = rsqrtf(ss / float(head_dim) + rms_eps);
    }
    float a[16], b[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      a[e] = r[i0 + e];
      b[e] = r[half + i0 + e];
      if (bias) {
        a[e] += to_f32(bias[f0 + i0 + e]);
        b[e] += to_f32(bias[f0 + half + i0 + e]);
      }
      if (nw) {
        a[e] *= inv_rms * to_f32(nw[i0 + e]);
        b[e] *= inv_rms * to_f32(nw[half + i0 + e]);
      }
    }
    if (is_q || is_k) {
      const float4 *cp = reinterpret_cast<const float4 *>(rope_cos + size_t(pos) * half + i0);
      const float4 *sp = reinterpret_cast<const float4 *>(rope_sin + size_t(pos) * half + i0);
#pragma unroll
      for (int e4 = 0; e4 < 4; ++e4) {
        const float4 c4 = cp[e4], s4 = sp[e4];
        const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int e = e4 * 4 + j;
          const float x1 = a[e], x2 = b[e];
          a[e] = x1 * cs[j] - x2 * sn[j];
          b[e] = x2 * cs[j] + x1 * sn[j];
        }
      }
    }
    store16<T>(dst + i0, a);
    store16<T>(dst + half + i0, b);
  }

  // One row (token) of a 128 x BN tile: BN / head_dim whole heads starting at column col0.
  template <int BN, class Acc>
  __device__ void operator()(const Acc &acc, int row, int col0, const GemmShape &s) const {
    const bool row_ok = row < s.M;
    const int half = head_dim / 2;
    int pos = 0, slot = -1;
    if (row_ok) {
      pos = positions[row];
      slot = slots[row];
    }
    for (int hl = 0; hl < BN / head_dim; ++hl) {
      const int f0 = col0 + hl * head_dim;  // warp-uniform
      if (f0 >= s.N) break;
      const int gh = f0 / head_dim;
      const bool is_q = gh < num_heads, is_k = !is_q && gh < num_heads + num_kv_heads;
      const T *nw = is_q ? q_norm : (is_k ? k_norm : nullptr);
      const int ta = hl * head_dim;  // accumulator column of this head
      // Destination row, or null when this row writes nothing for this head.
      T *dst = nullptr;
      bool rope_ok = true;
      if (row_ok && (is_q || is_k)) {
        rope_ok = pos >= 0 && pos < max_position;
        if (!rope_ok) report(FA_DEVERR_POSITION);
      }
      if (row_ok && rope_ok) {
        if (is_q) {
          dst = q_out + (size_t(row) * num_heads + gh) * head_dim;
        } else if (slot >= 0) {
          const int blk = slot / block_size, off = slot % block_size;
          if (blk < num_blocks) {
            const int kvh = gh - num_heads - (is_k ? 0 : num_kv_heads);
            dst = (is_k ? k_cache : v_cache) +
                  ((size_t(blk) * num_kv_heads + kvh) * block_size + off) * head_dim;
          } else {
            report(FA_DEVERR_SLOT);
          }
        } else if (slot < -1) {
          report(FA_DEVERR_SLOT);
        }
      }
      // RMSNorm over the head (after the bias, before RoPE: attention.rs:85-99).
      float inv_rms = 1.f;
      if (nw) {
        float ss = 0.f;
        for (int c = 0; c < head_dim / 32; ++c) {
          float v[32];
          acc.ld32(ta + c * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = v[e] + (bias ? to_f32(bias[f0 + c * 32 + e]) : 0.f);
            ss = fmaf(x, x, ss);
          }
        }
        inv_rms = rsqrtf(ss / float(head_dim) + rms_eps);
      }
      // Rotate-half RoPE pairs column i with column i + head_dim/2 (i < head_dim/2).
      for (int c = 0; c < half / 32; ++c) {
        float a[32], b[32];
        acc.ld32(ta + c * 32, a);
        acc.ld32(ta + half + c * 32, b);
        if (dst == nullptr) continue;
        const int i0 = c * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (bias) {
            a[e] += to_f32(bias[f0 + i0 + e]);
            b[e] += to_f32(bias[f0 + half + i0 + e]);
          }
          if (nw) {
            a[e] *= inv_rms * to_f32(nw[i0 + e]);
            b[e] *= inv_rms * to_f32(nw[half + i0 + e]);
          }
        }
        if (is_q || is_k) {
          const float4 *cp = reinterpret_cast<const float4 *>(rope_cos + size_t(pos) * half + i0);
          const float4 *sp = reinterpret_cast<const float4 *>(rope_sin + size_t(pos) * half + i0);
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 c4 = cp[e4], s4 = sp[e4];
            const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int e = e4 * 4 + j;
              const float x1 = a[e], x2 = b[e];
              a[e] = x1 * cs[j] - x2 * sn[j];
              b[e] = x2 * cs[j] + x1 * sn[j];
            }
          }
        }
        store32<T>(dst + i0, a);
        store32<T>(dst + half + i0, b);
      }
    }
  }
};

template <typename T>
struct ResidualEpilogue {
  T *out;                 // [M, N]
  const T *residual;      // [M, N] or null
  static constexpr bool kChunked = true;  // 32-column chunks are independent
  static constexpr bool kSplitUnits = false;

  __device__ void apply32(float (&v)[32], int row, int col, const GemmShape &s) const {
    const size_t base = size_t(row) * s.N + col;
    if (residual) {
      const uint4 *rp = reinterpret_cast<const uint4 *>(residual + base);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = rp[q];
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack2<T>(ww[j]);
          v[q * 8 + 2 * j] += f.x;
          v[q * 8 + 2 * j + 1] += f.y;
        }
      }
    }
    store32<T>(out + base, v);
  }

  template <int BN, class Acc>
  __device__ void operator()(const Acc &acc, int row, int col0, const GemmShape &s) const {
    const bool row_ok = row < s.M;
    for (int c = 0; c < BN / 32; ++c) {
      const int col = col0 + c * 32;  // warp-uniform
      if (col >= s.N) break;
      float v[32];
      acc.ld32(c * 32, v);
      if (row_ok) apply32(v, row, col, s);
    }
  }

  // Chunk c (32 columns) of a row whose accumulator is in shared memory (split-K path).
  template <class Acc>
  __device__ void chunk(const Acc &acc, int row, int col0, int c, const GemmShape &s) const {
    const int col = col0 + c * 32;
    if (row >= s.M || col >= s.N) return;
    float v[32];
    acc.ld32(c * 32, v);
    apply32(v, row, col, s);
  }
};

// f32 output, no other work: the logits of the lm_head projection (read back as f32 by the
// engine, engine.rs:221-222).
struct F32Epilogue {
  float *out;  // [M, N], N % 32 == 0, 16-byte aligned
  static constexpr bool kChunked = true;  // 32-column chunks are independent
  static constexpr bool kSplitUnits = false;

  __device__ void apply32(const float (&v)[32], int row, int col, const GemmShape &s) const {
    float4 *d = reinterpret_cast<float4 *>(out + size_t(row) * s.N + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) d[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }

  template <int BN, class Acc>
  __device__ void operator()(const Acc &acc, int row, int col0, const GemmShape &s) const {
    const bool row_ok = row < s.M;
    for (int c = 0; c < BN / 32; ++c) {
      const int col = col0 + c * 32;  // warp-uniform
      if (col >= s.N) break;
      float v[32];
      acc.ld32(c * 32, v);
      if (row_ok) apply32(v, row, col, s);
    }
  }

  // Chunk c (32 columns) of a row whose accumulator is in shared memory (split-K path).
  template <class Acc>
  __device__ void chunk(const Acc &acc, int row, int col0, int c, const GemmShape &s) const {
    const int col = col0 + c * 32;
    if (row >= s.M || col >= s.N) return;
    float v[32];
    acc.ld32(c * 32, v);
    apply32(v, row, col, s);
  }
};

// The final RMSNorm (CausalLM::forward, src/models/common/model.rs:56) of the last token of each
// sequence of a packed batch: the only rows whose logits the engine reads (engine.rs:221). One
// CTA per sequence; f32 math, one rounding to the model dtype (the GEMM operand). A sequence
// whose token range is empty or outside the batch gets a zero row and FA_DEVERR_SEQLEN.
constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    last_rows_norm_kernel(const T *hidden, const int32_t *cu_seqlens, int total_tokens,
                          const T *weight, float eps, int H, T *out) {
  __shared__ float s_red[kNormThreads / 32];
  const int seq = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) pdl_trigger();  // the lm_head GEMM may start loading weights
  const int a = cu_seqlens[seq], b = cu_seqlens[seq + 1];
  T *o = out + size_t(seq) * H;
  if (!(a >= 0 && b > a && b <= total_tokens)) {
    if (tid == 0) report(FA_DEVERR_SEQLEN);
    for (int i = tid; i < H; i += kNormThreads) o[i] = Elem<T>::from_f(0.f);
    return;
  }
  const T *x = hidden + size_t(b - 1) * H;
  float ss = 0.f;
  for (int i = tid; i < H; i += kNormThreads) {
    const float v = to_f32(x[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((tid & 31) == 0) s_red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += s_red[w];
  const float inv = rsqrtf(tot / float(H) + eps);
  for (int i = tid; i < H; i += kNormThreads) {
    const float wv = weight ? to_f32(weight[i]) : 1.f;
    o[i] = Elem<T>::from_f(to_f32(x[i]) * inv * wv);
  }
}

// ---- the persistent GEMM ---------------------------------------------------------------------

template <typename T, int BN, class Epi, int AROWS = 128>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_kernel(const __grid_constant__ GemmShape s, const __grid_constant__ Epi epi,
                   const __grid_constant__ CUtensorMap tm_a,
                   const __grid_constant__ CUtensorMap tm_b) {
  using C = GemmCfg<BN, AROWS>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tiles = s.tiles_m * s.tiles_n;
  const int num_k = (s.K + kGemmBK - 1) / kGemmBK;
  if (AROWS < 128 && s.M > AROWS) {  // uniform over the grid: every CTA leaves before any barrier
    if (tid == 0 && blockIdx.x == 0) report(FA_DEVERR_LAUNCH);
    return;
  }

  if (tid == 0) {
    for (int i = 0; i < C::NBARS; ++i)
      mbar_init(bar(i), (i == C::AEMPTY || i == C::AEMPTY + 1) ? 128 : 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(s_tmem), C::kTmemCols);
    tc::relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tmem = *s_tmem;
  if (tid == 0) pdl_trigger();  // the next kernel may start its prologue as SMs free up

  if (warp == 0) {
    // ================= TMA producer =================
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      // Weights do not depend on the preceding kernel: the first tile's first ring stages of B
      // are requested before waiting for it (programmatic dependent launch), A after.
      const int pre = blockIdx.x < tiles ? min(num_k, C::kStages) : 0;
      {
        const int n0 = blockIdx.x % s.tiles_n;
        for (int st = 0; st < pre; ++st) {
          mbar_arrive_expect_tx(bar(C::FULL + st), C::kStageBytes);
          tma_load_2d(sbase + st * C::kStageBytes + C::kABytes, &tm_b, bar(C::FULL + st),
                      st * kGemmBK, n0 * BN);
        }
      }
      pdl_wait();
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m = t / s.tiles_n, n = t % s.tiles_n;
        for (int kb = 0; kb < num_k; ++kb, ++it) {
          const int st = it % C::kStages;
          if (it >= C::kStages && !(ok = mbar_wait(bar(C::EMPTY + st), ((it / C::kStages) - 1) & 1)))
            break;
          const uint32_t a = sbase + st * C::kStageBytes;
          if (it >= pre) mbar_arrive_expect_tx(bar(C::FULL + st), C::kStageBytes);
          tma_load_2d(a, &tm_a, bar(C::FULL + st), kb * kGemmBK, m * 128);
          if (it >= pre) tma_load_2d(a + C::kABytes, &tm_b, bar(C::FULL + st), kb * kGemmBK, n * BN);
        }
      }
      if (!ok) report(FA_DEVERR_TIMEOUT);
    }
  } else if (warp == 1) {
    // ================= MMA issuer =================
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kBf16, 128, BN, false, false);
      int it = 0, tc_n = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc_n) {
        const int buf = tc_n & 1;
        if (tc_n >= 2 && !(ok = mbar_wait(bar(C::AEMPTY + buf), ((tc_n >> 1) - 1) & 1))) break;
        tc::fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < num_k; ++kb, ++it) {
          const int st = it % C::kStages;
          if (!(ok = mbar_wait(bar(C::FULL + st), (it / C::kStages) & 1))) break;
          tc::fence_after();
          const uint32_t a = sbase + st * C::kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk)
            tc::mma_ss(d, tc::sw128_desc(a + kk * 32, 16, 1024),
                       tc::sw128_desc(a + C::kABytes + kk * 32, 16, 1024), idesc,
                       (kb > 0 || kk > 0) ? 1u : 0u);
          tc::commit(bar(C::EMPTY + st));
        }
        if (!ok) break;
        tc::commit(bar(C::AFULL + buf));
      }
      if (!ok) report(FA_DEVERR_TIMEOUT);
      tc::commit(bar(C::DRAIN));  // every MMA issued above has completed once this arrives
      mbar_wait(bar(C::DRAIN), 0);
    }
  } else {
    // ================= epilogue: thread = output row of the tile =================
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    pdl_wait();  // the epilogue reads and writes memory the preceding kernel may use
    int tc_n = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tc_n) {
      const int buf = tc_n & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(C::AFULL + buf), (tc_n >> 1) & 1))) {
        if (lane == 0) report(FA_DEVERR_TIMEOUT);
        break;
      }
      tc::fence_after();
      const int m = t / s.tiles_n, n = t % s.tiles_n;
      epi.template operator()<BN>(TmemAcc{tmem + lane_off + buf * BN}, m * 128 + q * 32 + lane,
                                  n * BN, s);
      tc::fence_before();
      mbar_arrive(bar(C::AEMPTY + buf));
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::dealloc(tmem, C::kTmemCols);
  }
}

// ---- split-K over a thread-block cluster (small M) --------------------------------------------
//
// When the output has too few 128 x BN tiles to occupy the GPU (decode: 64 tokens), each tile is
// computed by a cluster of S CTAs that split K. Each CTA accumulates its K slice in TMEM, copies
// the f32 partial to its own shared memory, and signals every CTA of the cluster; CTA r then
// sums rows [r*R, (r+1)*R) of the tile's valid rows (R = ceil(valid / S)) over all S partials
// through distributed shared memory, once, with plain loads the compiler can overlap, writes the
// sums back over those rows of its own partial (no other CTA reads them there), and runs the
// epilogue on them from local shared memory. No global workspace; the waits between CTAs are
// bounded mbarrier waits.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster; orders shared-memory accesses across the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (the arrivals come from other CTAs).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t phase) {
  if (mbar_try_wait_cluster(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait_cluster(bar, phase)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

constexpr int kSplitMaxRanks = 8;

// One row of the tile, already summed over the cluster's partials, in this CTA's shared memory.
struct LocalAcc {
  const float *row;
  __device__ __forceinline__ void ld32(int col, float (&v)[32]) const {
    const float4 *p = reinterpret_cast<const float4 *>(row + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x = p[q];
      v[4 * q] = x.x;
      v[4 * q + 1] = x.y;
      v[4 * q + 2] = x.z;
      v[4 * q + 3] = x.w;
    }
  }
};

template <typename T, int BN, class Epi, int AROWS = 128>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_splitk_kernel(const __grid_constant__ GemmShape s, const __grid_constant__ Epi epi,
                          const __grid_constant__ CUtensorMap tm_a,
                          const __grid_constant__ CUtensorMap tm_b) {
  using C = GemmCfg<BN, AROWS>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kPitch = BN + 4;  // f32 row pitch of the partial (bank-conflict padding)
  static_assert(128 * kPitch * 4 <= C::kBarOff, "partial must fit in the operand ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint32_t *s_tmem = reinterpret_cast<uint32_t *>(smem + C::kMiscOff);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank(), nranks = cluster_nctarank();
  const int tile = int(cluster_id_x());
  const int m = tile / s.tiles_n, n = tile % s.tiles_n;
  const int num_k = (s.K + kGemmBK - 1) / kGemmBK;
  const int kb0 = int(int64_t(num_k) * rank / nranks), kb1 = int(int64_t(num_k) * (rank + 1) / nranks);
  // Barriers: FULL/EMPTY ring, AFULL (partial ready in TMEM), and AEMPTY reused as "every CTA's
  // partial is in its shared memory" (128 epilogue threads x nranks arrivals).
  const int PREADY = C::AEMPTY;
  if (AROWS < 128 && s.M > AROWS) {  // uniform over the grid: every CTA leaves before any barrier
    if (tid == 0 && blockIdx.x == 0) report(FA_DEVERR_LAUNCH);
    return;
  }

  if (tid == 0) {
    for (int i = 0; i < C::NBARS; ++i) mbar_init(bar(i), i == PREADY ? 128 * int(nranks) : 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::alloc(smem_u32(s_tmem), C::kTmemCols);
    tc::relinquish();
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  cluster_sync();  // every CTA's barriers are initialised before any remote arrive
  const uint32_t tmem = *s_tmem;
  if (tid == 0) pdl_trigger();  // the next kernel may start its prologue as SMs free up

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      // Weights do not depend on the preceding kernel: the first ring stages of B are requested
      // before waiting for it (programmatic dependent launch), A after.
      const int pre = min(kb1 - kb0, C::kStages);
      for (int st = 0; st < pre; ++st) {
        mbar_arrive_expect_tx(bar(C::FULL + st), C::kStageBytes);
        tma_load_2d(sbase + st * C::kStageBytes + C::kABytes, &tm_b, bar(C::FULL + st),
                    (kb0 + st) * kGemmBK, n * BN);
      }
      // The rest of this CTA's weight slice goes to L2 meanwhile (the decode-batch GEMMs this
      // kernel serves stream weights that are read exactly once).
      for (int kb = kb0 + pre; kb < kb1; ++kb) tma_prefetch_l2_2d(&tm_b, kb * kGemmBK, n * BN);
      pdl_wait();
      bool ok = true;
      for (int kb = kb0, it = 0; kb < kb1 && ok; ++kb, ++it) {
        const int st = it % C::kStages;
        if (it >= C::kStages && !(ok = mbar_wait(bar(C::EMPTY + st), ((it / C::kStages) - 1) & 1)))
          break;
        const uint32_t a = sbase + st * C::kStageBytes;
        if (it >= pre) mbar_arrive_expect_tx(bar(C::FULL + st), C::kStageBytes);
        tma_load_2d(a, &tm_a, bar(C::FULL + st), kb * kGemmBK, m * 128);
        if (it >= pre) tma_load_2d(a + C::kABytes, &tm_b, bar(C::FULL + st), kb * kGemmBK, n * BN);
      }
      if (!ok) report(FA_DEVERR_TIMEOUT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16(kBf16, 128, BN, false, false);
      bool ok = true;
      for (int kb = kb0, it = 0; kb < kb1; ++kb, ++it) {
        const int st = it % C::kStages;
        if (!(ok = mbar_wait(bar(C::FULL + st), (it / C::kStages) & 1))) break;
        tc::fence_after();
        const uint32_t a = sbase + st * C::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk)
          tc::mma_ss(tmem, tc::sw128_desc(a + kk * 32, 16, 1024),
                     tc::sw128_desc(a + C::kABytes + kk * 32, 16, 1024), idesc,
                     (kb > kb0 || kk > 0) ? 1u : 0u);
        tc::commit(bar(C::EMPTY + st));
      }
      if (!ok) report(FA_DEVERR_TIMEOUT);
      tc::commit(bar(C::AFULL));
      tc::commit(bar(C::DRAIN));  // every MMA issued above has completed once this arrives
      mbar_wait(bar(C::DRAIN), 0);
    }
  } else {
    const int q = warp & 3;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    const int r = q * 32 + lane;  // tile row of this thread's TMEM lane
    float *part = reinterpret_cast<float *>(smem);
    pdl_wait();  // the epilogue reads and writes memory the preceding kernel may use
    bool ok = __all_sync(0xffffffffu, mbar_wait(bar(C::AFULL), 0));
    if (ok) {
      tc::fence_after();
      // This CTA's partial -> shared memory (the operand ring is idle: every MMA has completed).
      const TmemAcc own{tmem + lane_off};
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        own.ld32(c * 32, v);
        float4 *dst = reinterpret_cast<float4 *>(part + r * kPitch + c * 32);
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
      }
    } else if (lane == 0) {
      report(FA_DEVERR_TIMEOUT);
    }
    tc::fence_before();
    // Tell every CTA of the cluster (this one included) that this thread's row is in place.
    for (uint32_t p = 0; p < nranks; ++p) mbar_arrive_remote(map_to_rank(bar(PREADY), p));
    ok = mbar_wait_cluster(bar(PREADY), 0) && ok;
    if (!ok) report(FA_DEVERR_TIMEOUT);
    // Rows [rank*R, rank*R + R) of the tile's valid rows: summed over all partials into this
    // CTA's own copy of those rows by all 128 epilogue threads (one float4 of one row each, the
    // loads from every rank independent), then the epilogue reads them locally. Every epilogue
    // thread reaches the named barrier, whatever its wait returned.
    const int valid = min(128, s.M - m * 128);
    const int R = (valid + int(nranks) - 1) / int(nranks);
    const int t = tid - 64;  // 0..127 over the four epilogue warps
    const int row0 = int(rank) * R;
    const int rows = max(0, min(R, valid - row0));
    if (ok) {
      namespace cg = cooperative_groups;
      cg::cluster_group cluster = cg::this_cluster();
      const float4 *src[kSplitMaxRanks];
#pragma unroll
      for (int p = 0; p < kSplitMaxRanks; ++p)
        src[p] = reinterpret_cast<const float4 *>(
            cluster.map_shared_rank(part, uint32_t(p) < nranks ? uint32_t(p) : 0u));
      float4 *own4 = reinterpret_cast<float4 *>(part);
      constexpr int kUnits = BN / 4;  // float4 per row
      for (int u = t; u < rows * kUnits; u += 128) {
        const int idx = (row0 + u / kUnits) * (kPitch / 4) + u % kUnits;
        float4 sum = src[0][idx];
#pragma unroll
        for (int p = 1; p < kSplitMaxRanks; ++p) {
          if (uint32_t(p) >= nranks) break;
          const float4 x = src[p][idx];
          sum.x += x.x;
          sum.y += x.y;
          sum.z += x.z;
          sum.w += x.w;
        }
        own4[idx] = sum;
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
    if (ok) {
      if constexpr (Epi::kChunked) {
        // One 32-column chunk per thread: every epilogue thread works, not one per row.
        constexpr int kChunks = BN / 32;
        for (int u = t; u < rows * kChunks; u += 128) {
          const int row = row0 + u / kChunks;
          epi.chunk(LocalAcc{part + row * kPitch}, m * 128 + row, n * BN, u % kChunks, s);
        }
      } else if constexpr (Epi::kSplitUnits) {
        // BN / 32 units per row (each 16 rotate-half pairs of one head) over all 128 threads.
        constexpr int kUnits = BN / 32;
        for (int u = t; u < rows * kUnits; u += 128) {
          const int row = row0 + u / kUnits;
          epi.template unit<BN>(LocalAcc{part + row * kPitch}, m * 128 + row, n * BN,
                                u % kUnits, s);
        }
      } else if (t < rows) {
        const int row = row0 + t;
        epi.template operator()<BN>(LocalAcc{part + row * kPitch}, m * 128 + row, n * BN, s);
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after();
    tc::dealloc(tmem, C::kTmemCols);
  }
  cluster_sync();  // no CTA leaves while another may still read its partial
}

}  // namespace fa
