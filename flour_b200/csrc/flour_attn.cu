// C ABI of libflour_attn.so: host-side validation, launch planning and dispatch to the
// sm_100a kernels. See include/flour_attn.h for the contract of every entry point.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <unordered_map>

#include "attn_generic.cuh"
#include "cache_ops.cuh"
#include "decode_sm100.cuh"
#include "gemm_sm100.cuh"
#include "prefill_sm100.cuh"
#include "flour_attn.h"

namespace {

thread_local char g_msg[512];

fa_status fail(fa_status st, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return st;
}

fa_status ok() {
  g_msg[0] = '\0';
  return FA_OK;
}

fa_status check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

int dtype_size(int32_t dt) { return dt == FA_F32 ? 4 : 2; }

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

fa_status check_layer(const fa_kv_layer *L, const char *who) {
  if (!L) return fail(FA_EINVAL, "%s: layer is NULL", who);
  if (!L->k_cache || !L->v_cache) return fail(FA_EINVAL, "%s: k_cache/v_cache is NULL", who);
  if (L->dtype != FA_F32 && L->dtype != FA_BF16 && L->dtype != FA_F16)
    return fail(FA_EINVAL, "%s: unknown dtype %d", who, L->dtype);
  if (L->num_blocks <= 0 || L->num_kv_heads <= 0 || L->block_size <= 0 || L->head_dim <= 0)
    return fail(FA_EINVAL, "%s: layer dims must be positive (blocks=%d kv_heads=%d bs=%d d=%d)",
                who, L->num_blocks, L->num_kv_heads, L->block_size, L->head_dim);
  return FA_OK;
}

// ---- tensor maps ----------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

fa_status get_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(FA_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return FA_OK;
}

// 2-D map over one K or V slab viewed as [rows = num_blocks*kv_heads*block_size, head_dim],
// box = 16 rows x 64 elements (128 B), 128-byte swizzle.
fa_status make_page_map(CUtensorMap *map, void *base, int64_t rows, int head_dim, int32_t dt) {
  if (fa_status s = get_encoder(); s != FA_OK) return s;
  const CUtensorMapDataType t =
      dt == FA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {cuuint64_t(head_dim), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(head_dim) * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, t, 2, base, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return FA_OK;
}

// 3-D map over packed queries [total_q, num_heads, 128] for the prefill kernel: one box is the
// n_rep heads of one KV group for tq consecutive tokens, 64 values of head_dim wide.
fa_status make_q_map(CUtensorMap *map, const void *q, int total_q, int num_heads, int n_rep, int tq,
                     int32_t dt) {
  if (fa_status s = get_encoder(); s != FA_OK) return s;
  const CUtensorMapDataType t =
      dt == FA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {128, cuuint64_t(num_heads), cuuint64_t(total_q)};
  cuuint64_t strides[2] = {256, cuuint64_t(num_heads) * 256};
  cuuint32_t box[3] = {64, cuuint32_t(n_rep), cuuint32_t(tq)};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, t, 3, const_cast<void *>(q), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ECUDA, "cuTensorMapEncodeTiled (queries) failed (%d)", int(r));
  return FA_OK;
}

// ---- decode planning --------------------------------------------------------------------

constexpr int kSmCount = 148;
// The split plan's CTA target: 12 per SM (see plan_decode). Three decode CTAs are resident per
// SM (2-stage rings), so this is four resident waves.
constexpr int kDecodeCtasPerSmTarget = 12;

struct DecodePlan {
  int pages_per_split = 0;
  int max_splits = 0;
};

// Split the context so that about 12 CTAs per SM cover the whole GPU, with at least 32 pages per
// split (8 per warp) and at most kDecodeMaxPagesPerSplit. That target measured best on B200 for
// C2 (U[512, 4096] contexts) with two resident CTAs per SM (six waves: four left a ragged last
// wave, eight or more paid more per-split overhead than they saved), and kept its edge once three
// became resident (C2 6015 -> 6185 GB/s; a 3-per-SM target of 18 CTAs per SM reached only 6090).
// The 32-page floor matters for small batches of short contexts, where the target would cut
// splits of 16 pages whose fixed per-CTA cost dominates (59 sequences of 1419 tokens, Qwen2-7B
// heads: 54.7 -> 45.0 us; C2 unchanged).
bool plan_decode(int num_seqs, int num_kv_heads, int max_context_len, DecodePlan *out) {
  const int max_pages = (max_context_len + fa::kPage - 1) / fa::kPage;
  const long units = long(num_seqs) * num_kv_heads;
  const long target = long(kSmCount) * kDecodeCtasPerSmTarget;
  const long want = std::max(1L, (target + units - 1) / units);
  int pps = int((max_pages + want - 1) / want);
  pps = std::max(pps, 32);
  pps = (pps + 3) / 4 * 4;
  pps = std::min(pps, fa::kDecodeMaxPagesPerSplit);
  const int splits = (max_pages + pps - 1) / pps;
  if (splits > fa::kDecodeMaxSplits) return false;
  out->pages_per_split = pps;
  out->max_splits = std::max(splits, 1);
  return true;
}

struct DecodeWorkspace {
  size_t counters_off, lse_off, o_off, bytes;
};

DecodeWorkspace decode_workspace_layout(int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                                        const DecodePlan &plan) {
  auto r256 = [](size_t x) { return (x + 255) / 256 * 256; };
  DecodeWorkspace w{};
  if (plan.max_splits <= 1) return w;
  w.counters_off = 0;
  w.lse_off = r256(size_t(num_seqs) * num_kv_heads * 4);
  w.o_off = w.lse_off + r256(size_t(num_seqs) * num_heads * plan.max_splits * 4);
  w.bytes = w.o_off + size_t(num_seqs) * num_heads * plan.max_splits * head_dim * 4;
  return w;
}

bool decode_fast_path(const fa_kv_layer *L, int n_rep, const void *q, const void *out) {
  return (L->dtype == FA_BF16 || L->dtype == FA_F16) && L->block_size == fa::kPage &&
         (L->head_dim == 64 || L->head_dim == 128) && n_rep >= 1 && n_rep <= 8 &&
         int64_t(L->num_blocks) * L->num_kv_heads * L->block_size < (int64_t(1) << 31) &&
         aligned(L->k_cache, 16) && aligned(L->v_cache, 16) && aligned(q, 16) &&
         aligned(out, 16);
}

template <typename T, int HD, int NSTAGE>
fa_status launch_decode_t(const fa::DecodeParams &p, const CUtensorMap &tk, const CUtensorMap &tv,
                          cudaStream_t stream) {
  using S = fa::DecodeSmem<HD, NSTAGE>;
  auto kern = fa::paged_decode_kernel<T, HD, NSTAGE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kAlloc);
  if (e != cudaSuccess) return fail(FA_ECUDA, "decode: set smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.max_splits, p.num_kv_heads, p.num_seqs);
  cfg.blockDim = dim3(fa::kDecodeThreads);
  cfg.dynamicSmemBytes = S::kAlloc;
  cfg.stream = stream;
  // Programmatic dependent launch: the CTAs may start while the preceding kernel finishes and
  // wait for it (griddepcontrol.wait) before touching any input, workspace or output.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p, tk, tv);
  if (e != cudaSuccess) return fail(FA_ECUDA, "paged_decode: launch: %s", cudaGetErrorString(e));
  return check_launch("paged_decode");
}

// Two ring stages per warp keep each decode CTA at 66 KB of shared memory, so three are resident
// per SM (with three stages only two fit): the same pages in flight per SM, and a third CTA's
// streaming hides the others' prologues and split-K merges (C2 6015 -> 6185 GB/s; C5's 59-sequence
// decode 38.2 -> 35.2 us per layer).
constexpr int kDecodeStages = 2;

// Split-K merge tickets must be zero when a decode launch starts. Every launch returns its own
// tickets to zero, but a caller workspace reused with another shape may hold split-K partials
// where the new tickets go (a launch's partials start right after its own tickets). Per
// workspace base pointer the library keeps:
//   clean:    a prefix that is zero whenever the next launch starts;
//   captured: the smallest ticket region of any launch recorded into a CUDA graph. A replay can
//             come at any time and leaves partials from that offset on, so `clean` never rises
//             above it.
// A launch with a smaller ticket region lowers `clean` to its own (its partials follow); one
// that reaches past `clean` zeroes the difference first, after which (when that memset runs
// eagerly, not into a graph) the prefix is clean up to its region, or to `captured`.
struct TicketState {
  size_t clean;
  size_t captured;
};
std::mutex g_ticket_mu;
std::unordered_map<uintptr_t, TicketState> g_ticket_state;

fa_status zero_stale_tickets(void *ws, size_t ticket_bytes, cudaStream_t stream) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess)
    return fail(FA_ECUDA, "decode: cudaStreamIsCapturing failed");
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(g_ticket_mu);
  const TicketState init{ticket_bytes, capturing ? ticket_bytes : SIZE_MAX};
  const auto [it, fresh] = g_ticket_state.try_emplace(reinterpret_cast<uintptr_t>(ws), init);
  if (fresh) return FA_OK;  // a workspace is zero-filled before its first use
  TicketState &s = it->second;
  if (capturing) s.captured = std::min(s.captured, ticket_bytes);
  if (ticket_bytes <= s.clean) {
    s.clean = ticket_bytes;
    return FA_OK;
  }
  const cudaError_t e =
      cudaMemsetAsync(static_cast<char *>(ws) + s.clean, 0, ticket_bytes - s.clean, stream);
  if (e != cudaSuccess) return fail(FA_ECUDA, "decode: zeroing merge tickets: %s", cudaGetErrorString(e));
  if (!capturing) s.clean = std::min(ticket_bytes, s.captured);
  return FA_OK;
}

// The new tokens' K/V of a fused append (fa_paged_decode_append).
struct AppendArgs {
  const void *key, *value;
  int64_t k_token, k_head, v_token, v_head;  // strides in elements
};

fa_status launch_decode(const fa_kv_layer *L, const void *q, void *out, const int32_t *ctx,
                        const int32_t *tables, int max_blocks, int num_seqs, int num_heads,
                        int n_rep, int max_context_len, float scale, int score_flow, void *ws,
                        size_t ws_bytes, cudaStream_t stream, const fa_tp_group *tp = nullptr,
                        bool caller_workspace = true, const AppendArgs *app = nullptr) {
  DecodePlan plan;
  if (!plan_decode(num_seqs, L->num_kv_heads, max_context_len, &plan))
    return fail(FA_EUNSUPPORTED, "decode: context of %d tokens needs more than %d splits",
                max_context_len, fa::kDecodeMaxSplits);
  const DecodeWorkspace w =
      decode_workspace_layout(num_seqs, num_heads, L->num_kv_heads, L->head_dim, plan);
  if (w.bytes > 0) {
    if (!ws) return fail(FA_EINVAL, "decode: workspace is NULL but %zu bytes are needed", w.bytes);
    if (ws_bytes < w.bytes)
      return fail(FA_ERANGE, "decode: workspace of %zu bytes, %zu needed", ws_bytes, w.bytes);
    if (!aligned(ws, 256)) return fail(FA_EINVAL, "decode: workspace must be 256-byte aligned");
    if (caller_workspace)
      if (fa_status s = zero_stale_tickets(ws, w.lse_off, stream); s != FA_OK) return s;
  }
  fa::DecodeParams p{};
  p.q = q;
  p.out = out;
  p.context_lens = ctx;
  p.block_tables = tables;
  char *wsb = static_cast<char *>(ws);
  p.counters = w.bytes ? reinterpret_cast<int32_t *>(wsb + w.counters_off) : nullptr;
  p.part_lse = w.bytes ? reinterpret_cast<float *>(wsb + w.lse_off) : nullptr;
  p.part_o = w.bytes ? reinterpret_cast<float *>(wsb + w.o_off) : nullptr;
  p.max_blocks_per_seq = max_blocks;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = L->num_kv_heads;
  p.n_rep = n_rep;
  p.num_blocks = L->num_blocks;
  p.pages_per_split = plan.pages_per_split;
  p.max_splits = plan.max_splits;
  p.max_context_len = max_context_len;
  p.scale_log2 = scale * fa::kLog2e;
  p.scale = scale;
  p.ref_scores = score_flow == FA_SCORES_REFERENCE;
  if (tp) {  // head-sharded: every rank's buffer, at this rank's head offset
    p.n_outs = tp->tp;
    p.out_heads = tp->tp * num_heads;
    p.out_head0 = tp->rank * num_heads;
    for (int r = 0; r < tp->tp; ++r) p.outs[r] = tp->out[r];
  }
  if (app) {
    p.new_k = app->key;
    p.new_v = app->value;
    p.nk_token = app->k_token;
    p.nk_head = app->k_head;
    p.nv_token = app->v_token;
    p.nv_head = app->v_head;
    p.k_pool = L->k_cache;
    p.v_pool = L->v_cache;
  }
  const int64_t rows = int64_t(L->num_blocks) * L->num_kv_heads * L->block_size;
  CUtensorMap tk, tv;
  if (fa_status s = make_page_map(&tk, L->k_cache, rows, L->head_dim, L->dtype); s != FA_OK) return s;
  if (fa_status s = make_page_map(&tv, L->v_cache, rows, L->head_dim, L->dtype); s != FA_OK) return s;
  if (L->dtype == FA_BF16) {
    if (L->head_dim == 128) return launch_decode_t<__nv_bfloat16, 128, kDecodeStages>(p, tk, tv, stream);
    return launch_decode_t<__nv_bfloat16, 64, kDecodeStages>(p, tk, tv, stream);
  }
  if (L->head_dim == 128) return launch_decode_t<__half, 128, kDecodeStages>(p, tk, tv, stream);
  return launch_decode_t<__half, 64, kDecodeStages>(p, tk, tv, stream);
}

fa_status launch_generic(const fa_kv_layer *L, const void *q, void *out, const int32_t *cu,
                         const int32_t *ctx, const int32_t *tables, int max_blocks, int num_seqs,
                         int num_heads, int n_rep, int total_q, float scale, int score_flow,
                         cudaStream_t stream) {
  if (L->head_dim > fa::kGenericMaxDim)
    return fail(FA_EUNSUPPORTED, "head_dim %d > %d is not supported", L->head_dim, fa::kGenericMaxDim);
  if (L->block_size > 1024)
    return fail(FA_EUNSUPPORTED, "block_size %d > 1024 is not supported", L->block_size);
  fa::GenericParams p{};
  p.q = q;
  p.out = out;
  p.k_cache = L->k_cache;
  p.v_cache = L->v_cache;
  p.cu_seqlens_q = cu;
  p.context_lens = ctx;
  p.block_tables = tables;
  p.max_blocks_per_seq = max_blocks;
  p.num_seqs = num_seqs;
  p.num_heads = num_heads;
  p.num_kv_heads = L->num_kv_heads;
  p.n_rep = n_rep;
  p.head_dim = L->head_dim;
  p.block_size = L->block_size;
  p.num_blocks = L->num_blocks;
  p.total_q = total_q;
  p.scale = scale;
  p.ref_scores = score_flow == FA_SCORES_REFERENCE;
  const size_t smem = fa::generic_smem_floats(L->block_size) * sizeof(float);
  dim3 grid(total_q, num_heads);
  auto launch = [&](auto kern) -> fa_status {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess)
      return fail(FA_ECUDA, "paged_attention (generic): set smem attribute: %s", cudaGetErrorString(e));
    kern<<<grid, fa::kGenericThreads, smem, stream>>>(p);
    return check_launch("paged_attention (generic)");
  };
  switch (L->dtype) {
    case FA_F32: return launch(fa::generic_attn_kernel<float>);
    case FA_BF16: return launch(fa::generic_attn_kernel<__nv_bfloat16>);
    default: return launch(fa::generic_attn_kernel<__half>);
  }
}

bool prefill_fast_path(const fa_kv_layer *L, int n_rep, int total_q, float scale, const void *q,
                       const void *out) {
  return (L->dtype == FA_BF16 || L->dtype == FA_F16) && L->block_size == fa::kPage &&
         L->head_dim == 128 && n_rep >= 1 && n_rep <= 128 && total_q >= 128 && scale > 0.f &&
         int64_t(L->num_blocks) * L->num_kv_heads * L->block_size < (int64_t(1) << 31) &&
         aligned(L->k_cache, 16) && aligned(L->v_cache, 16) && aligned(q, 16) && aligned(out, 32);
}

// Bytes of workspace the prefill kernel needs: two work counters (zero-filled once by the caller,
// returned to zero by the kernel).
constexpr size_t kPrefillWorkspace = 256;

int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kSmCount;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = kSmCount;
    cached[dev] = n;
  }
  return cached[dev];
}

template <typename T, bool kRef>
fa_status launch_prefill_t(const fa::PrefillParams &p, const CUtensorMap &tq, const CUtensorMap &tk,
                           const CUtensorMap &tv, int grid_x, cudaStream_t stream) {
  using S = fa::PrefillSmem;
  auto kern = fa::paged_prefill_kernel<T, kRef>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kAllocMax);
  if (e != cudaSuccess) return fail(FA_ECUDA, "prefill: set smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid_x));
  cfg.blockDim = dim3(fa::kPfThreads);
  cfg.dynamicSmemBytes = S::alloc(p.num_seqs);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];  // programmatic dependent launch: setup overlaps the predecessor
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p, tq, tk, tv);
  if (e != cudaSuccess) return fail(FA_ECUDA, "paged_prefill: launch: %s", cudaGetErrorString(e));
  return check_launch("paged_prefill");
}

fa_status launch_prefill(const fa_kv_layer *L, const void *q, void *out, const int32_t *cu,
                         const int32_t *ctx, const int32_t *tables, int max_blocks, int num_seqs,
                         int num_heads, int n_rep, int total_q, float scale, int score_flow,
                         void *ws, size_t ws_bytes, cudaStream_t stream) {
  if (!ws) return fail(FA_EINVAL, "prefill: workspace is NULL but %zu bytes are needed", kPrefillWorkspace);
  if (ws_bytes < kPrefillWorkspace)
    return fail(FA_ERANGE, "prefill: workspace of %zu bytes, %zu needed", ws_bytes, kPrefillWorkspace);
  if (!aligned(ws, 256)) return fail(FA_EINVAL, "prefill: workspace must be 256-byte aligned");
  fa::PrefillParams p{};
  p.out = out;
  p.counters = static_cast<int32_t *>(ws);
  p.max_blocks_per_seq = max_blocks;
  p.num_heads = num_heads;
  p.num_kv_heads = L->num_kv_heads;
  p.n_rep = n_rep;
  p.num_blocks = L->num_blocks;
  p.total_q = total_q;
  p.tq = 128 / n_rep;
  p.scale_log2 = scale * fa::kLog2e;
  p.scale = scale;
  const bool ref = score_flow == FA_SCORES_REFERENCE;
  const int64_t rows = int64_t(L->num_blocks) * L->num_kv_heads * L->block_size;
  CUtensorMap tmq, tk, tv;
  if (fa_status s = make_q_map(&tmq, q, total_q, num_heads, n_rep, p.tq, L->dtype); s != FA_OK) return s;
  if (fa_status s = make_page_map(&tk, L->k_cache, rows, 128, L->dtype); s != FA_OK) return s;
  if (fa_status s = make_page_map(&tv, L->v_cache, rows, 128, L->dtype); s != FA_OK) return s;
  // One persistent CTA per SM; at most kPfMaxSeqs sequences per launch (their chunk table lives
  // in shared memory), larger batches run as consecutive launches on the same stream.
  const int64_t chunk = 2 * p.tq;
  for (int s0 = 0; s0 < num_seqs; s0 += fa::kPfMaxSeqs) {
    p.num_seqs = std::min(fa::kPfMaxSeqs, num_seqs - s0);
    p.cu_seqlens_q = cu + s0;
    p.context_lens = ctx + s0;
    p.block_tables = tables + size_t(s0) * max_blocks;
    const int64_t items = ((int64_t(total_q) + chunk - 1) / chunk + p.num_seqs) * L->num_kv_heads;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>(sm_count(), items)));
    fa_status st =
        L->dtype == FA_BF16
            ? (ref ? launch_prefill_t<__nv_bfloat16, true>(p, tmq, tk, tv, grid, stream)
                   : launch_prefill_t<__nv_bfloat16, false>(p, tmq, tk, tv, grid, stream))
            : (ref ? launch_prefill_t<__half, true>(p, tmq, tk, tv, grid, stream)
                   : launch_prefill_t<__half, false>(p, tmq, tk, tv, grid, stream));
    if (st != FA_OK) return st;
  }
  return ok();
}

fa_status check_attention_args(const char *who, const fa_kv_layer *L, const void *q, const void *out,
                               const int32_t *ctx, const int32_t *tables, int max_blocks,
                               int num_seqs, int num_heads, int n_rep, int max_context_len,
                               float scale, int score_flow = FA_SCORES_F32) {
  if (fa_status s = check_layer(L, who); s != FA_OK) return s;
  if (!q || !out || !ctx || !tables) return fail(FA_EINVAL, "%s: NULL query/out/context_lens/block_tables", who);
  if (num_seqs < 0 || max_blocks <= 0) return fail(FA_EINVAL, "%s: num_seqs=%d max_blocks_per_seq=%d", who, num_seqs, max_blocks);
  if (n_rep <= 0 || num_heads != n_rep * L->num_kv_heads)
    return fail(FA_EINVAL, "%s: num_heads (%d) must equal n_rep (%d) * num_kv_heads (%d)", who,
                num_heads, n_rep, L->num_kv_heads);
  if (max_context_len < 0 || int64_t(max_context_len) > int64_t(max_blocks) * L->block_size)
    return fail(FA_ERANGE, "%s: max_context_len %d outside [0, %lld]", who, max_context_len,
                (long long)max_blocks * L->block_size);
  if (!std::isfinite(scale)) return fail(FA_EINVAL, "%s: scale is not finite", who);
  if (score_flow != FA_SCORES_F32 && score_flow != FA_SCORES_REFERENCE)
    return fail(FA_EINVAL, "%s: score_flow %d is not FA_SCORES_F32 or FA_SCORES_REFERENCE", who,
                score_flow);
  return FA_OK;
}

// ---- decode scratch for callers that cannot allocate ------------------------------------

// Split-K partials and merge tickets of fa_paged_decode_noalloc. Host code must not pass this
// symbol to a kernel (on the host it names a stand-in, not device memory): its device address
// comes from cudaGetSymbolAddress, looked up once per device with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FA_NOALLOC_DECODE_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {};

fa_status noalloc_scratch(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FA_ECUDA, "paged_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(FA_EUNSUPPORTED, "paged_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(FA_ECUDA, "paged_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FA_OK;
}

// ---- projection GEMMs ---------------------------------------------------------------------

// 2-D map over a row-major [rows, K] 16-bit matrix: box = box_rows x 64 elements (128 B),
// 128-byte swizzle (the K-major operand layout of the tcgen05 GEMM).
fa_status make_gemm_map(CUtensorMap *map, const void *base, int64_t rows, int64_t K, int32_t dt,
                        int box_rows, const char *who) {
  if (fa_status s = get_encoder(); s != FA_OK) return s;
  const CUtensorMapDataType t =
      dt == FA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  cuuint32_t box[2] = {uint32_t(fa::kGemmBK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, t, 2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d)", who, int(r));
  return FA_OK;
}

// 256-column output tiles when they alone fill the GPU, else 128 (more CTAs for small M). With
// several waves, 128 also wins when it cuts the columns of the busiest SM by more than 10 %
// (weight-streaming shapes such as a 64-row lm_head over a 128K vocabulary: 4 x 256 = 1024
// columns against 7 x 128 = 896).
int gemm_bn(int M, int N) {
  const int64_t m_tiles = (M + 127) / 128, sms = sm_count();
  const int64_t tiles256 = m_tiles * ((N + 255) / 256), tiles128 = m_tiles * ((N + 127) / 128);
  if (tiles256 < sms) return 128;
  const int64_t cols256 = (tiles256 + sms - 1) / sms * 256, cols128 = (tiles128 + sms - 1) / sms * 128;
  return cols128 * 10 < cols256 * 9 ? 128 : 256;
}

template <typename T, int BN, int AROWS, class Epi>
fa_status launch_gemm_rows(int M, int N, int K, const Epi &epi, const void *a, const void *b,
                           int32_t dt, cudaStream_t stream, const char *who) {
  using C = fa::GemmCfg<BN, AROWS>;
  fa::GemmShape s{M, N, K, (M + 127) / 128, (N + BN - 1) / BN};
  CUtensorMap ta, tb;
  if (fa_status st = make_gemm_map(&ta, a, M, K, dt, AROWS, who); st != FA_OK) return st;
  if (fa_status st = make_gemm_map(&tb, b, N, K, dt, BN, who); st != FA_OK) return st;
  auto kern = fa::gemm_tn_kernel<T, BN, Epi, AROWS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: set smem attribute: %s", who, cudaGetErrorString(e));
  const int grid = int(std::min<int64_t>(sm_count(), int64_t(s.tiles_m) * s.tiles_n));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(fa::kGemmThreads);
  cfg.dynamicSmemBytes = C::kAlloc;
  cfg.stream = stream;
  // Programmatic dependent launch: the prologue and the first weight stages overlap the tail of
  // the preceding kernel; the kernel waits for it before touching activations or outputs.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, s, epi, ta, tb);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: launch: %s", who, cudaGetErrorString(e));
  return check_launch(who);
}

// Batches of <= 64 rows on 128-wide tiles load 64-row A boxes: 8 ring stages instead of 6, more
// weight bytes in flight (the logits readback of a decode batch).
template <typename T, int BN, class Epi>
fa_status launch_gemm_t(int M, int N, int K, const Epi &epi, const void *a, const void *b,
                        int32_t dt, cudaStream_t stream, const char *who) {
  if constexpr (BN == 128)
    if (M <= 64) return launch_gemm_rows<T, 128, 64>(M, N, K, epi, a, b, dt, stream, who);
  return launch_gemm_rows<T, BN, 128>(M, N, K, epi, a, b, dt, stream, who);
}

// Split-K over a cluster of `ranks` CTAs per 128 x 128 tile (one tile per cluster).
template <typename T, int AROWS, class Epi>
fa_status launch_gemm_splitk_rows(int M, int N, int K, int ranks, const Epi &epi, const void *a,
                                  const void *b, int32_t dt, cudaStream_t stream, const char *who) {
  constexpr int BN = 128;
  using C = fa::GemmCfg<BN, AROWS>;
  fa::GemmShape s{M, N, K, (M + 127) / 128, (N + BN - 1) / BN};
  CUtensorMap ta, tb;
  if (fa_status st = make_gemm_map(&ta, a, M, K, dt, AROWS, who); st != FA_OK) return st;
  if (fa_status st = make_gemm_map(&tb, b, N, K, dt, BN, who); st != FA_OK) return st;
  auto kern = fa::gemm_tn_splitk_kernel<T, BN, Epi, AROWS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: set smem attribute: %s", who, cudaGetErrorString(e));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(s.tiles_m * s.tiles_n * ranks));
  cfg.blockDim = dim3(fa::kGemmThreads);
  cfg.dynamicSmemBytes = C::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(ranks);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch (as for the unsplit GEMM).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, s, epi, ta, tb);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: cluster launch: %s", who, cudaGetErrorString(e));
  return check_launch(who);
}

// Decode-sized batches (M <= 64) load 64-row A boxes: 8 ring stages instead of 6.
template <typename T, class Epi>
fa_status launch_gemm_splitk(int M, int N, int K, int ranks, const Epi &epi, const void *a,
                             const void *b, int32_t dt, cudaStream_t stream, const char *who) {
  if (M <= 64) return launch_gemm_splitk_rows<T, 64>(M, N, K, ranks, epi, a, b, dt, stream, who);
  return launch_gemm_splitk_rows<T, 128>(M, N, K, ranks, epi, a, b, dt, stream, who);
}

// How many clusters of `ranks` split-K CTAs can be resident at once (the driver's answer, which
// includes placing each cluster inside one GPC), cached per device and cluster size.
template <typename T, int AROWS, class Epi>
int splitk_max_clusters(int ranks) {
  static std::mutex mu;
  static std::unordered_map<int64_t, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const int64_t key = int64_t(dev) * 64 + ranks;
  std::lock_guard<std::mutex> lock(mu);
  if (auto it = cache.find(key); it != cache.end()) return it->second;
  using C = fa::GemmCfg<128, AROWS>;
  auto kern = fa::gemm_tn_splitk_kernel<T, 128, Epi, AROWS>;
  int n = 0;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(ranks));
    cfg.blockDim = dim3(fa::kGemmThreads);
    cfg.dynamicSmemBytes = C::kAlloc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(ranks);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
  }
  if (e != cudaSuccess) {  // a failed query only means "no split"
    n = 0;
    cudaGetLastError();
  }
  cache[key] = n;
  return n;
}

// How many CTAs split K when 128-wide tiles leave most SMs idle (1 = no split): the largest
// split, at least 4 K blocks per CTA, whose clusters all fit on the GPU at once. Clusters live
// inside one GPC, so the fit depends on the cluster size and not only on the CTA count (on B200,
// 32 tiles x 4 = 128 CTAs fit in one wave, 48 tiles x 3 = 144 do not).
template <typename T, class Epi>
int gemm_split_ranks(int M, int N, int K) {
  const int64_t tiles = int64_t((M + 127) / 128) * ((N + 127) / 128);
  const int num_k = (K + fa::kGemmBK - 1) / fa::kGemmBK;
  const int64_t max_r = std::min<int64_t>(
      std::min<int64_t>(fa::kSplitMaxRanks, num_k / 4), sm_count() / std::max<int64_t>(1, tiles));
  for (int r = int(max_r); r >= 2; --r) {
    const int fit = M <= 64 ? splitk_max_clusters<T, 64, Epi>(r)
                            : splitk_max_clusters<T, 128, Epi>(r);
    if (tiles <= fit) return r;
  }
  return 1;
}

template <typename T, class Epi>
fa_status launch_gemm(int M, int N, int K, const Epi &epi, const void *a, const void *b,
                      int32_t dt, cudaStream_t stream, const char *who) {
  if (const int r = gemm_split_ranks<T, Epi>(M, N, K); r >= 2)
    return launch_gemm_splitk<T>(M, N, K, r, epi, a, b, dt, stream, who);
  if (gemm_bn(M, N) == 256) return launch_gemm_t<T, 256>(M, N, K, epi, a, b, dt, stream, who);
  return launch_gemm_t<T, 128>(M, N, K, epi, a, b, dt, stream, who);
}

template <typename T>
fa_status launch_qkv(const fa_kv_layer *L, const fa_qkv_weights *w, const void *x,
                     const int32_t *pos, const int32_t *slots, int T_, void *q_out,
                     cudaStream_t stream) {
  fa::QkvEpilogue<T> epi{};
  epi.q_out = static_cast<T *>(q_out);
  epi.k_cache = static_cast<T *>(L->k_cache);
  epi.v_cache = static_cast<T *>(L->v_cache);
  epi.bias = static_cast<const T *>(w->bias);
  epi.q_norm = static_cast<const T *>(w->q_norm_weight);
  epi.k_norm = static_cast<const T *>(w->k_norm_weight);
  epi.rope_cos = w->rope_cos;
  epi.rope_sin = w->rope_sin;
  epi.positions = pos;
  epi.slots = slots;
  epi.rms_eps = w->rms_eps;
  epi.num_heads = w->num_heads;
  epi.num_kv_heads = L->num_kv_heads;
  epi.head_dim = L->head_dim;
  epi.num_blocks = L->num_blocks;
  epi.block_size = L->block_size;
  epi.max_position = w->max_position;
  const int N = (w->num_heads + 2 * L->num_kv_heads) * L->head_dim;
  return launch_gemm<T>(T_, N, w->hidden, epi, x, w->weight, L->dtype, stream, "qkv_rope_cache");
}

// Layers of one bundle: every layer must share layer 0's shape and dtype (one model's pool).
fa_status bundle_params(const fa_kv_layer *layers, int32_t num_layers,
                               const int32_t *block_ids, int32_t num_logical, const void *payload,
                               fa::BundleParams *p, int *vec, const char *who) {
  if (!layers) return fail(FA_EINVAL, "%s: layers is NULL", who);
  if (num_layers <= 0 || num_layers > FA_MAX_COPY_LAYERS)
    return fail(FA_EINVAL, "%s: num_layers %d outside [1, %d]", who, num_layers, FA_MAX_COPY_LAYERS);
  if (num_logical < 0 || num_logical > 65535)
    return fail(FA_EINVAL, "%s: num_blocks %d outside [0, 65535]", who, num_logical);
  const fa_kv_layer &L0 = layers[0];
  for (int l = 0; l < num_layers; ++l) {
    if (fa_status s = check_layer(&layers[l], who); s != FA_OK) return s;
    const fa_kv_layer &L = layers[l];
    if (L.num_blocks != L0.num_blocks || L.num_kv_heads != L0.num_kv_heads ||
        L.block_size != L0.block_size || L.head_dim != L0.head_dim || L.dtype != L0.dtype)
      return fail(FA_EINVAL, "%s: layer %d shape/dtype differs from layer 0", who, l);
    p->k[l] = static_cast<char *>(L.k_cache);
    p->v[l] = static_cast<char *>(L.v_cache);
  }
  if (num_logical > 0 && (!block_ids || !payload))
    return fail(FA_EINVAL, "%s: NULL block_ids/payload", who);
  p->block_ids = block_ids;
  p->payload = static_cast<char *>(const_cast<void *>(payload));
  p->block_bytes = int64_t(L0.num_kv_heads) * L0.block_size * L0.head_dim * dtype_size(L0.dtype);
  p->num_logical = num_logical;
  p->num_layers = num_layers;
  p->num_blocks = L0.num_blocks;
  int v = 16;
  auto fits = [&](int w) {
    if (p->block_bytes % w || !aligned(payload, w)) return false;
    for (int l = 0; l < num_layers; ++l)
      if (!aligned(p->k[l], w) || !aligned(p->v[l], w)) return false;
    return true;
  };
  while (v > 2 && !fits(v)) v >>= 1;
  if (!fits(v)) return fail(FA_EINVAL, "%s: misaligned caches or payload", who);
  *vec = v;
  return FA_OK;
}

template <bool kImport>
fa_status bundle_launch(const fa::BundleParams &p, int vec, cudaStream_t stream,
                               const char *who) {
  dim3 grid(2 * p.num_layers, p.num_logical);
  switch (vec) {
    case 16: fa::bundle_payload_kernel<16, kImport><<<grid, 256, 0, stream>>>(p); break;
    case 8: fa::bundle_payload_kernel<8, kImport><<<grid, 256, 0, stream>>>(p); break;
    case 4: fa::bundle_payload_kernel<4, kImport><<<grid, 256, 0, stream>>>(p); break;
    default: fa::bundle_payload_kernel<2, kImport><<<grid, 256, 0, stream>>>(p); break;
  }
  return check_launch(who);
}

}  // namespace

extern "C" {

int32_t fa_abi_version(void) { return 2; }

const char *fa_status_string(int32_t s) {
  switch (s) {
    case FA_OK: return "ok";
    case FA_EINVAL: return "invalid argument";
    case FA_ERANGE: return "out of range";
    case FA_ECUDA: return "CUDA error";
    case FA_ETIMEOUT: return "device wait timed out";
    case FA_EUNSUPPORTED: return "unsupported configuration";
    case FA_EDEVICE: return "kernel reported bad device data";
    default: return "unknown status";
  }
}

const char *fa_last_error_message(void) { return g_msg; }

fa_status fa_device_status(int32_t *status_out, int32_t clear, fa_stream_t stream) {
  if (!status_out) return fail(FA_EINVAL, "device_status: status_out is NULL");
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail(FA_ECUDA, "device_status: %s", cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, fa::g_status, sizeof(int));
  if (e != cudaSuccess) return fail(FA_ECUDA, "device_status: %s", cudaGetErrorString(e));
  if (clear) {
    const int z = 0;
    e = cudaMemcpyToSymbol(fa::g_status, &z, sizeof(int));
    if (e != cudaSuccess) return fail(FA_ECUDA, "device_status: %s", cudaGetErrorString(e));
  }
  *status_out = v;
  if (v & FA_DEVERR_TIMEOUT) return fail(FA_ETIMEOUT, "a device-side wait timed out (0x%x)", v);
  if (v) return fail(FA_EDEVICE, "kernels reported bad device data (0x%x)", v);
  return ok();
}

fa_status fa_reshape_and_cache(const fa_kv_layer *layer, const void *key, const void *value,
                               int64_t key_stride_token, int64_t key_stride_head,
                               int64_t value_stride_token, int64_t value_stride_head,
                               const int32_t *slot_mapping, int32_t num_tokens,
                               fa_stream_t stream) {
  if (fa_status s = check_layer(layer, "reshape_and_cache"); s != FA_OK) return s;
  if (num_tokens < 0) return fail(FA_EINVAL, "reshape_and_cache: num_tokens < 0");
  if (num_tokens == 0) return ok();
  if (!key || !value || !slot_mapping)
    return fail(FA_EINVAL, "reshape_and_cache: NULL key/value/slot_mapping");
  const int es = dtype_size(layer->dtype);
  fa::ReshapeParams p{};
  p.key = static_cast<const char *>(key);
  p.value = static_cast<const char *>(value);
  p.k_cache = static_cast<char *>(layer->k_cache);
  p.v_cache = static_cast<char *>(layer->v_cache);
  p.slot_mapping = slot_mapping;
  p.key_stride_token = key_stride_token * es;
  p.key_stride_head = key_stride_head * es;
  p.value_stride_token = value_stride_token * es;
  p.value_stride_head = value_stride_head * es;
  p.num_slots = int64_t(layer->num_blocks) * layer->block_size;
  p.num_tokens = num_tokens;
  p.num_kv_heads = layer->num_kv_heads;
  p.block_size = layer->block_size;
  p.row_bytes = layer->head_dim * es;
  // Widest vector every address and stride allows.
  int vec = 16;
  auto fits = [&](int v) {
    return p.row_bytes % v == 0 && aligned(key, v) && aligned(value, v) &&
           aligned(layer->k_cache, v) && aligned(layer->v_cache, v) && p.key_stride_token % v == 0 &&
           p.key_stride_head % v == 0 && p.value_stride_token % v == 0 &&
           p.value_stride_head % v == 0;
  };
  while (vec > 2 && !fits(vec)) vec >>= 1;
  if (!fits(vec)) return fail(FA_EINVAL, "reshape_and_cache: misaligned key/value/cache");
  const int64_t items = int64_t(num_tokens) * layer->num_kv_heads * (p.row_bytes / vec);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((items + threads - 1) / threads, int64_t(kSmCount) * 16);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(blocks));
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];  // programmatic dependent launch, as for the attention kernels
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (vec) {
    case 16: e = cudaLaunchKernelEx(&cfg, fa::reshape_and_cache_kernel<16>, p); break;
    case 8: e = cudaLaunchKernelEx(&cfg, fa::reshape_and_cache_kernel<8>, p); break;
    case 4: e = cudaLaunchKernelEx(&cfg, fa::reshape_and_cache_kernel<4>, p); break;
    default: e = cudaLaunchKernelEx(&cfg, fa::reshape_and_cache_kernel<2>, p); break;
  }
  if (e != cudaSuccess) return fail(FA_ECUDA, "reshape_and_cache: launch: %s", cudaGetErrorString(e));
  return check_launch("reshape_and_cache");
}

fa_status fa_copy_blocks(const fa_kv_layer *layers, int32_t num_layers, const int32_t *block_mapping,
                         int32_t num_pairs, fa_stream_t stream) {
  if (!layers) return fail(FA_EINVAL, "copy_blocks: layers is NULL");
  if (num_layers <= 0 || num_layers > FA_MAX_COPY_LAYERS)
    return fail(FA_EINVAL, "copy_blocks: num_layers %d outside [1, %d]", num_layers, FA_MAX_COPY_LAYERS);
  if (num_pairs < 0) return fail(FA_EINVAL, "copy_blocks: num_pairs < 0");
  if (num_pairs == 0) return ok();
  if (!block_mapping) return fail(FA_EINVAL, "copy_blocks: block_mapping is NULL");
  fa::CopyParams p{};
  const fa_kv_layer &L0 = layers[0];
  for (int l = 0; l < num_layers; ++l) {
    if (fa_status s = check_layer(&layers[l], "copy_blocks"); s != FA_OK) return s;
    const fa_kv_layer &L = layers[l];
    if (L.num_blocks != L0.num_blocks || L.num_kv_heads != L0.num_kv_heads ||
        L.block_size != L0.block_size || L.head_dim != L0.head_dim || L.dtype != L0.dtype)
      return fail(FA_EINVAL, "copy_blocks: layer %d shape/dtype differs from layer 0", l);
    p.k[l] = static_cast<char *>(L.k_cache);
    p.v[l] = static_cast<char *>(L.v_cache);
  }
  p.pairs = block_mapping;
  p.num_pairs = num_pairs;
  p.num_blocks = L0.num_blocks;
  p.block_bytes = int64_t(L0.num_kv_heads) * L0.block_size * L0.head_dim * dtype_size(L0.dtype);
  int vec = 16;
  auto fits = [&](int v) {
    if (p.block_bytes % v) return false;
    for (int l = 0; l < num_layers; ++l)
      if (!aligned(p.k[l], v) || !aligned(p.v[l], v)) return false;
    return true;
  };
  while (vec > 2 && !fits(vec)) vec >>= 1;
  if (!fits(vec)) return fail(FA_EINVAL, "copy_blocks: misaligned caches");
  dim3 grid(num_pairs, num_layers, 2);
  switch (vec) {
    case 16: fa::copy_blocks_kernel<16><<<grid, 256, 0, stream>>>(p); break;
    case 8: fa::copy_blocks_kernel<8><<<grid, 256, 0, stream>>>(p); break;
    case 4: fa::copy_blocks_kernel<4><<<grid, 256, 0, stream>>>(p); break;
    default: fa::copy_blocks_kernel<2><<<grid, 256, 0, stream>>>(p); break;
  }
  return check_launch("copy_blocks");
}

static fa_status block_copy(const fa_kv_layer *layer, int32_t block_id, void *kdst, const void *ksrc,
                            void *vdst, const void *vsrc, cudaStream_t stream, const char *who) {
  const size_t bytes =
      size_t(layer->num_kv_heads) * layer->block_size * layer->head_dim * dtype_size(layer->dtype);
  cudaError_t e = cudaMemcpyAsync(kdst, ksrc, bytes, cudaMemcpyDefault, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(vdst, vsrc, bytes, cudaMemcpyDefault, stream);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: %s", who, cudaGetErrorString(e));
  (void)block_id;
  return ok();
}

fa_status fa_write_block(const fa_kv_layer *layer, int32_t block_id, const void *key, const void *value,
                         fa_stream_t stream) {
  if (fa_status s = check_layer(layer, "write_block"); s != FA_OK) return s;
  if (!key || !value) return fail(FA_EINVAL, "write_block: NULL key/value");
  if (block_id < 0 || block_id >= layer->num_blocks)
    return fail(FA_ERANGE, "write_block: block_id %d outside [0, %d)", block_id, layer->num_blocks);
  const size_t off =
      size_t(block_id) * layer->num_kv_heads * layer->block_size * layer->head_dim * dtype_size(layer->dtype);
  return block_copy(layer, block_id, static_cast<char *>(layer->k_cache) + off, key,
                    static_cast<char *>(layer->v_cache) + off, value, stream, "write_block");
}

fa_status fa_read_block(const fa_kv_layer *layer, int32_t block_id, void *key, void *value,
                        fa_stream_t stream) {
  if (fa_status s = check_layer(layer, "read_block"); s != FA_OK) return s;
  if (!key || !value) return fail(FA_EINVAL, "read_block: NULL key/value");
  if (block_id < 0 || block_id >= layer->num_blocks)
    return fail(FA_ERANGE, "read_block: block_id %d outside [0, %d)", block_id, layer->num_blocks);
  const size_t off =
      size_t(block_id) * layer->num_kv_heads * layer->block_size * layer->head_dim * dtype_size(layer->dtype);
  return block_copy(layer, block_id, key, static_cast<const char *>(layer->k_cache) + off, value,
                    static_cast<const char *>(layer->v_cache) + off, stream, "read_block");
}

size_t fa_bundle_payload_bytes(const fa_kv_layer *layer, int32_t num_layers,
                               int32_t num_blocks) {
  if (!layer || num_layers <= 0 || num_blocks <= 0) return 0;
  return size_t(num_blocks) * size_t(num_layers) * 2 * size_t(layer->num_kv_heads) *
         size_t(layer->block_size) * size_t(layer->head_dim) * dtype_size(layer->dtype);
}

fa_status fa_export_bundle_payload(const fa_kv_layer *layers, int32_t num_layers,
                                   const int32_t *block_ids, int32_t num_blocks, void *payload,
                                   fa_stream_t stream) {
  const char *who = "export_bundle_payload";
  fa::BundleParams p{};
  int vec = 16;
  if (fa_status s = bundle_params(layers, num_layers, block_ids, num_blocks, payload, &p, &vec, who);
      s != FA_OK)
    return s;
  if (num_blocks == 0) return ok();
  return bundle_launch<false>(p, vec, stream, who);
}

fa_status fa_import_bundle_payload(const fa_kv_layer *layers, int32_t num_layers,
                                   const int32_t *block_ids, int32_t num_blocks,
                                   const void *payload, fa_stream_t stream) {
  const char *who = "import_bundle_payload";
  fa::BundleParams p{};
  int vec = 16;
  if (fa_status s = bundle_params(layers, num_layers, block_ids, num_blocks, payload, &p, &vec, who);
      s != FA_OK)
    return s;
  if (num_blocks == 0) return ok();
  return bundle_launch<true>(p, vec, stream, who);
}

fa_status fa_workspace_reset(const void *workspace) {
  if (!workspace) return fail(FA_EINVAL, "workspace_reset: workspace is NULL");
  std::lock_guard<std::mutex> lock(g_ticket_mu);
  g_ticket_state.erase(reinterpret_cast<uintptr_t>(workspace));
  return ok();
}

size_t fa_paged_attention_workspace_size(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                         int32_t head_dim, int32_t max_context_len,
                                         int32_t max_seqlen_q) {
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_context_len <= 0)
    return 0;
  if (max_seqlen_q != 1) return kPrefillWorkspace;
  DecodePlan plan;
  if (!plan_decode(num_seqs, num_kv_heads, max_context_len, &plan)) return 0;
  return decode_workspace_layout(num_seqs, num_heads, num_kv_heads, head_dim, plan).bytes;
}

fa_status fa_paged_decode(const fa_kv_layer *layer, const void *query, void *out,
                          const int32_t *context_lens, const int32_t *block_tables,
                          int32_t max_blocks_per_seq, int32_t num_seqs, int32_t num_heads,
                          int32_t n_rep, int32_t max_context_len, float scale,
                          int32_t score_flow, void *workspace, size_t workspace_bytes,
                          fa_stream_t stream) {
  if (fa_status s = check_attention_args("paged_decode", layer, query, out, context_lens,
                                         block_tables, max_blocks_per_seq, num_seqs, num_heads,
                                         n_rep, max_context_len, scale, score_flow);
      s != FA_OK)
    return s;
  if (num_seqs == 0) return ok();
  if (max_context_len < 1) return fail(FA_ERANGE, "paged_decode: max_context_len must be >= 1");
  if (num_seqs > 65535) return fail(FA_EUNSUPPORTED, "paged_decode: more than 65535 sequences per call");
  if (decode_fast_path(layer, n_rep, query, out))
    return launch_decode(layer, query, out, context_lens, block_tables, max_blocks_per_seq,
                         num_seqs, num_heads, n_rep, max_context_len, scale, score_flow, workspace,
                         workspace_bytes, stream);
  return launch_generic(layer, query, out, nullptr, context_lens, block_tables, max_blocks_per_seq,
                        num_seqs, num_heads, n_rep, num_seqs, scale, score_flow, stream);
}

fa_status fa_paged_decode_append(const fa_kv_layer *layer, const void *query, const void *key,
                                 const void *value, int64_t key_stride_token,
                                 int64_t key_stride_head, int64_t value_stride_token,
                                 int64_t value_stride_head, void *out, const int32_t *context_lens,
                                 const int32_t *block_tables, int32_t max_blocks_per_seq,
                                 int32_t num_seqs, int32_t num_heads, int32_t n_rep,
                                 int32_t max_context_len, float scale, int32_t score_flow,
                                 void *workspace, size_t workspace_bytes, fa_stream_t stream) {
  const char *who = "paged_decode_append";
  if (fa_status s = check_attention_args(who, layer, query, out, context_lens, block_tables,
                                         max_blocks_per_seq, num_seqs, num_heads, n_rep,
                                         max_context_len, scale, score_flow);
      s != FA_OK)
    return s;
  if (!key || !value) return fail(FA_EINVAL, "%s: key/value is NULL", who);
  if (key_stride_token < 0 || key_stride_head < 0 || value_stride_token < 0 || value_stride_head < 0)
    return fail(FA_EINVAL, "%s: negative key/value stride", who);
  if (num_seqs == 0) return ok();
  if (max_context_len < 1) return fail(FA_ERANGE, "%s: max_context_len must be >= 1", who);
  if (num_seqs > 65535) return fail(FA_EUNSUPPORTED, "%s: more than 65535 sequences per call", who);
  if (!decode_fast_path(layer, n_rep, query, out))
    return fail(FA_EUNSUPPORTED,
                "%s: needs a 16-bit pool, block_size 16, head_dim 64/128, n_rep <= 8 and 16-byte "
                "aligned buffers (use fa_reshape_and_cache + fa_paged_decode otherwise)", who);
  const AppendArgs app{key, value, key_stride_token, key_stride_head, value_stride_token,
                       value_stride_head};
  return launch_decode(layer, query, out, context_lens, block_tables, max_blocks_per_seq,
                       num_seqs, num_heads, n_rep, max_context_len, scale, score_flow, workspace,
                       workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr, true,
                       &app);
}

fa_status fa_paged_prefill(const fa_kv_layer *layer, const void *query, void *out,
                           const int32_t *cu_seqlens_q, const int32_t *context_lens,
                           const int32_t *block_tables, int32_t max_blocks_per_seq, int32_t num_seqs,
                           int32_t num_heads, int32_t n_rep, int32_t total_q, int32_t max_seqlen_q,
                           int32_t max_context_len, float scale, int32_t score_flow,
                           void *workspace, size_t workspace_bytes, fa_stream_t stream) {
  if (fa_status s = check_attention_args("paged_prefill", layer, query, out, context_lens,
                                         block_tables, max_blocks_per_seq, num_seqs, num_heads,
                                         n_rep, max_context_len, scale, score_flow);
      s != FA_OK)
    return s;
  if (!cu_seqlens_q) return fail(FA_EINVAL, "paged_prefill: cu_seqlens_q is NULL");
  if (total_q < 0 || max_seqlen_q < 0) return fail(FA_EINVAL, "paged_prefill: negative total_q/max_seqlen_q");
  if (max_seqlen_q > max_context_len)
    return fail(FA_ERANGE, "paged_prefill: max_seqlen_q %d > max_context_len %d", max_seqlen_q, max_context_len);
  if (total_q == 0 || num_seqs == 0) return ok();
  if (prefill_fast_path(layer, n_rep, total_q, scale, query, out))
    return launch_prefill(layer, query, out, cu_seqlens_q, context_lens, block_tables,
                          max_blocks_per_seq, num_seqs, num_heads, n_rep, total_q, scale,
                          score_flow, workspace, workspace_bytes, stream);
  return launch_generic(layer, query, out, cu_seqlens_q, context_lens, block_tables,
                        max_blocks_per_seq, num_seqs, num_heads, n_rep, total_q, scale, score_flow,
                        stream);
}

fa_status fa_paged_attention(const fa_kv_layer *layer, const void *query, void *out,
                             const int32_t *cu_seqlens_q, const int32_t *context_lens,
                             const int32_t *block_tables, int32_t max_blocks_per_seq,
                             int32_t num_seqs, int32_t num_heads, int32_t n_rep, int32_t total_q,
                             int32_t max_seqlen_q, int32_t max_context_len, float scale,
                             int32_t score_flow, void *workspace, size_t workspace_bytes,
                             fa_stream_t stream) {
  // Every sequence has exactly one query token when total_q == num_seqs and none has more
  // than one: that is the decode specialisation.
  if (max_seqlen_q == 1 && total_q == num_seqs)
    return fa_paged_decode(layer, query, out, context_lens, block_tables, max_blocks_per_seq,
                           num_seqs, num_heads, n_rep, max_context_len, scale, score_flow,
                           workspace, workspace_bytes, stream);
  return fa_paged_prefill(layer, query, out, cu_seqlens_q, context_lens, block_tables,
                          max_blocks_per_seq, num_seqs, num_heads, n_rep, total_q, max_seqlen_q,
                          max_context_len, scale, score_flow, workspace, workspace_bytes, stream);
}

fa_status fa_paged_decode_noalloc(const fa_kv_layer *layer, const void *query, void *out,
                                  const int32_t *context_lens, const int32_t *block_tables,
                                  int32_t max_blocks_per_seq, int32_t num_seqs, int32_t num_heads,
                                  int32_t n_rep, int32_t max_context_len, float scale,
                                  fa_stream_t stream) {
  if (fa_status s = check_attention_args("paged_decode_noalloc", layer, query, out, context_lens,
                                         block_tables, max_blocks_per_seq, num_seqs, num_heads,
                                         n_rep, max_context_len, scale);
      s != FA_OK)
    return s;
  if (num_seqs == 0) return ok();
  if (max_context_len < 1) return fail(FA_ERANGE, "paged_decode_noalloc: max_context_len must be >= 1");
  if (num_seqs > 65535) return fail(FA_EUNSUPPORTED, "paged_decode_noalloc: more than 65535 sequences per call");
  if (!decode_fast_path(layer, n_rep, query, out))  // the generic kernel uses no scratch
    return launch_generic(layer, query, out, nullptr, context_lens, block_tables,
                          max_blocks_per_seq, num_seqs, num_heads, n_rep, num_seqs, scale,
                          FA_SCORES_F32, stream);
  DecodePlan plan;
  if (!plan_decode(num_seqs, layer->num_kv_heads, max_context_len, &plan))
    return fail(FA_EUNSUPPORTED, "paged_decode_noalloc: context of %d tokens needs more than %d splits",
                max_context_len, fa::kDecodeMaxSplits);
  const DecodeWorkspace w =
      decode_workspace_layout(num_seqs, num_heads, layer->num_kv_heads, layer->head_dim, plan);
  if (w.bytes > FA_NOALLOC_DECODE_SCRATCH_BYTES)
    return fail(FA_ERANGE,
                "paged_decode_noalloc: %zu bytes of split-K scratch needed, the built-in buffer "
                "holds %u; call fa_paged_decode with a workspace instead",
                w.bytes, FA_NOALLOC_DECODE_SCRATCH_BYTES);
  void *scratch = nullptr;
  if (fa_status s = noalloc_scratch(&scratch); s != FA_OK) return s;
  if (w.bytes > 0) {
    // The merge tickets must start at zero; the previous call's contents are still there.
    const cudaError_t e = cudaMemsetAsync(static_cast<char *>(scratch) + w.counters_off, 0,
                                          size_t(num_seqs) * layer->num_kv_heads * sizeof(int32_t),
                                          stream);
    if (e != cudaSuccess) return fail(FA_ECUDA, "paged_decode_noalloc: %s", cudaGetErrorString(e));
  }
  return launch_decode(layer, query, out, context_lens, block_tables, max_blocks_per_seq, num_seqs,
                       num_heads, n_rep, max_context_len, scale, FA_SCORES_F32, scratch,
                       FA_NOALLOC_DECODE_SCRATCH_BYTES, stream, nullptr, false);
}

int32_t fa_gemm_tile_width(int32_t M, int32_t N, int32_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (gemm_split_ranks<__nv_bfloat16, fa::F32Epilogue>(M, N, K) >= 2) return 128;
  return gemm_bn(M, N);
}

fa_status fa_qkv_rope_cache(const fa_kv_layer *layer, const fa_qkv_weights *w, const void *x,
                            const int32_t *positions, const int32_t *slot_mapping,
                            int32_t num_tokens, void *q_out, fa_stream_t stream) {
  const char *who = "qkv_rope_cache";
  if (fa_status s = check_layer(layer, who); s != FA_OK) return s;
  if (!w) return fail(FA_EINVAL, "%s: weights is NULL", who);
  if (num_tokens < 0) return fail(FA_EINVAL, "%s: num_tokens %d < 0", who, num_tokens);
  if (num_tokens == 0) return ok();
  if (!x || !positions || !slot_mapping || !q_out || !w->weight || !w->rope_cos || !w->rope_sin)
    return fail(FA_EINVAL, "%s: NULL x/positions/slot_mapping/q_out/weight/rope tables", who);
  if (layer->dtype != FA_BF16 && layer->dtype != FA_F16)
    return fail(FA_EUNSUPPORTED, "%s: pool dtype must be bf16 or f16", who);
  if (layer->head_dim != 64 && layer->head_dim != 128)
    return fail(FA_EUNSUPPORTED, "%s: head_dim %d (64 or 128 supported)", who, layer->head_dim);
  if (w->num_heads <= 0 || w->num_heads % layer->num_kv_heads != 0)
    return fail(FA_EINVAL, "%s: num_heads %d is not a multiple of num_kv_heads %d", who,
                w->num_heads, layer->num_kv_heads);
  if (w->hidden <= 0 || w->hidden % 8 != 0)
    return fail(FA_EINVAL, "%s: hidden %d must be a positive multiple of 8", who, w->hidden);
  if (w->max_position <= 0) return fail(FA_EINVAL, "%s: max_position %d", who, w->max_position);
  if (!(w->rms_eps >= 0.f) || !std::isfinite(w->rms_eps))
    return fail(FA_EINVAL, "%s: rms_eps must be finite and >= 0", who);
  if (!aligned(x, 16) || !aligned(w->weight, 16) || !aligned(q_out, 32) ||
      !aligned(w->rope_cos, 16) || !aligned(w->rope_sin, 16) || !aligned(layer->k_cache, 32) ||
      !aligned(layer->v_cache, 32))
    return fail(FA_EINVAL, "%s: misaligned x/weight (16 B), q_out/pools (32 B) or tables (16 B)", who);
  if (int64_t(num_tokens) * w->num_heads * layer->head_dim >= (int64_t(1) << 40))
    return fail(FA_ERANGE, "%s: too many tokens", who);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return layer->dtype == FA_BF16
             ? launch_qkv<__nv_bfloat16>(layer, w, x, positions, slot_mapping, num_tokens, q_out, st)
             : launch_qkv<__half>(layer, w, x, positions, slot_mapping, num_tokens, q_out, st);
}

fa_status fa_o_proj_residual(const void *attn, const void *weight, const void *residual, void *out,
                             int32_t num_tokens, int32_t in_features, int32_t out_features,
                             int32_t dtype, fa_stream_t stream) {
  const char *who = "o_proj_residual";
  if (num_tokens < 0) return fail(FA_EINVAL, "%s: num_tokens %d < 0", who, num_tokens);
  if (num_tokens == 0) return ok();
  if (!attn || !weight || !out) return fail(FA_EINVAL, "%s: NULL attn/weight/out", who);
  if (dtype != FA_BF16 && dtype != FA_F16)
    return fail(dtype == FA_F32 ? FA_EUNSUPPORTED : FA_EINVAL, "%s: dtype %d (bf16 or f16)", who, dtype);
  if (in_features <= 0 || in_features % 8 != 0)
    return fail(FA_EINVAL, "%s: in_features %d must be a positive multiple of 8", who, in_features);
  if (out_features <= 0 || out_features % 32 != 0)
    return fail(FA_EINVAL, "%s: out_features %d must be a positive multiple of 32", who, out_features);
  if (!aligned(attn, 16) || !aligned(weight, 16) || !aligned(out, 32) ||
      (residual && !aligned(residual, 16)))
    return fail(FA_EINVAL, "%s: misaligned attn/weight/residual (16 B) or out (32 B)", who);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FA_BF16) {
    fa::ResidualEpilogue<__nv_bfloat16> epi{static_cast<__nv_bfloat16 *>(out),
                                            static_cast<const __nv_bfloat16 *>(residual)};
    return launch_gemm<__nv_bfloat16>(num_tokens, out_features, in_features, epi, attn, weight,
                                      dtype, st, who);
  }
  fa::ResidualEpilogue<__half> epi{static_cast<__half *>(out), static_cast<const __half *>(residual)};
  return launch_gemm<__half>(num_tokens, out_features, in_features, epi, attn, weight, dtype, st, who);
}

fa_status fa_last_token_logits(const void *hidden, const int32_t *cu_seqlens, int32_t num_seqs,
                               int32_t total_tokens, const void *norm_weight, float rms_eps,
                               const void *lm_head, int32_t hidden_size, int32_t vocab,
                               int32_t dtype, void *normed_out, float *logits_out,
                               fa_stream_t stream) {
  const char *who = "last_token_logits";
  if (num_seqs < 0) return fail(FA_EINVAL, "%s: num_seqs %d < 0", who, num_seqs);
  if (num_seqs == 0) return ok();
  if (!hidden || !cu_seqlens || !lm_head || !normed_out || !logits_out)
    return fail(FA_EINVAL, "%s: NULL hidden/cu_seqlens/lm_head/normed_out/logits_out", who);
  if (dtype != FA_BF16 && dtype != FA_F16)
    return fail(dtype == FA_F32 ? FA_EUNSUPPORTED : FA_EINVAL, "%s: dtype %d (bf16 or f16)", who, dtype);
  if (total_tokens < 1) return fail(FA_EINVAL, "%s: total_tokens %d < 1", who, total_tokens);
  if (hidden_size <= 0 || hidden_size % 8 != 0)
    return fail(FA_EINVAL, "%s: hidden_size %d must be a positive multiple of 8", who, hidden_size);
  if (vocab <= 0 || vocab % 32 != 0)
    return fail(FA_EINVAL, "%s: vocab %d must be a positive multiple of 32", who, vocab);
  if (num_seqs > 65535) return fail(FA_EUNSUPPORTED, "%s: more than 65535 sequences per call", who);
  if (!(rms_eps >= 0.f) || !std::isfinite(rms_eps))
    return fail(FA_EINVAL, "%s: rms_eps must be finite and >= 0", who);
  if (!aligned(hidden, 16) || !aligned(lm_head, 16) || !aligned(normed_out, 16) ||
      !aligned(logits_out, 16) || (norm_weight && !aligned(norm_weight, 2)))
    return fail(FA_EINVAL, "%s: misaligned hidden/lm_head/normed_out/logits_out (16 B)", who);
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FA_BF16) {
    using T = __nv_bfloat16;
    fa::last_rows_norm_kernel<T><<<num_seqs, fa::kNormThreads, 0, st>>>(
        static_cast<const T *>(hidden), cu_seqlens, total_tokens, static_cast<const T *>(norm_weight),
        rms_eps, hidden_size, static_cast<T *>(normed_out));
    if (fa_status s = check_launch(who); s != FA_OK) return s;
    return launch_gemm<T>(num_seqs, vocab, hidden_size, fa::F32Epilogue{logits_out}, normed_out,
                          lm_head, dtype, st, who);
  }
  using T = __half;
  fa::last_rows_norm_kernel<T><<<num_seqs, fa::kNormThreads, 0, st>>>(
      static_cast<const T *>(hidden), cu_seqlens, total_tokens, static_cast<const T *>(norm_weight),
      rms_eps, hidden_size, static_cast<T *>(normed_out));
  if (fa_status s = check_launch(who); s != FA_OK) return s;
  return launch_gemm<T>(num_seqs, vocab, hidden_size, fa::F32Epilogue{logits_out}, normed_out,
                        lm_head, dtype, st, who);
}

// ---- head-sharded decode ------------------------------------------------------------------

static_assert(FA_MAX_TP == fa::kMaxTp, "FA_MAX_TP and the kernel's rank limit differ");
static_assert(sizeof(fa_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");

fa_status fa_ipc_alloc(size_t bytes, void **ptr_out, fa_ipc_handle *handle_out) {
  if (!ptr_out || !handle_out) return fail(FA_EINVAL, "ipc_alloc: NULL output");
  *ptr_out = nullptr;
  if (bytes == 0) return fail(FA_EINVAL, "ipc_alloc: zero bytes");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(FA_ECUDA, "ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(FA_ECUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out->bytes, &h, sizeof(h));
  *ptr_out = p;
  return ok();
}

fa_status fa_ipc_free(void *ptr) {
  if (!ptr) return ok();
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(FA_ECUDA, "ipc_free: %s", cudaGetErrorString(e));
  return ok();
}

fa_status fa_ipc_open(const fa_ipc_handle *handle, void **ptr_out) {
  if (!handle || !ptr_out) return fail(FA_EINVAL, "ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(FA_ECUDA, "ipc_open: %s", cudaGetErrorString(e));
  return ok();
}

fa_status fa_ipc_close(void *ptr) {
  if (!ptr) return ok();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(FA_ECUDA, "ipc_close: %s", cudaGetErrorString(e));
  return ok();
}

static fa_status check_tp_group(const fa_tp_group *g, const char *who) {
  if (!g) return fail(FA_EINVAL, "%s: group is NULL", who);
  if (g->tp < 1 || g->tp > FA_MAX_TP)
    return fail(FA_EINVAL, "%s: tp %d outside [1, %d]", who, g->tp, FA_MAX_TP);
  if (g->rank < 0 || g->rank >= g->tp)
    return fail(FA_EINVAL, "%s: rank %d outside [0, %d)", who, g->rank, g->tp);
  for (int r = 0; r < g->tp; ++r) {
    if (!g->flags[r] || !aligned(g->flags[r], 4))
      return fail(FA_EINVAL, "%s: flags[%d] is NULL or misaligned", who, r);
  }
  return FA_OK;
}

fa_status fa_paged_decode_tp(const fa_tp_group *group, const fa_kv_layer *layer, const void *query,
                             const int32_t *context_lens, const int32_t *block_tables,
                             int32_t max_blocks_per_seq, int32_t num_seqs, int32_t num_heads,
                             int32_t n_rep, int32_t max_context_len, float scale,
                             int32_t score_flow, void *workspace, size_t workspace_bytes,
                             fa_stream_t stream) {
  const char *who = "paged_decode_tp";
  if (fa_status s = check_tp_group(group, who); s != FA_OK) return s;
  for (int r = 0; r < group->tp; ++r)
    if (!group->out[r] || !aligned(group->out[r], 16))
      return fail(FA_EINVAL, "%s: out[%d] is NULL or not 16-byte aligned", who, r);
  if (fa_status s = check_attention_args(who, layer, query, group->out[group->rank], context_lens,
                                         block_tables, max_blocks_per_seq, num_seqs, num_heads,
                                         n_rep, max_context_len, scale, score_flow);
      s != FA_OK)
    return s;
  if (num_seqs == 0) return ok();
  if (max_context_len < 1) return fail(FA_ERANGE, "%s: max_context_len must be >= 1", who);
  if (num_seqs > 65535) return fail(FA_EUNSUPPORTED, "%s: more than 65535 sequences per call", who);
  if (!decode_fast_path(layer, n_rep, query, group->out[group->rank]))
    return fail(FA_EUNSUPPORTED,
                "%s: needs a 16-bit pool, block_size 16, head_dim 64/128, n_rep <= 8 and "
                "16-byte aligned buffers", who);
  return launch_decode(layer, query, nullptr, context_lens, block_tables, max_blocks_per_seq,
                       num_seqs, num_heads, n_rep, max_context_len, scale, score_flow, workspace,
                       workspace_bytes, reinterpret_cast<cudaStream_t>(stream), group);
}

fa_status fa_tp_sync(const fa_tp_group *group, uint32_t epoch, int32_t mode, int64_t timeout_ns,
                     fa_stream_t stream) {
  const char *who = "tp_sync";
  if (fa_status s = check_tp_group(group, who); s != FA_OK) return s;
  if (mode < 1 || mode > (FA_TP_PUBLISH | FA_TP_WAIT))
    return fail(FA_EINVAL, "%s: mode %d (FA_TP_PUBLISH, FA_TP_WAIT or both)", who, mode);
  if (epoch == 0 && !group->epoch_counter)
    return fail(FA_EINVAL, "%s: epoch 0 (device epochs) needs group->epoch_counter", who);
  if ((mode & FA_TP_WAIT) && (timeout_ns < 1000 || timeout_ns > 10000000000LL))
    return fail(FA_ERANGE, "%s: timeout_ns %lld outside [1e3, 1e10]", who, (long long)timeout_ns);
  fa::TpFlagSlots slots{};
  for (int r = 0; r < group->tp; ++r) slots.slot[r] = group->flags[r] + group->rank;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];  // programmatic dependent launch, as for the decode
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, fa::tp_sync_kernel, slots,
                         static_cast<const uint32_t *>(group->flags[group->rank]), int(group->tp),
                         epoch, group->epoch_counter, int(mode), (unsigned long long)timeout_ns);
  if (e != cudaSuccess) return fail(FA_ECUDA, "%s: launch: %s", who, cudaGetErrorString(e));
  return check_launch(who);
}

}  // extern "C"

