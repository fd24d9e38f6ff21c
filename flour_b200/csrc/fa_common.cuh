// Shared device helpers for the sm_100a paged KV / paged attention kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "flour_attn.h"

namespace fa {

// Per-device status word: kernels OR FA_DEVERR_* bits into it instead of trapping.
__device__ int g_status;

__device__ __forceinline__ void report(int bits) { atomicOr(&g_status, bits); }

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

constexpr float kLog2e = 1.4426950408889634f;

// ---- element types --------------------------------------------------------------------

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Pack two floats into one 32-bit register of two 16-bit values (lo = a, hi = b).
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

// ---- the reference's score rounding (FA_SCORES_REFERENCE) ---------------------------------
// src/backend/cpu.rs:84-85 computes `(q.matmul(k^T) * scale).to_dtype(F32)` in the model dtype:
// the q.k product is rounded to the dtype, multiplied by the scale rounded to the dtype, and the
// product rounded again. With an f32 accumulator for q.k (the tensor cores' and the oracle's),
// these helpers reproduce those two roundings. A product of two 16-bit floats is exact in f32,
// so one hardware multiply rounded to nearest is the reference's single rounding of it. The
// transform is non-decreasing in `dot` (scale > 0), so it commutes with a row max.
template <typename T> __device__ __forceinline__ float ref_score(float dot, float scale_t);
template <> __device__ __forceinline__ float ref_score<float>(float dot, float scale_t) {
  return dot * scale_t;
}
template <> __device__ __forceinline__ float ref_score<__nv_bfloat16>(float dot, float scale_t) {
  return __bfloat162float(__hmul(__float2bfloat16_rn(dot), __float2bfloat16_rn(scale_t)));
}
template <> __device__ __forceinline__ float ref_score<__half>(float dot, float scale_t) {
  return __half2float(__hmul(__float2half_rn(dot), __float2half_rn(scale_t)));
}
// Two scores at once; `scale2` holds the rounded scale twice as a packed 16-bit pair.
template <typename T> __device__ __forceinline__ float2 ref_score2(float a, float b, uint32_t scale2);
template <>
__device__ __forceinline__ float2 ref_score2<__nv_bfloat16>(float a, float b, uint32_t scale2) {
  const __nv_bfloat162 v = __hmul2(__floats2bfloat162_rn(a, b),
                                   *reinterpret_cast<const __nv_bfloat162 *>(&scale2));
  return __bfloat1622float2(v);
}
template <> __device__ __forceinline__ float2 ref_score2<__half>(float a, float b, uint32_t scale2) {
  const __half2 v = __hmul2(__floats2half2_rn(a, b), *reinterpret_cast<const __half2 *>(&scale2));
  return __half22float2(v);
}

// ---- misc PTX ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// 2^x with the hardware approximation (ex2.approx, a single SFU instruction).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 256-bit global store (one full 32-byte sector); the address must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void *ptr, const uint32_t *r) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// The two values of a packed 16-bit pair as floats (lo, hi).
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t v);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2 *>(&v);
  return __half22float2(h);
}

// ---- programmatic dependent launch ------------------------------------------------------
// pdl_trigger: this CTA no longer holds back the next kernel on the stream, which may start
// (where it was launched with programmatic stream serialization) as SMs free up. pdl_wait: block
// until the preceding kernel has completed and its writes are visible. Both are no-ops for a
// launch without the programmatic attribute.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- mbarrier -------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}

// Upper bound on any single mbarrier wait. A healthy wait takes microseconds; hitting this
// means the copy it waits for will not arrive, and the caller reports FA_DEVERR_TIMEOUT.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded phase wait: true when the phase completed, false after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, phase)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---- TMA (no multicast anywhere in this library) -----------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled prefetch of one box into L2 (no shared memory, no completion signal).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// 2-D tiled load of one box into shared memory, completing on `bar` (complete_tx bytes).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// Same, with an L2 cache-policy hint (e.g. evict-first for data read exactly once).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap *map,
                                                 uint32_t bar, int32_t x, int32_t y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- warp-level tensor core path (ldmatrix / movmatrix / mma.sync) ------------------------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                 uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace fa
