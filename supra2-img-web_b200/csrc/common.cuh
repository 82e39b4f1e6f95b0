// Device helpers shared by the sm_100a kernels of libsupra_attn: mbarriers, bulk-async copies
// (the TMA engine's untiled form) with bounded waits, and the device status word.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace supra {

// ---- device status word ----------------------------------------------------------------------
// status[0] = first error code (DEV_* in kernels.h), status[1] = blockIdx.x of the reporter,
// status[2] = stage tag, status[3] = a detail word (e.g. the block counter a wait was for).
// The first reporter wins; the host reads and clears it at sync.
__device__ __forceinline__ void report_error(int32_t* status, int32_t code, int32_t stage, int32_t detail = 0) {
  if (atomicCAS(status, 0, code) == 0) {
    status[1] = (int32_t)blockIdx.x;
    status[2] = stage;
    status[3] = detail;
  }
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// One plain arrival (no transaction bytes).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (the bulk-copy engine).
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory accesses with later async-proxy accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete, for at most kWaitLimitNs. Returns
// false on timeout (the caller reports DEV_TIMEOUT and leaves); never spins forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---- bulk async copy global -> shared (no tensor map, this CTA only) --------------------------------
// Both addresses 16-byte aligned, bytes a multiple of 16. Completion is signalled on `bar` as
// transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- Ampere-style cp.async (4-byte granularity, any 4-byte aligned address) -----------------------
// src_bytes = 0 zero-fills the destination word.
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Score bias of a (query row i, key j) pair of one head from a T5 relative-bias table, in 32-bit
// index arithmetic: tab_h = table + h (the table is [buckets, H], buckets * H < 2^32), lut_c =
// rel_lut + rel_max (the bucket of relative position r at lut_c[r]), rel = j - i. Buckets of
// relative positions beyond rel_max equal those at +-rel_max (the bucket saturates at
// max_distance), so rel is clamped.
__device__ __forceinline__ float t5_table_bias(const float* __restrict__ tab_h, const int32_t* __restrict__ lut_c,
                                               int32_t rel_max, uint32_t H, int32_t rel) {
  rel = max(-rel_max, min(rel_max, rel));
  return __ldg(tab_h + (uint32_t)__ldg(lut_c + rel) * H);
}

// ops.linear's activations (app/gpu/gemm.js:28-36), kActGelu / kActGeluTanh / kActSilu: GELU in
// its erf form, GELU with the tanh approximation 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// SiLU x / (1 + e^-x).
__device__ __forceinline__ float linear_act(int act, float x) {
  if (act == kActGelu) return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
  if (act == kActGeluTanh) return 0.5f * x * (1.f + tanhf(0.79788456080286536f * (x + 0.044715f * x * x * x)));
  return x / (1.f + expf(-x));
}

// Tile index -> problem index: the largest p with begin[p] <= t (begin[0] == 0, ascending).
__device__ __forceinline__ int find_problem(const int32_t* __restrict__ begin, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(begin + mid) <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

}  // namespace supra
