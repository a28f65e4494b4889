// bnbq_async.cuh -- mbarrier / bulk-copy helpers (sm_90+ PTX) with bounded waits.
//
// Every wait is bounded in wall time (globaltimer, 1 s); on expiry it records the event
// in g_bnbq_wait_timeouts (read by bnbq_wait_timeouts()) and reports failure,
// so a kernel can stop instead of hanging the GPU. No cluster multicast is
// used anywhere: each CTA copies into its own shared memory.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace bnbq {

// Wait-timeout counter of the translation unit that includes this header
// (a module-scope device variable, one per device); read_wait_timeouts()
// returns it for the current device.
static __device__ unsigned int g_bnbq_wait_timeouts = 0;

static inline int read_wait_timeouts(unsigned int* out) {
  return cudaMemcpyFromSymbol(out, g_bnbq_wait_timeouts, sizeof(unsigned int)) == cudaSuccess ? 0 : -1;
}

// A wait gives up after this long (the kernels that wait run for microseconds;
// a translation unit whose waits are on other GPUs defines a longer default
// before including this header).
#ifndef BNBQ_WAIT_LIMIT_DEFAULT_NS
#define BNBQ_WAIT_LIMIT_DEFAULT_NS 1000000000ull  // 1 s
#endif
constexpr uint64_t kWaitLimitNs = BNBQ_WAIT_LIMIT_DEFAULT_NS;

// The limit the kernels of this translation unit read (per device). Tests
// shorten it to make a wait expire on purpose; 0 restores the default.
static __device__ uint64_t g_bnbq_wait_limit_ns = kWaitLimitNs;

// Waits for another GPU (the row-shard exchange) get a longer limit: a peer
// may legitimately start a call much later than this rank.
constexpr uint64_t kPeerWaitLimitNs = 10000000000ull;  // 10 s: a peer that is this late has failed
static __device__ uint64_t g_bnbq_peer_wait_limit_ns = kPeerWaitLimitNs;

// Sets both limits (ns for each; 0 restores the defaults).
static inline int write_wait_limit(uint64_t ns) {
  const uint64_t v = ns ? ns : kWaitLimitNs;
  const uint64_t vp = ns ? ns : kPeerWaitLimitNs;
  if (cudaMemcpyToSymbol(g_bnbq_wait_limit_ns, &v, sizeof(v)) != cudaSuccess) return -1;
  return cudaMemcpyToSymbol(g_bnbq_peer_wait_limit_ns, &vp, sizeof(vp)) == cudaSuccess ? 0 : -1;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// One test of the phase with the given parity; the hardware may suspend the
// thread for up to `hint_ns` while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete, for at most
// kWaitLimitNs of wall time (globaltimer); false on expiry (recorded).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  const uint64_t limit = g_bnbq_wait_limit_ns;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit) break;
  }
  atomicAdd(&g_bnbq_wait_timeouts, 1u);
  return false;
}

// Global -> this CTA's shared memory, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace bnbq
