// bnbq_peer.cuh -- the row-shard exchange's device side, shared by the
// standalone all-gather kernel (bnbq_peer.cu) and the matmul kernels that
// finish with the exchange themselves (bnbq_gemv.cu, bnbq_gemv_xtab.cu).
//
// Rank d's inbox is a uint64 array in two halves that alternate by the parity
// of the call's epoch e. Word r * n_total + c of a half holds output element
// (r, c) as value | e << 32: the 16-bit value and the epoch travel in one
// 8-byte store (single-copy atomic), so a receiver that sees the epoch sees
// the value. A sender stores into the peers' inboxes with relaxed
// system-scope stores (no fences); a receiver polls its own inbox (local
// memory) until the words carry e. The epoch lives in state[1] (state[0]
// counts the CTAs that have finished the call); the last CTA to finish stores
// it, after every thread of the call has read it.
#pragma once

#include <cstdint>

#include "bnbq_async.cuh"

namespace bnbq {

// Exchange mode of a matmul launch (inbox == nullptr: none). The matmul
// writes this rank's slice to its own output as usual and, in addition,
// stores every value into the peers' inboxes, polls for the other ranks'
// columns and writes them into y_full.
struct PeerOut {
  uint64_t* const* inbox;  // device array of `world` inbox pointers
  uint32_t* state;         // this rank's {finished CTAs, epoch}
  void* y_full;            // this rank's m x n_total output (16-bit values)
  int64_t n_total;         // columns of the full output
  int64_t ldf;             // y_full's row stride
  int64_t col0;            // this rank's first column
  int64_t half;            // words per inbox half
  int world, rank;
};

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The call's epoch (read after griddepcontrol.wait: the previous call's last
// CTA has stored it).
__device__ __forceinline__ uint32_t peer_epoch(const PeerOut& px) { return px.state[1] + 1u; }

// Value `bits` of output element (r, col0 + c) into every peer's inbox.
__device__ __forceinline__ void peer_send(const PeerOut& px, uint32_t epoch, int64_t r, int64_t c, uint16_t bits) {
  const int64_t w = ((epoch & 1u) ? px.half : 0) + r * px.n_total + px.col0 + c;
  const uint64_t word = uint64_t(epoch) << 32 | bits;
  for (int d = 1; d < px.world; ++d) {
    const int dst = px.rank + d < px.world ? px.rank + d : px.rank + d - px.world;
    st_relaxed_sys_u64(px.inbox[dst] + w, word);
  }
}

// The other ranks' columns of rows [0, m) into y_full, from this rank's own
// inbox: items tid, tid + step, ... of the m x (n_total - n_local) received
// elements, four polls in flight per thread. Waits are bounded from the
// start of the loop by the peer wait limit (10 s by default); false on
// expiry (the remaining items are skipped).
__device__ __forceinline__ bool peer_receive(const PeerOut& px, uint32_t epoch, int m, int64_t n_local,
                                             int64_t tid, int64_t step) {
  constexpr int kBatch = 4;
  const int64_t others = px.n_total - n_local;
  const int64_t recvs = int64_t(m) * others;
  const uint64_t limit = g_bnbq_peer_wait_limit_ns;
  const uint64_t t0 = global_ns();
  const uint64_t* mine = px.inbox[px.rank] + ((epoch & 1u) ? px.half : 0);
  uint16_t* y = static_cast<uint16_t*>(px.y_full);
  for (int64_t i0 = tid; i0 < recvs; i0 += kBatch * step) {
    uint64_t v[kBatch];
    int64_t r[kBatch], c[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int64_t i = i0 + j * step;
      r[j] = i / others;
      const int64_t o = i - r[j] * others;
      c[j] = o < px.col0 ? o : o + n_local;
      if (i < recvs) v[j] = ld_relaxed_sys_u64(mine + r[j] * px.n_total + c[j]);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i0 + j * step >= recvs) break;
      const uint64_t* p = mine + r[j] * px.n_total + c[j];
      while (uint32_t(v[j] >> 32) != epoch) {
        if (global_ns() - t0 > limit) return false;
        v[j] = ld_relaxed_sys_u64(p);
      }
      y[r[j] * px.ldf + c[j]] = uint16_t(v[j]);
    }
  }
  return true;
}

// One CTA has finished the call (one thread, after every thread of the CTA
// has read the epoch): counts an expiry and, for the last CTA, resets the
// counter and stores the epoch.
__device__ __forceinline__ void peer_finish_cta(const PeerOut& px, uint32_t epoch, bool expired) {
  if (expired) atomicAdd(&g_bnbq_wait_timeouts, 1u);
  const unsigned int total = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(&px.state[0], 1u) == total - 1) {
    px.state[0] = 0;
    px.state[1] = epoch;  // also after an expiry: stay in step with the peers that did send
  }
}

}  // namespace bnbq
