// bnbq_peer.cu -- all-gather of row-sharded GEMV/GEMM outputs over NVLink peer
// memory (the exchange step of the N-sharded matmul).
//
// Every rank computes y[:, col0 : col0 + n_local] with the fused kernels and
// then launches bnbq_peer_allgather_rows on the same stream (programmatic
// dependent launch: it starts while the matmul drains and waits for it with
// griddepcontrol.wait). Its CTAs store the rank's slice into the full-y buffer
// of EVERY rank with plain stores to peer memory (CUDA IPC mappings over
// NVLink; no multicast, no TMA).
//
// Two handshakes per call e (the epoch, kept in device memory in state[1] and
// advanced once per call, so replays of a captured CUDA graph stay in step):
//   ready -- once the kernel runs (after griddepcontrol.wait), everything
//            before it on this rank's stream has completed, including whatever
//            consumed the previous call's output. CTA 0 then publishes
//            ready = e in every rank's flag array, and no CTA stores into rank
//            d's buffer before rank d's ready has reached e. A fast peer can
//            therefore never overwrite a result this rank is still reading.
//   done  -- the last CTA to finish (a local arrival counter it resets) makes
//            the stores visible system-wide, publishes done = e in every
//            rank's flag array and waits until every peer's done has reached
//            e: on return every slice is in this rank's buffer.
// flags[d] is rank d's uint32[2 * world]: [0, world) done epochs by source
// rank, [world, 2 * world) ready epochs. Every wait is bounded in time; on
// expiry the kernel counts a timeout (bnbq_wait_timeouts), skips what waited
// and returns with the output incomplete.
#define BNBQ_WAIT_LIMIT_DEFAULT_NS 10000000000ull  // 10 s: a peer that is this late has failed
#include "bnbq_async.cuh"
#include "bnbq_common.cuh"

namespace bnbq {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait (one thread) until *p has reached `epoch` (wrap-around safe), at most
// the wait limit from t0; false on expiry (counted).
__device__ __forceinline__ bool wait_epoch(const uint32_t* p, uint32_t epoch, uint64_t t0) {
  const uint64_t limit = g_bnbq_wait_limit_ns;
  while (int32_t(ld_acquire_sys(p) - epoch) < 0) {
    if (global_ns() - t0 > limit) {
      atomicAdd(&g_bnbq_wait_timeouts, 1u);
      return false;
    }
    __nanosleep(128);
  }
  return true;
}

// y_local: m x n_local (row stride ld_local) 16-bit values; y_full[d]: rank d's
// m x ldy buffer; flags[d]: rank d's uint32[2 * world]; state: this rank's
// {arrived CTAs, epoch}.
__global__ void __launch_bounds__(256) peer_allgather_kernel(const uint16_t* y_local, int m, int64_t n_local,
                                                             int64_t ld_local, int64_t col0, int64_t ldy,
                                                             uint16_t* const* y_full, uint32_t* const* flags,
                                                             uint32_t* state, int world, int rank, int vec) {
  __shared__ uint32_t s_ready;  // bit d: rank d may be written
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the matmul that wrote y_local has completed
  const uint32_t epoch = state[1] + 1u;  // read before any CTA can advance it (advanced by the last CTA only)
  const uint32_t* mine = flags[rank];
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0)
      for (int d = 0; d < world; ++d) st_release_sys(flags[d] + world + rank, epoch);
    uint32_t ok = 0;
    const uint64_t t0 = global_ns();
    for (int d = 0; d < world; ++d)
      if (wait_epoch(mine + world + d, epoch, t0)) ok |= 1u << d;
    s_ready = ok;
  }
  __syncthreads();
  const uint32_t ready = s_ready;
  const int64_t per_row = vec ? n_local / 8 : n_local;  // 16-byte pieces or single values
  const int64_t total = int64_t(m) * per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row, c = i - r * per_row;
    if (vec) {
      const uint4 v = *reinterpret_cast<const uint4*>(y_local + r * ld_local + 8 * c);
      for (int d = 0; d < world; ++d)
        if (ready >> d & 1u) *reinterpret_cast<uint4*>(y_full[d] + r * ldy + col0 + 8 * c) = v;
    } else {
      const uint16_t v = y_local[r * ld_local + c];
      for (int d = 0; d < world; ++d)
        if (ready >> d & 1u) y_full[d][r * ldy + col0 + c] = v;
    }
  }
  __threadfence_system();  // this thread's peer stores, before the CTA reports
  __syncthreads();
  __shared__ int s_last;
  if (threadIdx.x == 0) s_last = atomicAdd(&state[0], 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  // last CTA of this rank: every CTA's stores are fenced (they fenced before arriving)
  state[0] = 0;  // no CTA of this launch touches the counter again
  __threadfence_system();
  for (int d = 0; d < world; ++d) st_release_sys(flags[d] + rank, epoch);
  const uint64_t t0 = global_ns();
  for (int src = 0; src < world; ++src)
    if (!wait_epoch(mine + src, epoch, t0)) break;
  state[1] = epoch;  // also after an expiry: stay in step with the peers that did publish
}

}  // namespace

int peer_wait_timeouts(unsigned int* out) { return read_wait_timeouts(out); }
int peer_set_wait_limit(uint64_t ns) { return write_wait_limit(ns); }

}  // namespace bnbq

using namespace bnbq;

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

// IPC export of the allocation that contains `ptr`: the 64-byte handle and the
// offset of `ptr` from the allocation's base (cudaIpcGetMemHandle wants a base).
extern "C" int bnbq_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return BNBQ_ERR_INVALID;
  static PFN_cuMemGetAddressRange_v3020 get_range = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!get_range) return BNBQ_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return BNBQ_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return BNBQ_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return BNBQ_OK;
}

// Map another process's allocation into the CURRENT device's context (peer
// access to the owner enabled as needed) and check that the mapping is device
// memory before any kernel touches it.
extern "C" int bnbq_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return BNBQ_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return BNBQ_ERR_CUDA;
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
    cudaIpcCloseMemHandle(p);
    return BNBQ_ERR_CUDA;
  }
  *base_out = p;
  return BNBQ_OK;
}

extern "C" int bnbq_ipc_close(void* base) {
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? BNBQ_OK : BNBQ_ERR_CUDA;
}

extern "C" int bnbq_peer_allgather_rows(int dtype, const void* y_local, int32_t m, int64_t n_local, int64_t ld_local,
                                        int64_t col0, int64_t ldy, void* const* y_full, uint32_t* const* flags,
                                        uint32_t* state, int32_t world, int32_t rank, void* stream) {
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (m < 0 || n_local < 0 || world < 1 || world > 32 || rank < 0 || rank >= world || ld_local < n_local ||
      col0 < 0 || ldy < col0 + n_local)
    return BNBQ_ERR_INVALID;
  if (!y_full || !flags || !state || (m > 0 && n_local > 0 && !y_local)) return BNBQ_ERR_INVALID;
  if (!aligned(y_local, 2) || !aligned(state, 4) || !aligned(y_full, 8) || !aligned(flags, 8))
    return BNBQ_ERR_MISALIGNED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  // 16-byte pieces when every row start on both sides is 16-byte aligned (the
  // full-y buffers themselves are 16-byte aligned allocations)
  const int vec = (n_local % 8 == 0 && col0 % 8 == 0 && ldy % 8 == 0 && ld_local % 8 == 0 && aligned(y_local, 16)) ? 1 : 0;
  const int64_t work = int64_t(m) * (vec ? n_local / 8 : n_local);
  int64_t grid = (work + 255) / 256;
  if (grid < 1) grid = 1;
  if (grid > int64_t(di.sm_count)) grid = di.sm_count;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, peer_allgather_kernel, static_cast<const uint16_t*>(y_local), int(m), n_local,
                         ld_local, col0, ldy, reinterpret_cast<uint16_t* const*>(y_full), flags, state, int(world),
                         int(rank), vec) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

// ---------------------------------------------------------------------------
// bnbq_peer_allgather_rows_noalloc: bnbq_peer_allgather_rows without the
// caller's `state` words, for callers that may not allocate device memory.
//
// Who needs it: code that runs the exchange where cudaMalloc is off limits --
// a custom-call handler inside a compiled program whose runtime owns the
// device memory (an XLA FFI handler receives only its operand and result
// buffers; the runtime has preallocated most of the memory, so cudaMalloc
// there can fail, and it would synchronise the device), or a serving loop held
// to a fixed memory plan. The state words must outlive every call (the epoch
// advances once per call, in step with the peers) and start at zero, so such
// a caller has nowhere to keep them. The flag arrays and full-y buffers are
// shared with the peers and are still the caller's (created once, with the
// group, by code that may allocate).
//
// Here the state lives in a fixed 256-byte array per device, held by every
// device that loads this library until the process exits: one {arrived CTAs,
// epoch} pair per exchange slot, kNoAllocExchanges (32) slots. A slot stands
// for one group's sequence of exchanges with one set of zeroed flag arrays;
// every rank of the group names the same slot on every call. Slots at or
// beyond 32 return BNBQ_ERR_TOO_LARGE.
namespace bnbq {
namespace {

constexpr int kNoAllocExchanges = 32;
constexpr int kNoAllocMaxDevices = 64;

// On the host this name is only a stand-in symbol, not a device address: a
// kernel given it would fault (or reach host memory). Host code passes the
// address that cudaGetSymbolAddress returns for the current device. Module
// loading zero-fills it, which is the state every slot must start from.
static __device__ __align__(256) uint32_t g_allgather_state[2 * kNoAllocExchanges];

std::mutex g_noalloc_mu;
uint32_t* g_noalloc_state[kNoAllocMaxDevices] = {};  // per device, once set up

// Set-up of the current device, once per process: the device address of its
// state array (loading the module if it is not loaded yet). Nothing is
// written: the array is zero from module load, the arrival counters return
// to zero at the end of every call, and the epochs must keep their values.
int noalloc_state(uint32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BNBQ_ERR_CUDA;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return BNBQ_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_state[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_allgather_state) != cudaSuccess || !p) return BNBQ_ERR_CUDA;
    g_noalloc_state[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_noalloc_state[dev];
  return BNBQ_OK;
}

}  // namespace
}  // namespace bnbq

// The set-up alone, for the current device: a caller that captures its
// exchanges into a CUDA graph or command buffer makes this call first (for
// example from a handler's prepare stage); otherwise the first exchange on a
// device does it.
extern "C" int bnbq_peer_allgather_noalloc_setup(void) {
  uint32_t* state = nullptr;
  return noalloc_state(&state);
}

// Puts slot `exchange` back to zero on `stream` (stream-ordered, no host
// synchronisation): for a slot taken over by another group or by a group with
// new, zeroed flag arrays. Every rank of the group resets the slot before its
// first exchange through it.
extern "C" int bnbq_peer_allgather_noalloc_reset(int32_t exchange, void* stream) {
  if (exchange < 0) return BNBQ_ERR_INVALID;
  if (exchange >= kNoAllocExchanges) return BNBQ_ERR_TOO_LARGE;
  uint32_t* state = nullptr;
  if (int st = noalloc_state(&state)) return st;
  if (cudaMemsetAsync(state + 2 * exchange, 0, 2 * sizeof(uint32_t), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return BNBQ_ERR_CUDA;
  return BNBQ_OK;
}

// Calls on one device share the array: two calls whose kernels overlap on
// the GPU with the same slot race on its counter and epoch.
extern "C" int bnbq_peer_allgather_rows_noalloc(int dtype, const void* y_local, int32_t m, int64_t n_local,
                                                int64_t ld_local, int64_t col0, int64_t ldy, void* const* y_full,
                                                uint32_t* const* flags, int32_t exchange, int32_t world,
                                                int32_t rank, void* stream) {
  if (exchange < 0) return BNBQ_ERR_INVALID;
  if (exchange >= kNoAllocExchanges) return BNBQ_ERR_TOO_LARGE;
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  uint32_t* state = nullptr;
  if (int st = noalloc_state(&state)) return st;
  return bnbq_peer_allgather_rows(dtype, y_local, m, n_local, ld_local, col0, ldy, y_full, flags,
                                  state + 2 * exchange, world, rank, stream);
}
