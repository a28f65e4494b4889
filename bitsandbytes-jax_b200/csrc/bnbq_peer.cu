// bnbq_peer.cu -- all-gather of row-sharded GEMV/GEMM outputs over NVLink peer
// memory (the exchange step of the N-sharded matmul).
//
// Every rank computes y[:, col0 : col0 + n_local] with the fused kernels and
// then launches bnbq_peer_allgather_rows on the same stream (programmatic
// dependent launch: it starts while the matmul drains and waits for it with
// griddepcontrol.wait).
//
// Protocol (device side in bnbq_peer.cuh): tagged words in a double-buffered
// inbox, one per rank.
//   * Rank d's inbox is a uint64 array of `inbox_words` words (zeroed once),
//     shared with the peers through CUDA IPC. Its two halves alternate by the
//     parity of the call's epoch e (kept in device memory in state[1] and
//     advanced once per call, so replays of a captured CUDA graph stay in
//     step). Word r * n_total + c of a half holds output element (r, c) as
//     value | e << 32 in one 8-byte store.
//   * Each CTA stores its share of this rank's slice into every peer's inbox
//     (plain relaxed system-scope stores over NVLink; no multicast, no TMA,
//     no fences) and straight into this rank's own output, then polls its
//     share of the other columns in its OWN inbox (local memory) until each
//     word carries epoch e, and unpacks it into the output. Peers never write
//     the output itself, so it stays valid until this rank's next call on
//     the stream.
//   * No handshake guards the inbox: a peer can store call e + 2 into the
//     half this rank reads for call e only after the peer finished call e + 1,
//     which needed this rank's call-(e + 1) slice, which this rank sends only
//     after its call-e kernel (and the matmul between them) has completed.
//   * A word can be mistaken for a current one only if it was written exactly
//     a multiple of 2^32 calls earlier and never since.
// The last CTA (a local arrival counter in state[0], which it resets) stores
// the epoch. Every wait is bounded in time from the start of the receive
// phase (10 s by default); on expiry the CTA counts a timeout
// (bnbq_wait_timeouts), leaves the words it did not receive unwritten in the
// output and returns.
//
// The matmul kernels that can finish with the exchange themselves (M <= 2,
// every CTA resident at once) take the same PeerOut and do both halves in
// their epilogue; bnbq_matmul_nf4_allgather picks them and falls back to the
// matmul plus this kernel.
#include "bnbq_common.cuh"
#include "bnbq_peer.cuh"

namespace bnbq {
namespace {

constexpr int kPeerMaxWorld = 64;
constexpr int kPeerThreads = 256;
constexpr int kPeerBatch = 4;  // words per thread with their loads in flight together

// y_local: m x n_local (row stride ld_local) 16-bit values; px: the exchange
// (its y_full is this rank's m x n_total output).
__global__ void __launch_bounds__(kPeerThreads) peer_allgather_kernel(const uint16_t* y_local, int m,
                                                                      int64_t n_local, int64_t ld_local, PeerOut px) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the matmul that wrote y_local has completed
  // every thread reads the epoch (stored by the last CTA only, once every
  // thread of the launch has read it and passed the final barrier)
  const uint32_t epoch = peer_epoch(px);
  const int64_t step = int64_t(gridDim.x) * kPeerThreads;
  const int64_t tid = int64_t(blockIdx.x) * kPeerThreads + threadIdx.x;
  uint16_t* y_full = static_cast<uint16_t*>(px.y_full);

  // send: this rank's slice into every peer's inbox and its own output
  const int64_t sends = int64_t(m) * n_local;
  for (int64_t i0 = tid; i0 < sends; i0 += kPeerBatch * step) {
    uint16_t v[kPeerBatch];
    int64_t r[kPeerBatch], c[kPeerBatch];
#pragma unroll
    for (int j = 0; j < kPeerBatch; ++j) {
      const int64_t i = i0 + j * step;
      r[j] = i / n_local;
      c[j] = i - r[j] * n_local;
      if (i < sends) v[j] = y_local[r[j] * ld_local + c[j]];
    }
#pragma unroll
    for (int j = 0; j < kPeerBatch; ++j) {
      if (i0 + j * step >= sends) break;
      peer_send(px, epoch, r[j], c[j], v[j]);
      y_full[r[j] * px.ldf + px.col0 + c[j]] = v[j];
    }
  }

  // receive: the other ranks' columns from this rank's own inbox
  const bool ok = peer_receive(px, epoch, m, n_local, tid, step);
  const int expired = __syncthreads_or(!ok);
  if (threadIdx.x == 0) peer_finish_cta(px, epoch, expired != 0);
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

namespace bnbq {

// Checks the exchange arguments shared by the standalone all-gather and the
// matmuls that end with it, and fills *px.
int peer_make(int dtype, int32_t m, int64_t n_local, int64_t col0, void* y_full, int64_t n_total, int64_t ldy,
              uint64_t* const* inbox, int64_t inbox_words, uint32_t* state, int32_t world, int32_t rank,
              PeerOut* px) {
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (m < 0 || n_local < 0 || world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world || col0 < 0 ||
      n_total < col0 + n_local || ldy < n_total || inbox_words < 0)
    return BNBQ_ERR_INVALID;
  if (world == 1 && (col0 != 0 || n_local != n_total)) return BNBQ_ERR_INVALID;  // no one else owns a column
  if (int64_t(m) * n_total > inbox_words / 2) return BNBQ_ERR_TOO_LARGE;
  if (!inbox || !state || (m > 0 && n_total > 0 && !y_full)) return BNBQ_ERR_INVALID;
  if (!aligned(y_full, 2) || !aligned(state, 4) || !aligned(inbox, 8)) return BNBQ_ERR_MISALIGNED;
  px->inbox = inbox;
  px->state = state;
  px->y_full = y_full;
  px->n_total = n_total;
  px->ldf = ldy;
  px->col0 = col0;
  px->half = inbox_words / 2;
  px->world = world;
  px->rank = rank;
  return BNBQ_OK;
}

// The standalone exchange kernel behind the matmul that wrote y_local.
int peer_allgather_launch(const void* y_local, int32_t m, int64_t n_local, int64_t ld_local, const PeerOut& px,
                          cudaStream_t stream) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  // one word per thread and pass, at most four CTAs per SM (all resident)
  const int64_t work = int64_t(m) * (n_local > px.n_total - n_local ? n_local : px.n_total - n_local);
  int64_t grid = (work + kPeerThreads - 1) / kPeerThreads;
  if (grid < 1) grid = 1;
  if (grid > 4 * int64_t(di.sm_count)) grid = 4 * int64_t(di.sm_count);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kPeerThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, peer_allgather_kernel, static_cast<const uint16_t*>(y_local), int(m), n_local,
                         ld_local, px) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

}  // namespace bnbq

extern "C" int bnbq_peer_allgather_rows(int dtype, const void* y_local, int32_t m, int64_t n_local, int64_t ld_local,
                                        int64_t col0, void* y_full, int64_t n_total, int64_t ldy,
                                        uint64_t* const* inbox, int64_t inbox_words, uint32_t* state, int32_t world,
                                        int32_t rank, void* stream) {
  PeerOut px;
  if (int st = peer_make(dtype, m, n_local, col0, y_full, n_total, ldy, inbox, inbox_words, state, world, rank, &px))
    return st;
  if (ld_local < n_local || (m > 0 && n_local > 0 && !y_local)) return BNBQ_ERR_INVALID;
  if (!aligned(y_local, 2)) return BNBQ_ERR_MISALIGNED;
  return peer_allgather_launch(y_local, m, n_local, ld_local, px, static_cast<cudaStream_t>(stream));
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
// a caller has nowhere to keep them. The inboxes (shared with the peers) and
// the output are still the caller's (the inboxes are created once, with the
// group, by code that may allocate).
//
// Here the state lives in a fixed 256-byte array per device, held by every
// device that loads this library until the process exits: one {arrived CTAs,
// epoch} pair per exchange slot, kNoAllocExchanges (32) slots. A slot stands
// for one group's sequence of exchanges with one set of zeroed inboxes;
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
// new, zeroed inboxes. Every rank of the group resets the slot before its
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
                                                int64_t ld_local, int64_t col0, void* y_full, int64_t n_total,
                                                int64_t ldy, uint64_t* const* inbox, int64_t inbox_words,
                                                int32_t exchange, int32_t world, int32_t rank, void* stream) {
  if (exchange < 0) return BNBQ_ERR_INVALID;
  if (exchange >= kNoAllocExchanges) return BNBQ_ERR_TOO_LARGE;
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  uint32_t* state = nullptr;
  if (int st = noalloc_state(&state)) return st;
  return bnbq_peer_allgather_rows(dtype, y_local, m, n_local, ld_local, col0, y_full, n_total, ldy, inbox,
                                  inbox_words, state + 2 * exchange, world, rank, stream);
}
