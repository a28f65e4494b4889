// bnbq_abi.cu -- device checks, status strings, diagnostics and the matmul router.
#include <map>
#include <mutex>
#include <tuple>

#include "bnbq_common.cuh"

namespace bnbq {

int gemv_validate(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                  int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                  const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                  void* y, int64_t ldy);
int gemv_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                int64_t absmax2_block0, void* y, int64_t ldy, cudaStream_t s);
int gemv_wait_timeouts(unsigned int* out);
int gemm_wait_timeouts(unsigned int* out);
int peer_wait_timeouts(unsigned int* out);
int xtab_wait_timeouts(unsigned int* out);
int quant_wait_timeouts(unsigned int* out);
int gemv_set_wait_limit(uint64_t ns);
int gemm_set_wait_limit(uint64_t ns);
int peer_set_wait_limit(uint64_t ns);
int xtab_set_wait_limit(uint64_t ns);
int quant_set_wait_limit(uint64_t ns);
int gemm_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                int64_t absmax2_block0, void* y, int64_t ldy, cudaStream_t s);

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_once[kMaxDevices];
DeviceInfo g_info[kMaxDevices];
int g_status[kMaxDevices];

__global__ void rcp_kernel(const float* in, float* out, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    out[i] = rcp_approx_ftz(in[i]);
}
}  // namespace

// Queried once per device; the kernels are built for sm_100a only.
namespace {
// (kernel, device) -> static shared memory and the dynamic shared memory
// attribute set so far; (kernel, device, threads, dynamic bytes) -> blocks per SM
struct FuncState {
  int static_smem = -1;
  int dyn_set = -1;
};
std::mutex g_func_mu;
std::map<std::pair<const void*, int>, FuncState> g_func;
std::map<std::tuple<const void*, int, int, size_t>, int> g_occ;
}  // namespace

int kernel_static_smem(const void* fn, int* bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BNBQ_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_func_mu);
  FuncState& f = g_func[{fn, dev}];
  if (f.static_smem < 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess) return BNBQ_ERR_CUDA;
    f.static_smem = int(fa.sharedSizeBytes);
  }
  *bytes = f.static_smem;
  return BNBQ_OK;
}

int kernel_reserve_smem(const void* fn, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BNBQ_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_func_mu);
  FuncState& f = g_func[{fn, dev}];
  if (bytes > f.dyn_set) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return BNBQ_ERR_CUDA;
    f.dyn_set = bytes;
  }
  return BNBQ_OK;
}

int kernel_occupancy(const void* fn, int threads, size_t dyn_bytes, int* per_sm) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BNBQ_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_func_mu);
  auto key = std::make_tuple(fn, dev, threads, dyn_bytes);
  auto it = g_occ.find(key);
  if (it == g_occ.end()) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, dyn_bytes) != cudaSuccess)
      return BNBQ_ERR_CUDA;
    it = g_occ.emplace(key, n).first;
  }
  *per_sm = it->second;
  return BNBQ_OK;
}

int device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BNBQ_ERR_CUDA;
  std::call_once(g_once[dev], [dev] {
    DeviceInfo di;
    int st = BNBQ_OK;
    if (cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&di.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&di.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&di.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      st = BNBQ_ERR_CUDA;
    else if (di.cc_major != 10 || di.cc_minor != 0)
      st = BNBQ_ERR_DEVICE;
    g_info[dev] = di;
    g_status[dev] = st;
  });
  *out = g_info[dev];
  return g_status[dev];
}

}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_matmul_nf4(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                               int64_t n_rows, int32_t blocksize, const float* absmax,
                               const uint8_t* absmax_q, const float* absmax2, const float* code2,
                               const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                               void* y, int64_t ldy, void* stream) {
  if (int st = gemv_validate(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                             offset, blocksize2, y, ldy))
    return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (m <= BNBQ_GEMV_MAX_M)
    return gemv_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                       offset, blocksize2, absmax2_block0, y, ldy, s);
  return gemm_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                     offset, blocksize2, absmax2_block0, y, ldy, s);
}

extern "C" int bnbq_gemv_nf4_ws(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                int64_t n_rows, int32_t blocksize, const float* absmax,
                                const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                void* y, int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream);

extern "C" int bnbq_matmul_nf4_ws(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                  int64_t n_rows, int32_t blocksize, const float* absmax,
                                  const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                  const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                  void* y, int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream) {
  if (m >= 1 && m <= BNBQ_GEMV_MAX_M)
    return bnbq_gemv_nf4_ws(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2, offset,
                            blocksize2, absmax2_block0, y, ldy, workspace, workspace_bytes, stream);
  return bnbq_matmul_nf4(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2, offset,
                         blocksize2, absmax2_block0, y, ldy, stream);
}

extern "C" int bnbq_rcp_approx_ftz(const float* in, float* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out))) return BNBQ_ERR_INVALID;
  if (!aligned(in, 4) || !aligned(out, 4)) return BNBQ_ERR_MISALIGNED;
  if (n == 0) return BNBQ_OK;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  int64_t grid = (n + 255) / 256;
  if (grid > int64_t(di.sm_count) * 8) grid = int64_t(di.sm_count) * 8;
  rcp_kernel<<<dim3(unsigned(grid)), 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, n);
  return launch_status();
}

extern "C" int bnbq_wait_timeouts(unsigned int* count) {
  if (!count) return BNBQ_ERR_INVALID;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  // one counter per source file with bounded waits (each has its own copy)
  unsigned int g = 0, h = 0, p = 0, t = 0, q = 0;
  if (gemv_wait_timeouts(&g) != 0 || gemm_wait_timeouts(&h) != 0 || peer_wait_timeouts(&p) != 0 ||
      xtab_wait_timeouts(&t) != 0 || quant_wait_timeouts(&q) != 0)
    return BNBQ_ERR_CUDA;
  *count = g + h + p + t + q;
  return BNBQ_OK;
}

extern "C" int bnbq_enable_peer_access(int peer_device) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BNBQ_ERR_CUDA;
  if (peer_device == dev) return BNBQ_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, dev, peer_device) != cudaSuccess) return BNBQ_ERR_CUDA;
  if (!can) return BNBQ_ERR_UNSUPPORTED;
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // clear the non-sticky status
    return BNBQ_OK;
  }
  return e == cudaSuccess ? BNBQ_OK : BNBQ_ERR_CUDA;
}

extern "C" int bnbq_set_wait_limit_ns(uint64_t ns) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if (gemv_set_wait_limit(ns) != 0 || gemm_set_wait_limit(ns) != 0 || peer_set_wait_limit(ns) != 0 ||
      xtab_set_wait_limit(ns) != 0 || quant_set_wait_limit(ns) != 0)
    return BNBQ_ERR_CUDA;
  return BNBQ_OK;
}

extern "C" const char* bnbq_error_string(int status) {
  switch (status) {
    case BNBQ_OK: return "ok";
    case BNBQ_ERR_INVALID: return "invalid argument";
    case BNBQ_ERR_UNSUPPORTED: return "unsupported dtype or shape";
    case BNBQ_ERR_MISALIGNED: return "misaligned pointer";
    case BNBQ_ERR_CUDA: return "CUDA error";
    case BNBQ_ERR_DEVICE: return "device is not sm_100 (B200)";
    case BNBQ_ERR_TOO_LARGE: return "larger than the fixed scratch of a no-allocation entry point";
    default: return "unknown status";
  }
}

extern "C" int bnbq_version(void) { return 100; }
