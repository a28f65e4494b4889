// bnbq_gemv_t.cu -- the backward of the fused matmul for a few rows of g:
// out[m, k] = sum_n g[m, n] * W[n, k] for an NF4 weight W (n_rows x K), never
// decoded to memory (the reference computes g @ w.dequantize(g.dtype),
// _matmul.py:67-68: the weight materialised in g's dtype, then a dense GEMM).
//
// Numerics: every weight is its exact dequantized float32 value,
// w = mul.ftz(T[q], a) with the block scale a (float32 absmax, or the
// double-quantized one decoded as QuantizedArray.dequantize does,
// array.py:95-108), multiplied by g in float32 and accumulated in float32 in a
// fixed order (rows of a warp in order, the warps of a CTA in order, the row
// parts in order), rounded once to g's dtype. A one-hot g returns the
// dequantized weight row, bitwise.
//
// Mapping. The columns are cut into groups of 256 (K % 256 == 0) and the rows
// into P parts; a unit is (part, group). One CTA per SM slot (persistent,
// two per SM) builds the byte -> (T[hi], T[lo]) pair table once (one copy per
// lane, so a warp's 32 pair loads hit 32 distinct banks) and walks its units.
// In a
// unit, lane l of every warp owns code word l of the group (columns 8l ..
// 8l + 7); warp w takes the part's rows w, w + 8, ..., loading the code words
// and scales of 8 rows before it decodes any (each row's 32 words are one
// coalesced 128-byte load). Per row: 4 pair loads, 4 packed mul.ftz by the
// block scale, 4 M packed FMAs with g. The 8 warps' sums meet in shared
// memory, are added in warp order, and the unit's 256 x M float32 partials go
// to the caller's workspace. A second kernel (programmatic dependent launch:
// it waits for the first with griddepcontrol.wait) adds each output's P
// partials in part order and rounds once. Deterministic; the workspace needs
// no initial contents.
//
// Measured on a B200 (config 2's weight, 4096 x 14336, M = 1): 67.7 us against
// 58.5 us for the reference's rule (our dequantize kernel, then cuBLAS). The
// kernel is memory-latency bound (long-scoreboard stalls first, 22 % issue
// active): a warp has only 8 rows x 128 bytes of codes in flight. So
// bnb_b200.matmul's backward keeps the rule, and this entry point is offered
// as the fused path that needs no dense weight in memory.
#include <atomic>

#include "bnbq_common.cuh"

namespace bnbq {
namespace {

constexpr int kTWarps = 8;
constexpr int kTThreads = kTWarps * 32;
constexpr int kTGroup = 256;               // columns per unit (one code word of 8 per lane)
constexpr int kTBatch = 8;                 // rows a warp loads before decoding them
constexpr int kTMaxRows = 512;             // rows per part at most
constexpr uint32_t kTPairBytes = 256 * 32 * 8;
constexpr int kTMaxM = 4;

struct GemvTArgs {
  const void* g;            // M x n_rows, row stride ldg elements
  const uint8_t* w;         // n_rows x K/2 code bytes
  const float* absmax;      // plain scales (absmax_q == nullptr)
  const uint8_t* absmax_q;  // double-quantized scales
  const float* absmax2;
  const float* code2;
  const float* offset;
  float* partial;           // [P][M][K]
  int64_t n_rows, ldg, block0;
  int k, log2_bs, log2_bs2, groups, parts, rows_per_part;
  int64_t units;
};

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

template <typename XT, int M, bool NESTED>
__global__ void __launch_bounds__(kTThreads, 2) gemv_t_kernel(const GemvTArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  float2* s_pair = reinterpret_cast<float2*>(smem);                       // [256][32]
  float* s_red = reinterpret_cast<float*>(smem + kTPairBytes);            // [8][M][256]
  float* s_g = s_red + kTWarps * M * kTGroup;                             // [M][rows_per_part]
  __shared__ float s_code2[256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  asm volatile("griddepcontrol.launch_dependents;");
  for (int b = warp; b < 256; b += kTWarps)
    s_pair[b * 32 + lane] = make_float2(kNF4Table[b >> 4], kNF4Table[b & 15]);
  float offset = 0.0f;
  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += kTThreads) s_code2[i] = a.code2[i];
    offset = __ldg(a.offset);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // g and the workspace: after the previous kernel
  const XT* g = static_cast<const XT*>(a.g);
  const uint32_t row_bytes = uint32_t(a.k) >> 1;
  for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x) {
    const int p = int(u / a.groups), gk = int(u % a.groups);
    const int64_t r0 = int64_t(p) * a.rows_per_part;
    const int nr = int(min(int64_t(a.rows_per_part), a.n_rows - r0));
    __syncthreads();  // the previous unit's s_g and s_red are no longer read (and the table is built)
    for (int i = tid; i < M * nr; i += kTThreads) {
      const int m = i / nr, r = i - m * nr;
      s_g[m * a.rows_per_part + r] = Elem<XT>::to_f32(g[int64_t(m) * a.ldg + r0 + r]);
    }
    __syncthreads();
    const int col = gk * kTGroup + 8 * lane;  // this lane's first column
    float2 acc[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.0f, 0.0f);
    for (int rb = warp; rb < nr; rb += kTWarps * kTBatch) {
      uint32_t cw[kTBatch];
      float sa[kTBatch];
      // loads of the batch: code words, then scales
#pragma unroll
      for (int i = 0; i < kTBatch; ++i) {
        const int r = rb + i * kTWarps;
        const int64_t row = r0 + min(r, nr - 1);
        cw[i] = __ldg(reinterpret_cast<const uint32_t*>(a.w + row * row_bytes + (col >> 1)));
      }
#pragma unroll
      for (int i = 0; i < kTBatch; ++i) {
        const int r = rb + i * kTWarps;
        const int64_t row = r0 + min(r, nr - 1);
        const int64_t blk = (row * a.k + col) >> a.log2_bs;
        if constexpr (NESTED) {
          const int q2 = __ldg(a.absmax_q + blk);
          const float a2 = __ldg(a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
          sa[i] = add_rn(mul_ftz(s_code2[q2], a2), offset);
        } else {
          sa[i] = __ldg(a.absmax + blk);
        }
      }
#pragma unroll
      for (int i = 0; i < kTBatch; ++i) {
        const int r = rb + i * kTWarps;
        if (r >= nr) break;  // warp-uniform
        float2 wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = (cw[i] >> (8 * j)) & 0xffu;
          wv[j] = mul_ftz2(s_pair[byte * 32 + lane], make_float2(sa[i], sa[i]));
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float gv = s_g[m * a.rows_per_part + r];
          const float2 g2 = make_float2(gv, gv);
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[m][j] = ffma2(wv[j], g2, acc[m][j]);
        }
      }
    }
    // the warps' sums, added in warp order
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float2*>(&s_red[(warp * M + m) * kTGroup + 8 * lane + 2 * j]) = acc[m][j];
    __syncthreads();
    for (int i = tid; i < M * kTGroup; i += kTThreads) {
      const int m = i / kTGroup, c = i - m * kTGroup;
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < kTWarps; ++w) v += s_red[(w * M + m) * kTGroup + c];
      __stcg(a.partial + (int64_t(p) * M + m) * a.k + int64_t(gk) * kTGroup + c, v);
    }
  }
}

// out[m, k] = round(sum over parts, in order, of partial[p][m][k])
template <typename XT, int M>
__global__ void __launch_bounds__(256) gemv_t_reduce_kernel(const float* partial, int parts, int k, void* out,
                                                            int64_t ldo) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // every partial of the first kernel is visible
  const int64_t total = int64_t(M) * k;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / k), c = int(i - int64_t(m) * k);
    float v = 0.0f;
    for (int p = 0; p < parts; ++p) v += __ldcg(partial + (int64_t(p) * M + m) * k + c);
    XT* o = static_cast<XT*>(out);
    if constexpr (Elem<XT>::kDtype == BNBQ_BF16) o[int64_t(m) * ldo + c] = __float2bfloat16_rn(v);
    else o[int64_t(m) * ldo + c] = __float2half_rn(v);
  }
}

// Rows per part: units (parts x groups) that fill `slots` CTA slots evenly,
// with as few parts (partials) as that allows.
void plan_parts(int64_t n_rows, int groups, int slots, int* parts, int* rows_per_part) {
  int best_p = 1;
  double best = -1.0;
  for (int p = 1; p <= 256; ++p) {
    const int64_t rpp = (n_rows + p - 1) / p;
    if (rpp > kTMaxRows) continue;
    if (int64_t(p - 1) * rpp >= n_rows) continue;  // an empty part
    const int64_t units = int64_t(p) * groups;
    const int64_t rounds = (units + slots - 1) / slots;
    const double eff = double(units) / double(rounds * slots) * (units >= slots ? 1.0 : double(units) / slots);
    if (eff > best + 0.02) {
      best = eff;
      best_p = p;
    }
  }
  *parts = best_p;
  *rows_per_part = int((n_rows + best_p - 1) / best_p);
}

size_t smem_for(int m, int rows_per_part) {
  return size_t(kTPairBytes) + size_t(kTWarps) * m * kTGroup * 4 + size_t(m) * rows_per_part * 4;
}

template <typename XT, int M, bool NESTED>
int launch_t(const GemvTArgs& a0, void* out, int64_t ldo, int64_t workspace_bytes, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  GemvTArgs a = a0;
  auto kern = gemv_t_kernel<XT, M, NESTED>;
  const size_t smem = smem_for(M, kTMaxRows);
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  int per_sm = 0;
  if (int st = kernel_occupancy(reinterpret_cast<const void*>(kern), kTThreads, smem, &per_sm)) return st;
  if (per_sm < 1) return BNBQ_ERR_UNSUPPORTED;
  const int slots = di.sm_count * per_sm;
  plan_parts(a.n_rows, a.groups, slots, &a.parts, &a.rows_per_part);
  if (workspace_bytes < int64_t(a.parts) * M * a.k * 4) return BNBQ_ERR_INVALID;  // (the plan's partials)
  a.units = int64_t(a.parts) * a.groups;
  int64_t grid = a.units < slots ? a.units : slots;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kTThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return BNBQ_ERR_CUDA;
  cudaLaunchConfig_t rc = cfg;
  const int64_t total = int64_t(M) * a.k;
  int64_t rgrid = (total + 255) / 256;
  if (rgrid > int64_t(di.sm_count) * 8) rgrid = int64_t(di.sm_count) * 8;
  rc.gridDim = dim3(unsigned(rgrid));
  rc.blockDim = dim3(256);
  rc.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&rc, gemv_t_reduce_kernel<XT, M>, static_cast<const float*>(a.partial), a.parts, a.k, out,
                         ldo) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, bool NESTED>
int launch_m(int m, const GemvTArgs& a, void* out, int64_t ldo, int64_t ws, cudaStream_t s) {
  switch (m) {
    case 1: return launch_t<XT, 1, NESTED>(a, out, ldo, ws, s);
    case 2: return launch_t<XT, 2, NESTED>(a, out, ldo, ws, s);
    case 3: return launch_t<XT, 3, NESTED>(a, out, ldo, ws, s);
    default: return launch_t<XT, 4, NESTED>(a, out, ldo, ws, s);
  }
}

}  // namespace
}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_gemv_t_nf4_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes) {
  if (!bytes || m < 1 || m > kTMaxM || k < 1 || n_rows < 1) return BNBQ_ERR_INVALID;
  if (k % kTGroup || n_rows > int64_t(kTMaxRows) * 256) return BNBQ_ERR_UNSUPPORTED;
  // the plan depends on the device (SM count, occupancy): the size of the
  // largest plan (256 parts) serves every device and shape of this m and k
  *bytes = int64_t(256) * m * k * 4;
  return BNBQ_OK;
}

extern "C" int bnbq_gemv_t_nf4_ws(int dtype, const void* g, int32_t m, int64_t n_rows, int64_t ldg, int32_t k,
                                  const uint8_t* w, int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                                  const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                                  int64_t absmax2_block0, void* out, int64_t ldo, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (m < 1 || m > kTMaxM || n_rows < 1 || k < 1 || ldg < n_rows || ldo < k) return BNBQ_ERR_INVALID;
  if (k % kTGroup || n_rows > int64_t(kTMaxRows) * 256) return BNBQ_ERR_UNSUPPORTED;
  const int l2 = log2_exact(blocksize);
  if (l2 < 3 || !g || !w || !out || !workspace) return BNBQ_ERR_INVALID;
  if (absmax_q) {
    if (!absmax2 || !code2 || !offset || log2_exact(blocksize2) < 0) return BNBQ_ERR_INVALID;
    if (!aligned(absmax2, 4) || !aligned(code2, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  } else {
    if (!absmax) return BNBQ_ERR_INVALID;
    if (!aligned(absmax, 4)) return BNBQ_ERR_MISALIGNED;
  }
  if (!aligned(g, 2) || !aligned(w, 16) || !aligned(out, 2) || !aligned(workspace, 16)) return BNBQ_ERR_MISALIGNED;
  GemvTArgs a{};
  a.g = g; a.w = w; a.absmax = absmax; a.absmax_q = absmax_q; a.absmax2 = absmax2; a.code2 = code2;
  a.offset = offset; a.partial = static_cast<float*>(workspace);
  a.n_rows = n_rows; a.ldg = ldg; a.block0 = absmax2_block0;
  a.k = k; a.log2_bs = l2; a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  a.groups = k / kTGroup;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool nested = absmax_q != nullptr;
  const int64_t ws = workspace_bytes;
  if (dtype == BNBQ_BF16)
    return nested ? launch_m<__nv_bfloat16, true>(m, a, out, ldo, ws, s)
                  : launch_m<__nv_bfloat16, false>(m, a, out, ldo, ws, s);
  return nested ? launch_m<__half, true>(m, a, out, ldo, ws, s) : launch_m<__half, false>(m, a, out, ldo, ws, s);
}
