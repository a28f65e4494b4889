// bnbq_gemv.cu -- fused NF4 dequantize-GEMV for 1 <= M <= 20 (CUDA cores).
//
// y[m, j] = sum_k x[m, k] * W[j, k], W NF4 (j < n_rows, k < K), never decoded to
// memory. Numerics as the reference GEMV (kernels/gemv.py:97-123): per
// 32-element chunk t = sum table[q] * x in float32 (here as two interleaved
// float32 partial sums, fma.rn.f32x2), then acc += a * t with the chunk's block
// scale a, and one rounding of the final sum to x's dtype. bs >= 32 and
// K % 32 == 0 keep a chunk inside one block. A one-hot x reproduces the
// dequantized weights bitwise: every product but one is an exact zero.
//
// Mapping. A CTA owns R consecutive rows over the whole K; its W warps split
// the K/32 chunks of those rows (thread t takes chunks t, t + 32W, ...), so a
// warp's code loads are one coalesced 512-byte run per row, and the host picks
// W so that K/32 divides evenly (e.g. K = 14336: 448 chunks = 2 x 7 warps x 32).
// CTAs are R rows, so N/R of them balance across the 148 SMs to within one CTA.
// x (M x K, <= 573 KB) is re-read from L1/L2 by every CTA; its loads are
// shared by the R rows of the CTA. Partial sums are reduced by warp
// butterflies and once through shared memory.
//
// The nested (double-quantized) scale is decoded per chunk and row:
//   a = fl32(mul.ftz(code2[absmax_q[blk]], absmax2[(block0 + blk) >> log2 bs2]) + offset)
// bitwise the value QuantizedArray.dequantize produces (array.py:95-108).
#include "bnbq_common.cuh"

namespace bnbq {
namespace {

struct GemvArgs {
  const void* x;
  const uint8_t* w;
  const float* absmax;
  const uint8_t* absmax_q;
  const float* absmax2;
  const float* code2;
  const float* offset;
  void* y;
  int64_t n_rows;
  int64_t ldy;
  int64_t block0;
  int k;
  int log2_bs;
  int log2_bs2;
};

template <typename XT>
__device__ __forceinline__ float2 unpack_x(uint32_t w) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) return unpack2_bf16(w);
  else return unpack2_f16(w);
}

template <typename XT>
__device__ __forceinline__ void store_y(void* y, int64_t i, float v) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(y)[i] = __float2half_rn(v);
}

constexpr int kMaxWarps = 8;

template <typename XT, int M, int R, bool NESTED>
__global__ void __launch_bounds__(kMaxWarps * 32)
gemv_kernel(GemvArgs a) {
  __shared__ float s_table[16];
  __shared__ float s_code2[NESTED ? 256 : 1];
  __shared__ float s_red[kMaxWarps][M * R];
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5;
  if (tid < 16) s_table[tid] = kNF4Table[tid];
  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += nthreads) s_code2[i] = __ldg(a.code2 + i);
  }
  __syncthreads();

  const int64_t row0 = int64_t(blockIdx.x) * R;
  const int cpr = a.k >> 5;  // chunks per row
  const float offset = NESTED ? __ldg(a.offset) : 0.0f;
  const XT* x = static_cast<const XT*>(a.x);

  int64_t rows[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rows[r] = min(row0 + r, a.n_rows - 1);  // clamp; results dropped

  float acc[M][R];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[m][r] = 0.0f;

  for (int c = tid; c < cpr; c += nthreads) {
    uint4 codes[R];
    float scale[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t e0 = rows[r] * a.k + int64_t(c) * 32;  // element index in this shard
      codes[r] = __ldg(reinterpret_cast<const uint4*>(a.w + (e0 >> 1)));
      const int64_t blk = e0 >> a.log2_bs;
      if constexpr (NESTED) {
        const int q2 = __ldg(a.absmax_q + blk);
        scale[r] = add_rn(mul_ftz(s_code2[q2], __ldg(a.absmax2 + ((a.block0 + blk) >> a.log2_bs2))), offset);
      } else {
        scale[r] = __ldg(a.absmax + blk);
      }
    }
    float2 t[M][R];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < R; ++r) t[m][r] = make_float2(0.0f, 0.0f);

#pragma unroll
    for (int i = 0; i < 4; ++i) {  // 8 elements: one 32-bit code word per row
      float wv[R][8];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t word = i == 0 ? codes[r].x : i == 1 ? codes[r].y : i == 2 ? codes[r].z : codes[r].w;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          wv[r][2 * j] = s_table[(word >> (8 * j + 4)) & 15u];  // high nibble first
          wv[r][2 * j + 1] = s_table[(word >> (8 * j)) & 15u];
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + int64_t(m) * a.k + c * 32 + i * 8));
        const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 xf = unpack_x<XT>(xs[j]);
#pragma unroll
          for (int r = 0; r < R; ++r) fma2(t[m][r], make_float2(wv[r][2 * j], wv[r][2 * j + 1]), xf);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < R; ++r) acc[m][r] = __fmaf_rn(scale[r], t[m][r].x + t[m][r].y, acc[m][r]);
  }

  // CTA reduction: butterfly within each warp, then across warps in smem.
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = acc[m][r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) s_red[warp][m * R + r] = v;
    }
  __syncthreads();
  const int nw = nthreads >> 5;
  for (int i = tid; i < M * R; i += nthreads) {
    float v = 0.0f;
    for (int w = 0; w < nw; ++w) v += s_red[w][i];
    const int m = i / R, r = i % R;
    if (row0 + r < a.n_rows) store_y<XT>(a.y, int64_t(m) * a.ldy + row0 + r, v);
  }
}

// Rows per CTA: enough to share each x load, few enough to keep registers.
constexpr int rows_for(int M) { return M <= 4 ? 4 : (M <= 8 ? 2 : 1); }

// Warps per CTA so that the K/32 chunks split evenly (fewest idle lanes).
int pick_warps(int cpr) {
  int best = 8;
  double best_eff = 0.0;
  for (int w = 8; w >= 4; --w) {
    const int slots = 32 * w;
    const int iters = (cpr + slots - 1) / slots;
    const double eff = double(cpr) / double(iters * slots);
    if (eff > best_eff + 1e-9) { best_eff = eff; best = w; }
  }
  return best;
}

template <typename XT, int M, bool NESTED>
int launch_m(const GemvArgs& a, cudaStream_t s) {
  constexpr int R = rows_for(M);
  const int warps = pick_warps(a.k >> 5);
  const int64_t grid = (a.n_rows + R - 1) / R;
  gemv_kernel<XT, M, R, NESTED><<<dim3(unsigned(grid)), dim3(warps * 32), 0, s>>>(a);
  return launch_status();
}

template <typename XT, bool NESTED, int M = 1>
int launch_dispatch(int m, const GemvArgs& a, cudaStream_t s) {
  if constexpr (M > BNBQ_GEMV_MAX_M) {
    return BNBQ_ERR_INVALID;
  } else {
    if (m == M) return launch_m<XT, M, NESTED>(a, s);
    return launch_dispatch<XT, NESTED, M + 1>(m, a, s);
  }
}

}  // namespace

// Validation shared with the GEMM path (bnbq_gemm.cu).
int gemv_validate(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                  int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                  const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                  void* y, int64_t ldy) {
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (m < 1 || k < 32 || (k & 31) || n_rows < 1 || ldy < n_rows) return BNBQ_ERR_INVALID;
  const int l2 = log2_exact(blocksize);
  if (l2 < 5) return BNBQ_ERR_INVALID;
  if (!x || !w || !y) return BNBQ_ERR_INVALID;
  if (absmax_q) {
    if (!absmax2 || !code2 || !offset || log2_exact(blocksize2) < 0) return BNBQ_ERR_INVALID;
    if (!aligned(absmax2, 4) || !aligned(code2, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  } else {
    if (!absmax) return BNBQ_ERR_INVALID;
    if (!aligned(absmax, 4)) return BNBQ_ERR_MISALIGNED;
  }
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 2)) return BNBQ_ERR_MISALIGNED;
  return BNBQ_OK;
}

int gemv_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                int64_t absmax2_block0, void* y, int64_t ldy, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  GemvArgs a{};
  a.x = x; a.w = w; a.absmax = absmax; a.absmax_q = absmax_q; a.absmax2 = absmax2;
  a.code2 = code2; a.offset = offset; a.y = y; a.n_rows = n_rows; a.ldy = ldy;
  a.block0 = absmax2_block0; a.k = k; a.log2_bs = log2_exact(blocksize);
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  const bool nested = absmax_q != nullptr;
  if (dtype == BNBQ_BF16)
    return nested ? launch_dispatch<__nv_bfloat16, true>(m, a, s) : launch_dispatch<__nv_bfloat16, false>(m, a, s);
  return nested ? launch_dispatch<__half, true>(m, a, s) : launch_dispatch<__half, false>(m, a, s);
}

}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_gemv_nf4(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                             int64_t n_rows, int32_t blocksize, const float* absmax,
                             const uint8_t* absmax_q, const float* absmax2, const float* code2,
                             const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                             void* y, int64_t ldy, void* stream) {
  if (int st = gemv_validate(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                             offset, blocksize2, y, ldy))
    return st;
  if (m > BNBQ_GEMV_MAX_M) return BNBQ_ERR_INVALID;
  return gemv_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2, offset,
                     blocksize2, absmax2_block0, y, ldy, static_cast<cudaStream_t>(stream));
}
