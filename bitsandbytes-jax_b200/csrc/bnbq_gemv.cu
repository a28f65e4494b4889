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
#include "bnbq_async.cuh"
#include "bnbq_common.cuh"
#include "bnbq_peer.cuh"

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

// v rounded to XT, as its 16 bits
template <typename XT>
__device__ __forceinline__ uint16_t bits_of(float v) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else return __half_as_ushort(__float2half_rn(v));
}

constexpr int kMaxWarps = 16;

// Per-thread loads of one 32-element chunk of R rows (the software-pipeline
// stage). XF: x of every batch row is prefetched with it (small M).
template <int M, int R, bool NESTED, bool XF>
struct Stage {
  uint4 codes[R];
  float scale_or_a2[R];  // plain: the absmax; nested: absmax2
  int q2[R];             // nested: absmax code
  uint4 x[XF ? M : 1][4];
};

template <typename XT, int M, int R, bool NESTED, bool XF>
__device__ __forceinline__ void load_stage(Stage<M, R, NESTED, XF>& st, const GemvArgs& a,
                                           const int64_t (&rows)[R], int c) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t e0 = rows[r] * a.k + int64_t(c) * 32;
    st.codes[r] = __ldg(reinterpret_cast<const uint4*>(a.w + (e0 >> 1)));
    const int64_t blk = e0 >> a.log2_bs;
    if constexpr (NESTED) {
      st.q2[r] = __ldg(a.absmax_q + blk);
      st.scale_or_a2[r] = __ldg(a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
    } else {
      st.scale_or_a2[r] = __ldg(a.absmax + blk);
    }
  }
  if constexpr (XF) {
    const XT* x = static_cast<const XT*>(a.x);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        st.x[m][i] = __ldg(reinterpret_cast<const uint4*>(x + int64_t(m) * a.k + c * 32 + i * 8));
  }
}

// Pair table in dynamic shared memory: entry b (a code byte: high nibble =
// even element, low nibble = odd element) is (table[b >> 4], table[b & 15]),
// replicated once per lane at [b][lane] (256 x 32 x 8 B = 64 KB), so that the
// 32 lanes of a warp read 32 distinct banks whatever their bytes are.
constexpr int kPairTableBytes = 256 * 32 * 8;
extern __shared__ float2 s_pair[];

// The same table in global memory, built at compile time, so a CTA can copy
// it into shared memory 16 bytes per thread at a time (the rows GEMV).
struct PairTable {
  float2 v[256 * 32];
  constexpr PairTable() : v() {
    constexpr float t[16] = {
        -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
        -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
        0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
        0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};
    for (int i = 0; i < 256 * 32; ++i) v[i] = float2{t[(i >> 5) >> 4], t[(i >> 5) & 15]};
  }
};
__device__ __align__(128) const PairTable g_pair_table{};

// Byte offset of (byte j of `word`, this lane) in s_pair: one prmt builds
// (byte << 8) | lane_x8, where lane_x8 = lane * 8 sits in byte 0 of `lane_b`.
__device__ __forceinline__ float2 pair_at(uint32_t word, uint32_t lane_b, int j) {
  const uint32_t off = __byte_perm(word, lane_b, 0x5504 | (j << 4));
  return *reinterpret_cast<const float2*>(reinterpret_cast<const char*>(s_pair) + off);
}

template <typename XT, int M, int R, bool NESTED, bool XF>
__device__ __forceinline__ void compute_stage(const Stage<M, R, NESTED, XF>& st, const GemvArgs& a,
                                              const float* s_code2, float offset, int c,
                                              uint32_t lane_b, float (&acc)[M][R]) {
  float scale[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if constexpr (NESTED) scale[r] = add_rn(mul_ftz(s_code2[st.q2[r]], st.scale_or_a2[r]), offset);
    else scale[r] = st.scale_or_a2[r];
  }
  float2 t[M][R];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) t[m][r] = make_float2(0.0f, 0.0f);
  const XT* x = static_cast<const XT*>(a.x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // 8 elements: one 32-bit code word per row
    float2 wv[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const uint32_t word = i == 0 ? st.codes[r].x : i == 1 ? st.codes[r].y : i == 2 ? st.codes[r].z : st.codes[r].w;
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[r][j] = pair_at(word, lane_b, j);
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      uint4 xv;
      if constexpr (XF) xv = st.x[m][i];
      else xv = __ldg(reinterpret_cast<const uint4*>(x + int64_t(m) * a.k + c * 32 + i * 8));
      const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xf = unpack_x<XT>(xs[j]);
#pragma unroll
        for (int r = 0; r < R; ++r) t[m][r] = __ffma2_rn(wv[r][j], xf, t[m][r]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[m][r] = __fmaf_rn(scale[r], t[m][r].x + t[m][r].y, acc[m][r]);
}

// Persistent: CTA b takes row groups b, b + gridDim.x, ... of R rows; its
// threads split each group's K/32 chunks (thread t: t, t + blockDim, ...).
// The loads of a thread's next chunk (of this group or the next) are issued
// before the current chunk is computed.
// Threads per CTA at most: wide CTAs for small M, 256 (255 registers) above.
constexpr int max_threads_for(int M) { return M == 1 ? kMaxWarps * 32 : 256; }

template <typename XT, int M, int R, bool NESTED>
__global__ void __launch_bounds__(max_threads_for(M))
gemv_kernel(GemvArgs a, int64_t n_groups) {
  constexpr bool XF = M <= 2;
  __shared__ float s_code2[NESTED ? 256 : 1];
  __shared__ float s_red[2][kMaxWarps][M * R];
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 256 * 32; i += nthreads) {
    const int b = i >> 5;
    s_pair[i] = make_float2(kNF4Table[b >> 4], kNF4Table[b & 15]);
  }
  const uint32_t lane_b = uint32_t(lane) * 8u;
  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += nthreads) s_code2[i] = __ldg(a.code2 + i);
  }
  __syncthreads();

  const int cpr = a.k >> 5;
  const float offset = NESTED ? __ldg(a.offset) : 0.0f;
  const int iters = (cpr + nthreads - 1) / nthreads;

  auto rows_of = [&](int64_t g, int64_t (&rows)[R]) {
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = min(g * R + r, a.n_rows - 1);  // clamp; results dropped
  };

  Stage<M, R, NESTED, XF> sa, sb;  // ping-pong stages, kept in registers
  int64_t g = blockIdx.x;
  if (g >= n_groups) return;
  int64_t rows[R];
  rows_of(g, rows);
  int it = 0;
  int c = min(tid, cpr - 1);
  load_stage<XT>(sa, a, rows, c);
  int parity = 0;
  float acc[M][R];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[m][r] = 0.0f;

  // Computes `cur` (this thread's chunk `c` of group `g`) after issuing the
  // loads of the following stage into `nxt`. Returns true when done.
  auto step = [&](Stage<M, R, NESTED, XF>& cur, Stage<M, R, NESTED, XF>& nxt) -> bool {
    int64_t g_next = g;
    int it_next = it + 1;
    if (it_next == iters) { g_next = g + gridDim.x; it_next = 0; }
    int64_t rows_next[R];
    const int c_next = min(tid + it_next * nthreads, cpr - 1);
    if (g_next < n_groups) {
      rows_of(g_next, rows_next);
      load_stage<XT>(nxt, a, rows_next, c_next);
    }
    if (tid + it * nthreads < cpr)
      compute_stage<XT>(cur, a, s_code2, offset, c, lane_b, acc);
    if (it_next == 0) {
      // group done: CTA reduction and store
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float v = acc[m][r];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0) s_red[parity][warp][m * R + r] = v;
          acc[m][r] = 0.0f;
        }
      __syncthreads();
      const int nw = nthreads >> 5;
      for (int i = tid; i < M * R; i += nthreads) {
        float v = 0.0f;
        for (int w = 0; w < nw; ++w) v += s_red[parity][w][i];
        const int m = i / R, r = i % R;
        const int64_t row = g * R + r;
        if (row < a.n_rows) store_y<XT>(a.y, int64_t(m) * a.ldy + row, v);
      }
      parity ^= 1;
      if (g_next >= n_groups) return true;
    }
    g = g_next;
    it = it_next;
    c = c_next;
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = rows_next[r];
    return false;
  };

  while (true) {
    if (step(sa, sb)) break;
    if (step(sb, sa)) break;
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined GEMV for M <= 2 (the decode batch sizes).
//
// One CTA per SM walks row groups g = blockIdx.x, blockIdx.x + gridDim.x, ...
// of R rows. A producer warp streams each group's codes (R rows x K/2 bytes,
// contiguous in HBM) and, when they are 16-byte aligned, its block scales
// (R x K/bs bytes of nested codes, or floats) into a ring of shared-memory
// stages with cp.async.bulk, completion counted on a per-stage "full"
// mbarrier. More than 100 KB per SM is in flight without using registers.
// Consumer thread t owns chunks t, t + 32*NC, ... of every row (SLOTS of
// them); its x never changes, so it is widened to float32 into registers once.
// The consumers write the pair table themselves while the first stages land
// (stores from the constant table: no 64 KB copy per CTA through L2).
// Per stage a thread decodes its chunks through the pair table and
// accumulates with fma.rn.f32x2. Partial sums leave each warp through a
// transposed butterfly into shared memory; a per-stage counter tells the last
// warp of the group to add them up and store y. No CTA-wide barrier runs in
// the loop, so warps drift apart and overlap their load, decode and fma phases.
// A stage is refilled only after every consumer warp has arrived on its
// "empty" mbarrier, the last warp after storing, so the partial-sum slot of a
// stage is never overwritten early.
// Programmatic dependent launch: weights and scales may be fetched before the
// preceding kernel in the stream finishes (they are never written by it);
// x is read and y written only after griddepcontrol.wait.
// Every wait is bounded; a timeout is recorded (bnbq_wait_timeouts) and the
// kernel stops early instead of hanging.

// ---------------------------------------------------------------------------
// Flat GEMV for small M: one CTA per R consecutive rows (the whole K), many
// CTAs per SM. Each thread owns SLOTS chunks of every row and issues all of
// its loads -- codes, block scales, then x -- before decoding anything, so the
// memory system sees ~256 bytes in flight per thread; the hardware CTA
// scheduler overlaps one CTA's loads with another's arithmetic. Decode uses
// the 16-entry table in shared memory: per code word, two shift-and-mask ops
// give 4 high-nibble and 4 low-nibble byte offsets, one prmt extracts each,
// one LDS reads the value. Partial sums: transposed warp butterfly, then one
// pass through shared memory. Programmatic dependent launch: weights and
// scales are requested before griddepcontrol.wait, x after it.

template <int N>
__device__ __forceinline__ float warp_reduce_many(float (&v)[N], int lane) {
  // halves the set of values at each of the first log2(N) steps; afterwards
  // lane l holds the sum of value (l >> (5 - log2 N)) when its low bits are 0
  int n = N;
  int o = 16;
#pragma unroll
  for (; o > 0 && n > 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
      if (j < n / 2) {
        const float send = upper ? v[j] : v[j + n / 2];
        const float keep = upper ? v[j + n / 2] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    n >>= 1;
  }
  float vs = v[0];
#pragma unroll
  for (; o > 0; o >>= 1) vs += __shfl_xor_sync(0xffffffffu, vs, o);
  return vs;
}

template <typename XT, int M, int R, bool NESTED, int SLOTS>
__global__ void __launch_bounds__(256)
gemv_flat_kernel(GemvArgs a) {
  __shared__ float s_table[16];
  __shared__ float s_code2[NESTED ? 256 : 1];
  __shared__ float s_red[8][M * R];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int cpr = a.k >> 5;
  const int64_t row0 = int64_t(blockIdx.x) * R;

  // ---- weights and scales (never written by the preceding kernel)
  uint4 codes[SLOTS][R];
  float sc[SLOTS][R];
  int q2[SLOTS][R];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) {
    const int c = min(tid + sl * nthreads, cpr - 1);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = min(row0 + r, a.n_rows - 1);
      const int64_t e0 = row * a.k + int64_t(c) * 32;
      codes[sl][r] = __ldg(reinterpret_cast<const uint4*>(a.w + (e0 >> 1)));
      const int64_t blk = e0 >> a.log2_bs;
      if constexpr (NESTED) {
        q2[sl][r] = __ldg(a.absmax_q + blk);
        sc[sl][r] = __ldg(a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
      } else {
        q2[sl][r] = 0;
        sc[sl][r] = __ldg(a.absmax + blk);
      }
    }
  }
  if (tid < 16) s_table[tid] = kNF4Table[tid];
  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += nthreads) s_code2[i] = __ldg(a.code2 + i);
  }
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x may come from the previous kernel
  const XT* x = static_cast<const XT*>(a.x);
  uint4 xv[SLOTS][M][4];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) {
    const int c = min(tid + sl * nthreads, cpr - 1);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        xv[sl][m][i] = __ldg(reinterpret_cast<const uint4*>(x + int64_t(m) * a.k + c * 32 + i * 8));
  }
  const float offset = NESTED ? __ldg(a.offset) : 0.0f;
  __syncthreads();

  float acc[M * R];
#pragma unroll
  for (int i = 0; i < M * R; ++i) acc[i] = 0.0f;
  const char* tbl = reinterpret_cast<const char*>(s_table);
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) {
    if (tid + sl * nthreads >= cpr) continue;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float scale = NESTED ? add_rn(mul_ftz(s_code2[q2[sl][r]], sc[sl][r]), offset) : sc[sl][r];
      const uint32_t words[4] = {codes[sl][r].x, codes[sl][r].y, codes[sl][r].z, codes[sl][r].w};
      float2 w2[16];
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        const uint32_t hi4 = (words[wi] >> 2) & 0x3c3c3c3cu;  // even elements' nibble x 4, per byte
        const uint32_t lo4 = (words[wi] << 2) & 0x3c3c3c3cu;  // odd elements'
#pragma unroll
        for (int j = 0; j < 4; ++j)
          w2[4 * wi + j] = make_float2(*reinterpret_cast<const float*>(tbl + __byte_perm(hi4, 0, 0x4440 + j)),
                                       *reinterpret_cast<const float*>(tbl + __byte_perm(lo4, 0, 0x4440 + j)));
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint32_t xw[16] = {xv[sl][m][0].x, xv[sl][m][0].y, xv[sl][m][0].z, xv[sl][m][0].w,
                                 xv[sl][m][1].x, xv[sl][m][1].y, xv[sl][m][1].z, xv[sl][m][1].w,
                                 xv[sl][m][2].x, xv[sl][m][2].y, xv[sl][m][2].z, xv[sl][m][2].w,
                                 xv[sl][m][3].x, xv[sl][m][3].y, xv[sl][m][3].z, xv[sl][m][3].w};
        float2 t[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) t[q] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int e = 0; e < 16; ++e) t[e & 3] = __ffma2_rn(w2[e], unpack_x<XT>(xw[e]), t[e & 3]);
        const float2 u = __fadd2_rn(__fadd2_rn(t[0], t[1]), __fadd2_rn(t[2], t[3]));
        acc[m * R + r] = __fmaf_rn(scale, u.x + u.y, acc[m * R + r]);
      }
    }
  }

  const float vs = warp_reduce_many<M * R>(acc, lane);
  constexpr int kBits = (M * R >= 8) ? 3 : (M * R >= 4 ? 2 : (M * R >= 2 ? 1 : 0));
  if ((lane & ((32 >> kBits) - 1)) == 0) {
    const int idx = lane >> (5 - kBits);
    if (idx < M * R) s_red[warp][idx] = vs;
  }
  __syncthreads();
  if (tid < M * R) {
    float v = 0.0f;
    const int nw = nthreads >> 5;
    for (int w = 0; w < nw; ++w) v += s_red[w][tid];
    const int m = tid / R, r = tid % R;
    const int64_t row = row0 + r;
    if (row < a.n_rows) store_y<XT>(a.y, int64_t(m) * a.ldy + row, v);
  }
}

// Threads per CTA for the flat kernel: <= 256, a multiple of 32, with the
// chunks of a row split into the fewest idle slots.
int flat_threads(int cpr, int max_slots, int* slots) {
  int best_t = 256, best_s = 1;
  double best_eff = -1.0;
  for (int w = 8; w >= 2; --w) {
    const int t = 32 * w;
    const int s = (cpr + t - 1) / t;
    if (s > max_slots) continue;
    const double eff = double(cpr) / double(s * t);
    if (eff > best_eff + 1e-9) { best_eff = eff; best_t = t; best_s = s; }
  }
  *slots = best_eff < 0 ? 0 : best_s;
  return best_t;
}

template <typename XT, int M, int R, bool NESTED, int SLOTS>
int launch_flat_t(const GemvArgs& a, int threads, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((a.n_rows + R - 1) / R));
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gemv_flat_kernel<XT, M, R, NESTED, SLOTS>, a) != cudaSuccess) return BNBQ_ERR_CUDA;
  return launch_status();
}

constexpr int kMaxRows = 4;
constexpr int kMaxStages = 8;
constexpr int kMaxGroupsPerFlush = 32;  // partial sums held in shared memory between flushes

// SIS: the block scales travel with the stage (a compile-time choice, so that
// the other layout's registers and code drop out). RG: the consumer warps form
// RG equal groups, group i taking rows [i R/RG, (i + 1) R/RG) of every stage
// (short rows: more warps than one row's chunks could keep busy).
template <typename XT, int M, int R, bool NESTED, int SLOTS, bool SIS, int RG, bool PX>
__global__ void __launch_bounds__(kMaxWarps * 32, 1)
gemv_bulk_kernel(GemvArgs a, int n_groups, int n_stages, uint32_t stage_bytes, PeerOut px) {
  static_assert(R % RG == 0, "row groups split the stage's rows evenly");
  constexpr int RT = R / RG;  // rows of a stage per consumer thread
  constexpr bool scales_in_stage = SIS;
  __shared__ __align__(16) float s_code2[256];
  __shared__ float s_part[kMaxGroupsPerFlush][kMaxWarps - 1][M * R];
  __shared__ __align__(8) uint64_t s_tbl_bar;
  __shared__ __align__(8) uint64_t s_done_bar;
  __shared__ volatile int s_abort;  // set by any thread whose wait expired
  __shared__ volatile int s_rx_expired;  // exchange mode: a wait for a peer expired
  char* stages = reinterpret_cast<char*>(s_pair) + kPairTableBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + size_t(n_stages) * stage_bytes);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int ncw = (blockDim.x >> 5) - 1;  // consumer warps; the last warp produces
  const int ncons = ncw * 32;
  const int wpg = RG == 1 ? ncw : ncw / RG;  // warps per row group (the host makes ncw a multiple of RG)
  const int gthreads = RG == 1 ? ncons : wpg * 32;  // threads per row group
  const int rgi = RG == 1 ? 0 : tid / gthreads;  // this thread's row group (consumers); constant for RG = 1
  const int lt = tid - rgi * gthreads;
  const int r0 = rgi * RT;         // its first row of a stage
  const int cpr = a.k >> 5;
  const uint32_t row_bytes = uint32_t(a.k) >> 1;
  const int spr = a.k >> a.log2_bs;  // scales per row (when K % bs == 0)
  const uint32_t scale_row_bytes = uint32_t(spr) * (NESTED ? 1u : 4u);
  const uint32_t codes_bytes = uint32_t(R) * row_bytes;
  if (n_stages < 1 || n_stages > kMaxStages) return;  // the host plans <= kMaxStages

  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == ncw) {  // ------------------------------------------- producer
    if (lane == 0) {
      s_abort = 0;
      s_rx_expired = 0;
      mbar_init(smem_u32(&s_tbl_bar), 1);
      mbar_init(smem_u32(&s_done_bar), uint32_t(ncw));
      for (int st = 0; st < n_stages; ++st) {
        mbar_init(smem_u32(bars + st), 1);                         // full
        mbar_init(smem_u32(bars + n_stages + st), uint32_t(ncw));  // empty
      }
      fence_mbar_init();
      // code2 first (the consumers build the pair table themselves)
      const uint32_t tb = smem_u32(&s_tbl_bar);
      mbar_arrive_expect_tx(tb, NESTED ? 1024u : 0u);
      if constexpr (NESTED) bulk_g2s(smem_u32(s_code2), a.code2, 1024, tb);
    }
    __syncthreads();  // barriers ready for everyone
    if (lane == 0) {
      int st = 0;
      uint32_t phase = 0;
      int i = 0;
      for (int g = blockIdx.x; g < n_groups && i < kMaxGroupsPerFlush; g += gridDim.x, ++i) {
        if (s_abort) break;
        if (i >= n_stages && !mbar_wait(smem_u32(bars + n_stages + st), phase ^ 1u)) {
          s_abort = 1;
          break;
        }
        // Every CTA asks for its first two stages only and waits for the first
        // before asking for more: the first stages of all CTAs then land ahead
        // of the bulk of the requests, and the consumers start sooner.
        if (i == 2 && n_stages > 2 && !mbar_wait(smem_u32(bars), 0)) {
          s_abort = 1;
          break;
        }
        const int64_t row0 = int64_t(g) * R;
        const uint32_t rows_in = uint32_t(min(int64_t(R), a.n_rows - row0));
        const uint32_t full = smem_u32(bars + st);
        const uint32_t dst = smem_u32(stages + size_t(st) * stage_bytes);
        mbar_arrive_expect_tx(full, rows_in * row_bytes + (scales_in_stage ? rows_in * scale_row_bytes : 0u));
        bulk_g2s(dst, a.w + row0 * int64_t(row_bytes), rows_in * row_bytes, full);
        if (scales_in_stage) {
          const void* src = NESTED ? static_cast<const void*>(a.absmax_q + row0 * spr)
                                   : static_cast<const void*>(a.absmax + row0 * spr);
          bulk_g2s(dst + codes_bytes, src, rows_in * scale_row_bytes, full);
        }
        if (++st == n_stages) { st = 0; phase ^= 1u; }
      }
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  __syncthreads();  // barriers initialised; code2 and the first stages are in flight
  const uint32_t lane_b = uint32_t(lane) * 8u;
  // The pair table, written by the consumer warps while the first stages
  // stream in: warp w fills rows w, w + ncw, ... (row b = 32 lane copies of
  // (T[b >> 4], T[b & 15]); b is warp-uniform, so the table reads broadcast).
  for (int b = warp; b < 256; b += ncw) s_pair[b * 32 + lane] = make_float2(kNF4Table[b >> 4], kNF4Table[b & 15]);
  named_bar_sync(1, ncons);

  // per (slot, row): the chunk's block within a group, relative to the group's
  // first block (K % bs == 0), or its global block for group g (otherwise)
  int cofs[SLOTS];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) cofs[sl] = min(lt + sl * gthreads, cpr - 1) * 32;
  auto block_of = [&](int g, int sl, int r) -> int64_t {
    const int64_t row = min(int64_t(g) * R + r, a.n_rows - 1);
    return (row * a.k + cofs[sl]) >> a.log2_bs;
  };
  // second-level scales (nested) two groups ahead; whole scales when they do
  // not travel with the stage
  float pre0[SLOTS][RT], pre1[SLOTS][RT];
  int preq0[SLOTS][RT], preq1[SLOTS][RT];
  // nested scales travelling with the stage: second-level scale of (slot,
  // row) = absmax2[(block0 + (g R + r) spr + bir[slot]) >> log2_bs2], in
  // 32-bit block numbers (the host checks that they fit)
  int bir[SLOTS];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) bir[sl] = cofs[sl] >> a.log2_bs;
  const int last_row_blk = int((a.n_rows - 1) * int64_t(spr));
  auto prefetch = [&](int g, float (&p)[SLOTS][RT], int (&q)[SLOTS][RT]) {
    if (NESTED && scales_in_stage) {
      const int gb = g * (R * spr);  // the group's first block
#pragma unroll
      for (int sl = 0; sl < SLOTS; ++sl)
#pragma unroll
        for (int rr = 0; rr < RT; ++rr) {
          q[sl][rr] = 0;
          const int rb = min(gb + (r0 + rr) * spr, last_row_blk);  // clamped rows: results dropped
          p[sl][rr] = g < n_groups ? __ldg(a.absmax2 + ((int(a.block0) + rb + bir[sl]) >> a.log2_bs2)) : 0.0f;
        }
      return;
    }
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl)
#pragma unroll
      for (int rr = 0; rr < RT; ++rr) {
        p[sl][rr] = 0.0f;
        q[sl][rr] = 0;
        if (g < n_groups && (NESTED || !scales_in_stage)) {
          const int64_t blk = block_of(g, sl, r0 + rr);
          if constexpr (NESTED) {
            p[sl][rr] = __ldg(a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
            if (!scales_in_stage) q[sl][rr] = __ldg(a.absmax_q + blk);
          } else {
            p[sl][rr] = __ldg(a.absmax + blk);
          }
        }
      }
  };
  prefetch(blockIdx.x, pre0, preq0);
  // within-group scale index of (slot, row) when scales travel with the stage
  // (row r's index = sidx0 + r * spr, K % bs == 0 there)
  int sidx0[SLOTS];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) sidx0[sl] = cofs[sl] >> a.log2_bs;

  asm volatile("griddepcontrol.wait;" ::: "memory");  // x may come from the previous kernel
  const XT* x = static_cast<const XT*>(a.x);
  float2 xr[SLOTS][M][16];
#pragma unroll
  for (int sl = 0; sl < SLOTS; ++sl) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + int64_t(m) * a.k + cofs[sl] + i * 8));
        xr[sl][m][4 * i + 0] = unpack_x<XT>(xv.x);
        xr[sl][m][4 * i + 1] = unpack_x<XT>(xv.y);
        xr[sl][m][4 * i + 2] = unpack_x<XT>(xv.z);
        xr[sl][m][4 * i + 3] = unpack_x<XT>(xv.w);
      }
  }
  const float offset = NESTED ? __ldg(a.offset) : 0.0f;
  bool ok = mbar_wait(smem_u32(&s_tbl_bar), 0);
  if (!ok) s_abort = 1;

  constexpr int kBits = (M * RT >= 8) ? 3 : (M * RT >= 4 ? 2 : (M * RT >= 2 ? 1 : 0));
  // lanes whose low bits are zero hold one of the M*RT warp sums after warp_reduce_many
  const bool holder = (lane & ((32 >> kBits) - 1)) == 0;
  const int hidx = lane >> (5 - kBits);

  int st = 0;
  uint32_t phase = 0;
  int gl = 0;
  for (int g = blockIdx.x; g < n_groups && gl < kMaxGroupsPerFlush; g += gridDim.x, ++gl) {
    if (!ok || s_abort) { ok = false; break; }
    ok = mbar_wait(smem_u32(bars + st), phase);
    if (!ok) { s_abort = 1; break; }
    const char* stage = stages + size_t(st) * stage_bytes;

    // a row's block scale, decoded where it is used (fewer live registers)
    auto scale_of = [&](int sl, int rr) -> float {
      if (scales_in_stage) {
        const int si = sidx0[sl] + (r0 + rr) * spr;
        if constexpr (NESTED) {
          const int q2 = reinterpret_cast<const uint8_t*>(stage + codes_bytes)[si];
          return add_rn(mul_ftz(s_code2[q2], pre0[sl][rr]), offset);
        } else {
          return reinterpret_cast<const float*>(stage + codes_bytes)[si];
        }
      } else {
        return NESTED ? add_rn(mul_ftz(s_code2[preq0[sl][rr]], pre0[sl][rr]), offset) : pre0[sl][rr];
      }
    };

    float acc[M * RT];
#pragma unroll
    for (int e = 0; e < M * RT; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int sl = 0; sl < SLOTS; ++sl) {
      const int c = lt + sl * gthreads;
      if (c < cpr) {
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const uint4 cw = *reinterpret_cast<const uint4*>(stage + (r0 + r) * row_bytes + c * 16);
          const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
          float2 t[M][4];
#pragma unroll
          for (int m = 0; m < M; ++m)
#pragma unroll
            for (int q = 0; q < 4; ++q) t[m][q] = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // 8 lookups, then their 4 fma chains per row of x
            float2 wv[8];
#pragma unroll
            for (int wi = 0; wi < 2; ++wi)
#pragma unroll
              for (int j = 0; j < 4; ++j) wv[4 * wi + j] = pair_at(words[2 * h + wi], lane_b, j);
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
              for (int e = 0; e < 8; ++e) t[m][e & 3] = __ffma2_rn(wv[e], xr[sl][m][8 * h + e], t[m][e & 3]);
          }
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float2 u = __fadd2_rn(__fadd2_rn(t[m][0], t[m][1]), __fadd2_rn(t[m][2], t[m][3]));
            acc[m * RT + r] = __fmaf_rn(scale_of(sl, r), u.x + u.y, acc[m * RT + r]);
          }
        }
      }
    }
    prefetch(g + int(gridDim.x), pre0, preq0);  // one group ahead
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(bars + n_stages + st));  // stage consumed
    if (++st == n_stages) { st = 0; phase ^= 1u; }

    const float vs = warp_reduce_many<M * RT>(acc, lane);
    if (holder && hidx < M * RT) s_part[gl][warp][hidx] = vs;
  }

  // Final sums: every consumer warp arrives on s_done (aborted or not); warp
  // 0 waits for all of them (bounded) and stores y. Row r of a stage is the
  // sum, in warp order, of its row group's warps' entries m * RT + r % RT.
  // Exchange mode: warp 0 also stores each value into the peers' inboxes;
  // then every consumer thread polls its share of the other ranks' columns
  // (the host launches at most one CTA per SM, so all CTAs are resident) and
  // the CTA reports that it has finished the call.
  __syncwarp();
  if (lane == 0) mbar_arrive(smem_u32(&s_done_bar));
  if constexpr (!PX) {  // the plain kernel: warp 0 alone finishes
    if (warp != 0) return;
    if (!mbar_wait(smem_u32(&s_done_bar), 0) || s_abort) return;
    for (int e = lane; e < gl * M * R; e += 32) {
      const int gi = e / (M * R), idx = e % (M * R);
      const int m = idx / R, r = idx % R;
      float v = 0.0f;
      if constexpr (RG == 1) {
        for (int w = 0; w < ncw; ++w) v += s_part[gi][w][idx];
      } else {
        const int w0 = (r / RT) * wpg, pi = m * RT + r % RT;
        for (int w = w0; w < w0 + wpg; ++w) v += s_part[gi][w][pi];
      }
      const int64_t row = (int64_t(blockIdx.x) + int64_t(gi) * gridDim.x) * R + r;
      if (row < a.n_rows) store_y<XT>(a.y, int64_t(m) * a.ldy + row, v);
    }
    return;
  }
  constexpr bool exchange = PX;
  const uint32_t epoch = exchange ? peer_epoch(px) : 0u;  // after griddepcontrol.wait
  if (warp == 0 && mbar_wait(smem_u32(&s_done_bar), 0) && !s_abort) {
    for (int e = lane; e < gl * M * R; e += 32) {
      const int gi = e / (M * R), idx = e % (M * R);
      const int m = idx / R, r = idx % R;
      const int w0 = (r / RT) * wpg, pi = m * RT + r % RT;
      float v = 0.0f;
      for (int w = w0; w < w0 + wpg; ++w) v += s_part[gi][w][pi];
      const int64_t row = (int64_t(blockIdx.x) + int64_t(gi) * gridDim.x) * R + r;
      if (row < a.n_rows) {
        store_y<XT>(a.y, int64_t(m) * a.ldy + row, v);
        if (exchange) peer_send(px, epoch, m, row, bits_of<XT>(v));
      }
    }
  }
  if constexpr (exchange) {
    if (!peer_receive(px, epoch, M, a.n_rows, int64_t(blockIdx.x) * ncons + tid, int64_t(gridDim.x) * ncons))
      s_rx_expired = 1;
    named_bar_sync(2, ncons);
    if (tid == 0) peer_finish_cta(px, epoch, s_rx_expired != 0);
  }
}

struct BulkPlan {
  int scales_in_stage = 0;
  int ncw = 0;      // consumer warps
  int slots = 0;    // chunks per consumer thread and row
  int rows = 0;     // R
  int groups = 1;   // RG: row groups of consumer warps
  uint32_t stage_bytes = 0;
};

// Chooses the consumer warps -- RG row groups of W warps, each thread owning
// `slots` 32-element chunks of its group's rows -- for the most lanes with
// work (at least 3/4 of the lanes busy; ties: fewer slots, then fewer warps),
// the rows per stage and whether the scales travel with the codes; stages are
// sized at launch. Row groups split a 4-row stage (RG = 2, 4) or a 3-row one
// (RG = 3).
bool plan_bulk(int m, int k, int log2_bs, bool nested, int smem_optin, BulkPlan* p) {
  const int cpr = k >> 5;
  double best_busy = -1.0;
  for (int rg = 1; rg <= 4; ++rg) {
    for (int w = 2; w * rg <= kMaxWarps - 1; ++w) {
      const int slots = (cpr + 32 * w - 1) / (32 * w);
      if (slots * m > 2) continue;
      const double eff = double(cpr) / double(slots * 32 * w);
      // row groups only for rows of >= 128 chunks (K >= 4096, measured); shorter rows
      // keep the flat kernel
      if (eff < 0.75 || w * rg < 4 || (rg > 1 && (slots > 1 || cpr < 128))) continue;
      const double busy = eff * w * rg;
      const bool better = busy > best_busy + 1e-9 ||
                          (busy > best_busy - 1e-9 && (slots < p->slots || (slots == p->slots && w * rg < p->ncw)));
      if (better) { best_busy = busy; p->ncw = w * rg; p->slots = slots; p->groups = rg; }
    }
  }
  if (p->ncw == 0) return false;
  const uint32_t row_bytes = uint32_t(k) >> 1;
  const bool whole_blocks = (k & ((1 << log2_bs) - 1)) == 0;
  const uint32_t srb = whole_blocks ? uint32_t(k >> log2_bs) * (nested ? 1u : 4u) : 0u;
  p->scales_in_stage = whole_blocks && (srb % 16 == 0);
  const size_t room = size_t(smem_optin) - size_t(kPairTableBytes) - 24 * 1024;  // static smem margin
  for (int R : {4, 3, 2, 1}) {
    if (p->groups == 1 ? R == 3 : (p->groups == 3 ? R != 3 : R != 4)) continue;
    const uint32_t sb = uint32_t(R) * (row_bytes + (p->scales_in_stage ? srb : 0u));
    if (room / (sb + 16) >= 4) {
      p->rows = R;
      p->stage_bytes = sb;
      return true;
    }
  }
  return false;
}

// px: the exchange mode (nullptr: none).
template <typename XT, int M, int R, bool NESTED, int SLOTS, int RG = 1>
int launch_bulk_t(const GemvArgs& a, const BulkPlan& p, const DeviceInfo& di, cudaStream_t s,
                  const PeerOut* xp = nullptr) {
  const bool px = xp != nullptr;
  auto kern = p.scales_in_stage ? (px ? gemv_bulk_kernel<XT, M, R, NESTED, SLOTS, true, RG, true>
                                      : gemv_bulk_kernel<XT, M, R, NESTED, SLOTS, true, RG, false>)
                                : (px ? gemv_bulk_kernel<XT, M, R, NESTED, SLOTS, false, RG, true>
                                      : gemv_bulk_kernel<XT, M, R, NESTED, SLOTS, false, RG, false>);
  int static_smem = 0;
  if (int st = kernel_static_smem(reinterpret_cast<const void*>(kern), &static_smem)) return st;
  const size_t room = size_t(di.smem_optin) - size_t(kPairTableBytes) - size_t(static_smem) - 1024;
  int stages = int(room / (p.stage_bytes + 16));
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return BNBQ_ERR_UNSUPPORTED;
  const size_t smem = size_t(kPairTableBytes) + size_t(stages) * p.stage_bytes + size_t(2 * stages) * 8;
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  const int64_t n_groups = (a.n_rows + R - 1) / R;
  if (n_groups > INT32_MAX / 2) return BNBQ_ERR_UNSUPPORTED;
  // the kernel numbers blocks in 32 bits when the scales travel with the stage
  if (p.scales_in_stage && a.block0 + ((a.n_rows * a.k) >> a.log2_bs) + R * int64_t(a.k >> a.log2_bs) >= INT32_MAX)
    return BNBQ_ERR_UNSUPPORTED;
  int64_t grid = n_groups < di.sm_count ? n_groups : di.sm_count;
  const int64_t min_grid = (n_groups + kMaxGroupsPerFlush - 1) / kMaxGroupsPerFlush;  // <= 32 groups per CTA
  if (grid < min_grid) grid = min_grid;
  // the exchange polls for peers from every CTA: all of them must be resident
  if (px && grid > di.sm_count) return BNBQ_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3((p.ncw + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, int(n_groups), stages, p.stage_bytes, px ? *xp : PeerOut{}) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, int M, bool NESTED>
int launch_bulk(const GemvArgs& a, const BulkPlan& p, const DeviceInfo& di, cudaStream_t s,
                const PeerOut* xp = nullptr) {
  if constexpr (M <= 2) {
    if (p.groups > 1) {  // short rows: one chunk per thread, row groups over a 4- or 3-row stage
      if (p.slots != 1) return BNBQ_ERR_UNSUPPORTED;
      switch (p.groups) {
        case 2: return launch_bulk_t<XT, M, 4, NESTED, 1, 2>(a, p, di, s, xp);
        case 3: return launch_bulk_t<XT, M, 3, NESTED, 1, 3>(a, p, di, s, xp);
        case 4: return launch_bulk_t<XT, M, 4, NESTED, 1, 4>(a, p, di, s, xp);
        default: return BNBQ_ERR_UNSUPPORTED;
      }
    }
    if (p.slots == 1) {
      switch (p.rows) {
        case 4: return launch_bulk_t<XT, M, 4, NESTED, 1>(a, p, di, s, xp);
        case 2: return launch_bulk_t<XT, M, 2, NESTED, 1>(a, p, di, s, xp);
        default: return launch_bulk_t<XT, M, 1, NESTED, 1>(a, p, di, s, xp);
      }
    }
    if constexpr (M == 1) {
      switch (p.rows) {
        case 4: return launch_bulk_t<XT, 1, 4, NESTED, 2>(a, p, di, s, xp);
        case 2: return launch_bulk_t<XT, 1, 2, NESTED, 2>(a, p, di, s, xp);
        default: return launch_bulk_t<XT, 1, 1, NESTED, 2>(a, p, di, s, xp);
      }
    }
  }
  return BNBQ_ERR_UNSUPPORTED;
}

// Rows per group: enough to share each x load, few enough to keep registers.
constexpr int rows_for(int M) { return M <= 2 ? 4 : (M <= 8 ? 2 : 1); }

// Threads per CTA (multiple of 32, <= 512) splitting the K/32 chunks of a
// row group with the fewest idle lanes.
int pick_threads(int cpr, int max_threads) {
  int best = 128;
  double best_eff = -1.0;
  for (int w = max_threads / 32; w >= 4; --w) {
    const int slots = 32 * w;
    const int iters = (cpr + slots - 1) / slots;
    const double eff = double(cpr) / double(iters * slots);
    if (eff > best_eff + 1e-9) { best_eff = eff; best = slots; }
  }
  return best;
}

template <typename XT, int M, bool NESTED>
int launch_m(const GemvArgs& a, cudaStream_t s) {
  constexpr int R = rows_for(M);
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if constexpr (M <= 2) {
    BulkPlan p;
    // bulk copies need 16-byte aligned sources: codes (checked by the caller),
    // code2, and the scale arrays when they travel with the stage
    const bool c2_ok = !NESTED || aligned(a.code2, 16);
    if (c2_ok && plan_bulk(M, a.k, a.log2_bs, NESTED, di.smem_optin, &p)) {
      if (p.scales_in_stage && !aligned(NESTED ? static_cast<const void*>(a.absmax_q)
                                              : static_cast<const void*>(a.absmax), 16))
        p.scales_in_stage = 0;
      const int st = launch_bulk<XT, M, NESTED>(a, p, di, s);
      if (st != BNBQ_ERR_UNSUPPORTED) return st;
    }
    int slots = 0;
    const int threads = flat_threads(a.k >> 5, 2, &slots);
    if (slots == 1) return launch_flat_t<XT, M, 4, NESTED, 1>(a, threads, s);
    if (slots == 2) return launch_flat_t<XT, M, 4, NESTED, 2>(a, threads, s);
  }
  const int threads = pick_threads(a.k >> 5, max_threads_for(M));
  const int64_t n_groups = (a.n_rows + R - 1) / R;
  auto kern = gemv_kernel<XT, M, R, NESTED>;
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), kPairTableBytes)) return st;
  int per_sm = 0;
  if (int st = kernel_occupancy(reinterpret_cast<const void*>(kern), threads, kPairTableBytes, &per_sm)) return st;
  per_sm = per_sm < 1 ? 1 : (per_sm > 2 ? 2 : per_sm);
  // One CTA per SM when that balances the groups to within 2%, else two.
  int64_t grid = di.sm_count;
  {
    const int64_t rounds1 = (n_groups + grid - 1) / grid;
    const double eff1 = double(n_groups) / double(rounds1 * grid);
    if (eff1 < 0.98 && per_sm >= 2) grid = int64_t(di.sm_count) * 2;
  }
  if (grid > n_groups) grid = n_groups;
  kern<<<dim3(unsigned(grid)), dim3(threads), kPairTableBytes, s>>>(a, n_groups);
  return launch_status();
}

// M > 2: the M = 2 (and M = 1) kernels over consecutive pairs of x rows. Each
// row's arithmetic is that of a single-row call; the weight, read from HBM by
// the first pass, is served from L2 (126 MB) to the following ones.
template <typename XT, bool NESTED>
int launch_pairs(int m, const GemvArgs& a, cudaStream_t s) {
  for (int m0 = 0; m0 < m; m0 += 2) {
    GemvArgs b = a;
    b.x = static_cast<const char*>(a.x) + size_t(m0) * size_t(a.k) * sizeof(XT);
    b.y = static_cast<char*>(a.y) + size_t(m0) * size_t(a.ldy) * sizeof(XT);
    const int st = (m - m0 >= 2) ? launch_m<XT, 2, NESTED>(b, s) : launch_m<XT, 1, NESTED>(b, s);
    if (st != BNBQ_OK) return st;
  }
  return BNBQ_OK;
}

// ------------------------------------------------------------ M = 3..20
// gemv_rows_kernel: lanes are weight rows, so x is shared by the 32 lanes of a
// warp (shared-memory broadcasts) and the weight is decoded once for all M rows
// of x. A CTA owns 32 rows; its 8 warps split K, each streaming its slice in
// 32-element stages through a D-deep per-warp ring filled by cp.async (no spin
// waits anywhere: cp.async.wait_group):
//   * codes (16 bytes per row) and the block scale (the float32 absmax, or the
//     4-byte word holding the nested code plus absmax2), one lane per row;
//   * x (MT rows x 32 columns of 16-bit values) in 16-byte pieces, converted
//     once per stage into a float32 tile the whole warp reads by broadcast.
// Each weight pair is scaled to its exact dequantized float32 value,
// mul.ftz(T[q], a), and accumulated with fma.rn.f32x2 into per-(x row) float2
// partials; the 8 warps' partials are summed in a fixed order in shared
// memory. A one-hot x therefore returns dequantize() bitwise.
constexpr int kRowsWarps = 8;

template <int MT>
struct RowsLayout {
  static constexpr int kDepth = MT <= 8 ? 8 : 4;             // stages in flight per warp
  static constexpr uint32_t kCodes = kDepth * 32 * 16;       // [depth][lane] 16 B
  static constexpr uint32_t kWords = kDepth * 32 * 4;        // [depth][lane] scale word
  static constexpr uint32_t kA2 = kDepth * 32 * 4;           // [depth][lane] absmax2
  static constexpr uint32_t kXRaw = kDepth * MT * 32 * 2;    // [depth][MT][32] 16-bit x
  static constexpr uint32_t kXF = MT * 32 * 4;               // [MT][32] float32 x
  static constexpr uint32_t kWarp = kCodes + kWords + kA2 + kXRaw + kXF;
  static constexpr uint32_t kPartials = kRowsWarps * MT * 32 * 4;
  static constexpr uint32_t kDynamic = kPairTableBytes + kRowsWarps * kWarp + kPartials;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <typename XT>
__device__ __forceinline__ float x_to_f32(uint16_t v) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) return __uint_as_float(uint32_t(v) << 16);
  else return __half2float(__ushort_as_half(v));
}

template <typename XT, int MT, bool NESTED>
__global__ void __launch_bounds__(kRowsWarps * 32, 1)
gemv_rows_kernel(GemvArgs a, int m_rows, int kw) {
  using L = RowsLayout<MT>;
  constexpr int D = L::kDepth;
  __shared__ float s_code2[NESTED ? 256 : 1];
  char* const dyn = reinterpret_cast<char*>(s_pair);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  char* const wb = dyn + kPairTableBytes + warp * L::kWarp;
  uint4* const s_codes = reinterpret_cast<uint4*>(wb);
  uint32_t* const s_word = reinterpret_cast<uint32_t*>(wb + L::kCodes);
  float* const s_a2 = reinterpret_cast<float*>(wb + L::kCodes + L::kWords);
  uint16_t* const s_xraw = reinterpret_cast<uint16_t*>(wb + L::kCodes + L::kWords + L::kA2);
  float* const s_xf = reinterpret_cast<float*>(wb + L::kCodes + L::kWords + L::kA2 + L::kXRaw);
  float* const s_part = reinterpret_cast<float*>(dyn + kPairTableBytes + kRowsWarps * L::kWarp);

  asm volatile("griddepcontrol.launch_dependents;");
  for (int i = tid; i < kPairTableBytes / 16; i += kRowsWarps * 32)
    reinterpret_cast<uint4*>(s_pair)[i] = reinterpret_cast<const uint4*>(g_pair_table.v)[i];
  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += kRowsWarps * 32) s_code2[i] = __ldg(a.code2 + i);
  }

  const int64_t row = min(int64_t(blockIdx.x) * 32 + lane, a.n_rows - 1);
  const int k0 = warp * kw;
  const int k1 = min(a.k, k0 + kw);
  const int nst = k1 > k0 ? (k1 - k0) >> 5 : 0;
  const char* const wrow = reinterpret_cast<const char*>(a.w) + row * int64_t(a.k >> 1);
  const int64_t rowk = row * int64_t(a.k);
  const uint16_t* const x = static_cast<const uint16_t*>(a.x);
  const int mx = m_rows < MT ? m_rows : MT;  // x rows actually copied

  auto issue_w = [&](int s) {  // weight codes and scale of stage s
    if (s < nst) {
      const int slot = s & (D - 1);
      const int kk = k0 + 32 * s;
      cp_async16(smem_u32(s_codes + slot * 32 + lane), wrow + (kk >> 1));
      const int64_t blk = (rowk + kk) >> a.log2_bs;
      if constexpr (NESTED) {
        cp_async4(smem_u32(s_word + slot * 32 + lane),
                  reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(a.absmax_q + blk) & ~uintptr_t(3)));
        cp_async4(smem_u32(s_a2 + slot * 32 + lane), a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
      } else {
        cp_async4(smem_u32(s_word + slot * 32 + lane), a.absmax + blk);
      }
    }
  };
  auto issue_x = [&](int s) {  // x[m][stage s], 4 pieces of 16 bytes per x row
    if (s < nst) {
      const int slot = s & (D - 1);
      const int kk = k0 + 32 * s;
      for (int c = lane; c < 4 * mx; c += 32) {
        const int m = c >> 2, part = c & 3;
        cp_async16(smem_u32(s_xraw + (slot * MT + m) * 32 + part * 8), x + int64_t(m) * a.k + kk + part * 8);
      }
    }
  };

  // weights do not depend on the previous kernel: start them before the wait
#pragma unroll
  for (int s = 0; s < D - 1; ++s) issue_w(s);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x may come from the previous kernel
  // group g holds stage g's x and, from g = D-1 on, stage g's weights too; the
  // prologue's weight copies ride in group 0, which completes first
#pragma unroll
  for (int s = 0; s < D - 1; ++s) {
    issue_x(s);
    cp_async_commit();
  }
  const float offset = NESTED ? __ldg(a.offset) : 0.0f;
  __syncthreads();  // pair table and code2 are in place

  float2 acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = make_float2(0.0f, 0.0f);
  const uint32_t lane_b = uint32_t(lane) * 8u;

  for (int s = 0; s < nst; ++s) {
    issue_w(s + D - 1);
    issue_x(s + D - 1);
    cp_async_commit();
    asm volatile("cp.async.wait_group %0;" ::"n"(D - 1) : "memory");  // this lane's stage-s copies
    __syncwarp();  // ... and every lane's (x pieces were copied by other lanes)
    const int slot = s & (D - 1);
#pragma unroll
    for (int m = 0; m < MT; ++m)
      s_xf[m * 32 + lane] = m < m_rows ? x_to_f32<XT>(s_xraw[(slot * MT + m) * 32 + lane]) : 0.0f;
    __syncwarp();
    const uint4 cw = s_codes[slot * 32 + lane];
    float sc;
    if constexpr (NESTED) {
      const int64_t blk = (rowk + k0 + 32 * s) >> a.log2_bs;
      const uint32_t sh = 8u * uint32_t(reinterpret_cast<uintptr_t>(a.absmax_q + blk) & 3);
      const uint32_t q = (s_word[slot * 32 + lane] >> sh) & 0xffu;
      sc = add_rn(mul_ftz(s_code2[q], s_a2[slot * 32 + lane]), offset);
    } else {
      sc = __uint_as_float(s_word[slot * 32 + lane]);
    }
    const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int e = 0; e < 16; e += 2) {  // pairs e and e+1: elements 2e .. 2e+3
      const float2 w0 = mul_ftz2(pair_at(words[e >> 2], lane_b, e & 3), make_float2(sc, sc));
      const float2 w1 = mul_ftz2(pair_at(words[e >> 2], lane_b, (e & 3) + 1), make_float2(sc, sc));
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float4 x4 = *reinterpret_cast<const float4*>(s_xf + m * 32 + 2 * e);  // broadcast
        acc[m] = __ffma2_rn(w0, make_float2(x4.x, x4.y), acc[m]);
        acc[m] = __ffma2_rn(w1, make_float2(x4.z, x4.w), acc[m]);
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");

#pragma unroll
  for (int m = 0; m < MT; ++m) s_part[(warp * MT + m) * 32 + lane] = acc[m].x + acc[m].y;
  __syncthreads();
  for (int e = tid; e < MT * 32; e += kRowsWarps * 32) {
    const int m = e >> 5, l = e & 31;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kRowsWarps; ++w) v += s_part[(w * MT + m) * 32 + l];
    const int64_t r = int64_t(blockIdx.x) * 32 + l;
    if (m < m_rows && r < a.n_rows) store_y<XT>(a.y, int64_t(m) * a.ldy + r, v);
  }
}

template <typename XT, int MT, bool NESTED>
int launch_rows_t(int m, const GemvArgs& a, const DeviceInfo& di, cudaStream_t s) {
  using L = RowsLayout<MT>;
  auto kern = gemv_rows_kernel<XT, MT, NESTED>;
  int static_smem = 0;
  if (int st = kernel_static_smem(reinterpret_cast<const void*>(kern), &static_smem)) return st;
  if (size_t(L::kDynamic) + size_t(static_smem) > size_t(di.smem_optin)) return BNBQ_ERR_UNSUPPORTED;
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(L::kDynamic))) return st;
  int kw = (a.k + kRowsWarps - 1) / kRowsWarps;
  kw = (kw + 31) & ~31;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((a.n_rows + 31) / 32));
  cfg.blockDim = dim3(kRowsWarps * 32);
  cfg.dynamicSmemBytes = L::kDynamic;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, m, kw) != cudaSuccess) return BNBQ_ERR_CUDA;
  return launch_status();
}

// M = 5..20: x rows rounded up to a multiple of 4 (the extra rows are zero).
template <typename XT, bool NESTED>
int launch_rows(int m, const GemvArgs& a, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if (a.n_rows > (int64_t(1) << 31) - 32) return BNBQ_ERR_UNSUPPORTED;
  if (m <= 8) return launch_rows_t<XT, 8, NESTED>(m, a, di, s);
  if (m <= 12) return launch_rows_t<XT, 12, NESTED>(m, a, di, s);
  if (m <= 16) return launch_rows_t<XT, 16, NESTED>(m, a, di, s);
  return launch_rows_t<XT, 20, NESTED>(m, a, di, s);
}

template <typename XT, bool NESTED, int M = 1>
int launch_dispatch(int m, const GemvArgs& a, cudaStream_t s) {
  if constexpr (M > BNBQ_GEMV_MAX_M) {
    return BNBQ_ERR_INVALID;
  } else {
    if (m == M) return launch_m<XT, M, NESTED>(a, s);
    if (M == 2) {  // M = 3, 4: two passes of the pipelined kernels; above: one pass of the rows kernel
      const int st = m > 4 ? launch_rows<XT, NESTED>(m, a, s) : BNBQ_ERR_UNSUPPORTED;
      return st == BNBQ_ERR_UNSUPPORTED ? launch_pairs<XT, NESTED>(m, a, s) : st;
    }
    return launch_dispatch<XT, NESTED, M + 1>(m, a, s);
  }
}

}  // namespace

int gemv_wait_timeouts(unsigned int* out) { return read_wait_timeouts(out); }
int gemv_set_wait_limit(uint64_t ns) { return write_wait_limit(ns); }

int gemm_precise_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                        int32_t blocksize, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                        const float* code2, const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                        void* y, int64_t ldy, cudaStream_t s);

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
  if (m >= 5) {  // the tensor cores with the GEMV's precision (hi + lo split), where the tile applies
    const int st = gemm_precise_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                                       offset, blocksize2, absmax2_block0, y, ldy, s);
    if (st != BNBQ_ERR_UNSUPPORTED) return st;
  }
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

namespace bnbq {
int64_t gemv_xtab_workspace_bytes(int m, int k, int64_t n_rows);
// The streaming kernel with the exchange in its epilogue (M <= 2, one pass),
// y = px.y_full's own columns; BNBQ_ERR_UNSUPPORTED where that kernel does not
// apply (the caller then runs the matmul and the standalone exchange).
int gemv_exchange_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                         int32_t blocksize, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                         const float* code2, const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                         const PeerOut& px, cudaStream_t s) {
  if (m < 1 || m > 2) return BNBQ_ERR_UNSUPPORTED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  GemvArgs a{};
  a.x = x; a.w = w; a.absmax = absmax; a.absmax_q = absmax_q; a.absmax2 = absmax2;
  a.code2 = code2; a.offset = offset; a.n_rows = n_rows;
  a.y = static_cast<char*>(px.y_full) + size_t(px.col0) * 2;
  a.ldy = px.ldf;
  a.block0 = absmax2_block0; a.k = k; a.log2_bs = log2_exact(blocksize);
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  const bool nested = absmax_q != nullptr;
  if (nested && !aligned(code2, 16)) return BNBQ_ERR_UNSUPPORTED;
  BulkPlan p;
  if (!plan_bulk(m, k, a.log2_bs, nested, di.smem_optin, &p)) return BNBQ_ERR_UNSUPPORTED;
  if (p.scales_in_stage &&
      !aligned(nested ? static_cast<const void*>(absmax_q) : static_cast<const void*>(absmax), 16))
    p.scales_in_stage = 0;
  const PeerOut* xp = &px;
  if (dtype == BNBQ_BF16) {
    if (m == 1)
      return nested ? launch_bulk<__nv_bfloat16, 1, true>(a, p, di, s, xp)
                    : launch_bulk<__nv_bfloat16, 1, false>(a, p, di, s, xp);
    return nested ? launch_bulk<__nv_bfloat16, 2, true>(a, p, di, s, xp)
                  : launch_bulk<__nv_bfloat16, 2, false>(a, p, di, s, xp);
  }
  if (m == 1)
    return nested ? launch_bulk<__half, 1, true>(a, p, di, s, xp) : launch_bulk<__half, 1, false>(a, p, di, s, xp);
  return nested ? launch_bulk<__half, 2, true>(a, p, di, s, xp) : launch_bulk<__half, 2, false>(a, p, di, s, xp);
}

int gemv_xtab_launch(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows, int blocksize,
                     const float* absmax, const uint8_t* absmax_q, const float* absmax2, const float* code2,
                     const float* offset, int blocksize2, int64_t absmax2_block0, void* y, int64_t ldy,
                     void* workspace, int64_t workspace_bytes, cudaStream_t s, const PeerOut* px = nullptr);
}  // namespace bnbq

namespace bnbq {
int gemv_xtab_applies(int m, int k, int64_t n_rows, int blocksize, const uint8_t* absmax_q, int blocksize2,
                      const void* workspace, int64_t workspace_bytes);
}  // namespace bnbq

namespace bnbq {
int gemv_xtab_set_policy(int policy);
}  // namespace bnbq

extern "C" int bnbq_set_gemv_policy(int32_t policy) { return gemv_xtab_set_policy(policy); }

extern "C" int bnbq_gemv_route(int32_t m, int32_t k, int64_t n_rows, int32_t blocksize, const uint8_t* absmax_q,
                               int32_t blocksize2, const void* workspace, int64_t workspace_bytes, int32_t* route) {
  if (!route || m < 1 || k < 1 || n_rows < 1) return BNBQ_ERR_INVALID;
  if (m > BNBQ_GEMV_MAX_M) {
    *route = BNBQ_ROUTE_GEMM;
    return BNBQ_OK;
  }
  const int st = gemv_xtab_applies(m, k, n_rows, blocksize, absmax_q, blocksize2, workspace, workspace_bytes);
  if (st != BNBQ_OK && st != BNBQ_ERR_UNSUPPORTED) return st;
  *route = st == BNBQ_OK ? BNBQ_ROUTE_TABLE_GEMV : BNBQ_ROUTE_GEMV;
  return BNBQ_OK;
}

extern "C" int bnbq_gemv_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes) {
  if (!bytes || m < 1 || k < 1 || n_rows < 1) return BNBQ_ERR_INVALID;
  *bytes = m <= BNBQ_GEMV_MAX_M ? gemv_xtab_workspace_bytes(m, k, n_rows) : 0;
  return BNBQ_OK;
}

namespace bnbq {
int64_t gemv_code8_workspace_bytes(int m, int k, int64_t n_rows);
int gemv_code8_launch(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows, int blocksize,
                      const float* code, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                      const float* code2, const float* offset, int blocksize2, int64_t absmax2_block0, void* y,
                      int64_t ldy, void* workspace, int64_t workspace_bytes, cudaStream_t s);
}  // namespace bnbq

extern "C" int bnbq_gemv_blockwise_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes) {
  if (!bytes || m < 1 || m > BNBQ_GEMV8_MAX_M || k < 1 || n_rows < 1) return BNBQ_ERR_INVALID;
  if (k % 128) return BNBQ_ERR_UNSUPPORTED;
  *bytes = gemv_code8_workspace_bytes(m, k, n_rows);
  return *bytes > 0 ? BNBQ_OK : BNBQ_ERR_UNSUPPORTED;
}

extern "C" int bnbq_gemv_blockwise_ws(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                      int64_t n_rows, int32_t blocksize, const float* code, const float* absmax,
                                      const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                      const float* offset, int32_t blocksize2, int64_t absmax2_block0, void* y,
                                      int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream) {
  if (int st = gemv_validate(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                             offset, blocksize2, y, ldy))
    return st;
  if (m > BNBQ_GEMV8_MAX_M || !code || workspace_bytes < 0 || !workspace) return BNBQ_ERR_INVALID;
  if (k % 128) return BNBQ_ERR_UNSUPPORTED;
  if (!aligned(code, 4)) return BNBQ_ERR_MISALIGNED;
  return gemv_code8_launch(dtype, x, m, k, w, n_rows, blocksize, code, absmax, absmax_q, absmax2, code2, offset,
                           blocksize2, absmax2_block0, y, ldy, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int bnbq_gemv_nf4_ws(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                int64_t n_rows, int32_t blocksize, const float* absmax,
                                const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                void* y, int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream) {
  if (int st = gemv_validate(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2,
                             offset, blocksize2, y, ldy))
    return st;
  if (m > BNBQ_GEMV_MAX_M || workspace_bytes < 0 || (workspace_bytes > 0 && !workspace)) return BNBQ_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int st = gemv_xtab_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2, offset,
                                  blocksize2, absmax2_block0, y, ldy, workspace, workspace_bytes, s);
  if (st != BNBQ_ERR_UNSUPPORTED) return st;
  return gemv_launch(dtype, x, m, k, w, n_rows, blocksize, absmax, absmax_q, absmax2, code2, offset,
                     blocksize2, absmax2_block0, y, ldy, s);
}

namespace bnbq {
int peer_make(int dtype, int32_t m, int64_t n_local, int64_t col0, void* y_full, int64_t n_total, int64_t ldy,
              uint64_t* const* inbox, int64_t inbox_words, uint32_t* state, int32_t world, int32_t rank,
              PeerOut* px);
int peer_allgather_launch(const void* y_local, int32_t m, int64_t n_local, int64_t ld_local, const PeerOut& px,
                          cudaStream_t stream);
}  // namespace bnbq

// The row-sharded matmul and its exchange in one call: M <= 2 runs ONE kernel
// chain that computes this rank's rows and, in its epilogue, stores them into
// the peers' inboxes and collects the other ranks' columns (the table GEMV's
// reduction or the streaming GEMV); other shapes run the matmul into y_full's
// own columns and then the standalone exchange kernel on them. The results
// are those of bnbq_matmul_nf4_ws on the rank's rows, bitwise.
extern "C" int bnbq_matmul_nf4_allgather(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w,
                                         int64_t n_local, int32_t blocksize, const float* absmax,
                                         const uint8_t* absmax_q, const float* absmax2, const float* code2,
                                         const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                                         void* y_full, int64_t n_total, int64_t ldy, int64_t col0,
                                         uint64_t* const* inbox, int64_t inbox_words, uint32_t* state,
                                         int32_t world, int32_t rank, void* workspace, int64_t workspace_bytes,
                                         void* stream) {
  PeerOut px;
  if (int st = peer_make(dtype, m, n_local, col0, y_full, n_total, ldy, inbox, inbox_words, state, world, rank, &px))
    return st;
  if (m < 1 || workspace_bytes < 0 || (workspace_bytes > 0 && !workspace)) return BNBQ_ERR_INVALID;
  void* y_own = static_cast<char*>(y_full) + size_t(col0) * 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_local > 0) {
    if (int st = gemv_validate(dtype, x, m, k, w, n_local, blocksize, absmax, absmax_q, absmax2, code2, offset,
                               blocksize2, y_own, ldy))
      return st;
    if (world == 1)  // nothing to exchange
      return bnbq_matmul_nf4_ws(dtype, x, m, k, w, n_local, blocksize, absmax, absmax_q, absmax2, code2, offset,
                                blocksize2, absmax2_block0, y_own, ldy, workspace, workspace_bytes, stream);
    if (m <= 2) {  // the kernel the plain call would run, in its exchange mode, when it has one
      const int table = gemv_xtab_applies(m, k, n_local, blocksize, absmax_q, blocksize2, workspace,
                                          workspace_bytes);
      if (table != BNBQ_OK && table != BNBQ_ERR_UNSUPPORTED) return table;
      const int st = table == BNBQ_OK
                         ? gemv_xtab_launch(dtype, x, m, k, w, n_local, blocksize, absmax, absmax_q, absmax2, code2,
                                            offset, blocksize2, absmax2_block0, y_own, ldy, workspace,
                                            workspace_bytes, s, &px)
                         : gemv_exchange_launch(dtype, x, m, k, w, n_local, blocksize, absmax, absmax_q, absmax2,
                                                code2, offset, blocksize2, absmax2_block0, px, s);
      if (st != BNBQ_ERR_UNSUPPORTED) return st;
    }
    if (int st = bnbq_matmul_nf4_ws(dtype, x, m, k, w, n_local, blocksize, absmax, absmax_q, absmax2, code2, offset,
                                    blocksize2, absmax2_block0, y_own, ldy, workspace, workspace_bytes, stream))
      return st;
  }
  return peer_allgather_launch(y_own, m, n_local, ldy, px, s);
}

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
