// bnbq_quant.cu -- blockwise quantize (NF4 and 8-bit) and the absmax mean.
//
// Per block of bs elements (reference kernels/quantize.py:128-193):
//   m = max.ftz(-FLT_MAX, abs.ftz(x_i)...)   (partial last block: zero padded)
//   r = rcp.approx.ftz(m)
//   code_i = choose(mul.ftz(x_i, r))
//
// Mapping. A lane owns 8 consecutive elements (one 16-byte load of a 16-bit
// type, two of float32), so a warp reads 256 contiguous elements per step.
// For bs <= 256 a block is L = bs/8 adjacent lanes and its absmax is a
// butterfly over those lanes; for bs > 256 a warp owns a whole block and loops
// over its bs/256 segments (values kept in registers up to bs = 1024, read
// again from L1/L2 above that). Warps pull work round-robin from a grid of a
// whole number of CTAs per SM; two segments per warp are in flight at once.
//
// Code choice, NF4 (reference's 15-compare count, kernels/quantize.py:91-95).
// Evaluated as one bucket lookup: u = fma(max(s,-1), 16, 2^23+16) rounds
// 16s+16 to an integer i = bits(u) & 63; the 33 buckets of width 1/16 hold at
// most one threshold each, so code = base[i] + (s > thr[i]). The tables are
// built per CTA from the thresholds' own buckets. (The equivalence with the
// 15-compare count is checked on the CPU for every float32 in [-1.01, 1.01].)
//
// Code choice, 8-bit (reference's binary search with midpoint rounding,
// kernels/quantize.py:102-125). For a strictly increasing finite codebook the
// search equals a count of 255 strict thresholds T_j (even j: the midpoint;
// odd j: the float just below the midpoint, or C[j] when the midpoint rounds
// onto it). Each CTA builds, from the codebook, a monotone bucket map over the
// float32 bits of s (sign, exponent, 4 mantissa bits; tiny and huge
// magnitudes clamped), base[b] = #thresholds in lower buckets, and the widest
// bucket's threshold count -> S search steps; then
//   code = base[bucket(s)] + (binary search of S steps over T[base ...]).
// Both tables are replicated per lane ([entry][32]) so a warp's random
// lookups never collide in a bank. Codebooks that are not strictly increasing,
// or whose buckets would need more than 4 steps, take the literal search.
#include <float.h>

#include "bnbq_common.cuh"

namespace bnbq {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// ------------------------------------------------------------------ tables

__device__ __forceinline__ int nf4_bucket(float s) {
  return int(__float_as_uint(__fmaf_rn(fmaxf(s, -1.0f), 16.0f, 8388624.0f)) & 63u);
}

// 8-bit bucket map over float32 bits (same as the CPU oracle's or_q8_bucket).
constexpr int kQ8MantBits = 4;
constexpr int kQ8ExpLo = 127 - 24;
constexpr int kQ8ExpHi = 127 + 2;
constexpr int kQ8NMag = (kQ8ExpHi - kQ8ExpLo) << kQ8MantBits;
constexpr int kQ8NB = 2 * kQ8NMag + 2;
constexpr int kQ8MaxSteps = 4;
constexpr int kQ8TLen = 255 + (1 << kQ8MaxSteps);  // +inf padded

__device__ __forceinline__ int q8_bucket(float s) {
  const uint32_t bits = __float_as_uint(fmaxf(s, -INFINITY));  // NaN -> -inf
  int mag = int((bits & 0x7fffffffu) >> (23 - kQ8MantBits));
  mag = min(max(mag, kQ8ExpLo << kQ8MantBits), kQ8ExpHi << kQ8MantBits) - (kQ8ExpLo << kQ8MantBits);
  const int sgn = int(bits) >> 31;
  return (kQ8NMag + 1) + (mag ^ sgn);
}

// The reference's literal search (slow path).
__device__ __forceinline__ int code8_search(const float* C, float x) {
  int pivot = 127, upper_pivot = 255, lower_pivot = 0;
  float lower = -1.0f, upper = 1.0f;
  float val = C[pivot];
#pragma unroll
  for (int i = 64; i > 0; i >>= 1) {
    const bool gt = x > val;
    lower_pivot = gt ? pivot : lower_pivot;
    lower = gt ? val : lower;
    upper_pivot = gt ? upper_pivot : pivot;
    upper = gt ? upper : val;
    pivot = gt ? pivot + i : pivot - i;
    val = C[pivot];
  }
  upper = upper_pivot == 255 ? C[255] : upper;
  lower = lower_pivot == 0 ? C[0] : lower;
  const int up = (x > __fmul_rn(__fadd_rn(upper, val), 0.5f)) ? upper_pivot : pivot;
  const int down = (x < __fmul_rn(__fadd_rn(lower, val), 0.5f)) ? lower_pivot : pivot;
  return x > val ? up : down;
}

struct QuantArgs {
  const void* x;
  int64_t n;
  int64_t nb;
  int log2_bs;
  uint8_t* q;
  float* absmax;
  const float* code;    // 8-bit only
  const float* offset;  // 8-bit only, nullable: x := fl32(x - offset)
};

// Shared memory of the 8-bit kernel.
struct Q8Smem {
  float code[256];
  float T[kQ8TLen];
  int bt[kQ8TLen];
  int maxwin;
  int steps;  // -1: literal search
  float T_rep[kQ8TLen * 32];
  uint8_t base_rep[kQ8NB * 32];
};

struct NF4Smem {
  float thr[64];
  int base[64];
};

__device__ void build_nf4_tables(NF4Smem& sm) {
  const int i = threadIdx.x;
  if (i < 64) {
    int b = 15;
    float t = INFINITY;
    if (i <= 32) {
      b = 0;
#pragma unroll
      for (int j = 0; j < 15; ++j) {
        const float tj = __uint_as_float(kNF4ThresholdBits[j]);
        const int bj = nf4_bucket(tj);
        b += (bj < i);
        if (bj == i) t = tj;
      }
    }
    sm.thr[i] = t;
    sm.base[i] = b;
  }
}

__device__ void build_q8_tables(Q8Smem& sm, const float* code) {
  const int tid = threadIdx.x;
  for (int j = tid; j < 256; j += kThreads) sm.code[j] = __ldg(code + j);
  if (tid == 0) sm.maxwin = 0;
  __syncthreads();
  bool ok = true;
  for (int j = tid; j < 256; j += kThreads) {
    const float c = sm.code[j];
    ok &= isfinite(c) && (j == 255 || c < sm.code[j + 1]);
  }
  ok = __syncthreads_and(ok);
  if (!ok) {
    if (tid == 0) sm.steps = -1;
    __syncthreads();
    return;
  }
  for (int j = tid; j < kQ8TLen; j += kThreads) {
    float t = INFINITY;
    if (j < 255) {
      const float c0 = sm.code[j], c1 = sm.code[j + 1];
      const float mid = __fmul_rn(__fadd_rn(c0, c1), 0.5f);
      t = !(j & 1) ? mid : (mid > c0 ? __int_as_float(__float_as_int(mid) + (mid > 0.0f ? -1 : 1)) : c0);
      // nextafter(mid, -inf): for mid == +0 step to -denorm_min
      if ((j & 1) && mid > c0 && mid == 0.0f) t = -__int_as_float(1);
    }
    sm.T[j] = t;
    sm.bt[j] = j < 255 ? q8_bucket(t) : kQ8NB;
  }
  __syncthreads();
  for (int b = tid; b < kQ8NB; b += kThreads) {
    int lo = 0, hi = 255;  // lower_bound of b in bt[0..255)
    while (lo < hi) { const int mid = (lo + hi) >> 1; if (sm.bt[mid] < b) lo = mid + 1; else hi = mid; }
    int lo2 = lo, hi2 = 255;  // upper_bound
    while (lo2 < hi2) { const int mid = (lo2 + hi2) >> 1; if (sm.bt[mid] <= b) lo2 = mid + 1; else hi2 = mid; }
    atomicMax(&sm.maxwin, lo2 - lo);
    for (int l = 0; l < 32; ++l) sm.base_rep[b * 32 + l] = uint8_t(lo);
  }
  for (int e = tid; e < kQ8TLen * 32; e += kThreads) sm.T_rep[e] = sm.T[e >> 5];
  __syncthreads();
  if (tid == 0) {
    int S = 0;
    while ((1 << S) - 1 < sm.maxwin) ++S;
    sm.steps = S <= kQ8MaxSteps ? S : -1;
  }
  __syncthreads();
}

template <int S>
__device__ __forceinline__ int code8_fast(const Q8Smem& sm, float s, int lane) {
  int c = sm.base_rep[q8_bucket(s) * 32 + lane];
#pragma unroll
  for (int st = S - 1; st >= 0; --st) {
    const float t = sm.T_rep[(c + (1 << st) - 1) * 32 + lane];
    c += (s > t) ? (1 << st) : 0;
  }
  return c;
}

// ----------------------------------------------------------- element loads

template <typename InT>
__device__ __forceinline__ void load8(const InT* x, int64_t e0, int64_t n, float (&v)[8]) {
  if (e0 + 8 <= n) {
    if constexpr (sizeof(InT) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(x + e0);
      const float4 b = *reinterpret_cast<const float4*>(x + e0 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      const uint4 w = *reinterpret_cast<const uint4*>(x + e0);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Elem<InT>::kDtype == BNBQ_BF16 ? unpack2_bf16(ws[j]) : unpack2_f16(ws[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (e0 + j < n) ? Elem<InT>::to_f32(x[e0 + j]) : 0.0f;
  }
}

// ------------------------------------------------------------------ codes

struct NF4Choose {
  const NF4Smem* sm;
  __device__ int operator()(float s, int) const {
    const int i = nf4_bucket(s);
    return sm->base[i] + (s > sm->thr[i]);
  }
};

template <int S>
struct Q8Choose {
  const Q8Smem* sm;
  __device__ int operator()(float s, int lane) const {
    if constexpr (S < 0) return code8_search(sm->code, s);
    else return code8_fast<S>(*sm, s, lane);
  }
};

// Codes of 8 scaled values, stored at their exact byte positions.
template <bool NF4, typename Choose>
__device__ __forceinline__ void emit_codes(const QuantArgs& a, int64_t e0, const float (&v)[8],
                                           float r, const Choose& choose, int lane) {
  int c[8];
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const float2 s = mul_ftz2(make_float2(v[j], v[j + 1]), make_float2(r, r));
    c[j] = choose(s.x, lane);
    c[j + 1] = choose(s.y, lane);
  }
  if constexpr (NF4) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) w |= uint32_t((c[2 * j] << 4) | c[2 * j + 1]) << (8 * j);
    if (e0 + 8 <= a.n) {
      *reinterpret_cast<uint32_t*>(a.q + (e0 >> 1)) = w;
    } else {
      const int64_t nq = (a.n + 1) >> 1;
      for (int j = 0; j < 4; ++j)
        if ((e0 >> 1) + j < nq) a.q[(e0 >> 1) + j] = uint8_t(w >> (8 * j));
    }
  } else {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo |= uint32_t(c[j]) << (8 * j);
      hi |= uint32_t(c[j + 4]) << (8 * j);
    }
    if (e0 + 8 <= a.n) {
      *reinterpret_cast<uint2*>(a.q + e0) = make_uint2(lo, hi);
    } else {
      for (int j = 0; j < 8; ++j)
        if (e0 + j < a.n) a.q[e0 + j] = uint8_t((j < 4 ? lo : hi) >> (8 * (j & 3)));
    }
  }
}

template <typename InT>
__device__ __forceinline__ void center(const QuantArgs& a, int64_t e0, float (&v)[8], float off) {
  if (a.offset) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (e0 + j < a.n) v[j] = sub_rn(v[j], off);  // padding stays 0 (array.py:201 pads after)
  }
}

// Raw 16-byte vectors of one lane's 8 elements (one for 16-bit types, two for
// float32), loaded early and unpacked when the segment is processed, so that
// a warp keeps several segments in flight at a modest register cost.
template <typename InT>
struct Raw8 {
  static constexpr int kVec = sizeof(InT) == 4 ? 2 : 1;
  uint4 w[kVec];
  bool full;
};

template <typename InT>
__device__ __forceinline__ void load_raw8(const InT* x, int64_t e0, int64_t n, Raw8<InT>& r) {
  r.full = e0 + 8 <= n;
  if (r.full) {
#pragma unroll
    for (int i = 0; i < Raw8<InT>::kVec; ++i) r.w[i] = *reinterpret_cast<const uint4*>(x + e0 + 4 * i);
  }
}

template <typename InT>
__device__ __forceinline__ void unpack_raw8(const InT* x, int64_t e0, int64_t n, const Raw8<InT>& r,
                                            float (&v)[8]) {
  if (!r.full) {  // partial segment at the end: element loads
    load8<InT>(x, e0, n, v);
    return;
  }
  if constexpr (sizeof(InT) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(&r.w[0]);
    const float4 b = *reinterpret_cast<const float4*>(&r.w[1]);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint32_t ws[4] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = Elem<InT>::kDtype == BNBQ_BF16 ? unpack2_bf16(ws[j]) : unpack2_f16(ws[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// bs <= 256: L = bs/8 lanes per block, one 256-element segment per warp step;
// U segments per warp are loaded before any is processed (4 for 16-bit inputs,
// 2 for float32: 2 KB per warp in flight either way).
template <typename InT, bool NF4, typename Choose>
__device__ void quant_small(const QuantArgs& a, const Choose& choose) {
  const InT* x = static_cast<const InT*>(a.x);
  const int lane = threadIdx.x & 31;
  const int L = 1 << (a.log2_bs - 3);
  const int64_t nseg = (a.n + 255) >> 8;
  const int64_t gw = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t tw = (int64_t(gridDim.x) * kThreads) >> 5;
  const float off = a.offset ? __ldg(a.offset) : 0.0f;
  constexpr int U = sizeof(InT) == 4 ? 2 : 4;
  for (int64_t seg0 = gw; seg0 < nseg; seg0 += tw * U) {
    Raw8<InT> raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t e0 = ((seg0 + u * tw) << 8) + lane * 8;
      load_raw8<InT>(x, e0, a.n, raw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t seg = seg0 + u * tw;
      if (seg >= nseg) break;  // warp-uniform
      const int64_t e0 = (seg << 8) + lane * 8;
      float v[8];
      unpack_raw8<InT>(x, e0, a.n, raw[u], v);
      center<InT>(a, e0, v, off);
      float m = -FLT_MAX;
#pragma unroll
      for (int j = 0; j < 8; ++j) m = max_abs_ftz(m, v[j]);
      for (int o = L >> 1; o > 0; o >>= 1) m = max_ftz(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float r = rcp_approx_ftz(m);
      const int64_t b = e0 >> a.log2_bs;
      if (b < a.nb) {
        if ((lane & (L - 1)) == 0) a.absmax[b] = m;
        if (e0 < a.n) emit_codes<NF4>(a, e0, v, r, choose, lane);
      }
    }
  }
}

// bs > 256: one block per warp; P = bs/256 segments; HOLD: keep values.
template <typename InT, bool NF4, int HOLD, typename Choose>
__device__ void quant_large(const QuantArgs& a, const Choose& choose) {
  const InT* x = static_cast<const InT*>(a.x);
  const int lane = threadIdx.x & 31;
  const int P = 1 << (a.log2_bs - 8);
  const int64_t gw = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t tw = (int64_t(gridDim.x) * kThreads) >> 5;
  const float off = a.offset ? __ldg(a.offset) : 0.0f;
  for (int64_t b = gw; b < a.nb; b += tw) {
    const int64_t base = b << a.log2_bs;
    float m = -FLT_MAX;
    float held[HOLD > 0 ? HOLD : 1][8];
    if constexpr (HOLD > 0) {
#pragma unroll
      for (int p = 0; p < HOLD; ++p) load8<InT>(x, base + p * 256 + lane * 8, a.n, held[p]);
#pragma unroll
      for (int p = 0; p < HOLD; ++p) {
        center<InT>(a, base + p * 256 + lane * 8, held[p], off);
#pragma unroll
        for (int j = 0; j < 8; ++j) m = max_abs_ftz(m, held[p][j]);
      }
    } else {
      for (int p0 = 0; p0 < P; p0 += 4) {
        float v[4][8];
#pragma unroll
        for (int p = 0; p < 4; ++p) load8<InT>(x, base + (p0 + p) * 256 + lane * 8, a.n, v[p]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          center<InT>(a, base + (p0 + p) * 256 + lane * 8, v[p], off);
#pragma unroll
          for (int j = 0; j < 8; ++j) m = max_abs_ftz(m, v[p][j]);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max_ftz(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float r = rcp_approx_ftz(m);
    if (lane == 0) a.absmax[b] = m;
    if constexpr (HOLD > 0) {
#pragma unroll
      for (int p = 0; p < HOLD; ++p) {
        const int64_t e0 = base + p * 256 + lane * 8;
        if (e0 < a.n) emit_codes<NF4>(a, e0, held[p], r, choose, lane);
      }
    } else {
      for (int p = 0; p < P; ++p) {
        const int64_t e0 = base + p * 256 + lane * 8;
        if (e0 >= a.n) break;
        float v[8];
        load8<InT>(x, e0, a.n, v);
        center<InT>(a, e0, v, off);
        emit_codes<NF4>(a, e0, v, r, choose, lane);
      }
    }
  }
}

template <typename InT, bool NF4, typename Choose>
__device__ __forceinline__ void quant_body(const QuantArgs& a, const Choose& choose) {
  if (a.log2_bs <= 8) quant_small<InT, NF4>(a, choose);
  else if (a.log2_bs == 9) quant_large<InT, NF4, 2>(a, choose);
  else if (a.log2_bs == 10) quant_large<InT, NF4, 4>(a, choose);
  else quant_large<InT, NF4, 0>(a, choose);
}

template <typename InT>
__global__ void __launch_bounds__(kThreads) quant_nf4_kernel(QuantArgs a) {
  __shared__ NF4Smem sm;
  build_nf4_tables(sm);
  __syncthreads();
  quant_body<InT, true>(a, NF4Choose{&sm});
}

template <typename InT>
__global__ void __launch_bounds__(kThreads) quant_8bit_kernel(QuantArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Q8Smem& sm = *reinterpret_cast<Q8Smem*>(smem_raw);
  build_q8_tables(sm, a.code);
  switch (sm.steps) {
    case 0: quant_body<InT, false>(a, Q8Choose<0>{&sm}); break;
    case 1: quant_body<InT, false>(a, Q8Choose<1>{&sm}); break;
    case 2: quant_body<InT, false>(a, Q8Choose<2>{&sm}); break;
    case 3: quant_body<InT, false>(a, Q8Choose<3>{&sm}); break;
    case 4: quant_body<InT, false>(a, Q8Choose<4>{&sm}); break;
    default: quant_body<InT, false>(a, Q8Choose<-1>{&sm}); break;
  }
}

template <typename Kern>
int launch_grid(Kern kern, size_t smem, int64_t work_warps, const QuantArgs& a, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  if (per_sm < 1) per_sm = 1;
  int64_t grid = int64_t(di.sm_count) * per_sm;
  const int64_t want = (work_warps + kWarps - 1) / kWarps;
  if (want < grid) grid = want > 0 ? want : 1;
  kern<<<dim3(unsigned(grid)), dim3(kThreads), smem, s>>>(a);
  return launch_status();
}

int check_quant(int dtype, const void* x, int64_t n, int32_t bs, uint8_t* q, float* absmax,
                QuantArgs* a) {
  if (dtype != BNBQ_F32 && dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (n < 0) return BNBQ_ERR_INVALID;
  a->log2_bs = log2_exact(bs);
  if (a->log2_bs < 3 || a->log2_bs > 12) return BNBQ_ERR_INVALID;
  if (n > 0 && (!x || !q || !absmax)) return BNBQ_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(q, 16) || !aligned(absmax, 4)) return BNBQ_ERR_MISALIGNED;
  a->x = x; a->n = n; a->nb = (n + bs - 1) / bs; a->q = q; a->absmax = absmax;
  return BNBQ_OK;
}

int64_t work_warps(const QuantArgs& a) {
  return a.log2_bs <= 8 ? (a.n + 255) >> 8 : a.nb;
}

// offset[0] = mean(absmax), float64 accumulation in a fixed order: one cluster
// of kMeanCtas CTAs; CTA c sums the strided elements c*1024 + t (+ i*kMeanCtas*1024)
// per thread, reduces its 1024 partials in a fixed tree, and rank 0 adds the
// CTAs' sums in rank order (distributed shared memory, between two cluster
// barriers that every thread passes).
constexpr int kMeanCtas = 8;

__global__ void __launch_bounds__(1024) mean_kernel(const float* a, int64_t n, float* out) {
  __shared__ double part[1024];
  __shared__ double ctas[kMeanCtas];
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  double s = 0.0;
  for (int64_t i = int64_t(rank) * 1024 + threadIdx.x; i < n; i += int64_t(kMeanCtas) * 1024) s += double(a[i]);
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = 512; w > 0; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (threadIdx.x == 0) {
    uint32_t dst;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(uint32_t(__cvta_generic_to_shared(&ctas[rank]))), "r"(0));
    asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(dst), "d"(part[0]) : "memory");
  }
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (rank == 0 && threadIdx.x == 0) {
    double t = 0.0;
    for (int c = 0; c < kMeanCtas; ++c) t += ctas[c];
    out[0] = float(t / double(n));
  }
}

}  // namespace
}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_quantize_nf4(int dtype, const void* x, int64_t n, int32_t blocksize,
                                 uint8_t* q, float* absmax, void* stream) {
  QuantArgs a{};
  if (int st = check_quant(dtype, x, n, blocksize, q, absmax, &a)) return st;
  if (n == 0) return BNBQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ww = work_warps(a);
  switch (dtype) {
    case BNBQ_F32: return launch_grid(quant_nf4_kernel<float>, 0, ww, a, s);
    case BNBQ_F16: return launch_grid(quant_nf4_kernel<__half>, 0, ww, a, s);
    default: return launch_grid(quant_nf4_kernel<__nv_bfloat16>, 0, ww, a, s);
  }
}

extern "C" int bnbq_quantize_blockwise(int dtype, const void* x, int64_t n, int32_t blocksize,
                                       const float* code, const float* offset, uint8_t* q,
                                       float* absmax, void* stream) {
  QuantArgs a{};
  if (int st = check_quant(dtype, x, n, blocksize, q, absmax, &a)) return st;
  if (n == 0) return BNBQ_OK;
  if (!code) return BNBQ_ERR_INVALID;
  if (!aligned(code, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  a.code = code;
  a.offset = offset;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t ww = work_warps(a);
  const size_t smem = sizeof(Q8Smem);
  switch (dtype) {
    case BNBQ_F32: return launch_grid(quant_8bit_kernel<float>, smem, ww, a, s);
    case BNBQ_F16: return launch_grid(quant_8bit_kernel<__half>, smem, ww, a, s);
    default: return launch_grid(quant_8bit_kernel<__nv_bfloat16>, smem, ww, a, s);
  }
}

extern "C" int bnbq_absmax_mean(const float* absmax, int64_t nb, float* offset, void* stream) {
  if (nb <= 0 || !absmax || !offset) return BNBQ_ERR_INVALID;
  if (!aligned(absmax, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kMeanCtas);
  cfg.blockDim = dim3(1024);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kMeanCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, mean_kernel, absmax, nb, offset) != cudaSuccess) return BNBQ_ERR_CUDA;
  return launch_status();
}
