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
// onto it). Each CTA builds, from the codebook, buckets of s by sign and by
// magnitude key |bits| >> shift (exponent and the top 23 - shift mantissa
// bits; magnitudes below the smallest threshold's key clamped into key 0),
// with as many mantissa bits as a 2 x 4096-entry table allows, so that no
// bucket holds two thresholds (the dynamic map gets 7). A threshold shares
// every bit above the low `shift` bits with the values of its bucket, so
// "s > T" compares those low bits, in reverse for negative values. One 32-bit
// word per bucket, E = base * 2^24 + an offset from the threshold's low bits,
// makes the compare a carry:
//   code = (E + low(s)) >> 24 (positive s),  (E - low(s)) >> 24 (negative s),
// base = thresholds in lower buckets. In a symmetric codebook the middle
// threshold is the float just below 0, whose tiny exponent would stretch the
// table; then the threshold of smallest magnitude stays out of the table and
// is compared directly. The per-element work (bucket, low bits, carry) is
// integer multiply-adds on the FMA pipe, not shifts and compares on the
// half-rate ALU pipe. Codebooks that are not strictly increasing, or whose
// thresholds would share a bucket, take the literal search.
#include <float.h>
#include <limits.h>

#include "bnbq_async.cuh"
#include "bnbq_common.cuh"

namespace bnbq {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// ------------------------------------------------------------------ tables

__device__ __forceinline__ int nf4_bucket(float s) {
  return int(__float_as_uint(__fmaf_rn(fmaxf(s, -1.0f), 16.0f, 8388624.0f)) & 63u);
}

// 8-bit bucket table (see the header): 2 * kQ8Keys entries at most.
constexpr int kQ8Keys = 4096;

// Per-element constants of the bucket map. The power-of-two multipliers are
// runtime values, so the compiler keeps the multiply-adds (FMA pipe) instead
// of turning them into shifts (ALU pipe).
struct Q8Map {
  int shift;         // low bits compared within a bucket
  int kmin;          // magnitude key of bucket 0 (the clamp bucket)
  int nkeys;         // magnitude buckets per sign
  uint32_t m_key;    // 2^(32 - shift): umulhi(u, m_key) = u >> shift
  uint32_t m_low;    // -2^shift: u + key * m_low = low bits
  uint32_t m_sgnk;   // 2^(31 - shift): sign bit's share of the key
  uint32_t m_two;    // 2: umulhi(u, 2) = sign bit
  uint32_t m_code;   // 256: umulhi(v, 256) = v >> 24
  int ex;            // 1: the smallest-magnitude threshold t_ex is compared directly
  float t_ex;
};

// Table index and low bits of s (NaN as -2: code 0, below every threshold;
// magnitudes from 2 on clamped into the top bucket, which holds no threshold).
__device__ __forceinline__ uint32_t q8_index(const Q8Map& m, float s, uint32_t& low, uint32_t& sg) {
  const uint32_t u = __float_as_uint(fmaxf(s, -2.0f));
  sg = __umulhi(u, m.m_two);
  const uint32_t kf = __umulhi(u, m.m_key);
  low = u + kf * m.m_low;
  const int k = max(int(kf - sg * m.m_sgnk) - m.kmin, 0);
  return sg * uint32_t(m.nkeys) + uint32_t(min(k, m.nkeys - 1));
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
  uint32_t two;         // 2, passed at run time (see gt01)
  int offset_in_arg;    // the offset is offset_value (computed by the same kernel), not *offset
  float offset_value;
  int cta0, ctas;       // the CTAs [cta0, cta0 + ctas) share the work (ctas == 0: the whole grid)
};

// This thread's warp among the working CTAs, and the number of their warps.
__device__ __forceinline__ void work_warp(const QuantArgs& a, int64_t& gw, int64_t& tw) {
  const int64_t ctas = a.ctas ? a.ctas : gridDim.x;
  gw = ((int64_t(blockIdx.x) - a.cta0) * kThreads + threadIdx.x) >> 5;
  tw = (ctas * kThreads) >> 5;
}

__device__ __forceinline__ float offset_of(const QuantArgs& a) {
  return a.offset ? (a.offset_in_arg ? a.offset_value : __ldg(a.offset)) : 0.0f;
}

// Shared memory of the 8-bit kernel.
struct Q8Smem {
  float code[256];
  float T[256];        // the 255 thresholds
  int ordc[256];       // bucket ordinals (monotone in value) of the table thresholds, ascending
  uint32_t lowc[256];  // their low bits
  Q8Map map;
  int kmin;
  unsigned long long exj;  // (magnitude bits << 8) | index of the smallest-magnitude threshold
  int mode;            // 1: bucket table, -1: literal search
  int okflag;
  uint32_t tab[2 * kQ8Keys];
};

// Bucket i: (its threshold or +inf, thresholds in lower buckets as int bits).
struct NF4Smem {
  float2 tb[64];
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
    sm.tb[i] = make_float2(t, __int_as_float(b));
  }
}

// (x > y) as 0/1 from the sign bit of fl(y - x) (IEEE subtraction keeps the
// sign of the exact difference; equal -> +0; a NaN x -> the positive default
// NaN), on the FMA pipe: `two` is a runtime 2, so umulhi is not turned into a
// shift.
__device__ __forceinline__ uint32_t gt01(float x, float y, uint32_t two) {
  return __umulhi(__float_as_uint(__fsub_rn(y, x)), two);
}

// Bucket ordinal of a table index (monotone in the value of s).
__device__ __forceinline__ int q8_ord(int idx, int nkeys) { return idx >= nkeys ? nkeys - 1 - (idx - nkeys) : nkeys + idx; }

__device__ void build_q8_tables(Q8Smem& sm, const float* code) {
  const int tid = threadIdx.x;
  static_assert(kThreads >= 255, "one threshold per thread");
  for (int j = tid; j < 256; j += kThreads) sm.code[j] = __ldg(code + j);
  if (tid == 0) { sm.mode = 1; sm.exj = ~0ull; }
  __syncthreads();
  bool ok = true;
  for (int j = tid; j < 256; j += kThreads) {
    const float c = sm.code[j];
    ok &= isfinite(c) && (j == 255 || c < sm.code[j + 1]);
  }
  if (!__syncthreads_and(ok)) {
    if (tid == 0) sm.mode = -1;
    __syncthreads();
    return;
  }
  float t = 0.0f;  // thread j < 255: threshold j
  if (tid < 255) {
    const float c0 = sm.code[tid], c1 = sm.code[tid + 1];
    const float mid = __fmul_rn(__fadd_rn(c0, c1), 0.5f);
    t = !(tid & 1) ? mid : (mid > c0 ? __int_as_float(__float_as_int(mid) + (mid > 0.0f ? -1 : 1)) : c0);
    // nextafter(mid, -inf): for mid == +0 step to -denorm_min
    if ((tid & 1) && mid > c0 && mid == 0.0f) t = -__int_as_float(1);
    sm.T[tid] = t;
    atomicMin(&sm.exj, (static_cast<unsigned long long>(__float_as_uint(t) & 0x7fffffffu) << 8) | unsigned(tid));
  }
  __syncthreads();
  const int jx = int(sm.exj & 255u);
  const uint32_t key2 = 0x40000000u;  // |bits| of 2.0: the top (clamp) bucket starts there
  // without, then with the smallest-magnitude threshold left out; largest mb that fits
  for (int ex = 0; ex < 2; ++ex) {
    for (int mb = 8; mb >= 1; --mb) {
      const int shift = 23 - mb;
      if (tid == 0) sm.kmin = INT_MAX;
      __syncthreads();
      const bool in_table = tid < 255 && !(ex && tid == jx);
      if (in_table) atomicMin(&sm.kmin, int((__float_as_uint(t) & 0x7fffffffu) >> shift));
      __syncthreads();
      const int kmin = sm.kmin - 1;  // clamp bucket below every threshold
      const int nkeys = int(key2 >> shift) - kmin + 1;
      if (kmin < 0 || nkeys > kQ8Keys) {
        __syncthreads();
        continue;
      }
      Q8Map m;
      m.shift = shift; m.kmin = kmin; m.nkeys = nkeys;
      m.m_key = 1u << (32 - shift); m.m_low = 0u - (1u << shift); m.m_sgnk = 1u << (31 - shift);
      m.m_two = 2u; m.m_code = 256u; m.ex = ex; m.t_ex = sm.T[jx];
      // every table threshold in a bucket of its own, none in a clamp bucket
      // (key 0 below the smallest threshold, key nkeys - 1 from |s| = 2 on)
      const int nin = 255 - ex;  // table thresholds, in value order at i = j - (j > jx)
      const int i = tid - (ex && tid > jx ? 1 : 0);
      uint32_t low = 0, sg = 0;
      const int idx = in_table ? int(q8_index(m, t, low, sg)) : 0;
      if (tid == 0) sm.okflag = 1;
      __syncthreads();
      if (in_table) {
        sm.ordc[i] = q8_ord(idx, nkeys);
        sm.lowc[i] = low;
        const int k = idx >= nkeys ? idx - nkeys : idx;
        if (k == 0 || k == nkeys - 1) sm.okflag = 0;
      }
      __syncthreads();
      if (in_table && i + 1 < nin && sm.ordc[i + 1] <= sm.ordc[i]) sm.okflag = 0;
      __syncthreads();
      if (sm.okflag) {
        const uint32_t mask = (1u << shift) - 1u;
        for (int b = tid; b < 2 * nkeys; b += kThreads) {
          const int o = q8_ord(b, nkeys);
          int lo = 0, hi = nin;  // table thresholds in lower buckets: lower_bound of o
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (sm.ordc[mid] < o) lo = mid + 1; else hi = mid;
          }
          const bool neg = b >= nkeys;
          uint32_t lt = neg ? 0u : mask;  // no threshold: the compare never carries
          if (lo < nin && sm.ordc[lo] == o) lt = sm.lowc[lo];
          sm.tab[b] = uint32_t(lo) * (1u << 24) + (neg ? (1u << 24) + lt - 1u : (1u << 24) - 1u - lt);
        }
        if (tid == 0) sm.map = m;
        __syncthreads();
        return;
      }
      __syncthreads();
    }
  }
  if (tid == 0) sm.mode = -1;
  __syncthreads();
}

// code = (E + low) >> 24 or (E - low) >> 24 (+ the directly compared threshold)
template <bool EX>
__device__ __forceinline__ int code8_table(const Q8Smem& sm, const Q8Map& m, float s) {
  uint32_t low, sg;
  const uint32_t idx = q8_index(m, s, low, sg);
  const uint32_t e = sm.tab[idx];
  int c = int(__umulhi(e + (1u - sg * m.m_two) * low, m.m_code));
  if constexpr (EX) c += int(gt01(s, m.t_ex, m.m_two));
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
  uint32_t two;  // 2 (runtime)
  __device__ int operator()(float s, int) const {
    const float2 e = sm->tb[nf4_bucket(s)];
    return __float_as_int(e.y) + (s > e.x ? 1 : 0);  // a plain compare measured faster here than gt01
  }
};

template <int MODE>  // 0: table, 1: table + one direct compare, -1: literal search
struct Q8Choose {
  const Q8Smem* sm;
  Q8Map m;
  __device__ int operator()(float s, int) const {
    if constexpr (MODE >= 0) return code8_table<MODE == 1>(*sm, m, s);
    else return code8_search(sm->code, s);
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
    // byte j = c[2j] * 16 + c[2j+1], little-endian: one multiply-add per code
    uint32_t w = uint32_t(c[6]);
    w = w * 16u + uint32_t(c[7]);
    w = w * 16u + uint32_t(c[4]);
    w = w * 16u + uint32_t(c[5]);
    w = w * 16u + uint32_t(c[2]);
    w = w * 16u + uint32_t(c[3]);
    w = w * 16u + uint32_t(c[0]);
    w = w * 16u + uint32_t(c[1]);
    if (e0 + 8 <= a.n) {
      *reinterpret_cast<uint32_t*>(a.q + (e0 >> 1)) = w;
    } else {
      const int64_t nq = (a.n + 1) >> 1;
      for (int j = 0; j < 4; ++j)
        if ((e0 >> 1) + j < nq) a.q[(e0 >> 1) + j] = uint8_t(w >> (8 * j));
    }
  } else {
    uint32_t lo = uint32_t(c[3]), hi = uint32_t(c[7]);
#pragma unroll
    for (int j = 2; j >= 0; --j) {
      lo = lo * 256u + uint32_t(c[j]);
      hi = hi * 256u + uint32_t(c[j + 4]);
    }
    if (e0 + 8 <= a.n) {
      *reinterpret_cast<uint2*>(a.q + e0) = make_uint2(lo, hi);
    } else {
      for (int j = 0; j < 8; ++j)
        if (e0 + j < a.n) a.q[e0 + j] = uint8_t((j < 4 ? lo : hi) >> (8 * (j & 3)));
    }
  }
}

// max.ftz over the warp of per-lane maxima that are >= 0 or -FLT_MAX (every
// input NaN): such floats order like their bit patterns as signed integers,
// so one redux replaces five shuffle-and-max steps.
__device__ __forceinline__ float warp_max_nonneg(float m) {
  int r;
  asm volatile("redux.sync.max.s32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(__float_as_int(m)));
  return __int_as_float(r);
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
  int64_t gw, tw;
  work_warp(a, gw, tw);
  const float off = offset_of(a);
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
      if (L == 32) m = warp_max_nonneg(m);
      else
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
  int64_t gw, tw;
  work_warp(a, gw, tw);
  const float off = offset_of(a);
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
    m = warp_max_nonneg(m);
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

// Blocks of up to 256 elements and larger blocks are separate kernels (LARGE),
// so that each gets its own register allocation and occupancy.
template <typename InT, bool NF4, bool LARGE, typename Choose>
__device__ __forceinline__ void quant_body(const QuantArgs& a, const Choose& choose) {
  if constexpr (!LARGE) quant_small<InT, NF4>(a, choose);
  else if (a.log2_bs == 9) quant_large<InT, NF4, 2>(a, choose);
  else if (a.log2_bs == 10) quant_large<InT, NF4, 4>(a, choose);
  else quant_large<InT, NF4, 0>(a, choose);
}

template <typename InT, bool LARGE>
__global__ void __launch_bounds__(kThreads) quant_nf4_kernel(QuantArgs a) {
  __shared__ NF4Smem sm;
  build_nf4_tables(sm);
  __syncthreads();
  quant_body<InT, true, LARGE>(a, NF4Choose{&sm, a.two});
}

template <typename InT, bool LARGE>
__global__ void __launch_bounds__(kThreads) quant_8bit_kernel(QuantArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Q8Smem& sm = *reinterpret_cast<Q8Smem*>(smem_raw);
  build_q8_tables(sm, a.code);
  if (sm.mode > 0 && !sm.map.ex) quant_body<InT, false, LARGE>(a, Q8Choose<0>{&sm, sm.map});
  else if (sm.mode > 0) quant_body<InT, false, LARGE>(a, Q8Choose<1>{&sm, sm.map});
  else quant_body<InT, false, LARGE>(a, Q8Choose<-1>{&sm, Q8Map{}});
}

template <typename Kern>
int launch_grid(Kern kern, size_t smem, int64_t work_warps, const QuantArgs& a, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if (smem > 48 * 1024)
    if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  int per_sm = 0;
  if (int st = kernel_occupancy(reinterpret_cast<const void*>(kern), kThreads, smem, &per_sm)) return st;
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
  a->x = x; a->n = n; a->nb = (n + bs - 1) / bs; a->q = q; a->absmax = absmax; a->two = 2u;
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

// --------------------------------------------- NF4 + double quantization, one launch
// quant_nf4_dq_kernel: the three steps of quantize(..., double_quant=True)
// (array.py:199-202) in one cooperative launch (every CTA resident). The grid
// is split: the first CTAs quantize x, the last a8.ctas CTAs -- as many as the
// nested pass fills -- build that pass's code tables meanwhile.
//   1. NF4 codes and float32 absmax of x, exactly as quant_nf4_kernel, by the
//      first CTAs, which then arrive on barrier 1.
//   2. The float64 mean of absmax in mean_kernel's summation order: CTAs
//      0 .. 31 wait for barrier 1; thread s of them forms mean_kernel's slot
//      sum s (elements s + j*8192 in order of j, 16 loads in flight) into the
//      workspace and arrives on barrier 2; CTA c < 8 waits for it, adds the
//      1024 slots of its c in mean_kernel's tree, stores the sum and arrives on
//      barrier 3.
//   3. The nested CTAs wait for barrier 3, add the 8 sums in order, so that
//      each holds offset = fl32(sum / nb), bitwise bnbq_absmax_mean's value,
//      and quantize absmax - offset with code2 in blocks of blocksize2,
//      exactly as quant_8bit_kernel with that offset.
// The barriers count arrivals on three workspace words that the host zeroes on
// the stream before the launch; only the CTAs that need a barrier wait on it,
// each wait bounded in time (an expiry is counted in the wait-timeout counter
// and the CTA stops: the outputs are then wrong).
struct DqWork {
  unsigned int arrived[3];  // CTAs that reached barrier 1, 2, 3
  unsigned int pad;
  double sums[kMeanCtas];
  double slots[kMeanCtas * 1024];
};

__device__ __forceinline__ void grid_arrive(unsigned int* arrived) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this CTA's outputs before its arrival
    atomicAdd(arrived, 1u);
  }
}

__device__ __forceinline__ bool grid_wait(const unsigned int* arrived, unsigned int target, int* s_fail) {
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    const uint64_t limit = g_bnbq_wait_limit_ns;
    unsigned int v;
    while (true) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(arrived) : "memory");
      if (v >= target) break;
      if (global_ns() - t0 > limit) {
        atomicAdd(&g_bnbq_wait_timeouts, 1u);
        *s_fail = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return *s_fail == 0;
}

template <typename InT, bool LARGE>
__global__ void __launch_bounds__(kThreads) quant_nf4_dq_kernel(QuantArgs a4, QuantArgs a8, DqWork* work) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Q8Smem& s8 = *reinterpret_cast<Q8Smem*>(smem_raw);
  __shared__ NF4Smem s4;
  __shared__ double part[1024];
  __shared__ int s_fail;
  if (threadIdx.x == 0) s_fail = 0;
  if (int(blockIdx.x) < a8.cta0) {  // ------------------------- 1. NF4 (and 2. the mean)
    build_nf4_tables(s4);
    __syncthreads();
    quant_body<InT, true, LARGE>(a4, NF4Choose{&s4, a4.two});
    grid_arrive(&work->arrived[0]);
    constexpr int64_t kSlots = int64_t(kMeanCtas) * 1024;
    constexpr int kSlotCtas = int(kSlots / kThreads);  // one slot per thread
    if (int(blockIdx.x) >= kSlotCtas) return;
    if (!grid_wait(&work->arrived[0], unsigned(a8.cta0), &s_fail)) return;
    {  // slot s sums elements s + j*8192 in order of j, 16 loads in flight
      const int64_t nb = a8.n;
      const float* am = static_cast<const float*>(a8.x);
      const int64_t slot = int64_t(blockIdx.x) * kThreads + threadIdx.x;
      double sum = 0.0;
      for (int64_t j0 = 0; slot + j0 * kSlots < nb; j0 += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int64_t i = slot + (j0 + u) * kSlots;
          v[u] = i < nb ? __ldcg(am + i) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u)
          if (slot + (j0 + u) * kSlots < nb) sum += double(v[u]);
      }
      __stcg(&work->slots[slot], sum);
    }
    grid_arrive(&work->arrived[1]);
    if (blockIdx.x >= kMeanCtas) return;
    if (!grid_wait(&work->arrived[1], unsigned(kSlotCtas), &s_fail)) return;
    const int c = int(blockIdx.x);
    for (int t = threadIdx.x; t < 1024; t += kThreads) part[t] = __ldcg(&work->slots[c * 1024 + t]);
    __syncthreads();
    for (int w = 512; w > 0; w >>= 1) {
      for (int t = threadIdx.x; t < w; t += kThreads) part[t] += part[t + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) __stcg(&work->sums[c], part[0]);
    grid_arrive(&work->arrived[2]);
    return;
  }
  // ------------------------------------------------------------------ 3. nested
  build_q8_tables(s8, a8.code);  // (ends with a CTA barrier)
  if (!grid_wait(&work->arrived[2], kMeanCtas, &s_fail)) return;
  double total = 0.0;
  for (int c = 0; c < kMeanCtas; ++c) total += __ldcg(&work->sums[c]);
  const float off = float(total / double(a8.n));
  if (int(blockIdx.x) == a8.cta0 && threadIdx.x == 0) *const_cast<float*>(a8.offset) = off;
  QuantArgs b = a8;
  b.offset_in_arg = 1;
  b.offset_value = off;
  if (s8.mode > 0 && !s8.map.ex) quant_body<float, false, false>(b, Q8Choose<0>{&s8, s8.map});
  else if (s8.mode > 0) quant_body<float, false, false>(b, Q8Choose<1>{&s8, s8.map});
  else quant_body<float, false, false>(b, Q8Choose<-1>{&s8, Q8Map{}});
}

template <typename InT, bool LARGE>
int launch_dq(const QuantArgs& a4, const QuantArgs& a8, DqWork* work, cudaStream_t s) {
  auto kern = quant_nf4_dq_kernel<InT, LARGE>;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  const size_t smem = sizeof(Q8Smem);
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  int per_sm = 0;
  if (int st = kernel_occupancy(reinterpret_cast<const void*>(kern), kThreads, smem, &per_sm)) return st;
  if (per_sm < 1) return BNBQ_ERR_UNSUPPORTED;
  int64_t grid = int64_t(di.sm_count) * per_sm;  // every CTA resident (cooperative launch)
  const int64_t want = (work_warps(a4) + kWarps - 1) / kWarps;
  if (want < grid) grid = want;
  if (grid < 64) grid = 64;  // 32 CTAs for the mean's slots, and the nested pass
  if (grid > int64_t(di.sm_count) * per_sm) return BNBQ_ERR_UNSUPPORTED;
  // the nested pass (1/64 of the NF4 pass's elements for blocksize 64) on the
  // last CTAs of the grid: as many as its work fills, at most 1/16 of the grid
  // (measured: the NF4 pass slows in proportion to the CTAs it loses); the
  // NF4 pass, and the mean, on the others
  static_assert(1024 % kThreads == 0, "whole CTAs per mean slot group");
  const int64_t cap3 = grid / 16 > 8 ? grid / 16 : 8;
  int64_t ctas3 = (work_warps(a8) + kWarps - 1) / kWarps;
  ctas3 = ctas3 < 1 ? 1 : (ctas3 > cap3 ? cap3 : ctas3);
  QuantArgs a = a4, b = a8;
  a.cta0 = 0;
  a.ctas = int(grid - ctas3);
  b.cta0 = int(grid - ctas3);
  b.ctas = int(ctas3);
  if (cudaMemsetAsync(work->arrived, 0, sizeof(work->arrived), s) != cudaSuccess) return BNBQ_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, b, work) != cudaSuccess) return BNBQ_ERR_CUDA;
  return launch_status();
}

}  // namespace

int quant_wait_timeouts(unsigned int* out) { return read_wait_timeouts(out); }
int quant_set_wait_limit(uint64_t ns) { return write_wait_limit(ns); }
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
    case BNBQ_F32:
      return a.log2_bs > 8 ? launch_grid(quant_nf4_kernel<float, true>, 0, ww, a, s)
                           : launch_grid(quant_nf4_kernel<float, false>, 0, ww, a, s);
    case BNBQ_F16:
      return a.log2_bs > 8 ? launch_grid(quant_nf4_kernel<__half, true>, 0, ww, a, s)
                           : launch_grid(quant_nf4_kernel<__half, false>, 0, ww, a, s);
    default:
      return a.log2_bs > 8 ? launch_grid(quant_nf4_kernel<__nv_bfloat16, true>, 0, ww, a, s)
                           : launch_grid(quant_nf4_kernel<__nv_bfloat16, false>, 0, ww, a, s);
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
    case BNBQ_F32:
      return a.log2_bs > 8 ? launch_grid(quant_8bit_kernel<float, true>, smem, ww, a, s)
                           : launch_grid(quant_8bit_kernel<float, false>, smem, ww, a, s);
    case BNBQ_F16:
      return a.log2_bs > 8 ? launch_grid(quant_8bit_kernel<__half, true>, smem, ww, a, s)
                           : launch_grid(quant_8bit_kernel<__half, false>, smem, ww, a, s);
    default:
      return a.log2_bs > 8 ? launch_grid(quant_8bit_kernel<__nv_bfloat16, true>, smem, ww, a, s)
                           : launch_grid(quant_8bit_kernel<__nv_bfloat16, false>, smem, ww, a, s);
  }
}

extern "C" int bnbq_quantize_nf4_dq(int dtype, const void* x, int64_t n, int32_t blocksize, const float* code2,
                                    int32_t blocksize2, uint8_t* q, float* absmax, uint8_t* absmax_q,
                                    float* absmax2, float* offset, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  QuantArgs a4{};
  if (int st = check_quant(dtype, x, n, blocksize, q, absmax, &a4)) return st;
  if (n == 0 || !code2 || !absmax_q || !absmax2 || !offset || !workspace) return BNBQ_ERR_INVALID;
  if (workspace_bytes < int64_t(sizeof(DqWork))) return BNBQ_ERR_INVALID;
  if (!aligned(code2, 4) || !aligned(absmax2, 4) || !aligned(offset, 4) || !aligned(absmax_q, 16) ||
      !aligned(workspace, 16))
    return BNBQ_ERR_MISALIGNED;
  QuantArgs a8{};
  if (int st = check_quant(BNBQ_F32, absmax, a4.nb, blocksize2, absmax_q, absmax2, &a8)) return st;
  if (a8.log2_bs > 8) return BNBQ_ERR_UNSUPPORTED;  // the nested pass takes blocks of up to 256
  a8.code = code2;
  a8.offset = offset;
  if (!aligned(absmax, 16)) return BNBQ_ERR_MISALIGNED;  // (the nested pass reads it as 16-byte vectors)
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DqWork* w = static_cast<DqWork*>(workspace);
  switch (dtype) {
    case BNBQ_F32:
      return a4.log2_bs > 8 ? launch_dq<float, true>(a4, a8, w, s) : launch_dq<float, false>(a4, a8, w, s);
    case BNBQ_F16:
      return a4.log2_bs > 8 ? launch_dq<__half, true>(a4, a8, w, s) : launch_dq<__half, false>(a4, a8, w, s);
    default:
      return a4.log2_bs > 8 ? launch_dq<__nv_bfloat16, true>(a4, a8, w, s)
                            : launch_dq<__nv_bfloat16, false>(a4, a8, w, s);
  }
}

extern "C" int64_t bnbq_quantize_nf4_dq_workspace_bytes(void) { return int64_t(sizeof(DqWork)); }

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
