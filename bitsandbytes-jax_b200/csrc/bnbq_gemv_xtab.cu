// bnbq_gemv_xtab.cu -- fused NF4 GEMV for one or two rows of x (the decode
// batch sizes), with x held in a shared-memory table of pair sums.
//
// y[m, r] = sum_k x[m, k] * W[r, k] for an NF4 weight W (n_rows x K), never
// decoded to memory.
//
// Decode. K is cut into groups of GK elements (GK = 256 for one row of x, 128
// for two). For the group a CTA works on, a 128 KB table in shared memory holds
// for every element pair j of the group and every code byte b (high nibble =
// the even element, as the codes are packed) the float32 partial sum
//     P[j][b][m] = fma(T[b & 15], x[m][2j + 1], T[b >> 4] * x[m][2j]).
// One code byte -- two weights -- then costs one table load and one add; the
// weight itself is never formed. A warp takes 32 weight rows of a group (lane
// l = row l). Lane l reads the code words w of its row in a lane-dependent
// order (a different word for every lane at every step), and entry (j, b)
// lives in the bank of j's word w = j >> 2: the 32 lanes' table loads always
// hit 32 distinct banks, whatever the code bytes are. The table is placed at a
// 64 KB-aligned shared address and entry (j, b) sits at byte offset
//     ((j >> 1) & 1) << 16 | b << 8 | (j & 1) << 7 | w << 2   (one row of x)
//     ((j >> 1) & 1) << 16 | b << 8 | (j & 1) << 7 | w << 3   (two rows: float2)
// so one byte permute -- the code byte dropped into bits 8-15 of the word's
// base address -- forms the address of a table load, whose constant part
// ((j & 3) of the pair) is the load's immediate offset. The two halves of a
// warp are served separately by 64-bit loads, and for two rows of x the lanes
// of each half read distinct words.
//
// Scales. The words of a block are summed first; each block's scale a -- the
// float32 absmax, or, double-quantized, fl32(mul.ftz(code2[q2], absmax2[..]) +
// offset) exactly as QuantizedArray.dequantize forms it (array.py:95-108) -- is
// applied once per block and lane: acc = fma.rn.ftz(a, block sum, acc). With a
// one-hot x every table value but one is +0 or -0 and the remaining one is
// T[q] itself, so the result is mul.ftz(T[q], a) rounded once to x's dtype: the
// dequantized weight, bitwise (as kernels/gemv.py:97-123 gives it).
//
// Work. A unit is (group, 32-row block); the units, in group-major order, are
// split evenly over one CTA per SM, so a CTA's units span one group or two (the
// table is rebuilt between them, all consumer warps at a barrier). Each CTA
// processes its units starting from its first row block 0, so that all CTAs
// walk the row blocks together and read whole rows of W at a time. Two
// producer warps, taking turns, stream each unit's 32 x GK/2 code bytes with
// one TMA load into a ring of shared-memory stages placed around the table
// (mbarrier full/empty pairs); the consumer warps take the units round-robin,
// copy a unit's codes
// into registers (releasing the stage at once) and fetch their row's scale
// words one unit ahead. Every unit's 32 (x M) float32 results go to the
// caller's workspace. A second, small kernel (launched right behind, waiting
// for this one with griddepcontrol.wait, so that all partials are visible
// without fences or counters) adds each row's partials in a fixed order,
// rounds once to x's dtype and writes y. Results are deterministic, and the
// workspace needs no initial contents.
//
// Every mbarrier wait is bounded in time; on an expiry the CTA stops working,
// still waits (bounded) for every copy it issued and counts the expiry
// (bnbq_wait_timeouts); y is then wrong.
//
// Programmatic dependent launch: the producers start streaming codes, and
// the consumers load the double-quantization constants, before the previous
// kernel on the stream has finished (the weight is an input that kernel does
// not write); x, the workspace and y are touched only after
// griddepcontrol.wait.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "bnbq_async.cuh"
#include "bnbq_common.cuh"
#include "bnbq_peer.cuh"

namespace bnbq {
namespace {

constexpr uint32_t kTabBytes = 131072;  // the pair table, for either row count
constexpr uint32_t kTabAlign = 65536;   // its shared address has zero bits 8-15
constexpr int kRows = 32;               // weight rows per unit (one per lane)
constexpr int kMaxStages = 56;
constexpr int kProducers = 2;  // producer warps per CTA (TMA issue is per-thread latency-bound)
constexpr int kMaxDevices = 64;
constexpr uint32_t kPairTableBytesT = 256 * 32 * 8;  // the backward's byte -> (T[hi], T[lo]) table, one copy per lane

// Which GEMV a call with a workspace gets: 0 automatic -- the table GEMV when
// the weight has at least 1.5 output rows per element of K (wide weights:
// there it measured faster; the streaming row kernels win on long rows) --,
// 1 the table GEMV whenever it applies, 2 never.
std::atomic<int> g_table_policy{0};


constexpr int gcd(int a, int b) { return b == 0 ? a : gcd(b, a % b); }
constexpr int lcm(int a, int b) { return a / gcd(a, b) * b; }

template <int M>
struct Cfg {
  // consumer warps; the ring is a whole number of rounds of them, so a slot is
  // always taken by the same consumer warp and filled by the same producer
  static constexpr int kConsumers = M == 1 ? 11 : 14;
  static constexpr int kRound = lcm(kConsumers, kProducers);
  static constexpr int kGroupK = M == 1 ? 256 : 128;          // elements of K per table
  static constexpr int kWords = kGroupK / 8;                   // 32-bit code words per row and group
  static constexpr uint32_t kStageBytes = kRows * kWords * 4;  // 4 KB / 2 KB of codes per unit
};

struct XtabArgs {
  const void* x;
  const float* absmax;      // plain scales (absmax_q == nullptr)
  const uint8_t* absmax_q;  // double-quantized scales
  const float* absmax2;
  const float* code2;
  const float* offset;
  void* y;
  float* partial;      // [row_blocks][groups][M][32]
  int64_t n_rows, ldy, block0, units;
  int k, log2_bs, log2_bs2, groups, row_blocks;
  uint32_t dyn_bytes;  // dynamic shared memory of the launch
};

// Shared-memory loads by 32-bit shared-window address. The code-word load
// carries a memory clobber so that it stays after the wait for its stage.
__device__ __forceinline__ uint32_t lds_code(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
template <int OFF>
__device__ __forceinline__ float lds_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(a), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ float2 lds_f32x2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2+%3];" : "=f"(v.x), "=f"(v.y) : "r"(a), "n"(OFF));
  return v;
}
__device__ __forceinline__ void sts_f32(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void sts_f32x2(uint32_t a, float v0, float v1) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v0), "f"(v1) : "memory");
}

__device__ __forceinline__ float fma_ftz(float a, float b, float c) {
  float r;
  asm("fma.rn.ftz.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {  // two add.rn.f32 in one instruction
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pr;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "add.rn.f32x2 pr, pa, pb;\n\tmov.b64 {%0, %1}, pr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
// Read-only global loads kept where they are written (issued a unit ahead of use).
__device__ __forceinline__ uint32_t ldg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void ldg_u32x2(const void* p, uint32_t& a, uint32_t& b) {
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "l"(p));
}
__device__ __forceinline__ uint32_t ldg_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_u8(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return v & 0xffu;
}
__device__ __forceinline__ float ldg_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldcg4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

template <typename XT>
__device__ __forceinline__ void store_y(void* y, int64_t i, float v) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(y)[i] = __float2half_rn(v);
}

// 8 consecutive elements of x as float32 (one 16-byte load).
template <typename XT>
__device__ __forceinline__ void load_x8(float (&v)[8], const XT* p) {
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f;
    if constexpr (Elem<XT>::kDtype == BNBQ_BF16) f = unpack2_bf16(u[i]);
    else f = unpack2_f16(u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// x's elements of group g that this thread's table entries need: pairs
// 4 jq .. 4 jq + 3, for every row of x.
template <typename XT, int M>
__device__ __forceinline__ void load_group_x(float (&xs)[M][8], const XtabArgs& a, int g, int lane) {
  const int jq = M == 1 ? lane : (lane & 15);
  const XT* x = static_cast<const XT*>(a.x);
#pragma unroll
  for (int m = 0; m < M; ++m) load_x8<XT>(xs[m], x + int64_t(m) * a.k + int64_t(g) * Cfg<M>::kGroupK + 8 * jq);
}

// Byte offset of entry (pair j, code byte b) in the table.
template <int M>
__device__ __forceinline__ uint32_t entry_offset(int j, int b) {
  return (uint32_t((j >> 1) & 1) << 16) | (uint32_t(b) << 8) | (uint32_t(j & 1) << 7) | (uint32_t(j >> 2) << (M == 1 ? 2 : 3));
}

// The pair table from this thread's x values, written by the consumer warps
// (warp cw of ncw). A thread owns the pairs j with j >> 2 == jq (its bank);
// the (j & 3, high nibble) combinations are spread over the warps (and, for
// two rows, the half-warps); each writes the 16 entries of its low nibbles.
template <int M>
__device__ __forceinline__ void build_table(uint32_t tab, const float (&xs)[M][8], int cw, int ncw, int lane) {
  const int jq = M == 1 ? lane : (lane & 15);
  const int slot = M == 1 ? cw : 2 * cw + (lane >> 4);
  const int nslots = M == 1 ? ncw : 2 * ncw;
  const float t_lane = kNF4Table[lane & 15];
#pragma unroll
  for (int jl = 0; jl < 4; ++jl) {
    for (int hi = ((slot - 16 * jl) % nslots + nslots) % nslots; hi < 16; hi += nslots) {
      // (one row of x: hi is the same across the warp; two rows: the halves may differ)
      const float thi = M == 1 ? __shfl_sync(0xffffffffu, t_lane, hi) : kNF4Table[hi];
      float u[M];
#pragma unroll
      for (int m = 0; m < M; ++m) u[m] = __fmul_rn(thi, xs[m][2 * jl]);
      const uint32_t base = tab + entry_offset<M>(4 * jq + jl, hi * 16);
#pragma unroll
      for (int lo = 0; lo < 16; ++lo) {
        const float t = kNF4Table[lo];
        if constexpr (M == 1) sts_f32(base + (lo << 8), __fmaf_rn(t, xs[0][2 * jl + 1], u[0]));
        else sts_f32x2(base + (lo << 8), __fmaf_rn(t, xs[0][2 * jl + 1], u[0]), __fmaf_rn(t, xs[1][2 * jl + 1], u[1]));
      }
    }
  }
}

// The scale words of one unit for this lane's row: the NB double-quantized
// codes (one aligned load) and the one or two absmax2 values they use, or NB
// plain float32 scales.
template <int NB, bool NESTED>
struct ScaleWords {
  uint32_t q[NESTED ? (NB + 3) / 4 : 1];
  float v[NESTED ? 2 : NB];
  int64_t gb0;
  bool valid;
};

template <int M, int NB, bool NESTED, int GK = Cfg<M>::kGroupK>
__device__ __forceinline__ void fetch_scales(ScaleWords<NB, NESTED>& s, const XtabArgs& a, int g, int rb, int lane) {
  const int64_t row = int64_t(rb) * kRows + lane;
  s.valid = row < a.n_rows;
  if (!s.valid) return;
  const int64_t bpr = int64_t(a.k) >> a.log2_bs;  // blocks per row
  s.gb0 = row * bpr + ((int64_t(g) * GK) >> a.log2_bs);
  if constexpr (NESTED) {
    if constexpr (NB == 8) {
      ldg_u32x2(a.absmax_q + s.gb0, s.q[0], s.q[1]);
    } else if constexpr (NB == 4) {
      s.q[0] = ldg_u32(a.absmax_q + s.gb0);
    } else if constexpr (NB == 2) {
      s.q[0] = ldg_u16(a.absmax_q + s.gb0);
    } else {
      s.q[0] = ldg_u8(a.absmax_q + s.gb0);
    }
    const int64_t i0 = (a.block0 + s.gb0) >> a.log2_bs2;
    const int64_t i1 = (a.block0 + s.gb0 + NB - 1) >> a.log2_bs2;
    s.v[0] = ldg_f32(a.absmax2 + i0);
    s.v[1] = ldg_f32(a.absmax2 + i1);
  } else {
#pragma unroll
    for (int b = 0; b < NB; ++b) s.v[b] = ldg_f32(a.absmax + s.gb0 + b);
  }
}

// a_rot[p] = the scale of the block this lane visits in phase p, block (p + al) mod NB.
template <int NB, bool NESTED>
__device__ __forceinline__ void decode_scales(float (&a_rot)[NB], const ScaleWords<NB, NESTED>& s, const XtabArgs& a,
                                              const float* s_code2, float offset, int al) {
#pragma unroll
  for (int p = 0; p < NB; ++p) {
    const int blk = (p + al) & (NB - 1);
    if (!s.valid) {
      a_rot[p] = 0.0f;
      continue;
    }
    if constexpr (NESTED) {
      uint32_t word = s.q[0];
      if constexpr (NB == 8) word = blk < 4 ? s.q[0] : s.q[(NB + 3) / 4 - 1];
      const uint32_t q2 = (word >> (8 * (blk & 3))) & 0xffu;
      const int64_t i0 = (a.block0 + s.gb0) >> a.log2_bs2;
      const float a2 = ((a.block0 + s.gb0 + blk) >> a.log2_bs2) != i0 ? s.v[1] : s.v[0];
      a_rot[p] = add_rn(mul_ftz(s_code2[q2], a2), offset);
    } else {
      float v = s.v[0];
#pragma unroll
      for (int b = 1; b < NB; ++b)
        if (blk == b) v = s.v[b];
      a_rot[p] = v;
    }
  }
}

// Walk order of a lane's code words within a unit: phase p covers block
// (p + al) mod NB, and within it the lane starts at word (orot mod WB). Word
// (p, s) is wbase(p) + o(s) with wbase(p) = ((p + al) mod NB) * WB and
// o(s) = (s + orot) mod WB.
template <int M, int NB>
struct Walk {
  static constexpr int GW = Cfg<M>::kWords;
  static constexpr int WB = GW / NB;
  int al, orot;
  __device__ __forceinline__ explicit Walk(int lane) {
    const int li = M == 1 ? lane : (lane & 15);
    al = li / WB;
    orot = M == 1 ? lane : li + (lane >> 4);
  }
  __device__ __forceinline__ int wbase(int p) const { return ((p + al) & (NB - 1)) * WB; }
  __device__ __forceinline__ int o(int s) const { return (s + orot) & (WB - 1); }
};

// The unit's code words of this lane's row, from its stage into registers in
// walk order (conflict-free: the lanes' words differ at every step).
template <int M, int NB>
__device__ __forceinline__ void load_codes(uint32_t (&cw)[NB][Walk<M, NB>::WB], uint32_t row_codes,
                                           const uint32_t (&cb)[NB], const uint32_t (&co)[Walk<M, NB>::WB]) {
#pragma unroll
  for (int p = 0; p < NB; ++p)
#pragma unroll
    for (int s = 0; s < Walk<M, NB>::WB; ++s) cw[p][s] = lds_code(row_codes + cb[p] + co[s]);
}

// The unit's dot products for this lane's row, from its code words. Word
// (p, s)'s table entries are at prmt(code byte i into bits 8-15 of
// tp[p] + to[s]) + the pair's constant offset. Per block, the words' values
// are summed pairwise into a two-lane accumulator in walk order, then scaled
// once: acc = fma.ftz(a, sum, acc). All table loads of a batch of words are
// issued before their adds.
template <int M, int NB>
__device__ __forceinline__ void unit_dot(const uint32_t (&cw)[NB][Walk<M, NB>::WB], const uint32_t (&tp)[NB],
                                         const uint32_t (&to)[Walk<M, NB>::WB], const float (&a_rot)[NB],
                                         float (&acc)[M]) {
  constexpr int WB = Walk<M, NB>::WB;
  constexpr int kBatch = WB < 8 ? WB : 8;
  // pairs j & 3 = 1, 2, 3: entry offsets 128, 64 K, 64 K + 128 from pair 0's; the 64 K is
  // added to the base (a second base register) rather than to the load
  constexpr int kOff1 = 1 << 7, kOff3 = 1 << 7;
#pragma unroll
  for (int p = 0; p < NB; ++p) {
    float2 ps[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ps[m] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int s0 = 0; s0 < WB; s0 += kBatch) {
      if constexpr (M == 1) {
        float v[kBatch][4];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const uint32_t c = cw[p][s0 + j];
          const uint32_t tw = tp[p] + to[s0 + j], tw2 = tw + (1u << 16);
          v[j][0] = lds_f32<0>(__byte_perm(c, tw, 0x7604));
          v[j][1] = lds_f32<kOff1>(__byte_perm(c, tw, 0x7614));
          v[j][2] = lds_f32<0>(__byte_perm(c, tw2, 0x7624));
          v[j][3] = lds_f32<kOff3>(__byte_perm(c, tw2, 0x7634));
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          ps[0] = add2(ps[0], add2(make_float2(v[j][0], v[j][2]), make_float2(v[j][1], v[j][3])));
      } else {
        float2 v[kBatch][4];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const uint32_t c = cw[p][s0 + j];
          const uint32_t tw = tp[p] + to[s0 + j], tw2 = tw + (1u << 16);
          v[j][0] = lds_f32x2<0>(__byte_perm(c, tw, 0x7604));
          v[j][1] = lds_f32x2<kOff1>(__byte_perm(c, tw, 0x7614));
          v[j][2] = lds_f32x2<0>(__byte_perm(c, tw2, 0x7624));
          v[j][3] = lds_f32x2<kOff3>(__byte_perm(c, tw2, 0x7634));
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const float2 h01 = add2(v[j][0], v[j][1]), h23 = add2(v[j][2], v[j][3]);
          ps[0] = add2(ps[0], make_float2(h01.x, h23.x));
          ps[1] = add2(ps[1], make_float2(h01.y, h23.y));
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = fma_ftz(a_rot[p], ps[m].x + ps[m].y, acc[m]);
  }
}

// The reduction of the split-K partials: y[m, r] = round(sum over groups, in
// order, of partial[rb][g][m][r % 32]). A CTA of kRedThreads threads takes one
// row block and one row of x: thread t adds the groups g = t / 32, t / 32 + 8,
// ... of row t % 32, and the eight warps' sums are added in warp order.
// Exchange mode (px.inbox != nullptr; the host has checked that every CTA can
// be resident at once): the rows are also stored into the peers' inboxes,
// then every thread polls its share of the other ranks' columns into
// px.y_full and the CTA reports that it has finished the call.
constexpr int kRedThreads = 256;

template <typename XT, int M>
__global__ void __launch_bounds__(kRedThreads) gemv_xtab_reduce_kernel(const float* partial, int groups,
                                                                       int row_blocks, int64_t n_rows, void* y,
                                                                       int64_t ldy, PeerOut px) {
  __shared__ float s_sum[kRedThreads / 32][kRows];
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // every partial of the GEMV kernel is visible
  const int rb = int(blockIdx.x) / M, m = int(blockIdx.x) % M;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float* p = partial + (int64_t(rb) * groups * M + m) * kRows + lane;
  constexpr int kBatch = 8;
  float sum = 0.0f;
  for (int g0 = w; g0 < groups; g0 += 8 * kBatch) {
    float v[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int g = g0 + 8 * b;
      v[b] = g < groups ? __ldcg(p + int64_t(g) * M * kRows) : 0.0f;
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) sum += v[b];
  }
  s_sum[w][lane] = sum;
  __syncthreads();
  const bool exchange = px.inbox != nullptr;
  const uint32_t epoch = exchange ? peer_epoch(px) : 0u;  // after griddepcontrol.wait
  if (w == 0) {
    float t = s_sum[0][lane];
#pragma unroll
    for (int i = 1; i < kRedThreads / 32; ++i) t += s_sum[i][lane];
    const int64_t r = int64_t(rb) * kRows + lane;
    if (r < n_rows) {
      store_y<XT>(y, int64_t(m) * ldy + r, t);
      if (exchange) {
        if constexpr (Elem<XT>::kDtype == BNBQ_BF16) peer_send(px, epoch, m, r, __bfloat16_as_ushort(__float2bfloat16_rn(t)));
        else peer_send(px, epoch, m, r, __half_as_ushort(__float2half_rn(t)));
      }
    }
  }
  if (!exchange) return;
  const bool ok = peer_receive(px, epoch, M, n_rows, int64_t(blockIdx.x) * kRedThreads + threadIdx.x,
                               int64_t(gridDim.x) * kRedThreads);
  const int expired = __syncthreads_or(!ok);
  if (threadIdx.x == 0) peer_finish_cta(px, epoch, expired != 0);
}

// A CTA's units [u0, u1) (group-major numbering) in processing order: from
// the first unit that starts a group (row block 0), to the end, then the
// units before it. Every CTA then walks the row blocks in about the same
// order at the same time, so the code slabs that all CTAs read at a given
// moment are the same whole rows of W: contiguous memory, not 128-byte
// pieces strided by a row.
struct Order {
  uint32_t u0, u1, us, n1, rbs;
  __device__ __forceinline__ Order(int64_t a, int64_t b, int row_blocks) {
    u0 = uint32_t(a);
    u1 = uint32_t(b);
    rbs = uint32_t(row_blocks);
    const uint32_t up = (u0 + rbs - 1) / rbs * rbs;  // first group start at or after u0
    us = up < u1 ? up : u0;
    n1 = u1 - us;
  }
  __device__ __forceinline__ uint32_t unit(uint32_t p) const { return p < n1 ? us + p : u0 + (p - n1); }
  __device__ __forceinline__ void at(uint32_t p, int& g, int& rb) const {
    const uint32_t u = unit(p);
    g = int(u / rbs);
    rb = int(u - uint32_t(g) * rbs);
  }
  // (g, rb) of position p + step from (g, rb) of position p (p + step < n)
  __device__ __forceinline__ void advance(uint32_t p, uint32_t step, int& g, int& rb) const {
    if (p < n1 && p + step >= n1) {  // wraps to the units before us
      at(p + step, g, rb);
      return;
    }
    rb += int(step);
    while (rb >= int(rbs)) {
      rb -= int(rbs);
      ++g;
    }
  }
  // end (exclusive) of the run of positions from p that share p's group
  __device__ __forceinline__ uint32_t seg_end(uint32_t p) const {
    const uint32_t u = unit(p);
    const uint32_t gend = (u / rbs + 1) * rbs;
    return p < n1 ? min(u1, gend) - us : n1 + (min(us, gend) - u0);
  }
};

template <typename XT, int M, int NB, bool NESTED>
__global__ void __launch_bounds__((Cfg<M>::kConsumers + kProducers) * 32, 1)
    gemv_xtab_kernel(const __grid_constant__ CUtensorMap tmap, const XtabArgs a) {
  constexpr uint32_t kStage = Cfg<M>::kStageBytes;
  constexpr int GW = Cfg<M>::kWords;
  constexpr int WB = Walk<M, NB>::WB;
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ float s_code2[256];
  __shared__ __align__(8) uint64_t s_bar[2 * kMaxStages];
  __shared__ volatile int s_abort;
  __shared__ volatile int s_next[kProducers];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = int(blockDim.x >> 5) - kProducers;  // consumer warps; the last kProducers warps produce
  const int64_t u0 = int64_t(blockIdx.x) * a.units / gridDim.x;
  const int64_t u1 = int64_t(blockIdx.x + 1) * a.units / gridDim.x;
  const int n_units = int(u1 - u0);
  const Order ord(u0, u1, a.row_blocks);
  // Shared layout: stages below the table (from the dynamic base up to the
  // 64 KB-aligned table), the table, stages above it.
  const uint32_t dyn0 = smem_u32(smem);
  const uint32_t tab = (dyn0 + kTabAlign - 1) & ~(kTabAlign - 1);
  const int s_lo = int((tab - dyn0) / kStage);
  int S = s_lo + int((dyn0 + a.dyn_bytes - (tab + kTabBytes)) / kStage);
  if (S > kMaxStages) S = kMaxStages;
  S -= S % Cfg<M>::kRound;
  const uint32_t stage_hi = tab + kTabBytes;
  const uint32_t full0 = smem_u32(s_bar), empty0 = full0 + 8u * kMaxStages;

  if (threadIdx.x == 0) {
    s_abort = S < Cfg<M>::kRound || dyn0 + a.dyn_bytes < tab + kTabBytes;  // (the host sizes the launch for this)
    for (int q = 0; q < kProducers; ++q) s_next[q] = -1;  // set by producer q when it stops
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8u * s, 1);   // the producer's arrival (plus the copy's bytes)
      mbar_init(empty0 + 8u * s, 1);  // the one consumer warp that took the unit
    }
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");
  if (s_abort) {  // a layout this kernel cannot use: count it like an expired wait, write nothing
    if (threadIdx.x == 0) atomicAdd(&g_bnbq_wait_timeouts, 1u);
    return;
  }
  auto stage_addr = [&](int slot) -> uint32_t {
    return slot < s_lo ? dyn0 + uint32_t(slot) * kStage : stage_hi + uint32_t(slot - s_lo) * kStage;
  };

  if (warp >= ncw) {  // ----------------------------------------------- producers
    // producer q issues positions q, q + P, ...: the slots q, q + P, ... and
    // every use of them (S is a multiple of P), in order, each after the
    // slot's previous use has been taken (its empty barrier)
    const int q = warp - ncw;
    if (lane == 0 && q < n_units) {
      if (q == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
      int i = q, slot = q % S, g, rb;
      uint32_t use = uint32_t(q / S);
      ord.at(uint32_t(q), g, rb);
      bool ok = true;
      int unissued = 0x7fffffff;  // first position of this producer not issued
      while (true) {
        if (use > 0) ok = mbar_wait(empty0 + 8u * slot, (use - 1u) & 1u);
        if (!ok || s_abort) {
          unissued = i;
          break;
        }
        const uint32_t full = full0 + 8u * slot;
        mbar_arrive_expect_tx(full, kStage);
        tma_load_2d(stage_addr(slot), &tmap, g * (GW * 4), rb * kRows, full);
        if (i + kProducers >= n_units) break;
        ord.advance(uint32_t(i), kProducers, g, rb);
        i += kProducers;
        slot += kProducers;
        if (slot >= S) {
          slot -= S;
          ++use;
        }
      }
      if (!ok) {
        __threadfence_block();
        s_abort = 1;
      }
      s_next[q] = unissued;
    } else if (lane == 0) {
      s_next[q] = 0x7fffffff;
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int ncons = ncw * 32;
  float offset = 0.0f;
  if constexpr (NESTED) {  // constants of the weight: before waiting for the previous kernel
    for (int i = threadIdx.x; i < 256; i += ncons) s_code2[i] = a.code2[i];
    offset = *a.offset;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x and the workspace: after the previous kernel
  const Walk<M, NB> wk(lane);
  // word (p, s): code at row_codes + cb[p] + co[s]; table base tp[p] + to[s]
  uint32_t cb[NB], co[WB], tp[NB], to[WB];
#pragma unroll
  for (int p = 0; p < NB; ++p) {
    cb[p] = uint32_t(wk.wbase(p)) * 4u;
    tp[p] = tab + uint32_t(wk.wbase(p)) * (4u * M);
  }
#pragma unroll
  for (int s = 0; s < WB; ++s) {
    co[s] = uint32_t(wk.o(s)) * 4u;
    to[s] = uint32_t(wk.o(s)) * (4u * M);
  }
  const uint32_t lane_row = uint32_t(lane) * (GW * 4);

  // this warp's positions: i = warp, warp + ncw, ...
  int g = 0, rb = 0;
  ScaleWords<NB, NESTED> sw;
  if (warp < n_units) {
    ord.at(uint32_t(warp), g, rb);
    fetch_scales<M, NB, NESTED>(sw, a, g, rb, lane);
  }
  float xs[M][8];
  {
    int g0, rb0;
    ord.at(0u, g0, rb0);
    load_group_x<XT, M>(xs, a, g0, lane);
  }
  int i = warp;
  int slot = warp % S;
  uint32_t parity = uint32_t((warp / S) & 1);
  uint32_t seg = 0;
  while (seg < uint32_t(n_units)) {
    const uint32_t seg_end = ord.seg_end(seg);
    named_bar_sync(1, ncons);  // the previous group's table is no longer read
    build_table<M>(tab, xs, warp, ncw, lane);
    if (seg_end < uint32_t(n_units)) {  // the next group's x, in flight during this segment
      int gx, rbx;
      ord.at(seg_end, gx, rbx);
      load_group_x<XT, M>(xs, a, gx, lane);
    }
    named_bar_sync(1, ncons);  // the table (and code2) are complete
    for (; i < int(seg_end); i += ncw) {
      bool ok;
      if (s_abort) {  // drain: wait (bounded) only for copies that were issued
        ok = false;
        const int q = i % kProducers;
        const uint64_t t0 = global_ns();
        while (s_next[q] < 0 && global_ns() - t0 < g_bnbq_wait_limit_ns) {
        }
        if (i < s_next[q]) mbar_wait(full0 + 8u * slot, parity);
      } else {
        // this warp took the slot's previous use itself (S is a multiple of
        // ncw), so the parity wait can only see this use's data
        ok = mbar_wait(full0 + 8u * slot, parity);
        ok = __shfl_sync(0xffffffffu, ok, 0);  // one decision for the warp
        if (!ok) s_abort = 1;
      }
      uint32_t cw[NB][WB];
      if (ok) load_codes<M, NB>(cw, stage_addr(slot) + lane_row, cb, co);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8u * slot);  // the stage is free again
      slot += ncw;  // this warp's next position (ncw < S: at most one wrap)
      if (slot >= S) {
        slot -= S;
        parity ^= 1u;
      }
      float a_rot[NB];
      decode_scales<NB, NESTED>(a_rot, sw, a, s_code2, offset, wk.al);
      const int gc = g, rbc = rb;
      if (i + ncw < n_units) {
        ord.advance(uint32_t(i), uint32_t(ncw), g, rb);
        fetch_scales<M, NB, NESTED>(sw, a, g, rb, lane);
      }
      if (ok) {
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        unit_dot<M, NB>(cw, tp, to, a_rot, acc);
        float* part = a.partial + ((int64_t(rbc) * a.groups + gc) * M) * kRows;
#pragma unroll
        for (int m = 0; m < M; ++m) __stcg(part + m * kRows + lane, acc[m]);
      }
    }
    seg = seg_end;
  }

}

// ---------------------------------------------------------------------------
// 8-bit codebook weights (quantize_blockwise: one code byte per element, a
// 256-entry float32 codebook): gemv_code8_kernel, for 1 to 4 rows of x.
// The reference has no fused path for them (its router sends them to
// x @ dequantize(w).T, _matmul.py:74-79); the numerics here are those of the
// NF4 GEMV: float32 products of x with the exact codebook value, block sums,
// the block's scale applied once (acc = fma.rn.ftz(a, block sum, 0), a being
// the float32 absmax or the double-quantized one decoded as
// QuantizedArray.dequantize does), the blocks, then the groups, added in a
// fixed order, one rounding to x's dtype. A one-hot x gives
// mul.ftz(code[q], a) rounded once: the dequantized weight, bitwise.
// Layout: units of (128 elements of K, 32 rows), streamed by the same
// producers as the NF4 kernels (the unit is again 32 rows x 128 bytes); lane l
// owns code word l -- elements 4l .. 4l + 3 -- of every row of its unit, with
// x's 4 matching elements in registers. The codebook sits in shared memory
// once per lane, entry (code c, lane l) at c << 8 | l << 2 of a 64 KB-aligned
// table, so one byte permute forms each load's address and the 32 lanes'
// loads always hit 32 distinct banks, whatever the codes are.
// Row sums without selects: at slot s lane l takes row s ^ l of the unit
// (its code-word loads hit bank l too). At the butterfly level with lane mask
// m the lane adds its partner's slot s + m into its slot s (s & m == 0); both
// hold the same row, because (s + m) ^ (l ^ m) = s ^ l. The levels inside a
// block (m < 32 / NB lanes) run first, each block's sum then gets its scale
// -- lane r decoded the NB scales of row r and hands the one a lane needs to
// it with one shuffle --, and the remaining levels add a row's blocks,
// leaving row l of the unit in lane l.
constexpr int kGroupK8 = 128;         // elements of K per unit
constexpr uint32_t kTab8Bytes = 65536;  // 256 codes x 256-byte rows (32 lanes used)

template <int M>
struct Cfg8 {
  static constexpr int kConsumers = M >= 3 ? 8 : 16;  // (registers: 4 x M values per lane and row)
  static constexpr int kRound = lcm(kConsumers, kProducers);
};

template <typename XT, int M, int NB, bool NESTED>
__global__ void __launch_bounds__((Cfg8<M>::kConsumers + kProducers) * 32, 1)
    gemv_code8_kernel(const __grid_constant__ CUtensorMap tmap, const XtabArgs a, const float* __restrict__ code) {
  constexpr uint32_t kStage = kRows * kGroupK8;  // 4 KB
  constexpr int LPB = 32 / NB;
  static_assert(LPB >= 2, "two or more code words per block");
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ float s_code2[256];
  __shared__ __align__(8) uint64_t s_bar[2 * kMaxStages];
  __shared__ volatile int s_abort;
  __shared__ volatile int s_next[kProducers];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = int(blockDim.x >> 5) - kProducers;
  const int64_t u0 = int64_t(blockIdx.x) * a.units / gridDim.x;
  const int64_t u1 = int64_t(blockIdx.x + 1) * a.units / gridDim.x;
  const int n_units = int(u1 - u0);
  const Order ord(u0, u1, a.row_blocks);
  const uint32_t dyn0 = smem_u32(smem);
  const uint32_t tab = (dyn0 + kTabAlign - 1) & ~(kTabAlign - 1);
  const int s_lo = int((tab - dyn0) / kStage);
  int S = s_lo + int((dyn0 + a.dyn_bytes - (tab + kTab8Bytes)) / kStage);
  if (S > kMaxStages) S = kMaxStages;
  S -= S % Cfg8<M>::kRound;
  const uint32_t stage_hi = tab + kTab8Bytes;
  const uint32_t full0 = smem_u32(s_bar), empty0 = full0 + 8u * kMaxStages;

  if (threadIdx.x == 0) {
    s_abort = S < Cfg8<M>::kRound || dyn0 + a.dyn_bytes < tab + kTab8Bytes;
    for (int q = 0; q < kProducers; ++q) s_next[q] = -1;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");
  if (s_abort) {
    if (threadIdx.x == 0) atomicAdd(&g_bnbq_wait_timeouts, 1u);
    return;
  }
  auto stage_addr = [&](int slot) -> uint32_t {
    return slot < s_lo ? dyn0 + uint32_t(slot) * kStage : stage_hi + uint32_t(slot - s_lo) * kStage;
  };

  if (warp >= ncw) {  // ----------------------------------------------- producers
    const int q = warp - ncw;
    if (lane == 0 && q < n_units) {
      if (q == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
      int i = q, slot = q % S, g, rb;
      uint32_t use = uint32_t(q / S);
      ord.at(uint32_t(q), g, rb);
      bool ok = true;
      int unissued = 0x7fffffff;
      while (true) {
        if (use > 0) ok = mbar_wait(empty0 + 8u * slot, (use - 1u) & 1u);
        if (!ok || s_abort) {
          unissued = i;
          break;
        }
        const uint32_t full = full0 + 8u * slot;
        mbar_arrive_expect_tx(full, kStage);
        tma_load_2d(stage_addr(slot), &tmap, g * kGroupK8, rb * kRows, full);
        if (i + kProducers >= n_units) break;
        ord.advance(uint32_t(i), kProducers, g, rb);
        i += kProducers;
        slot += kProducers;
        if (slot >= S) {
          slot -= S;
          ++use;
        }
      }
      if (!ok) {
        __threadfence_block();
        s_abort = 1;
      }
      s_next[q] = unissued;
    } else if (lane == 0) {
      s_next[q] = 0x7fffffff;
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int ncons = ncw * 32;
  // the codebook, one copy per lane (weight constants: before the wait)
  for (int c = warp; c < 256; c += ncw) sts_f32(tab + (uint32_t(c) << 8) + uint32_t(lane) * 4u, __ldg(code + c));
  float offset = 0.0f;
  if constexpr (NESTED) {
    for (int i = threadIdx.x; i < 256; i += ncons) s_code2[i] = a.code2[i];
    offset = *a.offset;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  named_bar_sync(1, ncons);  // the codebook (and code2) are complete
  const uint32_t base = tab + uint32_t(lane) * 4u;
  const uint32_t word_ofs = uint32_t(lane) * 4u;
  const int qs = lane / LPB;
  const XT* xg = static_cast<const XT*>(a.x);

  int g = 0, rb = 0;
  ScaleWords<NB, NESTED> sw;
  uint2 xw[M];  // x's 4 elements of this lane for the unit, per row of x
  auto fetch_x = [&](int gg) {
#pragma unroll
    for (int m = 0; m < M; ++m)
      xw[m] = __ldg(reinterpret_cast<const uint2*>(xg + int64_t(m) * a.k + int64_t(gg) * kGroupK8 + 4 * lane));
  };
  if (warp < n_units) {
    ord.at(uint32_t(warp), g, rb);
    fetch_scales<M, NB, NESTED, kGroupK8>(sw, a, g, rb, lane);
    fetch_x(g);
  }
  int slot = warp % S;
  uint32_t parity = uint32_t((warp / S) & 1);
  for (int i = warp; i < n_units; i += ncw) {
    bool ok;
    if (s_abort) {
      ok = false;
      const int q = i % kProducers;
      const uint64_t t0 = global_ns();
      while (s_next[q] < 0 && global_ns() - t0 < g_bnbq_wait_limit_ns) {
      }
      if (i < s_next[q]) mbar_wait(full0 + 8u * slot, parity);
    } else {
      ok = mbar_wait(full0 + 8u * slot, parity);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) s_abort = 1;
    }
    uint32_t cw[kRows];
    if (ok) {
      const uint32_t st = stage_addr(slot) + word_ofs;
#pragma unroll
      for (int s = 0; s < kRows; ++s) cw[s] = lds_code(st + (uint32_t(s ^ lane) << 7));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * slot);
    slot += ncw;
    if (slot >= S) {
      slot -= S;
      parity ^= 1u;
    }
    float a_own[NB];
    decode_scales<NB, NESTED>(a_own, sw, a, s_code2, offset, 0);
    float xv[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float2 f0, f1;
      if constexpr (Elem<XT>::kDtype == BNBQ_BF16) {
        f0 = unpack2_bf16(xw[m].x);
        f1 = unpack2_bf16(xw[m].y);
      } else {
        f0 = unpack2_f16(xw[m].x);
        f1 = unpack2_f16(xw[m].y);
      }
      xv[m][0] = f0.x;
      xv[m][1] = f0.y;
      xv[m][2] = f1.x;
      xv[m][3] = f1.y;
    }
    const int gc = g, rbc = rb;
    if (i + ncw < n_units) {
      ord.advance(uint32_t(i), uint32_t(ncw), g, rb);
      fetch_scales<M, NB, NESTED, kGroupK8>(sw, a, g, rb, lane);
      fetch_x(g);
    }
    if (ok) {
      float acc[NB][M];
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        // this lane's 4 elements of row slot LPB t + k, per row of x
        auto row_dot = [&](int k, float (&r)[M]) {
          const uint32_t c = cw[LPB * t + k];
          const float w0 = lds_f32<0>(__byte_perm(c, base, 0x7604));
          const float w1 = lds_f32<0>(__byte_perm(c, base, 0x7614));
          const float w2 = lds_f32<0>(__byte_perm(c, base, 0x7624));
          const float w3 = lds_f32<0>(__byte_perm(c, base, 0x7634));
#pragma unroll
          for (int m = 0; m < M; ++m)
            r[m] = __fmaf_rn(w3, xv[m][3], __fmaf_rn(w2, xv[m][2], __fmaf_rn(w1, xv[m][1], w0 * xv[m][0])));
        };
        // the first level as the slots are made (fewer live values)
        float v[LPB / 2][M];
#pragma unroll
        for (int k = 0; k < LPB / 2; ++k) {
          float hi[M];
          row_dot(k, v[k]);
          row_dot(k + LPB / 2, hi);
#pragma unroll
          for (int m = 0; m < M; ++m) v[k][m] += __shfl_xor_sync(0xffffffffu, hi[m], LPB / 2);
        }
#pragma unroll
        for (int mk = LPB / 4; mk >= 1; mk >>= 1)
#pragma unroll
          for (int k = 0; k < mk; ++k)
#pragma unroll
            for (int m = 0; m < M; ++m) v[k][m] += __shfl_xor_sync(0xffffffffu, v[k + mk][m], mk);
        float give = a_own[0];
#pragma unroll
        for (int p = 1; p < NB; ++p)
          if ((qs ^ t) == p) give = a_own[p];
        const float at = __shfl_xor_sync(0xffffffffu, give, LPB * t);
#pragma unroll
        for (int m = 0; m < M; ++m) acc[t][m] = fma_ftz(at, v[0][m], 0.0f);
      }
#pragma unroll
      for (int mk = NB / 2; mk >= 1; mk >>= 1)
#pragma unroll
        for (int t = 0; t < mk; ++t)
#pragma unroll
          for (int m = 0; m < M; ++m) acc[t][m] += __shfl_xor_sync(0xffffffffu, acc[t + mk][m], LPB * mk);
      float* part = a.partial + ((int64_t(rbc) * a.groups + gc) * M) * kRows + lane;
#pragma unroll
      for (int m = 0; m < M; ++m) __stcg(part + m * kRows, acc[0][m]);
    }
  }
}

// ---------------------------------------------------------------------------
// The backward of the fused matmul for a few rows of g (gemv_t_kernel):
// out[m, k] = sum_n g[m, n] * W[n, k], W NF4 (n_rows x K) never decoded to
// memory; the reference computes g @ w.dequantize(g.dtype) (_matmul.py:67-68).
// Units are the table GEMV's (256 columns x 32 rows, one TMA tile), taken in
// plain unit order (column group major) from the same producers and ring.
// Lane l owns code word l (columns 8l .. 8l + 7) of the group; for each row of
// its unit it reads the row's word (the warp reads the row's 128 contiguous
// bytes), the row's block scale (decoded by the lane that owns the row and
// passed through a per-warp shared array) and g's values of the row, and
// accumulates g * w, w = mul.ftz(T[q], a) exactly (the pair table gives T of
// both nibbles), in float32, over every unit it takes of a column group. A
// warp stores one partial per column group it touched (zeros for a group of
// its CTA it had no unit of); a second kernel adds, per output, the partials
// of the CTAs that covered its group, in CTA, group-segment and warp order,
// and rounds once. A one-hot g returns the dequantized weight row bitwise.
constexpr int kTConsumers = 12;
constexpr int kTRound = lcm(kTConsumers, kProducers);

struct GemvTArgs {
  const void* g;   // M x n_rows, row stride ldg
  float* partial;  // [grid][maxseg][kTConsumers][M][256]
  XtabArgs x;      // the weight's scales, sizes and block numbering, as fetch_scales reads them
  int64_t ldg, units;
  int groups, row_blocks, maxseg;
  uint32_t dyn_bytes;
};

template <typename XT, int M, int NB, bool NESTED>
__global__ void __launch_bounds__((kTConsumers + kProducers) * 32, 1)
    gemv_t_kernel(const __grid_constant__ CUtensorMap tmap, const GemvTArgs a) {
  constexpr uint32_t kStage = kRows * 128;
  constexpr int LPB = 32 / NB;  // lanes per block
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ float s_code2[256];
  __shared__ __align__(8) uint64_t s_bar[2 * kMaxStages];
  __shared__ volatile int s_abort;
  __shared__ volatile int s_next[kProducers];
  __shared__ float s_a[kTConsumers][kRows][NB];
  __shared__ float s_gv[kTConsumers][M][kRows];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncw = kTConsumers;
  const int64_t u0 = int64_t(blockIdx.x) * a.units / gridDim.x;
  const int64_t u1 = int64_t(blockIdx.x + 1) * a.units / gridDim.x;
  const int n_units = int(u1 - u0);
  const int g_first = int(u0 / a.row_blocks);
  float2* s_pair = reinterpret_cast<float2*>(smem);  // [256][32]
  const uint32_t stage0 = smem_u32(smem) + kPairTableBytesT;
  int S = int((a.dyn_bytes - kPairTableBytesT) / kStage);
  if (S > kMaxStages) S = kMaxStages;
  S -= S % kTRound;
  const uint32_t full0 = smem_u32(s_bar), empty0 = full0 + 8u * kMaxStages;
  if (threadIdx.x == 0) {
    s_abort = S < kTRound;
    for (int q = 0; q < kProducers; ++q) s_next[q] = -1;
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;");
  if (s_abort) {
    if (threadIdx.x == 0) atomicAdd(&g_bnbq_wait_timeouts, 1u);
    return;
  }
  if (warp >= ncw) {  // ----------------------------------------------- producers
    const int q = warp - ncw;
    if (lane == 0 && q < n_units) {
      if (q == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap) : "memory");
      int i = q, slot = q % S;
      uint32_t use = uint32_t(q / S);
      bool ok = true;
      int unissued = 0x7fffffff;
      while (true) {
        if (use > 0) ok = mbar_wait(empty0 + 8u * slot, (use - 1u) & 1u);
        if (!ok || s_abort) {
          unissued = i;
          break;
        }
        const int64_t u = u0 + i;
        const int g = int(u / a.row_blocks), rb = int(u % a.row_blocks);
        const uint32_t full = full0 + 8u * slot;
        mbar_arrive_expect_tx(full, kStage);
        tma_load_2d(stage0 + uint32_t(slot) * kStage, &tmap, g * 128, rb * kRows, full);
        if (i + kProducers >= n_units) break;
        i += kProducers;
        slot += kProducers;
        if (slot >= S) {
          slot -= S;
          ++use;
        }
      }
      if (!ok) {
        __threadfence_block();
        s_abort = 1;
      }
      s_next[q] = unissued;
    } else if (lane == 0) {
      s_next[q] = 0x7fffffff;
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int ncons = ncw * 32;
  for (int b = warp; b < 256; b += ncw) s_pair[b * 32 + lane] = make_float2(kNF4Table[b >> 4], kNF4Table[b & 15]);
  float offset = 0.0f;
  if constexpr (NESTED) {
    for (int i = threadIdx.x; i < 256; i += ncons) s_code2[i] = a.x.code2[i];
    offset = *a.x.offset;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // g and the workspace: after the previous kernel
  named_bar_sync(1, ncons);
  const XT* gp = static_cast<const XT*>(a.g);
  const int qs = lane / LPB;
  const int nseg = int((u1 - 1) / a.row_blocks) - g_first + 1;
  float* part_cta = a.partial + int64_t(blockIdx.x) * a.maxseg * ncw * M * 256;
  auto flush = [&](int seg, const float2 (&acc)[M][4]) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float* dst = part_cta + ((int64_t(seg) * ncw + warp) * M + m) * 256 + 8 * lane;
      __stcg(reinterpret_cast<float4*>(dst), make_float4(acc[m][0].x, acc[m][0].y, acc[m][1].x, acc[m][1].y));
      __stcg(reinterpret_cast<float4*>(dst + 4), make_float4(acc[m][2].x, acc[m][2].y, acc[m][3].x, acc[m][3].y));
    }
  };
  float2 acc[M][4];
#pragma unroll
  for (int m = 0; m < M; ++m)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.0f, 0.0f);
  int cur = 0;  // the segment (column group - g_first) acc belongs to
  ScaleWords<NB, NESTED> sw;
  float gv[M];
  auto fetch_g = [&](int rb) {
    const int64_t row = int64_t(rb) * kRows + lane;
#pragma unroll
    for (int m = 0; m < M; ++m) gv[m] = row < a.x.n_rows ? Elem<XT>::to_f32(gp[int64_t(m) * a.ldg + row]) : 0.0f;
  };
  if (warp < n_units) {
    const int64_t u = u0 + warp;
    fetch_scales<1, NB, NESTED>(sw, a.x, int(u / a.row_blocks), int(u % a.row_blocks), lane);
    fetch_g(int(u % a.row_blocks));
  }
  int slot = warp % S;
  uint32_t parity = uint32_t((warp / S) & 1);
  for (int i = warp; i < n_units; i += ncw) {
    bool ok;
    if (s_abort) {
      ok = false;
      const int q = i % kProducers;
      const uint64_t t0 = global_ns();
      while (s_next[q] < 0 && global_ns() - t0 < g_bnbq_wait_limit_ns) {
      }
      if (i < s_next[q]) mbar_wait(full0 + 8u * slot, parity);
    } else {
      ok = mbar_wait(full0 + 8u * slot, parity);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) s_abort = 1;
    }
    uint32_t cw[kRows];
    if (ok) {
      const uint32_t st = stage0 + uint32_t(slot) * kStage + uint32_t(lane) * 4u;
#pragma unroll
      for (int r = 0; r < kRows; ++r) cw[r] = lds_code(st + uint32_t(r) * 128u);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8u * slot);
    slot += ncw;
    if (slot >= S) {
      slot -= S;
      parity ^= 1u;
    }
    const int64_t u = u0 + i;
    const int seg = int(u / a.row_blocks) - g_first;
    // this row's block scales and g values, for the warp's lanes to read
    float a_own[NB];
    decode_scales<NB, NESTED>(a_own, sw, a.x, s_code2, offset, 0);
#pragma unroll
    for (int p = 0; p < NB; ++p) s_a[warp][lane][p] = a_own[p];
#pragma unroll
    for (int m = 0; m < M; ++m) s_gv[warp][m][lane] = gv[m];
    __syncwarp();
    if (i + ncw < n_units) {
      const int64_t un = u0 + i + ncw;
      fetch_scales<1, NB, NESTED>(sw, a.x, int(un / a.row_blocks), int(un % a.row_blocks), lane);
      fetch_g(int(un % a.row_blocks));
    }
    if (seg != cur) {  // a new column group: store the finished ones (zeros for skipped)
      for (; cur < seg; ++cur) {
        flush(cur, acc);
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.0f, 0.0f);
      }
    }
    if (ok) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const float sa = s_a[warp][r][qs];
        float2 wv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t byte = (cw[r] >> (8 * j)) & 0xffu;
          wv[j] = mul_ftz2(s_pair[byte * 32 + lane], make_float2(sa, sa));
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const float gr = s_gv[warp][m][r];
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[m][j] = __ffma2_rn(wv[j], make_float2(gr, gr), acc[m][j]);
        }
      }
    }
    __syncwarp();  // s_a and s_gv are rewritten for the next unit
  }
  for (; cur < nseg; ++cur) {
    flush(cur, acc);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.0f, 0.0f);
  }
}

// The CTA of a grid of G over U units (CTA b: units [b U / G, (b + 1) U / G))
// that holds unit u.
__device__ __forceinline__ int64_t cta_of(int64_t u, int64_t units, int64_t grid) {
  return ((u + 1) * grid + units - 1) / units - 1;
}

template <typename XT, int M>
__global__ void __launch_bounds__(256) gemv_t_reduce_kernel(const float* partial, int64_t units, int64_t grid,
                                                            int row_blocks, int maxseg, int k, void* out,
                                                            int64_t ldo) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // every partial of the first kernel is visible
  const int64_t total = int64_t(M) * k;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int m = int(i / k), c = int(i - int64_t(m) * k);
    const int g = c >> 8, cc = c & 255;
    const int64_t b_lo = cta_of(int64_t(g) * row_blocks, units, grid);
    const int64_t b_hi = cta_of(int64_t(g + 1) * row_blocks - 1, units, grid);
    float v = 0.0f;
    for (int64_t b = b_lo; b <= b_hi; ++b) {
      const int g0 = int((b * units / grid) / row_blocks);
      const float* p = partial + ((b * maxseg + (g - g0)) * kTConsumers * M + m) * 256 + cc;
      for (int w = 0; w < kTConsumers; ++w) v += __ldcg(p + int64_t(w) * M * 256);
    }
    XT* o = static_cast<XT*>(out);
    if constexpr (Elem<XT>::kDtype == BNBQ_BF16) o[int64_t(m) * ldo + c] = __float2bfloat16_rn(v);
    else o[int64_t(m) * ldo + c] = __float2half_rn(v);
  }
}

// --------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Workspace: the partials of the split K (any initial contents).
constexpr int64_t kMaxRowBlocks = int64_t(1) << 24;

int64_t workspace_bytes_for(int m, int k, int64_t n_rows) {
  const int gk = m == 1 ? Cfg<1>::kGroupK : Cfg<2>::kGroupK;
  const int mm = m == 1 ? 1 : 2;
  const int64_t rbs = (n_rows + kRows - 1) / kRows;
  const int64_t groups = k / gk;
  return rbs * groups * mm * kRows * 4;
}

// Dynamic shared memory of a launch: all the block may have, less its static
// arrays. The kernel places the table at a 64 KB-aligned address inside it and
// the stages below and above it; the alignment can cost up to one stage.
int dyn_bytes(const DeviceInfo& di) { return (di.smem_optin - 4096) / 1024 * 1024; }

template <int M>
bool fits(int dyn) {
  return dyn >= int(kTabBytes + kTabAlign) && (dyn - int(kTabBytes)) / int(Cfg<M>::kStageBytes) - 1 >= Cfg<M>::kRound;
}

template <typename XT, int M, int NB, bool NESTED>
int launch_t(const CUtensorMap& map, const XtabArgs& a0, const DeviceInfo& di, cudaStream_t s, const PeerOut* xp) {
  constexpr uint32_t kStage = Cfg<M>::kStageBytes;
  auto kern = gemv_xtab_kernel<XT, M, NB, NESTED>;
  XtabArgs a = a0;
  const int ncw = Cfg<M>::kConsumers;
  const int nwarps = ncw + kProducers;
  // All the shared memory the block may have, less its static arrays; the
  // kernel places the table at a 64 KB-aligned address inside it and the
  // stages around it (at least ncw + 2 of them).
  // The table then fits whatever the dynamic base address below 64 KB is, and
  // what it leaves below and above the table holds the stages.
  const int dyn = dyn_bytes(di);
  if (!fits<M>(dyn)) return BNBQ_ERR_UNSUPPORTED;
  a.dyn_bytes = uint32_t(dyn);
  if (xp) {  // the exchange polls for peers from every reduction CTA: all must be resident
    int per_sm = 0;
    if (int st = kernel_occupancy(reinterpret_cast<const void*>(gemv_xtab_reduce_kernel<XT, M>), kRedThreads, 0,
                                  &per_sm))
      return st;
    if (int64_t(a.row_blocks) * M > int64_t(per_sm) * di.sm_count) return BNBQ_ERR_UNSUPPORTED;
  }
  static std::atomic<int> attr_set[kMaxDevices];  // per device: the attribute is set once
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BNBQ_ERR_CUDA;
  if (attr_set[dev].load(std::memory_order_acquire) != dyn) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
      return BNBQ_ERR_CUDA;
    attr_set[dev].store(dyn, std::memory_order_release);
  }
  int64_t grid = di.sm_count;
  if (grid > a.units) grid = a.units;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(unsigned(nwarps * 32));
  cfg.dynamicSmemBytes = size_t(dyn);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, map, a) != cudaSuccess) return BNBQ_ERR_CUDA;
  // the reduction, behind it on the stream
  cudaLaunchConfig_t rc = cfg;
  rc.gridDim = dim3(unsigned(int64_t(a.row_blocks) * M));
  rc.blockDim = dim3(kRedThreads);
  rc.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&rc, gemv_xtab_reduce_kernel<XT, M>, static_cast<const float*>(a.partial), a.groups,
                         a.row_blocks, a.n_rows, a.y, a.ldy, xp ? *xp : PeerOut{}) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, int M, bool NESTED>
int launch_nb(int nb, const CUtensorMap& map, const XtabArgs& a, const DeviceInfo& di, cudaStream_t s,
              const PeerOut* xp) {
  switch (nb) {
    case 1: return launch_t<XT, M, 1, NESTED>(map, a, di, s, xp);
    case 2: return launch_t<XT, M, 2, NESTED>(map, a, di, s, xp);
    case 4: return launch_t<XT, M, 4, NESTED>(map, a, di, s, xp);
    case 8:
      if constexpr (M == 1) return launch_t<XT, M, 8, NESTED>(map, a, di, s, xp);
      else return BNBQ_ERR_UNSUPPORTED;
    default: return BNBQ_ERR_UNSUPPORTED;
  }
}

// One pass over rows [m0, m0 + mm) of x (mm = 1 or 2).
template <typename XT>
int launch_rows(int mm, const XtabArgs& base, const uint8_t* w, bool nested, const DeviceInfo& di, const PeerOut* xp,
                cudaStream_t s) {
  const int gk = mm == 1 ? Cfg<1>::kGroupK : Cfg<2>::kGroupK;
  const int bs = 1 << base.log2_bs;
  const int nb = bs >= gk ? 1 : gk / bs;
  XtabArgs a = base;
  a.groups = base.k / gk;
  a.row_blocks = int((base.n_rows + kRows - 1) / kRows);
  a.units = int64_t(a.groups) * a.row_blocks;

  auto encode = encoder();
  if (!encode) return BNBQ_ERR_CUDA;
  CUtensorMap map;
  const cuuint64_t dims[2] = {cuuint64_t(base.k / 2), cuuint64_t(base.n_rows)};
  const cuuint64_t strides[1] = {cuuint64_t(base.k / 2)};
  const cuuint32_t box[2] = {cuuint32_t(gk / 2), cuuint32_t(kRows)};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return BNBQ_ERR_UNSUPPORTED;
  if (mm == 1)
    return nested ? launch_nb<XT, 1, true>(nb, map, a, di, s, xp) : launch_nb<XT, 1, false>(nb, map, a, di, s, xp);
  return nested ? launch_nb<XT, 2, true>(nb, map, a, di, s, xp) : launch_nb<XT, 2, false>(nb, map, a, di, s, xp);
}

// ---- 8-bit codebook weights
int64_t code8_workspace_bytes(int m, int k, int64_t n_rows) {
  const int64_t rbs = (n_rows + kRows - 1) / kRows;
  return rbs * (k / kGroupK8) * m * kRows * 4;
}

template <typename XT, int M, int NB, bool NESTED>
int launch_code8_t(const CUtensorMap& map, const XtabArgs& a0, const float* code, const DeviceInfo& di,
                   cudaStream_t s) {
  auto kern = gemv_code8_kernel<XT, M, NB, NESTED>;
  XtabArgs a = a0;
  const int dyn = dyn_bytes(di);
  if (dyn < int(kTab8Bytes + kTabAlign) || (dyn - int(kTab8Bytes)) / (kRows * kGroupK8) - 1 < Cfg8<M>::kRound)
    return BNBQ_ERR_UNSUPPORTED;
  a.dyn_bytes = uint32_t(dyn);
  static std::atomic<int> attr_set[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BNBQ_ERR_CUDA;
  if (attr_set[dev].load(std::memory_order_acquire) != dyn) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
      return BNBQ_ERR_CUDA;
    attr_set[dev].store(dyn, std::memory_order_release);
  }
  int64_t grid = di.sm_count;
  if (grid > a.units) grid = a.units;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(unsigned((Cfg8<M>::kConsumers + kProducers) * 32));
  cfg.dynamicSmemBytes = size_t(dyn);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, map, a, code) != cudaSuccess) return BNBQ_ERR_CUDA;
  cudaLaunchConfig_t rc = cfg;
  rc.gridDim = dim3(unsigned(int64_t(a.row_blocks) * M));
  rc.blockDim = dim3(kRedThreads);
  rc.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&rc, gemv_xtab_reduce_kernel<XT, M>, static_cast<const float*>(a.partial), a.groups,
                         a.row_blocks, a.n_rows, a.y, a.ldy, PeerOut{}) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, int M, bool NESTED>
int launch_code8_nb(int nb, const CUtensorMap& map, const XtabArgs& a, const float* code, const DeviceInfo& di,
                    cudaStream_t s) {
  switch (nb) {
    case 1: return launch_code8_t<XT, M, 1, NESTED>(map, a, code, di, s);
    case 2: return launch_code8_t<XT, M, 2, NESTED>(map, a, code, di, s);
    case 4: return launch_code8_t<XT, M, 4, NESTED>(map, a, code, di, s);
    default: return BNBQ_ERR_UNSUPPORTED;
  }
}

template <typename XT, int M>
int launch_code8_m(int nb, bool nested, const CUtensorMap& map, const XtabArgs& a, const float* code,
                   const DeviceInfo& di, cudaStream_t s) {
  return nested ? launch_code8_nb<XT, M, true>(nb, map, a, code, di, s)
                : launch_code8_nb<XT, M, false>(nb, map, a, code, di, s);
}

// ---- the backward (gemv_t_kernel)
struct TPlan {
  int64_t grid, units;
  int maxseg;
};

TPlan plan_t(int64_t n_rows, int k, int sm_count) {
  TPlan p;
  const int rbs = int((n_rows + kRows - 1) / kRows);
  p.units = int64_t(k / 256) * rbs;
  p.grid = p.units < sm_count ? p.units : sm_count;
  p.maxseg = 1;
  for (int64_t b = 0; b < p.grid; ++b) {
    const int64_t u0 = b * p.units / p.grid, u1 = (b + 1) * p.units / p.grid;
    const int nseg = int((u1 - 1) / rbs - u0 / rbs + 1);
    p.maxseg = nseg > p.maxseg ? nseg : p.maxseg;
  }
  return p;
}

int64_t t_workspace_bytes(int m, const TPlan& p) { return p.grid * p.maxseg * kTConsumers * m * 256 * 4; }

template <typename XT, int M, int NB, bool NESTED>
int launch_gemv_t(const CUtensorMap& map, const GemvTArgs& a0, const TPlan& p, void* out, int64_t ldo,
                  const DeviceInfo& di, cudaStream_t s) {
  auto kern = gemv_t_kernel<XT, M, NB, NESTED>;
  GemvTArgs a = a0;
  int static_smem = 0;
  if (int st = kernel_static_smem(reinterpret_cast<const void*>(kern), &static_smem)) return st;
  const int dyn = (di.smem_optin - static_smem - 1024) / 1024 * 1024;
  if (dyn < int(kPairTableBytesT) + kTRound * kRows * 128) return BNBQ_ERR_UNSUPPORTED;
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), dyn)) return st;
  a.dyn_bytes = uint32_t(dyn);
  a.units = p.units;
  a.maxseg = p.maxseg;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p.grid));
  cfg.blockDim = dim3(unsigned((kTConsumers + kProducers) * 32));
  cfg.dynamicSmemBytes = size_t(dyn);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, map, a) != cudaSuccess) return BNBQ_ERR_CUDA;
  cudaLaunchConfig_t rc = cfg;
  const int64_t total = int64_t(M) * a.x.k;
  int64_t rgrid = (total + 255) / 256;
  if (rgrid > int64_t(di.sm_count) * 8) rgrid = int64_t(di.sm_count) * 8;
  rc.gridDim = dim3(unsigned(rgrid));
  rc.blockDim = dim3(256);
  rc.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&rc, gemv_t_reduce_kernel<XT, M>, static_cast<const float*>(a.partial), p.units, p.grid,
                         a.row_blocks, p.maxseg, a.x.k, out, ldo) != cudaSuccess)
    return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, int M, bool NESTED>
int launch_gemv_t_nb(int nb, const CUtensorMap& map, const GemvTArgs& a, const TPlan& p, void* out, int64_t ldo,
                     const DeviceInfo& di, cudaStream_t s) {
  switch (nb) {
    case 1: return launch_gemv_t<XT, M, 1, NESTED>(map, a, p, out, ldo, di, s);
    case 2: return launch_gemv_t<XT, M, 2, NESTED>(map, a, p, out, ldo, di, s);
    case 4: return launch_gemv_t<XT, M, 4, NESTED>(map, a, p, out, ldo, di, s);
    case 8: return launch_gemv_t<XT, M, 8, NESTED>(map, a, p, out, ldo, di, s);
    default: return BNBQ_ERR_UNSUPPORTED;
  }
}

template <typename XT, bool NESTED>
int launch_gemv_t_m(int m, int nb, const CUtensorMap& map, const GemvTArgs& a, const TPlan& p, void* out,
                    int64_t ldo, const DeviceInfo& di, cudaStream_t s) {
  switch (m) {
    case 1: return launch_gemv_t_nb<XT, 1, NESTED>(nb, map, a, p, out, ldo, di, s);
    case 2: return launch_gemv_t_nb<XT, 2, NESTED>(nb, map, a, p, out, ldo, di, s);
    case 3: return launch_gemv_t_nb<XT, 3, NESTED>(nb, map, a, p, out, ldo, di, s);
    default: return launch_gemv_t_nb<XT, 4, NESTED>(nb, map, a, p, out, ldo, di, s);
  }
}

}  // namespace

int xtab_wait_timeouts(unsigned int* out) { return read_wait_timeouts(out); }
int xtab_set_wait_limit(uint64_t ns) { return write_wait_limit(ns); }

int gemv_xtab_set_policy(int policy) {
  if (policy < 0 || policy > 2) return BNBQ_ERR_INVALID;
  g_table_policy.store(policy, std::memory_order_relaxed);
  return BNBQ_OK;
}

// Bytes of workspace the table GEMV needs for m rows of x (0 when it does not
// apply to m).
int64_t gemv_xtab_workspace_bytes(int m, int k, int64_t n_rows) {
  if (m < 1 || m > 4 || n_rows < 1 || n_rows > kMaxRowBlocks * kRows || k < 1) return 0;
  return workspace_bytes_for(m, k, n_rows);
}

// BNBQ_ERR_UNSUPPORTED when the table GEMV does not take this call (the caller
// then uses the other GEMV kernels).
// BNBQ_OK when the table GEMV takes a call of this shape (with a workspace of
// workspace_bytes at `workspace`), else BNBQ_ERR_UNSUPPORTED (or a device error).
int gemv_xtab_applies(int m, int k, int64_t n_rows, int blocksize, const uint8_t* absmax_q, int blocksize2,
                      const void* workspace, int64_t workspace_bytes) {
  if (m < 1 || m > 4 || !workspace || n_rows < 1 || n_rows > kMaxRowBlocks * kRows) return BNBQ_ERR_UNSUPPORTED;
  const int policy = g_table_policy.load(std::memory_order_relaxed);
  if (policy == 2 || (policy == 0 && 2 * n_rows < 3 * int64_t(k))) return BNBQ_ERR_UNSUPPORTED;
  if (k % Cfg<1>::kGroupK != 0) return BNBQ_ERR_UNSUPPORTED;  // (covers the two-row group too)
  const int l2 = log2_exact(blocksize);
  if (l2 < 5) return BNBQ_ERR_UNSUPPORTED;
  const int nb_max = blocksize >= 256 ? 1 : 256 / blocksize;
  if (absmax_q) {
    if (log2_exact(blocksize2) < 0 || blocksize2 < nb_max) return BNBQ_ERR_UNSUPPORTED;
    if (!aligned(absmax_q, uint64_t(nb_max))) return BNBQ_ERR_UNSUPPORTED;
  }
  if (workspace_bytes < workspace_bytes_for(m, k, n_rows) || !aligned(workspace, 256)) return BNBQ_ERR_UNSUPPORTED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  if (!fits<1>(dyn_bytes(di)) || (m >= 2 && !fits<2>(dyn_bytes(di)))) return BNBQ_ERR_UNSUPPORTED;
  return BNBQ_OK;
}

// px != nullptr: the exchange mode (one pass, M <= 2), y = px->y_full's own
// columns; y and ldy are then ignored.
int gemv_xtab_launch(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows, int blocksize,
                     const float* absmax, const uint8_t* absmax_q, const float* absmax2, const float* code2,
                     const float* offset, int blocksize2, int64_t absmax2_block0, void* y, int64_t ldy,
                     void* workspace, int64_t workspace_bytes, cudaStream_t s, const PeerOut* px) {
  if (int st = gemv_xtab_applies(m, k, n_rows, blocksize, absmax_q, blocksize2, workspace, workspace_bytes))
    return st;
  if (px) {
    if (m > 2) return BNBQ_ERR_UNSUPPORTED;
    y = static_cast<char*>(px->y_full) + size_t(px->col0) * 2;
    ldy = px->ldf;
  }
  const int l2 = log2_exact(blocksize);
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  XtabArgs a{};
  a.absmax = absmax;
  a.absmax_q = absmax_q;
  a.absmax2 = absmax2;
  a.code2 = code2;
  a.offset = offset;
  a.partial = static_cast<float*>(workspace);
  a.n_rows = n_rows;
  a.ldy = ldy;
  a.block0 = absmax2_block0;
  a.k = k;
  a.log2_bs = l2;
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  const size_t es = dtype == BNBQ_F32 ? 4 : 2;
  const bool nested = absmax_q != nullptr;
  // passes of two rows, then one of one row (m = 1, 3)
  for (int m0 = 0; m0 < m;) {
    const int mm = (m - m0 >= 2) ? 2 : 1;
    a.x = static_cast<const char*>(x) + size_t(m0) * size_t(k) * es;
    a.y = static_cast<char*>(y) + size_t(m0) * size_t(ldy) * es;
    int st;
    if (dtype == BNBQ_BF16) st = launch_rows<__nv_bfloat16>(mm, a, w, nested, di, px, s);
    else if (dtype == BNBQ_F16) st = launch_rows<__half>(mm, a, w, nested, di, px, s);
    else return BNBQ_ERR_UNSUPPORTED;
    if (st != BNBQ_OK) return st;
    m0 += mm;
  }
  return BNBQ_OK;
}


// ---- 8-bit codebook weights: the fused GEMV (gemv_code8_kernel)
int64_t gemv_code8_workspace_bytes(int m, int k, int64_t n_rows) {
  if (m < 1 || m > 4 || k < kGroupK8 || k % kGroupK8 || n_rows < 1 || n_rows > kMaxRowBlocks * kRows) return 0;
  return code8_workspace_bytes(m, k, n_rows);
}

int gemv_code8_launch(int dtype, const void* x, int m, int k, const uint8_t* w, int64_t n_rows, int blocksize,
                      const float* code, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                      const float* code2, const float* offset, int blocksize2, int64_t absmax2_block0, void* y,
                      int64_t ldy, void* workspace, int64_t workspace_bytes, cudaStream_t s) {
  if (m < 1 || m > 4 || k % kGroupK8 || n_rows < 1 || n_rows > kMaxRowBlocks * kRows) return BNBQ_ERR_UNSUPPORTED;
  const int l2 = log2_exact(blocksize);
  if (l2 < 5) return BNBQ_ERR_INVALID;
  const int nb = blocksize >= kGroupK8 ? 1 : kGroupK8 / blocksize;
  if (absmax_q) {
    if (log2_exact(blocksize2) < 0 || blocksize2 < nb) return BNBQ_ERR_UNSUPPORTED;
    if (!aligned(absmax_q, uint64_t(nb))) return BNBQ_ERR_MISALIGNED;
  }
  if (!workspace || workspace_bytes < gemv_code8_workspace_bytes(m, k, n_rows) || !aligned(workspace, 256))
    return BNBQ_ERR_INVALID;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  auto encode = encoder();
  if (!encode) return BNBQ_ERR_CUDA;
  CUtensorMap map;
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(n_rows)};
  const cuuint64_t strides[1] = {cuuint64_t(k)};
  const cuuint32_t box[2] = {cuuint32_t(kGroupK8), cuuint32_t(kRows)};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return BNBQ_ERR_UNSUPPORTED;
  XtabArgs a{};
  a.absmax = absmax;
  a.absmax_q = absmax_q;
  a.absmax2 = absmax2;
  a.code2 = code2;
  a.offset = offset;
  a.partial = static_cast<float*>(workspace);
  a.n_rows = n_rows;
  a.ldy = ldy;
  a.block0 = absmax2_block0;
  a.k = k;
  a.log2_bs = l2;
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  a.groups = k / kGroupK8;
  a.row_blocks = int((n_rows + kRows - 1) / kRows);
  a.units = int64_t(a.groups) * a.row_blocks;
  const bool nested = absmax_q != nullptr;
  // one pass over the weight for all m rows of x
  a.x = x;
  a.y = y;
  if (dtype == BNBQ_BF16) {
    switch (m) {
      case 1: return launch_code8_m<__nv_bfloat16, 1>(nb, nested, map, a, code, di, s);
      case 2: return launch_code8_m<__nv_bfloat16, 2>(nb, nested, map, a, code, di, s);
      case 3: return launch_code8_m<__nv_bfloat16, 3>(nb, nested, map, a, code, di, s);
      default: return launch_code8_m<__nv_bfloat16, 4>(nb, nested, map, a, code, di, s);
    }
  }
  if (dtype == BNBQ_F16) {
    switch (m) {
      case 1: return launch_code8_m<__half, 1>(nb, nested, map, a, code, di, s);
      case 2: return launch_code8_m<__half, 2>(nb, nested, map, a, code, di, s);
      case 3: return launch_code8_m<__half, 3>(nb, nested, map, a, code, di, s);
      default: return launch_code8_m<__half, 4>(nb, nested, map, a, code, di, s);
    }
  }
  return BNBQ_ERR_UNSUPPORTED;
}

}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_gemv_t_nf4_workspace_bytes(int32_t m, int32_t k, int64_t n_rows, int64_t* bytes) {
  if (!bytes || m < 1 || m > 4 || k < 1 || n_rows < 1) return BNBQ_ERR_INVALID;
  if (k % 256 || n_rows > kMaxRowBlocks * kRows) return BNBQ_ERR_UNSUPPORTED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  *bytes = t_workspace_bytes(m, plan_t(n_rows, k, di.sm_count));
  return BNBQ_OK;
}

extern "C" int bnbq_gemv_t_nf4_ws(int dtype, const void* g, int32_t m, int64_t n_rows, int64_t ldg, int32_t k,
                                  const uint8_t* w, int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                                  const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                                  int64_t absmax2_block0, void* out, int64_t ldo, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  if (dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (m < 1 || m > 4 || n_rows < 1 || k < 1 || ldg < n_rows || ldo < k) return BNBQ_ERR_INVALID;
  if (k % 256 || n_rows > kMaxRowBlocks * kRows) return BNBQ_ERR_UNSUPPORTED;
  const int l2 = log2_exact(blocksize);
  if (l2 < 5 || !g || !w || !out || !workspace) return BNBQ_ERR_INVALID;
  const int nb = blocksize >= 256 ? 1 : 256 / blocksize;
  if (absmax_q) {
    if (!absmax2 || !code2 || !offset || log2_exact(blocksize2) < 0) return BNBQ_ERR_INVALID;
    if (blocksize2 < nb) return BNBQ_ERR_UNSUPPORTED;
    if (!aligned(absmax2, 4) || !aligned(code2, 4) || !aligned(offset, 4) || !aligned(absmax_q, uint64_t(nb)))
      return BNBQ_ERR_MISALIGNED;
  } else {
    if (!absmax) return BNBQ_ERR_INVALID;
    if (!aligned(absmax, 4)) return BNBQ_ERR_MISALIGNED;
  }
  if (!aligned(g, 2) || !aligned(w, 16) || !aligned(out, 2) || !aligned(workspace, 16)) return BNBQ_ERR_MISALIGNED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  const TPlan p = plan_t(n_rows, k, di.sm_count);
  if (workspace_bytes < t_workspace_bytes(m, p)) return BNBQ_ERR_INVALID;
  auto encode = encoder();
  if (!encode) return BNBQ_ERR_CUDA;
  CUtensorMap map;
  const cuuint64_t dims[2] = {cuuint64_t(k / 2), cuuint64_t(n_rows)};
  const cuuint64_t strides[1] = {cuuint64_t(k / 2)};
  const cuuint32_t box[2] = {128u, cuuint32_t(kRows)};
  const cuuint32_t estr[2] = {1, 1};
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return BNBQ_ERR_UNSUPPORTED;
  GemvTArgs a{};
  a.g = g;
  a.partial = static_cast<float*>(workspace);
  a.ldg = ldg;
  a.row_blocks = int((n_rows + kRows - 1) / kRows);
  a.groups = k / 256;
  a.x.absmax = absmax;
  a.x.absmax_q = absmax_q;
  a.x.absmax2 = absmax2;
  a.x.code2 = code2;
  a.x.offset = offset;
  a.x.n_rows = n_rows;
  a.x.block0 = absmax2_block0;
  a.x.k = k;
  a.x.log2_bs = l2;
  a.x.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool nested = absmax_q != nullptr;
  if (dtype == BNBQ_BF16)
    return nested ? launch_gemv_t_m<__nv_bfloat16, true>(m, nb, map, a, p, out, ldo, di, s)
                  : launch_gemv_t_m<__nv_bfloat16, false>(m, nb, map, a, p, out, ldo, di, s);
  return nested ? launch_gemv_t_m<__half, true>(m, nb, map, a, p, out, ldo, di, s)
                : launch_gemv_t_m<__half, false>(m, nb, map, a, p, out, ldo, di, s);
}
