// bnbq_gemm.cu -- fused NF4 dequantize-GEMM for M > 20 on the 5th-generation
// tensor cores (tcgen05.mma, operands and accumulator in tensor memory).
//
// y = x @ W.T for x (M, K) bf16/f16 and an NF4 weight W (N, K). It replaces the
// reference's fallback for large batches, `xm @ w.dequantize(xm.dtype).T`
// (bnb_jax/_matmul.py:58-59): the dense weight is never written to HBM. Every
// weight element is decoded to x's dtype as dtype(mul.ftz(table[q], a)) -- the
// value dequantize() produces, bit for bit -- and the products are accumulated
// in float32 by the tensor cores, so the result equals the fallback's up to the
// order of summation.
//
// One CTA computes a tile of 128 weight rows (the MMA's M, one tensor-memory
// lane per row) by BN rows of x (the MMA's N, 32..256), K in stages of 64:
//   TMA warp               one thread copies the stage's 128 x 32 bytes of NF4 codes and the BN x 64
//                          tile of x (128-byte swizzle) into a shared-memory ring
//                          slot; completion counted in bytes.
//   scale warp             asynchronous copies (cp.async, completion counted on
//                          the stage's barrier) of the block scales of the stage's
//                          128 rows: float32 absmax, or the nested code word and
//                          absmax2; the ring's depth is the prefetch distance.
//   decoder groups         DG groups of 4 warps (DG = 2; 4 for the precise split),
//                          group g taking stages g, g+DG, ...;
//                          thread t of a group owns weight row t: it decodes the
//                          row's block scale a (nested: code2[q] * absmax2 +
//                          offset) and builds the 16-entry table dtype(mul.ftz(T[q], a)) in
//                          registers (two byte planes), decodes the 64 codes with
//                          byte permutes and writes them with tcgen05.st into its
//                          lane of an A slot in tensor memory (32 columns; a ring
//                          of SA slots, separate from the shared-memory ring).
//   precise split (GEMV)   the weight's exact float32 value w as hi = RN(w) plus
//                          lo = RZ(w - hi) in x's dtype: two A terms, two MMAs per
//                          K step into the same accumulator. Each decoder lane keeps
//                          its block's 16 (hi | lo << 16) words in a warp-private
//                          shared table [q][lane] (bank = lane) and decodes a value
//                          with one load. Rounding hi + lo gives hi back in every
//                          case, so a one-hot x returns the decoded weights bitwise.
//   MMA warp               tensor memory allocation; one thread issues the stage's
//                          four K=16 MMAs (A from tensor memory, x from shared
//                          memory) and a tcgen05.commit that frees the ring slot
//                          and, SA stages later, the A slot.
//   epilogue (decoders)    tcgen05.ld of the accumulator lanes, rounding to x's
//                          dtype, stores of y.
// Every wait is bounded in time. On expiry the CTA stops issuing work, waits
// (bounded) for the copies and MMAs it started, frees its tensor memory and
// returns without writing y; the expiry is counted (bnbq_wait_timeouts).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "bnbq_async.cuh"
#include "bnbq_common.cuh"

namespace bnbq {

int gemv_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                int32_t blocksize, const float* absmax, const uint8_t* absmax_q,
                const float* absmax2, const float* code2, const float* offset, int32_t blocksize2,
                int64_t absmax2_block0, void* y, int64_t ldy, cudaStream_t s);

namespace {

constexpr int kBM = 128;                        // weight rows per CTA (MMA M)
constexpr int kBK = 64;                         // K per stage
constexpr int kMaxStages = 12;                  // shared-memory ring slots
constexpr int kMaxASlots = 6;                   // tensor-memory A slots
constexpr uint32_t kCodeBytes = kBM * kBK / 2;  // 4 KB of codes per stage
constexpr uint32_t kScaleBytes = 4 * kBM * 4;   // per row, up to two blocks: scale word and absmax2
constexpr uint32_t kAColsPerStage = kBK / 2;    // 64 16-bit values = 32 columns

// Tile configuration: BN rows of x, DG decoder groups of 4 warps; the tiles up to
// 64 wide run two CTAs per SM.
template <int BN, bool PRECISE = false>
struct Tile {
  static constexpr int kDG = PRECISE ? 4 : 2;  // the precise split decodes twice as much per stage
  static constexpr uint32_t kACols = PRECISE ? 2 * kAColsPerStage : kAColsPerStage;  // hi (+ lo) terms
  static constexpr int kWarpTma = 4 * kDG, kWarpScale = kWarpTma + 1, kWarpMma = kWarpTma + 2;
  static constexpr int kThreads = (kWarpMma + 1) * 32;
  static constexpr bool kPair = BN <= 64 && !PRECISE;  // the precise (GEMV) tiles run one CTA per SM
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kBBytes + kCodeBytes + kScaleBytes;  // a multiple of 1024
  // precise decoders: a warp-private 16 x 32 table of (hi | lo << 16) words after the ring
  static constexpr uint32_t kTableBytes = PRECISE ? 4 * kDG * 16 * 32 * 4 : 0;
};

struct GemmArgs {
  const uint8_t* absmax_q;
  const float* absmax;
  const float* absmax2;
  const float* code2;
  const float* offset;
  void* y;
  int64_t n_rows;
  int64_t k;
  int64_t ldy;
  int64_t block0;
  int m;
  int log2_bs;
  int log2_bs2;
  int n_stages;
  int n_aslots;
  uint32_t tmem_cols;
  int kb_per_split;  // K blocks per CTA of a cluster along K (gridDim.z CTAs)
};

// Shared-memory matrix descriptor (sm_100 format) of a K-major tile in the
// canonical 128-byte-swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes
// apart. Fields: start address >> 4 (bits 0-13), leading byte offset (16-29,
// unused for this layout), stride byte offset >> 4 (32-45), version 1 (46-47),
// layout type SWIZZLE_128B = 2 (61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return uint64_t((smem_addr >> 4) & 0x3fffu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor of kind::f16: f32 accumulator (bits 4-5 = 1), A and B
// of x's type (bits 7-9 and 10-12: 0 f16, 1 bf16), both K-major (bits 15, 16 = 0),
// N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t instr_desc(bool bf16, int bn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (uint32_t(bn >> 3) << 17) |
         (uint32_t(kBM >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem_d] (+)= A[tmem_a] x B[desc_b]: A read from tensor memory, B from shared memory.
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t desc_b, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 4-byte asynchronous global -> shared copy; completion is signalled by cp_async_arrive.
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Arrive on `bar` once all of this thread's earlier cp.async copies are complete
// (the arrival is part of the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <typename XT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) return pack2_bf16(lo, hi);
  else return pack2_f16(lo, hi);
}

// Round-toward-zero pair conversion (the residual term of the precise split).
template <typename XT>
__device__ __forceinline__ uint32_t pack2_rz(float lo, float hi) {
  uint32_t r;
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) asm("cvt.rz.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else asm("cvt.rz.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename XT>
__device__ __forceinline__ float2 unpack2x(uint32_t w) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) return unpack2_bf16(w);
  else return unpack2_f16(w);
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of this CTA's shared address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

template <typename XT>
__device__ __forceinline__ void store_out(void* y, int64_t i, float v) {
  if constexpr (Elem<XT>::kDtype == BNBQ_BF16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(y)[i] = __float2half_rn(v);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// The 16 values dtype(mul.ftz(T[q], a)) of one block as two byte planes:
// byte i of lo[j] (hi[j]) is the low (high) byte of entry 4j + i.
template <typename XT>
__device__ __forceinline__ void block_table(float a, uint32_t (&lo)[4], uint32_t (&hi)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t p0 = pack2<XT>(mul_ftz(kNF4Table[4 * j], a), mul_ftz(kNF4Table[4 * j + 1], a));
    const uint32_t p1 = pack2<XT>(mul_ftz(kNF4Table[4 * j + 2], a), mul_ftz(kNF4Table[4 * j + 3], a));
    lo[j] = prmt(p0, p1, 0x6420);
    hi[j] = prmt(p0, p1, 0x7531);
  }
}

// One 32-bit word of packed codes (byte b: value 2b in the high nibble, 2b+1 in
// the low nibble) -> four words of two 16-bit values, value 2i in the low half
// of word i. Per group of four codes: the low three bits of each code pick a
// byte from entries 0-7 and from entries 8-15, bit 3 picks between the two.
__device__ __forceinline__ void decode_word(uint32_t w, const uint32_t (&lo)[4], const uint32_t (&hi)[4],
                                            uint32_t* out) {
  const uint32_t sel = w & 0x77777777u;
  const uint32_t half = ((w >> 1) & 0x44444444u) | 0x32103210u;
#pragma unroll
  for (int g = 0; g < 2; ++g) {  // prmt reads the low 16 bits of its selector
    const uint32_t s = g ? sel >> 16 : sel;
    const uint32_t h = g ? half >> 16 : half;
    const uint32_t l = prmt(prmt(lo[0], lo[1], s), prmt(lo[2], lo[3], s), h);
    const uint32_t u = prmt(prmt(hi[0], hi[1], s), prmt(hi[2], hi[3], s), h);
    // byte i of l/u belongs to code nibble i: values 2g*2+1, 2g*2, 2g*2+3, 2g*2+2
    out[2 * g] = prmt(l, u, 0x4051);
    out[2 * g + 1] = prmt(l, u, 0x6273);
  }
}

template <typename XT, int BN, bool NESTED, bool PRECISE>
__global__ void __launch_bounds__(Tile<BN, PRECISE>::kThreads, Tile<BN, PRECISE>::kPair ? 2 : 1)
gemm_kernel(const GemmArgs a, const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w) {
  using T = Tile<BN, PRECISE>;
  constexpr uint32_t kACols = T::kACols;
  constexpr int DG = T::kDG;
  constexpr uint32_t kBBytes = T::kBBytes, kStage = T::kStageBytes;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ float s_code2[NESTED ? 256 : 1];
  __shared__ __align__(8) uint64_t s_bar[3 * kMaxStages + 2 * kMaxASlots + 1];
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_abort;

  const int S = a.n_stages, SA = a.n_aslots;
  if (S <= SA || S > kMaxStages || SA <= DG || SA > kMaxASlots) return;  // uniform: before any barrier
  // 1024-byte aligned ring (the 128-byte swizzle pattern follows address bits 7-9)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t ring = (raw + 1023u) & ~1023u;
  unsigned char* const ring_ptr = smem_raw + (ring - raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // this CTA's K blocks: [kb_begin, kb_begin + kblocks) (the whole K unless split)
  const int kb_begin = int(blockIdx.z) * a.kb_per_split;
  const int kb_all = int(a.k / kBK);
  const int kblocks = (kb_all - kb_begin) < a.kb_per_split ? (kb_all - kb_begin) : a.kb_per_split;
  const int m0 = int(blockIdx.x) * BN;
  const int64_t n0 = int64_t(blockIdx.y) * kBM;
  const uint32_t bar0 = smem_u32(s_bar);
  auto tma_full = [&](int st) { return bar0 + 8u * uint32_t(st); };
  auto scale_full = [&](int st) { return bar0 + 8u * uint32_t(kMaxStages + st); };
  auto slot_empty = [&](int st) { return bar0 + 8u * uint32_t(2 * kMaxStages + st); };
  auto a_full = [&](int sa) { return bar0 + 8u * uint32_t(3 * kMaxStages + sa); };
  const uint32_t done = bar0 + 8u * uint32_t(3 * kMaxStages + 2 * kMaxASlots);

  if constexpr (NESTED) {
    for (int i = tid; i < 256; i += T::kThreads) s_code2[i] = __ldg(a.code2 + i);
  }
  if (tid == 0) {
    s_abort = 0;
    for (int st = 0; st < S; ++st) {
      mbar_init(tma_full(st), 1);
      mbar_init(scale_full(st), 32);
      mbar_init(slot_empty(st), 1);
    }
    for (int sa = 0; sa < SA; ++sa) mbar_init(a_full(sa), 4 * 32);
    mbar_init(done, 1);
    fence_mbar_init();
  }
  if (warp == T::kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(a.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;  // accumulator: columns [0, BN); A slot sa: BN + kACols sa

  if (warp == T::kWarpTma) {
    // -------------------------------------------------------- TMA producer
    // The warp runs the loop converged; lane 0 issues.
    int issued = 0;
    for (int kb = 0, st = 0, u = 0; kb < kblocks; ++kb) {
      if (__any_sync(0xffffffffu, s_abort)) break;
      if (u > 0 && !__all_sync(0xffffffffu, mbar_wait(slot_empty(st), uint32_t(u - 1) & 1u))) {
        s_abort = 1;
        break;
      }
      if (lane == 0) {
        const uint32_t slot = ring + uint32_t(st) * kStage;
        mbar_arrive_expect_tx(tma_full(st), kBBytes + kCodeBytes);
        tma_load_2d(slot, &tmap_x, (kb_begin + kb) * kBK, m0, tma_full(st));
        tma_load_2d(slot + kBBytes, &tmap_w, (kb_begin + kb) * (kBK / 2), int(n0), tma_full(st));
      }
      __syncwarp();
      issued = kb + 1;
      if (++st == S) { st = 0; ++u; }
    }
    // no copy may still be writing this CTA's shared memory when it exits
    for (int kb = issued > S ? issued - S : 0; kb < issued; ++kb) mbar_wait(tma_full(kb % S), uint32_t(kb / S) & 1u);
  } else if (warp == T::kWarpScale) {
    // --------------------------------------------------------- block scales
    // lane l copies rows l, l+32, l+64, l+96; blocksize 32 has two blocks per stage.
    // Slot layout: word[j][row] (float32 absmax, or the 4-byte-aligned word holding
    // the nested code) at 0, absmax2[j][row] at 2 * 128 * 4. The aligned word may
    // take up to 3 bytes from either side of absmax_q; they lie in the same aligned
    // word as a byte of absmax_q and are never used.
    const int nj = a.log2_bs == 5 ? 2 : 1;
    int64_t rowk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t r = n0 + lane + 32 * i;
      rowk[i] = (r < a.n_rows ? r : a.n_rows - 1) * a.k;
    }
    for (int kb = 0, st = 0, u = 0; kb < kblocks; ++kb) {
      if (s_abort) break;
      if (u > 0 && !mbar_wait(slot_empty(st), uint32_t(u - 1) & 1u)) { s_abort = 1; break; }
      const uint32_t sp = ring + uint32_t(st) * kStage + kBBytes + kCodeBytes;
      for (int j = 0; j < nj; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t blk = (rowk[i] + int64_t(kb_begin + kb) * kBK + 32 * j) >> a.log2_bs;
          const uint32_t o = uint32_t(j * kBM + lane + 32 * i) * 4u;
          if constexpr (NESTED) {
            cp_async4(sp + o, reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(a.absmax_q + blk) &
                                                          ~uintptr_t(3)));
            cp_async4(sp + 2u * kBM * 4u + o, a.absmax2 + ((a.block0 + blk) >> a.log2_bs2));
          } else {
            cp_async4(sp + o, a.absmax + blk);
          }
        }
      cp_async_arrive(scale_full(st));
      if (++st == S) { st = 0; ++u; }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight at exit
  } else if (warp == T::kWarpMma) {
    // ------------------------------------------------------------ MMA issue
    // The warp runs the loop converged; lane 0 issues the MMAs and commits (a
    // commit tracks the MMAs of the thread that executes it). a_full implies the
    // stage's x tile has landed: the decoders passed tma_full before arriving.
    const uint32_t idesc = instr_desc(Elem<XT>::kDtype == BNBQ_BF16, BN);
    for (int kb = 0, st = 0, sa = 0, ua = 0; kb < kblocks; ++kb) {
      if (!__all_sync(0xffffffffu, mbar_wait(a_full(sa), uint32_t(ua) & 1u))) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint64_t db = sw128_desc(ring + uint32_t(st) * kStage);
        const uint32_t ta = tmem + uint32_t(BN) + uint32_t(sa) * kACols;
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {  // K = 16 per MMA: 8 columns of A, 32 bytes of B's rows
          mma_ts(tmem, ta + uint32_t(8 * j), db + uint64_t(2 * j), idesc, (kb | j) ? 1u : 0u);
          if constexpr (PRECISE)  // the residual term, same B
            mma_ts(tmem, ta + kAColsPerStage + uint32_t(8 * j), db + uint64_t(2 * j), idesc, 1u);
        }
        mma_commit(slot_empty(st));  // ring slot st and A slot sa are free once these MMAs have read them
      }
      __syncwarp();
      if (++st == S) st = 0;
      if (++sa == SA) { sa = 0; ++ua; }
    }
    if (lane == 0) mma_commit(done);  // every MMA issued above has completed
    __syncwarp();
  } else {
    // ------------------------------------------------------------- decoders
    const int g = warp >> 2, wq = warp & 3;
    const int t = wq * 32 + lane;  // weight row n0 + t, tensor-memory lane t
    const uint32_t lane_addr = tmem + (uint32_t(wq * 32) << 16);
    const bool two = a.log2_bs == 5;
    const float offset = NESTED ? __ldg(a.offset) : 0.0f;
    const int64_t row = n0 + t < a.n_rows ? n0 + t : a.n_rows - 1;
    const int64_t rowk = row * a.k;
    // block scale j (0, or 1 for the second half of a blocksize-32 stage)
    auto scale = [&](const unsigned char* sp, int kb, int j) -> float {
      const uint32_t word = reinterpret_cast<const uint32_t*>(sp)[j * kBM + t];
      if constexpr (NESTED) {
        const int64_t blk = (rowk + int64_t(kb_begin + kb) * kBK + 32 * j) >> a.log2_bs;
        const uint32_t q = (word >> (8 * uint32_t(reinterpret_cast<uintptr_t>(a.absmax_q + blk) & 3))) & 0xffu;
        const float a2 = reinterpret_cast<const float*>(sp + 2 * kBM * 4)[j * kBM + t];
        return add_rn(mul_ftz(s_code2[q], a2), offset);
      } else {
        return __uint_as_float(word);
      }
    };
    // stage kb: ring slot st (use u), A slot sa; the A slot was last read by the
    // MMAs of stage kb - SA, whose commit completes ring slot pst (use pu < 0: none)
    int st = g, u = 0, sa = g, pst = g - SA + S, pu = -1;  // DG < SA < S
    for (int kb = g; kb < kblocks; kb += DG) {
      if (__any_sync(0xffffffffu, s_abort)) break;
      bool ok = mbar_wait(tma_full(st), uint32_t(u) & 1u) && mbar_wait(scale_full(st), uint32_t(u) & 1u);
      if (ok && pu >= 0) ok = mbar_wait(slot_empty(pst), uint32_t(pu) & 1u);
      if (!__all_sync(0xffffffffu, ok)) { s_abort = 1; break; }
      tc_fence_after();
      const unsigned char* slot = ring_ptr + size_t(st) * kStage;
      const unsigned char* sp = slot + kBBytes + kCodeBytes;
      const uint4 c0 = *reinterpret_cast<const uint4*>(slot + kBBytes + 32 * t);
      const uint4 c1 = *reinterpret_cast<const uint4*>(slot + kBBytes + 32 * t + 16);
      const uint32_t cols = lane_addr + uint32_t(BN) + uint32_t(sa) * kACols;
      uint32_t v[16], lo[4], hi[4];
      if constexpr (PRECISE) {
        // lane-private table: entry q of this lane at tab[q * 32 + lane] (bank = lane)
        uint32_t* const tab = reinterpret_cast<uint32_t*>(ring_ptr + size_t(S) * kStage) + warp * (16 * 32);
        auto build = [&](float a_) {
#pragma unroll
          for (int q = 0; q < 16; q += 2) {
            const float w0 = mul_ftz(kNF4Table[q], a_), w1 = mul_ftz(kNF4Table[q + 1], a_);
            const uint32_t p = pack2<XT>(w0, w1);  // hi terms, nearest
            const float2 h = unpack2x<XT>(p);
            const uint32_t r = pack2_rz<XT>(isinf(h.x) ? 0.0f : sub_rn(w0, h.x), isinf(h.y) ? 0.0f : sub_rn(w1, h.y));
            tab[q * 32 + lane] = prmt(p, r, 0x5410);        // (hi, lo) of entry q
            tab[(q + 1) * 32 + lane] = prmt(p, r, 0x7632);  // of entry q + 1
          }
        };
        // 4 code words (32 values) -> 16 words of hi pairs and 16 of lo pairs
        auto decode4 = [&](const uint32_t (&wd)[4], uint32_t (&vh)[16], uint32_t (&vl)[16]) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t e0 = tab[((wd[i] >> (8 * b + 4)) & 15u) * 32 + lane];  // value 2b: high nibble
              const uint32_t e1 = tab[((wd[i] >> (8 * b)) & 15u) * 32 + lane];
              vh[4 * i + b] = prmt(e0, e1, 0x5410);
              vl[4 * i + b] = prmt(e0, e1, 0x7632);
            }
        };
        const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w}, w1[4] = {c1.x, c1.y, c1.z, c1.w};
        uint32_t vl[16];
        build(scale(sp, kb, 0));
        decode4(w0, v, vl);
        tmem_st16(cols, v);
        tmem_st16(cols + kAColsPerStage, vl);
        if (two) build(scale(sp, kb, 1));
        decode4(w1, v, vl);
        tmem_st16(cols + 16, v);
        tmem_st16(cols + kAColsPerStage + 16, vl);
      } else {
        block_table<XT>(scale(sp, kb, 0), lo, hi);
        decode_word(c0.x, lo, hi, v + 0);
        decode_word(c0.y, lo, hi, v + 4);
        decode_word(c0.z, lo, hi, v + 8);
        decode_word(c0.w, lo, hi, v + 12);
        tmem_st16(cols, v);
        if (two) block_table<XT>(scale(sp, kb, 1), lo, hi);
        decode_word(c1.x, lo, hi, v + 0);
        decode_word(c1.y, lo, hi, v + 4);
        decode_word(c1.z, lo, hi, v + 8);
        decode_word(c1.w, lo, hi, v + 12);
        tmem_st16(cols + 16, v);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(a_full(sa));
      st += DG;
      if (st >= S) { st -= S; ++u; }
      sa += DG;
      if (sa >= SA) sa -= SA;
      pst += DG;
      if (pst >= S) { pst -= S; ++pu; }
    }
  }

  // -------------------------------------------------------------- epilogue
  const bool finished = mbar_wait(done, 0);  // all issued MMAs have completed
  const int C = int(gridDim.z);             // CTAs of the cluster along K
  const int g = warp >> 2, wq = warp & 3;
  const int64_t n = n0 + wq * 32 + lane;
  const uint32_t lane_addr = tmem + (uint32_t(wq * 32) << 16);
  // group g handles accumulator columns [g kCols, (g + 1) kCols), whole 16-column loads
  constexpr int kCols = BN / DG >= 16 ? BN / DG : 16;
  const int col_end = (g + 1) * kCols < BN ? (g + 1) * kCols : BN;
  if (C == 1) {
    if (warp < 4 * DG && __all_sync(0xffffffffu, finished && !s_abort)) {
      tc_fence_after();
#pragma unroll 1
      for (int col = g * kCols; col < col_end && m0 + col < a.m; col += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + uint32_t(col), r);
        if (n < a.n_rows) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int mrow = m0 + col + j;
            if (mrow < a.m) store_out<XT>(a.y, int64_t(mrow) * a.ldy + n, __uint_as_float(r[j]));
          }
        }
      }
    }
  } else {
    // K split over the cluster: ranks 1..C-1 store their partial tiles into
    // rank 0's ring (free once every CTA's main loop is over: first cluster
    // barrier); rank 0 adds them in rank order after the second barrier. Every
    // thread of every CTA passes both barriers on every path.
    const uint32_t rank = cluster_rank();
    tc_fence_before();
    cluster_sync();
    if (rank > 0 && warp < 4 * DG) {
      tc_fence_after();
      const uint32_t dst = map_to_rank(ring, 0);
#pragma unroll 1
      for (int col = g * kCols; col < col_end; col += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + uint32_t(col), r);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          st_cluster_f32(dst + 4u * uint32_t(((int(rank) - 1) * BN + col + j) * kBM + wq * 32 + lane),
                         __uint_as_float(r[j]));
      }
    }
    cluster_sync();
    if (rank == 0 && warp < 4 * DG && __all_sync(0xffffffffu, finished && !s_abort)) {
      tc_fence_after();
      const float* part = reinterpret_cast<const float*>(ring_ptr);
#pragma unroll 1
      for (int col = g * kCols; col < col_end && m0 + col < a.m; col += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + uint32_t(col), r);
        if (n < a.n_rows) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v = __uint_as_float(r[j]);
            for (int p = 1; p < C; ++p) v += part[((p - 1) * BN + col + j) * kBM + wq * 32 + lane];
            const int mrow = m0 + col + j;
            if (mrow < a.m) store_out<XT>(a.y, int64_t(mrow) * a.ldy + n, v);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == T::kWarpMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols));
  }
}

// --------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// 2-D row-major tensor map: `cols` x `rows` elements, row pitch `pitch` bytes.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t cols, uint64_t rows,
               uint64_t pitch, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  auto encode = get_encode();
  if (!encode) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t pow2_at_least(uint32_t v) {
  uint32_t c = 32;
  while (c < v) c <<= 1;
  return c;
}

template <typename XT, int BN, bool NESTED, bool PRECISE>
int launch_t(GemmArgs a, const void* x, const uint8_t* w, const DeviceInfo& di, cudaStream_t s, int max_split) {
  using T = Tile<BN, PRECISE>;
  CUtensorMap map_x, map_w;
  const CUtensorMapDataType dt =
      Elem<XT>::kDtype == BNBQ_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (!encode_2d(&map_x, dt, x, uint64_t(a.k), uint64_t(a.m), uint64_t(a.k) * 2, kBK, BN,
                 CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, uint64_t(a.k / 2), uint64_t(a.n_rows),
                 uint64_t(a.k / 2), kBK / 2, kBM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return BNBQ_ERR_CUDA;
  auto kern = gemm_kernel<XT, BN, NESTED, PRECISE>;
  int static_smem = 0;
  if (int st = kernel_static_smem(reinterpret_cast<const void*>(kern), &static_smem)) return st;
  // Paired tiles take just under half of the SM's shared memory (so that no
  // third CTA becomes resident and waits in tcgen05.alloc) and at most 256
  // tensor-memory columns each.
  const size_t smem_cap = T::kPair ? size_t(di.smem_optin) / 2 - size_t(static_smem) - 1024
                                   : size_t(di.smem_optin) - size_t(static_smem);
  int stages = int((smem_cap - 1024 - T::kTableBytes) / T::kStageBytes);
  stages = stages < kMaxStages ? stages : kMaxStages;
  const uint32_t tmem_budget = T::kPair ? 256u : 512u;
  int aslots = int((tmem_budget - uint32_t(BN)) / T::kACols);
  aslots = aslots < kMaxASlots ? aslots : kMaxASlots;
  aslots = aslots < stages - 1 ? aslots : stages - 1;
  if (stages <= aslots || aslots <= T::kDG) return BNBQ_ERR_UNSUPPORTED;
  a.n_stages = stages;
  a.n_aslots = aslots;
  a.tmem_cols = pow2_at_least(uint32_t(BN) + uint32_t(aslots) * T::kACols);
  const size_t smem = T::kPair ? (smem_cap / 1024) * 1024 : size_t(stages) * T::kStageBytes + T::kTableBytes + 1024;
  if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  // K split across a cluster when the tiles alone leave SMs idle: about one CTA
  // per SM, at most 8 (portable cluster size), each with >= 2 K blocks, and
  // the partial tiles of ranks 1.. must fit in rank 0's ring.
  const int64_t tiles = int64_t((a.m + BN - 1) / BN) * ((a.n_rows + kBM - 1) / kBM);
  const int kb_all = a.k / kBK;
  int split = tiles >= di.sm_count ? 1 : int(di.sm_count / tiles);
  split = split < max_split ? split : max_split;
  split = split < kb_all / 2 ? split : kb_all / 2;
  const int fit = 1 + int((size_t(stages) * T::kStageBytes) / (size_t(kBM) * BN * 4));
  split = split < fit ? split : fit;
  if (split < 1) split = 1;
  a.kb_per_split = (kb_all + split - 1) / split;
  split = (kb_all + a.kb_per_split - 1) / a.kb_per_split;  // no empty CTA
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((a.m + BN - 1) / BN), unsigned((a.n_rows + kBM - 1) / kBM), unsigned(split));
  cfg.blockDim = dim3(T::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = unsigned(split);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, map_x, map_w) != cudaSuccess) return BNBQ_ERR_CUDA;
  return launch_status();
}

template <typename XT, bool NESTED>
int launch_bn(const GemmArgs& a, const void* x, const uint8_t* w, const DeviceInfo& di, cudaStream_t s) {
  if (a.m <= 32) return launch_t<XT, 32, NESTED, false>(a, x, w, di, s, 8);
  if (a.m <= 64) return launch_t<XT, 64, NESTED, false>(a, x, w, di, s, 8);
  if (a.m <= 128) return launch_t<XT, 128, NESTED, false>(a, x, w, di, s, 8);
  return launch_t<XT, 256, NESTED, false>(a, x, w, di, s, 8);
}

}  // namespace

int gemm_wait_timeouts(unsigned int* out) { return read_wait_timeouts(out); }
int gemm_set_wait_limit(uint64_t ns) { return write_wait_limit(ns); }

// The GEMV's numerics on the tensor cores, for 1 <= m <= 32: every weight as
// the exact dequantized float32 value split into hi + lo terms of x's dtype,
// f32 accumulation, K split across a cluster to occupy the SMs. Returns
// BNBQ_ERR_UNSUPPORTED where the tile does not apply (K % 64, sizes).
int gemm_precise_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                        int32_t blocksize, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                        const float* code2, const float* offset, int32_t blocksize2, int64_t absmax2_block0,
                        void* y, int64_t ldy, cudaStream_t s) {
  if (m < 1 || m > 32 || (k % kBK) != 0 || n_rows > (int64_t(1) << 31) - kBM || (n_rows + kBM - 1) / kBM > 65535)
    return BNBQ_ERR_UNSUPPORTED;
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  GemmArgs a{};
  a.absmax_q = absmax_q; a.absmax = absmax; a.absmax2 = absmax2; a.code2 = code2; a.offset = offset;
  a.y = y; a.n_rows = n_rows; a.k = k; a.ldy = ldy; a.block0 = absmax2_block0; a.m = m;
  a.log2_bs = log2_exact(blocksize);
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  const bool nested = absmax_q != nullptr;
  if (dtype == BNBQ_BF16)
    return nested ? launch_t<__nv_bfloat16, 32, true, true>(a, x, w, di, s, 8)
                  : launch_t<__nv_bfloat16, 32, false, true>(a, x, w, di, s, 8);
  return nested ? launch_t<__half, 32, true, true>(a, x, w, di, s, 8)
                : launch_t<__half, 32, false, true>(a, x, w, di, s, 8);
}

// Arguments are validated by the caller (gemv_validate). Shapes outside the
// tile's reach (K not a multiple of 64, more than 2^31 - 128 weight rows or
// 65535 row tiles) run as GEMV passes of up to 20 rows of x each.
int gemm_launch(int dtype, const void* x, int32_t m, int32_t k, const uint8_t* w, int64_t n_rows,
                int32_t blocksize, const float* absmax, const uint8_t* absmax_q, const float* absmax2,
                const float* code2, const float* offset, int32_t blocksize2, int64_t absmax2_block0, void* y,
                int64_t ldy, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  GemmArgs a{};
  a.absmax_q = absmax_q; a.absmax = absmax; a.absmax2 = absmax2; a.code2 = code2; a.offset = offset;
  a.y = y; a.n_rows = n_rows; a.k = k; a.ldy = ldy; a.block0 = absmax2_block0; a.m = m;
  a.log2_bs = log2_exact(blocksize);
  a.log2_bs2 = absmax_q ? log2_exact(blocksize2) : 0;
  const int64_t n_tiles = (n_rows + kBM - 1) / kBM;
  int st = BNBQ_ERR_UNSUPPORTED;
  if ((k % kBK) == 0 && n_rows <= (int64_t(1) << 31) - kBM && n_tiles <= 65535) {
    const bool nested = absmax_q != nullptr;
    if (dtype == BNBQ_BF16)
      st = nested ? launch_bn<__nv_bfloat16, true>(a, x, w, di, s) : launch_bn<__nv_bfloat16, false>(a, x, w, di, s);
    else
      st = nested ? launch_bn<__half, true>(a, x, w, di, s) : launch_bn<__half, false>(a, x, w, di, s);
  }
  if (st != BNBQ_ERR_UNSUPPORTED) return st;
  const size_t esz = 2;
  for (int r0 = 0; r0 < m; r0 += BNBQ_GEMV_MAX_M) {
    const int mm = m - r0 < BNBQ_GEMV_MAX_M ? m - r0 : BNBQ_GEMV_MAX_M;
    st = gemv_launch(dtype, static_cast<const char*>(x) + size_t(r0) * size_t(k) * esz, mm, k, w, n_rows, blocksize,
                     absmax, absmax_q, absmax2, code2, offset, blocksize2, absmax2_block0,
                     static_cast<char*>(y) + size_t(r0) * size_t(ldy) * esz, ldy, s);
    if (st != BNBQ_OK) return st;
  }
  return BNBQ_OK;
}

}  // namespace bnbq
