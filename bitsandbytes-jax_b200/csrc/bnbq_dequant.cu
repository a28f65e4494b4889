// bnbq_dequant.cu -- blockwise dequantize (NF4 / 8-bit, plain and double-quantized).
//
// Element i decodes as  out[i] = T(mul.ftz(table[code_i], a_{i / bs}))
// (reference kernels/dequantize.py:39-69), with a_b either the stored float32
// absmax or, for a double-quantized array, the nested scale decoded in-kernel:
//   a_b = fl32(mul.ftz(code2[absmax_q[b]], absmax2[b >> log2 bs2]) + offset)
// which is bitwise the reference's chain (array.py:95-97, :107-108).
//
// Layout and mapping. The output is cut into 16-byte vectors (8 elements of a
// 16-bit type, 4 of float32); each thread of a persistent grid (a whole number
// of CTAs per SM) streams vectors with stride gridDim*blockDim, so every warp
// store is one fully coalesced 512-byte run and every code load a coalesced
// 64..256-byte run. Several vectors per thread per iteration keep loads in
// flight (unroll_for).
// bs >= 8 guarantees a vector never straddles two blocks.
// The NF4 table lives in shared memory (16 floats, conflict-free). The 8-bit
// codebook is replicated once per lane (256 x 32 floats): a lane reads its own
// copy, so a warp's 32 random code lookups hit 32 distinct banks.
// A partial last vector (n % EPV != 0) is finished by one thread with scalar
// loads and stores, so no byte outside the exact buffers is touched.
#include "bnbq_common.cuh"

namespace bnbq {
namespace {

constexpr int kThreads = 256;
// Output vectors per thread per iteration (their code loads are issued
// together): measured on config 3, 8 for 8-bit codes to 16-bit outputs and 2
// for float32 outputs (whose 16-byte vector holds only 4 elements) keep HBM
// busiest; NF4 (half the code bytes per vector) keeps 4.
template <typename OutT, bool NF4>
constexpr int unroll_for() { return NF4 ? 4 : (sizeof(OutT) == 4 ? 2 : 8); }

template <typename OutT>
struct Vec;  // 16 bytes of output
template <> struct Vec<float> {
  static constexpr int kEPV = 4;
  __device__ static uint4 pack(const float (&v)[4]) {
    return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                      __float_as_uint(v[3]));
  }
  __device__ static void store1(void* out, int64_t i, float v) { static_cast<float*>(out)[i] = v; }
};
template <> struct Vec<__nv_bfloat16> {
  static constexpr int kEPV = 8;
  __device__ static uint4 pack(const float (&v)[8]) {
    return make_uint4(pack2_bf16(v[0], v[1]), pack2_bf16(v[2], v[3]), pack2_bf16(v[4], v[5]),
                      pack2_bf16(v[6], v[7]));
  }
  __device__ static void store1(void* out, int64_t i, float v) {
    static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  }
};
template <> struct Vec<__half> {
  static constexpr int kEPV = 8;
  __device__ static uint4 pack(const float (&v)[8]) {
    return make_uint4(pack2_f16(v[0], v[1]), pack2_f16(v[2], v[3]), pack2_f16(v[4], v[5]),
                      pack2_f16(v[6], v[7]));
  }
  __device__ static void store1(void* out, int64_t i, float v) {
    static_cast<__half*>(out)[i] = __float2half_rn(v);
  }
};

struct DequantArgs {
  const uint8_t* q;
  const float* absmax;     // plain scales (nullptr when nested)
  const float* code;       // 8-bit codebook (nullptr for NF4)
  const uint8_t* absmax_q; // nested: 8-bit codes of the scales
  const float* absmax2;    // nested: second-level scales
  const float* code2;      // nested: second-level codebook
  const float* offset;     // nested: offset; plain 8-bit f32: optional post-add
  void* out;
  int64_t n;
  int log2_bs;
  int log2_bs2;
};

// Shared memory: NF4 -> 16-entry table; 8-bit -> lane-replicated codebook
// [256][32]; nested adds the 256-entry code2.
template <bool NF4, bool NESTED>
struct Smem {
  static constexpr int kTable = NF4 ? 16 : 256 * 32;
  static constexpr int kCode2 = NESTED ? 256 : 0;
  static constexpr size_t kBytes = sizeof(float) * (kTable + kCode2);
};

template <bool NESTED>
__device__ __forceinline__ float block_scale(const DequantArgs& a, const float* s_code2,
                                             int64_t blk, float offset) {
  if constexpr (NESTED) {
    const int q2 = __ldg(a.absmax_q + blk);
    return add_rn(mul_ftz(s_code2[q2], __ldg(a.absmax2 + (blk >> a.log2_bs2))), offset);
  } else {
    return __ldg(a.absmax + blk);
  }
}

template <typename OutT, bool NF4, bool NESTED, bool POSTADD>
__global__ void __launch_bounds__(kThreads)
dequant_kernel(DequantArgs a) {
  constexpr int EPV = Vec<OutT>::kEPV;
  constexpr int CB = NF4 ? EPV / 2 : EPV;  // code bytes per vector
  constexpr int kUnroll = unroll_for<OutT, NF4>();
  extern __shared__ float smem[];
  float* s_table = smem;
  float* s_code2 = smem + Smem<NF4, NESTED>::kTable;
  const int lane = threadIdx.x & 31;

  if constexpr (NF4) {
    if (threadIdx.x < 16) s_table[threadIdx.x] = kNF4Table[threadIdx.x];
  } else {
    for (int i = threadIdx.x; i < 256 * 32; i += kThreads) s_table[i] = __ldg(a.code + (i >> 5));
  }
  if constexpr (NESTED) {
    for (int i = threadIdx.x; i < 256; i += kThreads) s_code2[i] = __ldg(a.code2 + i);
  }
  __syncthreads();

  const float offset = (NESTED || POSTADD) ? __ldg(a.offset) : 0.0f;
  const int64_t nvec = a.n / EPV;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  const int shift = a.log2_bs - (EPV == 8 ? 3 : 2);  // vector index -> block index

  auto decode = [&](uint64_t codes, float scale, float (&v)[EPV]) {
#pragma unroll
    for (int j = 0; j < EPV; j += 2) {
      float t0, t1;
      if constexpr (NF4) {
        const uint32_t byte = uint32_t(codes >> (4 * j)) & 0xffu;
        t0 = s_table[byte >> 4];   // element j: high nibble (dequantize.py:59-62)
        t1 = s_table[byte & 15u];
      } else {
        t0 = s_table[((uint32_t(codes >> (8 * j)) & 0xffu) << 5) + lane];
        t1 = s_table[((uint32_t(codes >> (8 * j + 8)) & 0xffu) << 5) + lane];
      }
      const float2 r = mul_ftz2(make_float2(t0, t1), make_float2(scale, scale));
      v[j] = r.x;
      v[j + 1] = r.y;
      if constexpr (POSTADD) {
        v[j] = add_rn(v[j], offset);
        v[j + 1] = add_rn(v[j + 1], offset);
      }
    }
  };

  for (int64_t base = int64_t(blockIdx.x) * kThreads + threadIdx.x; base < nvec;
       base += stride * kUnroll) {
    uint64_t codes[kUnroll];
    float scale[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = base + u * stride;
      codes[u] = 0;
      scale[u] = 0.0f;
      if (v < nvec) {
        const uint8_t* src = a.q + v * CB;
        if constexpr (CB == 8) codes[u] = *reinterpret_cast<const uint64_t*>(src);
        else if constexpr (CB == 4) codes[u] = *reinterpret_cast<const uint32_t*>(src);
        else codes[u] = *reinterpret_cast<const uint16_t*>(src);
        scale[u] = block_scale<NESTED>(a, s_code2, v >> shift, offset);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = base + u * stride;
      if (v < nvec) {
        float vals[EPV];
        decode(codes[u], scale[u], vals);
        *reinterpret_cast<uint4*>(static_cast<char*>(a.out) + v * 16) = Vec<OutT>::pack(vals);
      }
    }
  }

  // ragged tail: fewer than EPV elements after the last whole vector
  if (blockIdx.x == 0 && threadIdx.x == 0 && nvec * EPV < a.n) {
    for (int64_t i = nvec * EPV; i < a.n; ++i) {
      float t;
      if constexpr (NF4) {
        const uint32_t byte = a.q[i >> 1];
        t = s_table[(i & 1) ? (byte & 15u) : (byte >> 4)];
      } else {
        t = s_table[(uint32_t(a.q[i]) << 5) + lane];
      }
      float v = mul_ftz(t, block_scale<NESTED>(a, s_code2, i >> a.log2_bs, offset));
      if constexpr (POSTADD) v = add_rn(v, offset);
      Vec<OutT>::store1(a.out, i, v);
    }
  }
}

template <typename OutT, bool NF4, bool NESTED, bool POSTADD>
int launch_t(const DequantArgs& a, cudaStream_t s) {
  DeviceInfo di;
  if (int st = device_info(&di)) return st;
  constexpr int EPV = Vec<OutT>::kEPV;
  auto kern = dequant_kernel<OutT, NF4, NESTED, POSTADD>;
  constexpr size_t smem = Smem<NF4, NESTED>::kBytes;
  if (smem > 48 * 1024)
    if (int st = kernel_reserve_smem(reinterpret_cast<const void*>(kern), int(smem))) return st;
  int per_sm = 0;
  if (int st = kernel_occupancy(reinterpret_cast<const void*>(kern), kThreads, smem, &per_sm)) return st;
  if (per_sm < 1) per_sm = 1;
  const int64_t nvec = a.n / EPV;
  constexpr int kUnroll = unroll_for<OutT, NF4>();
  const int64_t want = (nvec + int64_t(kThreads) * kUnroll - 1) / (int64_t(kThreads) * kUnroll);
  int64_t grid = int64_t(di.sm_count) * per_sm;
  if (want < grid) grid = want > 0 ? want : 1;
  kern<<<dim3(unsigned(grid)), dim3(kThreads), smem, s>>>(a);
  return launch_status();
}

template <bool NF4, bool NESTED, bool POSTADD>
int dispatch(int dtype, const DequantArgs& a, cudaStream_t s) {
  switch (dtype) {
    case BNBQ_F32: return launch_t<float, NF4, NESTED, POSTADD>(a, s);
    case BNBQ_F16: if constexpr (!POSTADD) return launch_t<__half, NF4, NESTED, false>(a, s); break;
    case BNBQ_BF16: if constexpr (!POSTADD) return launch_t<__nv_bfloat16, NF4, NESTED, false>(a, s); break;
    default: break;
  }
  return BNBQ_ERR_UNSUPPORTED;
}

int check_common(int dtype, const uint8_t* q, int64_t n, int32_t bs, void* out, int* log2_bs) {
  if (dtype != BNBQ_F32 && dtype != BNBQ_F16 && dtype != BNBQ_BF16) return BNBQ_ERR_UNSUPPORTED;
  if (n < 0) return BNBQ_ERR_INVALID;
  *log2_bs = log2_exact(bs);
  if (*log2_bs < 3) return BNBQ_ERR_INVALID;
  if (n > 0 && (!q || !out)) return BNBQ_ERR_INVALID;
  if (!aligned(q, 16) || !aligned(out, 16)) return BNBQ_ERR_MISALIGNED;
  return BNBQ_OK;
}

}  // namespace
}  // namespace bnbq

using namespace bnbq;

extern "C" int bnbq_dequantize_nf4(int dtype, const uint8_t* q, const float* absmax, int64_t n,
                                   int32_t blocksize, void* out, void* stream) {
  DequantArgs a{};
  if (int st = check_common(dtype, q, n, blocksize, out, &a.log2_bs)) return st;
  if (n == 0) return BNBQ_OK;
  if (!absmax) return BNBQ_ERR_INVALID;
  if (!aligned(absmax, 4)) return BNBQ_ERR_MISALIGNED;
  a.q = q; a.absmax = absmax; a.out = out; a.n = n;
  return dispatch<true, false, false>(dtype, a, static_cast<cudaStream_t>(stream));
}

extern "C" int bnbq_dequantize_blockwise(int dtype, const uint8_t* q, const float* absmax,
                                         const float* code, int64_t n, int32_t blocksize,
                                         const float* offset, void* out, void* stream) {
  DequantArgs a{};
  if (int st = check_common(dtype, q, n, blocksize, out, &a.log2_bs)) return st;
  if (n == 0) return BNBQ_OK;
  if (!absmax || !code) return BNBQ_ERR_INVALID;
  if (offset && dtype != BNBQ_F32) return BNBQ_ERR_UNSUPPORTED;
  if (!aligned(absmax, 4) || !aligned(code, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  a.q = q; a.absmax = absmax; a.code = code; a.offset = offset; a.out = out; a.n = n;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return offset ? dispatch<false, false, true>(dtype, a, s) : dispatch<false, false, false>(dtype, a, s);
}

extern "C" int bnbq_dequantize_nf4_nested(int dtype, const uint8_t* q, const uint8_t* absmax_q,
                                          const float* absmax2, const float* code2,
                                          const float* offset, int64_t n, int32_t blocksize,
                                          int32_t blocksize2, void* out, void* stream) {
  DequantArgs a{};
  if (int st = check_common(dtype, q, n, blocksize, out, &a.log2_bs)) return st;
  a.log2_bs2 = log2_exact(blocksize2);
  if (a.log2_bs2 < 0) return BNBQ_ERR_INVALID;
  if (n == 0) return BNBQ_OK;
  if (!absmax_q || !absmax2 || !code2 || !offset) return BNBQ_ERR_INVALID;
  if (!aligned(absmax2, 4) || !aligned(code2, 4) || !aligned(offset, 4)) return BNBQ_ERR_MISALIGNED;
  a.q = q; a.absmax_q = absmax_q; a.absmax2 = absmax2; a.code2 = code2; a.offset = offset;
  a.out = out; a.n = n;
  return dispatch<true, true, false>(dtype, a, static_cast<cudaStream_t>(stream));
}

extern "C" int bnbq_dequantize_blockwise_nested(int dtype, const uint8_t* q, const float* code,
                                                const uint8_t* absmax_q, const float* absmax2,
                                                const float* code2, const float* offset, int64_t n,
                                                int32_t blocksize, int32_t blocksize2, void* out,
                                                void* stream) {
  DequantArgs a{};
  if (int st = check_common(dtype, q, n, blocksize, out, &a.log2_bs)) return st;
  a.log2_bs2 = log2_exact(blocksize2);
  if (a.log2_bs2 < 0) return BNBQ_ERR_INVALID;
  if (n == 0) return BNBQ_OK;
  if (!code || !absmax_q || !absmax2 || !code2 || !offset) return BNBQ_ERR_INVALID;
  if (!aligned(code, 4) || !aligned(absmax2, 4) || !aligned(code2, 4) || !aligned(offset, 4))
    return BNBQ_ERR_MISALIGNED;
  a.q = q; a.code = code; a.absmax_q = absmax_q; a.absmax2 = absmax2; a.code2 = code2;
  a.offset = offset; a.out = out; a.n = n;
  return dispatch<false, true, false>(dtype, a, static_cast<cudaStream_t>(stream));
}
