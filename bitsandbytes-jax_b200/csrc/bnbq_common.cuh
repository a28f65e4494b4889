// bnbq_common.cuh -- shared device helpers for the sm_100a quantization kernels.
//
// The fast-math operations bitsandbytes' kernels are built with (and which the
// reference spells out in PTX, src/bnb_jax/kernels/_ptx.py:15-33) are written
// here as explicit PTX with an explicit rounding mode, so that ptxas can neither
// contract them into FMAs nor change their flush behaviour:
//   mul.rn.ftz.f32 / .f32x2, abs.ftz + max.ftz, rcp.approx.ftz.f32.
// Additions that the reference performs in IEEE float32 (XLA adds) use
// add.rn.f32 / sub.rn.f32 without .ftz.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bnbq.h"

namespace bnbq {

// ----------------------------------------------------------------- PTX math

__device__ __forceinline__ float mul_ftz(float a, float b) {
  float r;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Two independent mul.rn.ftz.f32 in one packed sm_100 instruction.
__device__ __forceinline__ float2 mul_ftz2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pr;\n\t"
      "mov.b64 pa, {%2, %3};\n\t"
      "mov.b64 pb, {%4, %5};\n\t"
      "mul.rn.ftz.f32x2 pr, pa, pb;\n\t"
      "mov.b64 {%0, %1}, pr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// acc += a * b on two lanes, one rounding each (fma.rn.f32x2).
__device__ __forceinline__ void fma2(float2& acc, float2 a, float2 b) {
  asm("{\n\t.reg .b64 pa, pb, pc;\n\t"
      "mov.b64 pa, {%2, %3};\n\t"
      "mov.b64 pb, {%4, %5};\n\t"
      "mov.b64 pc, {%0, %1};\n\t"
      "fma.rn.f32x2 pc, pa, pb, pc;\n\t"
      "mov.b64 {%0, %1}, pc;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
}

// fmaxf(m, fabsf(x)) with subnormals flushed (kernels/_ptx.py:25-28).
__device__ __forceinline__ float max_abs_ftz(float m, float x) {
  float r;
  asm("{\n\t.reg .f32 t;\n\tabs.ftz.f32 t, %2;\n\tmax.ftz.f32 %0, %1, t;\n\t}"
      : "=f"(r) : "f"(m), "f"(x));
  return r;
}

__device__ __forceinline__ float max_ftz(float a, float b) {
  float r;
  asm("max.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float rcp_approx_ftz(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

__device__ __forceinline__ float add_rn(float a, float b) {
  float r;
  asm("add.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float sub_rn(float a, float b) {
  float r;
  asm("sub.rn.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// ------------------------------------------------------------ element types

template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kDtype = BNBQ_F32;
  __device__ static float to_f32(float v) { return v; }
};
template <> struct Elem<__half> {
  static constexpr int kDtype = BNBQ_F16;
  __device__ static float to_f32(__half v) { return __half2float(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kDtype = BNBQ_BF16;
  __device__ static float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
};

// Two float32 -> one packed pair, round to nearest (cvt.rn.{bf16,f16}x2.f32):
// `lo` lands in the low half (lower address), `hi` in the high half.
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack2_f16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Unpack a 32-bit word holding two 16-bit elements into float32 (exact).
__device__ __forceinline__ float2 unpack2_bf16(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float2 unpack2_f16(uint32_t w) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

// ----------------------------------------------------------------- constants

// NF4 table (reference kernels/dequantize.py:27-32).
__device__ __constant__ static const float kNF4Table[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

// NF4 decision thresholds as float32 bits (reference kernels/quantize.py:46-50).
__device__ __constant__ static const uint32_t kNF4ThresholdBits[15] = {
    0xbf591cd9u, 0xbf1c5270u, 0xbeeb8480u, 0xbeadea76u, 0xbe703cecu,
    0xbe0d38bcu, 0xbd3a7871u, 0x3d22faffu, 0x3df64863u, 0x3e5067e0u,
    0x3e9582d4u, 0x3ec753f9u, 0x3f006d03u, 0x3f248dafu, 0x3f5c89d9u};

// --------------------------------------------------------------- host side

struct DeviceInfo {
  int sm_count = 0;
  int smem_optin = 0;  // max dynamic shared memory per block (opt-in), bytes
  int cc_major = 0;
  int cc_minor = 0;
};

// Per-device attributes, queried once per device (thread-safe).
int device_info(DeviceInfo* out);

// Kernel launch attributes on the current device, each CUDA query made once
// per (kernel, device) and then served from a table (a launch then costs no
// attribute round trips): the kernel's static shared memory; its maximum
// dynamic shared memory raised to at least `bytes` (set only when it grows);
// its resident blocks per SM for (threads, dynamic bytes).
int kernel_static_smem(const void* fn, int* bytes);
int kernel_reserve_smem(const void* fn, int bytes);
int kernel_occupancy(const void* fn, int threads, size_t dyn_bytes, int* per_sm);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int l = 0;
  while ((int64_t(1) << l) < v) ++l;
  return l;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BNBQ_OK : BNBQ_ERR_CUDA;
}

}  // namespace bnbq
