// ffi_xla.cc -- XLA FFI custom-call handlers over the C ABI (include/bnbq.h),
// the binding that replaces the reference's cutejax.call sites:
//   kernels/quantize.py:226-233    (nf4=True / nf4=False)  -> BnbqQuantizeNf4 / BnbqQuantizeBlockwise
//   array.py:200                   (jnp.mean of absmax)   -> BnbqAbsmaxMean
//   kernels/dequantize.py:110-116  (nf4 / 8-bit)          -> BnbqDequantizeNf4 / BnbqDequantizeBlockwise
//   array.py:95-108                (nested decode chain)  -> BnbqDequantizeNf4Nested / BnbqDequantizeBlockwiseNested
//   kernels/gemv.py:195-204 and _matmul.py:46-60 (GEMV, and the M > 20 route) -> BnbqMatmulNf4
// and three with no cutejax.call of their own in the reference:
//   _matmul.py:74-79 -> 58-59  (8-bit weights: the dequantize fallback)   -> BnbqGemvBlockwise
//   _matmul.py:67-68           (the custom VJP's g @ w.dequantize())      -> BnbqGemvTNf4
//   array.py:199-202           (quantize_nf4, jnp.mean, quantize_blockwise) -> BnbqQuantizeNf4Dq
//
// Built by build.py only where jaxlib's FFI headers are found
// (jax.ffi.include_dir(), or the BNBQ_XLA_FFI_INCLUDE environment variable),
// into libbnbq_xla.so linked against libbnbq.so; the image this package is
// developed on has no jaxlib, so there it is not compiled.
//
// Every handler is stateless: it reads its buffers' element type and sizes,
// passes device pointers and XLA's stream to one C-ABI call and maps the
// status to an FFI error. Nothing is allocated: the matmul's workspace (the
// table GEMV's split-K partials; bnbq_gemv_workspace_bytes) is an extra
// result buffer that XLA allocates and the caller discards.
#include <cuda_runtime_api.h>

#include <cstdint>
#include <string>

#include "bnbq.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error Check(int status, const char* what) {
  if (status == BNBQ_OK) return ffi::Error::Success();
  const std::string msg = std::string(what) + ": " + bnbq_error_string(status);
  switch (status) {
    case BNBQ_ERR_UNSUPPORTED:
      return ffi::Error(ffi::ErrorCode::kUnimplemented, msg);
    case BNBQ_ERR_CUDA:
      return ffi::Error(ffi::ErrorCode::kInternal, msg);
    default:
      return ffi::Error(ffi::ErrorCode::kInvalidArgument, msg);
  }
}

// The C ABI's dtype code of a 16/32-bit float buffer; -1 for anything else.
int DtypeOf(ffi::DataType t) {
  switch (t) {
    case ffi::DataType::F32: return BNBQ_F32;
    case ffi::DataType::F16: return BNBQ_F16;
    case ffi::DataType::BF16: return BNBQ_BF16;
    default: return -1;
  }
}

ffi::Error BadType(const char* what) {
  return ffi::Error(ffi::ErrorCode::kUnimplemented, std::string(what) + ": unsupported element type");
}

// ------------------------------------------------------------- quantize

ffi::Error QuantizeNf4(cudaStream_t s, ffi::AnyBuffer x, ffi::Result<ffi::Buffer<ffi::U8>> q,
                       ffi::Result<ffi::Buffer<ffi::F32>> absmax, int64_t blocksize) {
  const int dt = DtypeOf(x.element_type());
  if (dt < 0) return BadType("quantize_nf4");
  return Check(bnbq_quantize_nf4(dt, x.untyped_data(), int64_t(x.element_count()), int32_t(blocksize),
                                 q->typed_data(), absmax->typed_data(), s),
               "quantize_nf4");
}

// `offset` holds one float32 subtracted from x before the block max (the
// centring of a nested absmax); an empty buffer means none.
ffi::Error QuantizeBlockwise(cudaStream_t s, ffi::AnyBuffer x, ffi::Buffer<ffi::F32> code,
                             ffi::Buffer<ffi::F32> offset, ffi::Result<ffi::Buffer<ffi::U8>> q,
                             ffi::Result<ffi::Buffer<ffi::F32>> absmax, int64_t blocksize) {
  const int dt = DtypeOf(x.element_type());
  if (dt < 0) return BadType("quantize_blockwise");
  const float* off = offset.element_count() ? offset.typed_data() : nullptr;
  return Check(bnbq_quantize_blockwise(dt, x.untyped_data(), int64_t(x.element_count()), int32_t(blocksize),
                                       code.typed_data(), off, q->typed_data(), absmax->typed_data(), s),
               "quantize_blockwise");
}

ffi::Error AbsmaxMean(cudaStream_t s, ffi::Buffer<ffi::F32> absmax, ffi::Result<ffi::Buffer<ffi::F32>> offset) {
  return Check(bnbq_absmax_mean(absmax.typed_data(), int64_t(absmax.element_count()), offset->typed_data(), s),
               "absmax_mean");
}

// ----------------------------------------------------------- dequantize

ffi::Error DequantizeNf4(cudaStream_t s, ffi::Buffer<ffi::U8> q, ffi::Buffer<ffi::F32> absmax,
                         ffi::Result<ffi::AnyBuffer> out, int64_t blocksize) {
  const int dt = DtypeOf(out->element_type());
  if (dt < 0) return BadType("dequantize_nf4");
  return Check(bnbq_dequantize_nf4(dt, q.typed_data(), absmax.typed_data(), int64_t(out->element_count()),
                                   int32_t(blocksize), out->untyped_data(), s),
               "dequantize_nf4");
}

ffi::Error DequantizeBlockwise(cudaStream_t s, ffi::Buffer<ffi::U8> q, ffi::Buffer<ffi::F32> absmax,
                               ffi::Buffer<ffi::F32> code, ffi::Buffer<ffi::F32> offset,
                               ffi::Result<ffi::AnyBuffer> out, int64_t blocksize) {
  const int dt = DtypeOf(out->element_type());
  if (dt < 0) return BadType("dequantize_blockwise");
  const float* off = offset.element_count() ? offset.typed_data() : nullptr;
  return Check(bnbq_dequantize_blockwise(dt, q.typed_data(), absmax.typed_data(), code.typed_data(),
                                         int64_t(out->element_count()), int32_t(blocksize), off,
                                         out->untyped_data(), s),
               "dequantize_blockwise");
}

ffi::Error DequantizeNf4Nested(cudaStream_t s, ffi::Buffer<ffi::U8> q, ffi::Buffer<ffi::U8> absmax_q,
                               ffi::Buffer<ffi::F32> absmax2, ffi::Buffer<ffi::F32> code2,
                               ffi::Buffer<ffi::F32> offset, ffi::Result<ffi::AnyBuffer> out, int64_t blocksize,
                               int64_t blocksize2) {
  const int dt = DtypeOf(out->element_type());
  if (dt < 0) return BadType("dequantize_nf4_nested");
  return Check(bnbq_dequantize_nf4_nested(dt, q.typed_data(), absmax_q.typed_data(), absmax2.typed_data(),
                                          code2.typed_data(), offset.typed_data(), int64_t(out->element_count()),
                                          int32_t(blocksize), int32_t(blocksize2), out->untyped_data(), s),
               "dequantize_nf4_nested");
}

ffi::Error DequantizeBlockwiseNested(cudaStream_t s, ffi::Buffer<ffi::U8> q, ffi::Buffer<ffi::F32> code,
                                     ffi::Buffer<ffi::U8> absmax_q, ffi::Buffer<ffi::F32> absmax2,
                                     ffi::Buffer<ffi::F32> code2, ffi::Buffer<ffi::F32> offset,
                                     ffi::Result<ffi::AnyBuffer> out, int64_t blocksize, int64_t blocksize2) {
  const int dt = DtypeOf(out->element_type());
  if (dt < 0) return BadType("dequantize_blockwise_nested");
  return Check(bnbq_dequantize_blockwise_nested(dt, q.typed_data(), code.typed_data(), absmax_q.typed_data(),
                                                absmax2.typed_data(), code2.typed_data(), offset.typed_data(),
                                                int64_t(out->element_count()), int32_t(blocksize),
                                                int32_t(blocksize2), out->untyped_data(), s),
               "dequantize_blockwise_nested");
}

// --------------------------------------------------------------- matmul

// y (M, n_rows) = x (M, K) @ W.T. `absmax` is the float32 scales when
// `nested` is 0, else the uint8 codes of the double-quantized scales with
// absmax2 / code2 / offset (the unused buffers may be empty). `workspace` is
// a uint8 result of bnbq_gemv_workspace_bytes(M, K, n_rows) bytes (may be
// empty: the kernels without split-K partials run then).
ffi::Error MatmulNf4(cudaStream_t s, ffi::AnyBuffer x, ffi::Buffer<ffi::U8> w, ffi::AnyBuffer absmax,
                     ffi::Buffer<ffi::F32> absmax2, ffi::Buffer<ffi::F32> code2, ffi::Buffer<ffi::F32> offset,
                     ffi::Result<ffi::AnyBuffer> y, ffi::Result<ffi::Buffer<ffi::U8>> workspace, int64_t n_rows,
                     int64_t blocksize, int64_t nested, int64_t blocksize2) {
  const int dt = DtypeOf(x.element_type());
  if (dt != BNBQ_F16 && dt != BNBQ_BF16) return BadType("matmul_nf4");
  const auto dims = x.dimensions();
  if (dims.size() != 2) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "matmul_nf4: x must be (M, K)");
  const int32_t m = int32_t(dims[0]), k = int32_t(dims[1]);
  const float* a = nested ? nullptr : static_cast<const float*>(absmax.untyped_data());
  const uint8_t* aq = nested ? static_cast<const uint8_t*>(absmax.untyped_data()) : nullptr;
  return Check(bnbq_matmul_nf4_ws(dt, x.untyped_data(), m, k, w.typed_data(), n_rows, int32_t(blocksize), a, aq,
                                  nested ? absmax2.typed_data() : nullptr, nested ? code2.typed_data() : nullptr,
                                  nested ? offset.typed_data() : nullptr, nested ? int32_t(blocksize2) : 0, 0,
                                  y->untyped_data(), n_rows, workspace->untyped_data(),
                                  int64_t(workspace->size_bytes()), s),
               "matmul_nf4");
}

// y (M, n_rows) = x (M, K) @ W.T for an 8-bit blockwise weight with codebook
// `code`; scales as MatmulNf4. `workspace`: a uint8 result of
// bnbq_gemv_blockwise_workspace_bytes(M, K, n_rows) bytes.
ffi::Error GemvBlockwise(cudaStream_t s, ffi::AnyBuffer x, ffi::Buffer<ffi::U8> w, ffi::Buffer<ffi::F32> code,
                         ffi::AnyBuffer absmax, ffi::Buffer<ffi::F32> absmax2, ffi::Buffer<ffi::F32> code2,
                         ffi::Buffer<ffi::F32> offset, ffi::Result<ffi::AnyBuffer> y,
                         ffi::Result<ffi::Buffer<ffi::U8>> workspace, int64_t n_rows, int64_t blocksize,
                         int64_t nested, int64_t blocksize2) {
  const int dt = DtypeOf(x.element_type());
  if (dt != BNBQ_F16 && dt != BNBQ_BF16) return BadType("gemv_blockwise");
  const auto dims = x.dimensions();
  if (dims.size() != 2) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "gemv_blockwise: x must be (M, K)");
  const int32_t m = int32_t(dims[0]), k = int32_t(dims[1]);
  const float* a = nested ? nullptr : static_cast<const float*>(absmax.untyped_data());
  const uint8_t* aq = nested ? static_cast<const uint8_t*>(absmax.untyped_data()) : nullptr;
  return Check(bnbq_gemv_blockwise_ws(dt, x.untyped_data(), m, k, w.typed_data(), n_rows, int32_t(blocksize),
                                      code.typed_data(), a, aq, nested ? absmax2.typed_data() : nullptr,
                                      nested ? code2.typed_data() : nullptr, nested ? offset.typed_data() : nullptr,
                                      nested ? int32_t(blocksize2) : 0, 0, y->untyped_data(), n_rows,
                                      workspace->untyped_data(), int64_t(workspace->size_bytes()), s),
               "gemv_blockwise");
}

// out (M, K) = g (M, n_rows) @ W for an NF4 weight of n_rows x K: the VJP's
// backward for up to 4 rows of g. `workspace`: a uint8 result of
// bnbq_gemv_t_nf4_workspace_bytes(M, K, n_rows) bytes.
ffi::Error GemvTNf4(cudaStream_t s, ffi::AnyBuffer g, ffi::Buffer<ffi::U8> w, ffi::AnyBuffer absmax,
                    ffi::Buffer<ffi::F32> absmax2, ffi::Buffer<ffi::F32> code2, ffi::Buffer<ffi::F32> offset,
                    ffi::Result<ffi::AnyBuffer> out, ffi::Result<ffi::Buffer<ffi::U8>> workspace, int64_t k,
                    int64_t blocksize, int64_t nested, int64_t blocksize2) {
  const int dt = DtypeOf(g.element_type());
  if (dt != BNBQ_F16 && dt != BNBQ_BF16) return BadType("gemv_t_nf4");
  const auto dims = g.dimensions();
  if (dims.size() != 2) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "gemv_t_nf4: g must be (M, N)");
  const int32_t m = int32_t(dims[0]);
  const int64_t n_rows = dims[1];
  const float* a = nested ? nullptr : static_cast<const float*>(absmax.untyped_data());
  const uint8_t* aq = nested ? static_cast<const uint8_t*>(absmax.untyped_data()) : nullptr;
  return Check(bnbq_gemv_t_nf4_ws(dt, g.untyped_data(), m, n_rows, n_rows, int32_t(k), w.typed_data(),
                                  int32_t(blocksize), a, aq, nested ? absmax2.typed_data() : nullptr,
                                  nested ? code2.typed_data() : nullptr, nested ? offset.typed_data() : nullptr,
                                  nested ? int32_t(blocksize2) : 0, 0, out->untyped_data(), k,
                                  workspace->untyped_data(), int64_t(workspace->size_bytes()), s),
               "gemv_t_nf4");
}

// quantize(x, "nf4", blocksize, double_quant=True) in one launch: codes,
// absmax, the nested codes and scales and the offset. `workspace`: a uint8
// result of bnbq_quantize_nf4_dq_workspace_bytes() bytes.
ffi::Error QuantizeNf4Dq(cudaStream_t s, ffi::AnyBuffer x, ffi::Buffer<ffi::F32> code2,
                         ffi::Result<ffi::Buffer<ffi::U8>> q, ffi::Result<ffi::Buffer<ffi::F32>> absmax,
                         ffi::Result<ffi::Buffer<ffi::U8>> absmax_q, ffi::Result<ffi::Buffer<ffi::F32>> absmax2,
                         ffi::Result<ffi::Buffer<ffi::F32>> offset, ffi::Result<ffi::Buffer<ffi::U8>> workspace,
                         int64_t blocksize, int64_t blocksize2) {
  const int dt = DtypeOf(x.element_type());
  if (dt < 0) return BadType("quantize_nf4_dq");
  return Check(bnbq_quantize_nf4_dq(dt, x.untyped_data(), int64_t(x.element_count()), int32_t(blocksize),
                                    code2.typed_data(), int32_t(blocksize2), q->typed_data(), absmax->typed_data(),
                                    absmax_q->typed_data(), absmax2->typed_data(), offset->typed_data(),
                                    workspace->untyped_data(), int64_t(workspace->size_bytes()), s),
               "quantize_nf4_dq");
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_quantize_nf4_ffi, QuantizeNf4,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("blocksize"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_quantize_blockwise_ffi, QuantizeBlockwise,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int64_t>("blocksize"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_absmax_mean_ffi, AbsmaxMean,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>());

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_dequantize_nf4_ffi, DequantizeNf4,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("blocksize"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_dequantize_blockwise_ffi, DequantizeBlockwise,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("blocksize"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_dequantize_nf4_nested_ffi, DequantizeNf4Nested,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("blocksize2"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_dequantize_blockwise_nested_ffi, DequantizeBlockwiseNested,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("blocksize2"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_matmul_nf4_ffi, MatmulNf4,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int64_t>("n_rows")
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("nested")
                                  .Attr<int64_t>("blocksize2"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_gemv_blockwise_ffi, GemvBlockwise,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int64_t>("n_rows")
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("nested")
                                  .Attr<int64_t>("blocksize2"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_gemv_t_nf4_ffi, GemvTNf4,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int64_t>("k")
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("nested")
                                  .Attr<int64_t>("blocksize2"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(bnbq_quantize_nf4_dq_ffi, QuantizeNf4Dq,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int64_t>("blocksize")
                                  .Attr<int64_t>("blocksize2"));
