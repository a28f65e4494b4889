// A minimal stand-in for the subset of jaxlib's xla/ffi/api/ffi.h that
// csrc/ffi_xla.cc uses, written from the API's published shape (class and
// method names, handler binding by template chain). It exists only so that a
// CPU test can type-check the handlers' calls into include/bnbq.h with
// g++ -fsyntax-only where jaxlib is absent; it is not the real API and
// nothing links against it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace xla::ffi {

enum class DataType { INVALID, PRED, S8, S16, S32, S64, U8, U16, U32, U64, F16, F32, F64, BF16 };
enum class ErrorCode { kOk, kInvalidArgument, kUnimplemented, kInternal };

class Error {
 public:
  Error() = default;
  Error(ErrorCode code, std::string message) : code_(code), message_(std::move(message)) {}
  static Error Success() { return Error(); }

 private:
  ErrorCode code_ = ErrorCode::kOk;
  std::string message_;
};

template <typename T>
struct Span {
  const T* data;
  size_t n;
  size_t size() const { return n; }
  const T& operator[](size_t i) const { return data[i]; }
};

class AnyBuffer {
 public:
  DataType element_type() const { return type_; }
  void* untyped_data() const { return data_; }
  size_t element_count() const { return count_; }
  size_t size_bytes() const { return bytes_; }
  Span<int64_t> dimensions() const { return {dims_.data(), dims_.size()}; }

 private:
  DataType type_ = DataType::INVALID;
  void* data_ = nullptr;
  size_t count_ = 0, bytes_ = 0;
  std::vector<int64_t> dims_;
};

template <DataType T>
struct NativeType;
template <>
struct NativeType<DataType::U8> {
  using type = uint8_t;
};
template <>
struct NativeType<DataType::F32> {
  using type = float;
};

constexpr DataType U8 = DataType::U8;
constexpr DataType F32 = DataType::F32;

template <DataType T>
class Buffer {
 public:
  using Native = typename NativeType<T>::type;
  Native* typed_data() const { return data_; }
  void* untyped_data() const { return data_; }
  size_t element_count() const { return count_; }
  size_t size_bytes() const { return count_ * sizeof(Native); }

 private:
  Native* data_ = nullptr;
  size_t count_ = 0;
};

template <typename T>
class Result {
 public:
  T* operator->() { return &value_; }

 private:
  T value_;
};

template <typename T>
struct PlatformStream {};

struct Binding {
  template <typename T>
  Binding Ctx() const { return *this; }
  template <typename T>
  Binding Arg() const { return *this; }
  template <typename T>
  Binding Ret() const { return *this; }
  template <typename T>
  Binding Attr(const char*) const { return *this; }
};

struct Ffi {
  static Binding Bind() { return {}; }
};

}  // namespace xla::ffi

// The real macro defines an exported handler symbol bound to `impl`; here it
// only takes the handler's address, so an undefined name still fails.
#define XLA_FFI_DEFINE_HANDLER_SYMBOL(name, impl, binding) \
  extern "C" const void* name##_stub_ref() {               \
    (void)(binding);                                       \
    return reinterpret_cast<const void*>(&impl);           \
  }
