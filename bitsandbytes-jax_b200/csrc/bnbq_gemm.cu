// bnbq_gemm.cu -- fused NF4 dequantize-GEMM for M > 20 (tcgen05 / TMEM).
#include "bnbq_common.cuh"

namespace bnbq {

int gemm_launch(int, const void*, int32_t, int32_t, const uint8_t*, int64_t, int32_t, const float*,
                const uint8_t*, const float*, const float*, const float*, int32_t, int64_t, void*,
                int64_t, cudaStream_t) {
  return BNBQ_ERR_UNSUPPORTED;
}

}  // namespace bnbq
