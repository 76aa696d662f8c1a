// Prefill W4A16 / W8A16 GEMM on tcgen05 (sm_100a).  Until the tensor-core
// pipeline lands these report UNSUPPORTED and the caller uses the generic
// CUDA kernel.
#include "b2_common.cuh"

int b2_detail_w4_gemm(const void*, const void*, void*, const void*, const void*,
                      int64_t, int64_t, int64_t, int64_t, int, cudaStream_t) {
  return B2_ERR_UNSUPPORTED;
}

int b2_detail_w8_gemm(const void*, const void*, void*, const void*, const void*,
                      int64_t, int64_t, int64_t, int, cudaStream_t) {
  return B2_ERR_UNSUPPORTED;
}
