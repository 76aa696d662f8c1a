// FlashAttention forward (sm_100a).
#include "b2_common.cuh"

extern "C" int b2_flash_attn_fwd(const void*, const void*, const void*, void*, int64_t, int64_t, int64_t,
                                 int64_t, int64_t, int64_t, const int64_t*, const int64_t*, const int64_t*,
                                 const int64_t*, float, int, int, void*) {
  b2::set_error("flash_attn_fwd: not built yet");
  return B2_ERR_UNSUPPORTED;
}
