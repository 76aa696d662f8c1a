// KDA chunked gated-delta-rule forward (sm_100a).
#include "b2_common.cuh"

extern "C" size_t b2_kda_workspace_size(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t) { return 0; }

extern "C" int b2_kda_fwd(const void*, const void*, const void*, const float*, const void*, const float*,
                          void*, float*, void*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float,
                          int, void*) {
  b2::set_error("kda_fwd: not built yet");
  return B2_ERR_UNSUPPORTED;
}
