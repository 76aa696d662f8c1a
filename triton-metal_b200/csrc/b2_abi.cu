// C-ABI bookkeeping: version, the thread-local last-error message, the
// device error word of the bounded waits, and tensor-map encoding.
#include "b2_common.cuh"
#include <string.h>

namespace b2 {
// Device-side error word: bounded waits record a non-zero code here.
__device__ unsigned int g_device_error = 0;

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

unsigned int* device_error_word() {
  static unsigned int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<unsigned int*>(p);
  }
  return cache[dev];
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cache[dev]) cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev);
  return cache[dev] > 0 ? cache[dev] : 148;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return false;
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u", (int)r,
              (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
    return false;
  }
  return true;
}
}  // namespace b2

extern "C" int b2_version(void) { return 10000; }  // 1.0.0

extern "C" const char* b2_last_error(void) { return b2::g_last_error; }

// Synchronise the stream, then read and clear the device error word.
extern "C" int b2_device_error(void* stream, unsigned int* code) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) {
    b2::set_error("device_error: stream sync failed: %s", cudaGetErrorString(e));
    return B2_ERR_LAUNCH;
  }
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, b2::g_device_error, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(b2::g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) {
    b2::set_error("device_error: %s", cudaGetErrorString(e));
    return B2_ERR_LAUNCH;
  }
  if (code) *code = v;
  if (v) {
    b2::set_error("a bounded device wait ran out (code 0x%x)", v);
    return B2_ERR_TIMEOUT;
  }
  return B2_OK;
}
