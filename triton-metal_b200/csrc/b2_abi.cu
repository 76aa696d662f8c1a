// C-ABI bookkeeping: version, the thread-local last-error message, the
// device error word of the bounded waits, and tensor-map encoding.
#include "b2_common.cuh"
#include <string.h>
#include <mutex>

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

// A tensor map encodes only the address, shape, strides, box and modes, so a
// map built once is valid for every later call with the same arguments.  A
// small per-thread direct-mapped cache saves the driver call (~1 us of host
// time) on the repeated small launches of a decode loop.
namespace {
struct TmapKey {
  const void* base;
  uint64_t inner, outer, stride;
  uint32_t box_inner, box_outer;
  int dt, swizzle;
  bool operator==(const TmapKey& o) const {
    return base == o.base && inner == o.inner && outer == o.outer && stride == o.stride &&
           box_inner == o.box_inner && box_outer == o.box_outer && dt == o.dt && swizzle == o.swizzle;
  }
};
struct TmapEntry {
  bool valid;
  TmapKey key;
  CUtensorMap map;
};
constexpr int kTmapCache = 256;
thread_local TmapEntry t_tmap_cache[kTmapCache];
}  // namespace

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  const TmapKey key{base, inner, outer, row_stride_bytes, box_inner, box_outer, (int)dt, (int)swizzle};
  uint64_t h = reinterpret_cast<uintptr_t>(base) >> 4;
  h ^= inner * 0x9E3779B97F4A7C15ull ^ outer * 0xC2B2AE3D27D4EB4Full ^ ((uint64_t)box_inner << 32 | box_outer) ^
       ((uint64_t)dt << 8 | (uint64_t)swizzle);
  h ^= h >> 29;
  TmapEntry& e = t_tmap_cache[h % kTmapCache];
  if (e.valid && e.key == key) {
    *map = e.map;
    return true;
  }
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
  e.valid = true;
  e.key = key;
  e.map = *map;
  return true;
}

bool make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t (&dims)[3],
                  const uint64_t (&strides_bytes)[2], const uint32_t (&box)[3], CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return false;
  }
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  const cuuint32_t bx[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), d, st, bx, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    return false;
  }
  return true;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device)
// and size instead of on every launch.
void set_max_smem(const void* func, int bytes) {
  struct Entry {
    const void* func;
    int dev, bytes;
  };
  static std::mutex mu;
  static Entry done[256];
  static int n = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i)
      if (done[i].func == func && done[i].dev == dev && done[i].bytes >= bytes) return;
  }
  cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (done[i].func == func && done[i].dev == dev) {
      if (bytes > done[i].bytes) done[i].bytes = bytes;
      return;
    }
  if (n < 256) done[n++] = Entry{func, dev, bytes};
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
