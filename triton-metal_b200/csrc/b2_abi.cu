// C-ABI bookkeeping: version and the thread-local last-error message.
#include "b2_common.cuh"
#include <string.h>

namespace b2 {
static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}
}  // namespace b2

extern "C" int b2_version(void) { return 10000; }  // 1.0.0

extern "C" const char* b2_last_error(void) { return b2::g_last_error; }
