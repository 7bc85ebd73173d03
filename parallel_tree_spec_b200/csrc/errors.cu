// Error reporting for the C ABI (thread-local last message).
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace pts {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

}  // namespace pts

extern "C" const char* pts_last_error(void) { return pts::g_last_error; }

extern "C" int pts_version(void) { return 1; }
