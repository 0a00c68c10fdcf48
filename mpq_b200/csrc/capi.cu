// Library-level C-ABI entry points: version and the last error message.
#include <stdarg.h>
#include <stdio.h>
#include "common.cuh"

namespace mpq {
static thread_local char g_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}
}  // namespace mpq

MPQ_API const char* mpq_last_error(void) { return mpq::g_last_error; }

MPQ_API int mpq_abi_version(void) { return 1; }
