// Thread-local last-error storage behind swl_last_error().
#include "common.h"

namespace swl {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

const char* last_error() { return g_last_error.c_str(); }

}  // namespace swl

SWL_EXPORT const char* swl_last_error(void) { return swl::last_error(); }

SWL_EXPORT int swl_abi_version(void) { return 1; }
