// Thread-local last-error storage behind swl_last_error().
#include "common.h"
#include "launch.h"

#include <atomic>

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

static std::atomic<int> g_pdl{1};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

}  // namespace swl

SWL_EXPORT const char* swl_last_error(void) { return swl::last_error(); }

SWL_EXPORT int swl_abi_version(void) { return 1; }

// Switches programmatic dependent launch for every later kernel launch of the
// library (on by default); returns the previous setting.
SWL_EXPORT int swl_set_pdl(int on) { return swl::g_pdl.exchange(on ? 1 : 0); }
