// Thread-local error messages behind bt_last_error().
#include "common.cuh"

namespace bt {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_last_error; }

}  // namespace bt

extern "C" const char* bt_last_error(void) { return bt::last_error(); }

extern "C" const char* bt_version(void) { return "boonta_b200 0.1 (sm_100a)"; }
