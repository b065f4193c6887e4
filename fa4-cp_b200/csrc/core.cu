// Library core: version and the per-thread last-error text.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace fa4cp {

static thread_local char t_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace fa4cp

extern "C" int fa4cp_version(void) { return 100; }

extern "C" const char* fa4cp_last_error(void) { return fa4cp::t_last_error; }

