// Library-wide C entry points: version string and per-thread error messages.
#include "lf_common.cuh"

#include <stdarg.h>

namespace lf {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_err[0] = '\0'; }

}  // namespace lf

extern "C" const char* lf_version(void) { return "loopfuse_b200 0.1 sm_100a"; }
extern "C" const char* lf_last_error(void) { return lf::g_err; }
