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

static DeviceErrorReader g_readers[16];
static int g_n_readers = 0;

bool register_device_error_reader(DeviceErrorReader fn) {
    if (g_n_readers < 16) g_readers[g_n_readers++] = fn;
    return true;
}

}  // namespace lf

extern "C" const char* lf_version(void) { return "loopfuse_b200 0.1 sm_100a"; }
extern "C" const char* lf_last_error(void) { return lf::g_err; }

extern "C" int lf_device_status(int* out) {
    LF_CHECK_ARG(out != nullptr, "device_status: out is null");
    int first = 0;
    for (int i = 0; i < lf::g_n_readers; ++i) {
        const int v = lf::g_readers[i]();
        if (v < 0) return lf::set_error(LF_ECUDA, "device_status: reading an error word failed");
        if (first == 0) first = v;
    }
    *out = first;
    lf::clear_error();
    return LF_OK;
}
