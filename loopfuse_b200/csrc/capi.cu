// Library-wide C entry points: version string and per-thread error messages.
#include "lf_common.cuh"

#include <stdarg.h>
#include <stdlib.h>

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

// cuCtxGetCurrent / cuCtxGetId, looked up through the runtime so that the library links against
// the runtime alone.
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

int current_context_id(unsigned long long* id) {
    static std::once_flag once;
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(f);
    });
    LF_CHECK_ARG(get_current != nullptr && get_id != nullptr,
                 "context: the driver has no cuCtxGetCurrent / cuCtxGetId");
    void* ctx = nullptr;
    LF_CHECK_ARG(get_current(&ctx) == 0, "context: cuCtxGetCurrent failed");
    if (ctx == nullptr) {                 // nothing current yet: bind the device's primary context
        int dev = 0;
        LF_CHECK_CUDA(cudaGetDevice(&dev));
        LF_CHECK_CUDA(cudaSetDevice(dev));
        LF_CHECK_ARG(get_current(&ctx) == 0 && ctx != nullptr, "context: no current context");
    }
    LF_CHECK_ARG(get_id(ctx, id) == 0, "context: cuCtxGetId failed");
    return LF_OK;
}

constexpr int kMaxReaders = 64;
static DeviceErrorReader g_readers[kMaxReaders];
static int g_n_readers = 0;

// Runs at library load, once per translation unit.  Past the table's size a unit's reports
// would be lost without a sign, so loading fails instead.
bool register_device_error_reader(DeviceErrorReader fn) {
    if (g_n_readers >= kMaxReaders) {
        fprintf(stderr, "loopfuse_b200: more than %d device error words; raise kMaxReaders\n",
                kMaxReaders);
        abort();
    }
    g_readers[g_n_readers++] = fn;
    return true;
}

}  // namespace lf

extern "C" const char* lf_version(void) { return "loopfuse_b200 0.1 sm_100a"; }
extern "C" const char* lf_last_error(void) { return lf::g_err; }

extern "C" int lf_device_status(int* out) {
    LF_CHECK_ARG(out != nullptr, "device_status: out is null");
    // The first unit (in load order) holding a report gives it up; other units keep theirs for
    // the next call, so repeated calls drain every report.
    int first = 0;
    for (int i = 0; i < lf::g_n_readers && first == 0; ++i) {
        const int v = lf::g_readers[i]();
        if (v < 0) return lf::set_error(LF_ECUDA, "device_status: reading an error word failed");
        first = v;
    }
    *out = first;
    lf::clear_error();
    return LF_OK;
}
