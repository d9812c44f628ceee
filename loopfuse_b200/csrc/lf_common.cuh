// Shared helpers for the sm_100a kernels: status/error plumbing, bf16 unpacking,
// streaming 128-bit loads.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "../../include/loopfuse_b200.h"

namespace lf {

// Records the message returned by lf_last_error() for this host thread.
int set_error(int code, const char* fmt, ...);
void clear_error();

#define LF_CHECK_ARG(cond, ...)                         \
    do {                                                \
        if (!(cond)) return ::lf::set_error(LF_EINVAL, __VA_ARGS__); \
    } while (0)

#define LF_CHECK_CUDA(expr)                                                       \
    do {                                                                          \
        cudaError_t e_ = (expr);                                                  \
        if (e_ != cudaSuccess)                                                    \
            return ::lf::set_error(LF_ECUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

// Id of the CUDA context current on this thread: the driver's context id, unique for the life of
// the process.  When no context is current, the device's primary context is made current first.
int current_context_id(unsigned long long* id);

// A set-up step that belongs to a CUDA context (a kernel's shared-memory opt-in, say), run the
// first time each context reaches the call site that owns this object.  It is keyed on the
// context id rather than the device ordinal, so after a device reset, or with another context
// current on the same device, the step runs again instead of being skipped.  Past kSlots
// contexts the oldest entry makes room; its step then simply runs again if that context returns.
class PerContextOnce {
  public:
    template <class F>
    int run(F&& setup) {
        unsigned long long id = 0;
        const int rc = current_context_id(&id);
        if (rc != LF_OK) return rc;
        std::lock_guard<std::mutex> lock(mu_);
        for (int i = 0; i < n_; ++i)
            if (ids_[i] == id) return LF_OK;
        const int rs = setup();
        if (rs != LF_OK) return rs;
        ids_[next_] = id;
        next_ = (next_ + 1) % kSlots;
        if (n_ < kSlots) ++n_;
        return LF_OK;
    }

  private:
    static constexpr int kSlots = 64;
    std::mutex mu_;
    unsigned long long ids_[kSlots] = {};
    int n_ = 0, next_ = 0;
};

// After a <<<>>> launch: report configuration errors without synchronising.
inline int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(LF_ECUDA, "%s launch: %s", what, cudaGetErrorString(e));
    clear_error();
    return LF_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// bf16 bit patterns -> fp32: a bf16 is the high half of the fp32 with the same value.
__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_rn(float f) {
    uint16_t r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
    return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// 16-byte streaming load: read-only path, not kept in L1 (K/V pages are read once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device-side error reporting.  Each translation unit gets its own error word (device code is
// compiled per unit, without cross-unit device linking); a kernel whose bounded wait gave up,
// or that met a bad page id, stores a site code there instead of faulting or hanging.  Each
// unit registers a reader at load time, and lf_device_status() collects and clears them all.
using DeviceErrorReader = int (*)();
bool register_device_error_reader(DeviceErrorReader fn);

static __device__ int g_device_error = 0;

static int take_device_error() {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v != 0) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    }
    return v;
}

static const bool g_device_error_registered = register_device_error_reader(&take_device_error);

}  // namespace lf
