// Diagnostic entry point: exercises the failure path every pipelined kernel here relies on.
//
// The tcgen05 kernels never spin without a limit: each mbarrier wait gives up after a wall-clock
// limit, marks the block as aborted, unwinds and records a site code in the device error word
// that lf_device_status() reads.  lf_selftest_bounded_wait runs that same wait (mbar_wait) on a
// barrier that nothing ever arrives at, with a short limit, so a caller -- or a test -- can see
// the expiry reported and the context left usable, without provoking a real pipeline failure.
#include "lf_common.cuh"
#include "sm100_primitives.cuh"

namespace lf {
namespace selftest {

constexpr int kSite = 77;   // reported as 100 + kSite, like the attention kernels' sites

__global__ void bounded_wait_kernel(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar_word;
    __shared__ int err;
    const uint32_t bar = sm100::smem_addr(&bar_word);
    if (threadIdx.x == 0) {
        sm100::mbar_init(bar, 1);                  // expects one arrival, which never comes
        err = 0;
        sm100::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !sm100::mbar_wait(bar, 0, &err, kSite, limit_ns))
        atomicCAS(&g_device_error, 0, 100 + err);
}

}  // namespace selftest
}  // namespace lf

extern "C" int lf_selftest_bounded_wait(unsigned timeout_us, void* stream) {
    LF_CHECK_ARG(timeout_us >= 1 && timeout_us <= 100000,
                 "selftest: timeout_us must be 1..100000 (got %u)", timeout_us);
    lf::selftest::bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<unsigned long long>(timeout_us) * 1000ull);
    return lf::launch_status("selftest bounded wait");
}
