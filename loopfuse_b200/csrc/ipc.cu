// Sharing one device buffer with the other processes of a node (head-tensor-parallel decode:
// every rank's combine kernel stores its heads into every rank's output buffer).
//
// The buffers are ordinary caching-allocator memory.  An IPC handle names a whole allocation,
// so the exporter also reports the buffer's offset inside it (the allocation's base comes from
// cuMemGetAddressRange); the importer opens the allocation (peer access enabled on demand) and
// adds the offset.  The mappings are plain peer-to-peer ones.
#include "lf_common.cuh"

#include <cuda.h>
#include <cstring>

namespace {

using PFN_range = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_range range_fn() {
    static PFN_range fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_range>(ptr);
    }
    return fn;
}

}  // namespace

using namespace lf;

extern "C" int lf_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
    LF_CHECK_ARG(ptr && handle_out && offset_out, "ipc export: null argument");
    PFN_range fn = range_fn();
    if (fn == nullptr) return set_error(LF_ECUDA, "cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_error(LF_ECUDA, "ipc export: pointer is not device memory");
    cudaIpcMemHandle_t h;
    LF_CHECK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
    clear_error();
    return LF_OK;
}

extern "C" int lf_ipc_import(const void* handle, void** base_out) {
    LF_CHECK_ARG(handle && base_out, "ipc import: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    LF_CHECK_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
    clear_error();
    return LF_OK;
}

extern "C" int lf_ipc_close(void* base) {
    LF_CHECK_ARG(base != nullptr, "ipc close: null pointer");
    LF_CHECK_CUDA(cudaIpcCloseMemHandle(base));
    clear_error();
    return LF_OK;
}
