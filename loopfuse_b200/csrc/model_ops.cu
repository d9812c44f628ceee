// Elementwise decoder ops around the attention path: residual add + RMSNorm, and the SwiGLU
// gate.  Each replaces a chain of ~7 (norm) or ~3 (gate) separate elementwise passes over HBM
// with one; both are bandwidth-bound, 16-byte vectors, fp32 arithmetic.
//
// The reference's fused_ln_qkv (kernels/triton/fused_ln_qkv.py:27-72) keeps a LayerNorm in
// registers ahead of its QKV product; here the norm is RMSNorm (Llama) and the GEMM stays a
// library call, so the kernel fuses the residual add into the norm instead.
#include "lf_common.cuh"

#include <cuda_bf16.h>

namespace lf {
namespace model {

constexpr int kNormThreads = 256;
constexpr int kNormVecs = 4;                       // vectors of 8 per thread: dim <= 8192

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack2(float a, float b) {    // one packed conversion
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// One CTA per row.
__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(uint16_t* __restrict__ x, const uint16_t* __restrict__ delta,
                   const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int dim, float eps) {
    __shared__ float red[kNormThreads / 32];
    const long row = blockIdx.x;
    uint16_t* xr = x + row * dim;
    const int nvec = dim / 8;
    float v[kNormVecs][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
        const int vi = i * kNormThreads + threadIdx.x;
        if (vi < nvec) {
            uint4 a = *reinterpret_cast<const uint4*>(xr + vi * 8);
            const uint32_t* aw = reinterpret_cast<const uint32_t*>(&a);
            if (delta != nullptr) {
                const uint4 d = *reinterpret_cast<const uint4*>(delta + row * dim + vi * 8);
                const uint32_t* dw = reinterpret_cast<const uint32_t*>(&d);
                uint4 s;
                uint32_t* sw = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
                for (int k = 0; k < 4; ++k) sw[k] = pack2(lo_f(aw[k]) + lo_f(dw[k]), hi_f(aw[k]) + hi_f(dw[k]));
                *reinterpret_cast<uint4*>(xr + vi * 8) = s;
                a = s;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[i][2 * k] = lo_f(aw[k]);
                v[i][2 * k + 1] = hi_f(aw[k]);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
        }
    }
    if (w == nullptr) return;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < kNormThreads / 32; ++k) tot += red[k];
    const float r = rsqrtf(tot / static_cast<float>(dim) + eps);
    uint16_t* orow = out + row * dim;
#pragma unroll
    for (int i = 0; i < kNormVecs; ++i) {
        const int vi = i * kNormThreads + threadIdx.x;
        if (vi < nvec) {
            const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
            const uint32_t* ww = reinterpret_cast<const uint32_t*>(&wv);
            uint4 o;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t nrm = pack2(v[i][2 * k] * r, v[i][2 * k + 1] * r);   // bf16(x * r)
                ow[k] = pack2(lo_f(nrm) * lo_f(ww[k]), hi_f(nrm) * hi_f(ww[k]));
            }
            *reinterpret_cast<uint4*>(orow + vi * 8) = o;
        }
    }
}

// out[r][j] = bf16(bf16(silu(g)) * u) with g = gu[r][j], u = gu[r][ffn + j].  grid.x walks the
// vectors of a row, grid.y the rows (grid-stride).
__global__ void swiglu_kernel(const uint16_t* __restrict__ gu, uint16_t* __restrict__ out, int rows,
                              int ffn) {
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (c >= ffn) return;
    for (int r = blockIdx.y; r < rows; r += gridDim.y) {
        const uint16_t* grow = gu + (long)r * 2 * ffn;
        const uint4 g = *reinterpret_cast<const uint4*>(grow + c);
        const uint4 u = *reinterpret_cast<const uint4*>(grow + ffn + c);
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g);
        const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float g0 = lo_f(gw[k]), g1 = hi_f(gw[k]);
            const uint32_t sl = pack2(g0 / (1.f + expf(-g0)), g1 / (1.f + expf(-g1)));   // bf16(silu)
            ow[k] = pack2(lo_f(sl) * lo_f(uw[k]), hi_f(sl) * hi_f(uw[k]));
        }
        *reinterpret_cast<uint4*>(out + (long)r * ffn + c) = o;
    }
}

}  // namespace model
}  // namespace lf

using namespace lf;

extern "C" int lf_add_rmsnorm(lf_bf16* x, const lf_bf16* delta, const lf_bf16* w, lf_bf16* out,
                              int rows, int dim, float eps, void* stream) {
    LF_CHECK_ARG(rows >= 0 && dim > 0 && dim % 8 == 0 && dim <= model::kNormThreads * model::kNormVecs * 8,
                 "add_rmsnorm: dim must be a positive multiple of 8, at most %d",
                 model::kNormThreads * model::kNormVecs * 8);
    LF_CHECK_ARG(x != nullptr && (w == nullptr || out != nullptr), "add_rmsnorm: null pointer");
    LF_CHECK_ARG(aligned16(x) && aligned16(delta) && aligned16(w) && aligned16(out),
                 "add_rmsnorm: buffers must be 16-byte aligned");
    if (rows == 0) { clear_error(); return LF_OK; }
    model::add_rmsnorm_kernel<<<rows, model::kNormThreads, 0, (cudaStream_t)stream>>>(
        x, delta, w, out, dim, eps);
    return launch_status("add_rmsnorm");
}

extern "C" int lf_swiglu(const lf_bf16* gu, lf_bf16* out, int rows, int ffn, void* stream) {
    LF_CHECK_ARG(rows >= 0 && ffn > 0 && ffn % 8 == 0, "swiglu: ffn must be a positive multiple of 8");
    LF_CHECK_ARG(gu && out && aligned16(gu) && aligned16(out), "swiglu: null or unaligned buffer");
    if (rows == 0) { clear_error(); return LF_OK; }
    const int bx = (ffn / 8 + 255) / 256;
    int by = (148 * 16 + bx - 1) / bx;
    if (by > rows) by = rows;
    if (by > 65535) by = 65535;
    model::swiglu_kernel<<<dim3(bx, by), 256, 0, (cudaStream_t)stream>>>(gu, out, rows, ffn);
    return launch_status("swiglu");
}
