// Paged-decode constants shared by decode.cu, decode_mma.cu and decode_prefix.cu, and the lane
// layout and reductions of the CUDA-core shared-prefix kernel (decode_prefix.cu, head_dim 64):
// a page row of D bf16 is read by D/8 lanes, 16 bytes each.
#pragma once

#include "lf_common.cuh"

namespace lf {
namespace decode {

constexpr int kPage = LF_PAGE_SIZE;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;

template <int D, int G>
struct Cfg {
    static constexpr int LPT = D / 8;            // lanes per token row (16 B per lane)
    static constexpr int TPI = 32 / LPT;         // token rows per load instruction
    static constexpr int ROWS = kPage / TPI;     // load instructions per page per operand
    static constexpr int LOG_LPT = (LPT == 16) ? 4 : (LPT == 8 ? 3 : 2);
    static constexpr int LOG_G = (G == 8) ? 3 : (G == 4 ? 2 : (G == 2 ? 1 : 0));
    static constexpr int H = (LOG_G < LOG_LPT) ? LOG_G : LOG_LPT;   // halving steps
    static_assert((1 << H) == G, "group size must fit the lanes of a row");
};

// Head whose full score lane chunk c ends up holding after the reduce-scatter.
template <int D, int G>
__device__ __forceinline__ int head_of_chunk(int c) {
    using C = Cfg<D, G>;
    int h = 0;
#pragma unroll
    for (int s = 0; s < C::H; ++s) h += ((c >> (C::LOG_LPT - 1 - s)) & 1) * (G >> (s + 1));
    return h;
}

// Chunk index (within a row's lanes) that holds head g's score with low bits zero.
template <int D, int G>
__device__ __forceinline__ int chunk_of_head(int g) {
    using C = Cfg<D, G>;
    int c = 0;
#pragma unroll
    for (int s = 0; s < C::H; ++s) c |= ((g >> (C::H - 1 - s)) & 1) << (C::LOG_LPT - 1 - s);
    return c;
}

template <int D, int G>
__device__ __forceinline__ float reduce_scatter_row(float (&v)[G], int c) {
    using C = Cfg<D, G>;
#pragma unroll
    for (int s = 0; s < C::H; ++s) {
        const int bit = C::LPT >> (s + 1);
        const bool upper = (c & bit) != 0;
        const int half = G >> (s + 1);
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float keep = upper ? v[half + i] : v[i];
            const float send = upper ? v[i] : v[half + i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
    }
    float r = v[0];
#pragma unroll
    for (int bit = C::LPT >> (C::H + 1); bit >= 1; bit >>= 1) r += __shfl_xor_sync(0xffffffffu, r, bit);
    return r;
}

// Page id from a block table, checked against the pool size.  A bad id is replaced by page 0
// (an in-bounds read whose result is wrong but harmless) and reported through the library's
// device error word instead of faulting.
__device__ __forceinline__ int checked_page(int page, int num_pages) {
    if (static_cast<unsigned>(page) >= static_cast<unsigned>(num_pages)) {
        atomicCAS(&g_device_error, 0, 200);
        return 0;
    }
    return page;
}

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
    f[0] = bf16lo_to_f32(w.x); f[1] = bf16hi_to_f32(w.x);
    f[2] = bf16lo_to_f32(w.y); f[3] = bf16hi_to_f32(w.y);
    f[4] = bf16lo_to_f32(w.z); f[5] = bf16hi_to_f32(w.z);
    f[6] = bf16lo_to_f32(w.w); f[7] = bf16hi_to_f32(w.w);
}

}  // namespace decode
}  // namespace lf
