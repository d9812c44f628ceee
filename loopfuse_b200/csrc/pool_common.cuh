// Metadata view and block-wide helpers shared by the pool kernels (pool.cu, pool_dedup.cu).
#pragma once

#include "lf_common.cuh"

#include <climits>

namespace lf {
namespace pool {

constexpr int kMetaThreads = 1024;
// Sessions a reserve checks for repeated ids with a shared-memory bitmap (32 KB); larger
// pools use the exact pairwise scan.
constexpr int kDupBits = 1 << 18;

struct Meta {
    int32_t* fq;
    int32_t* rc;
    int32_t* bt;
    int32_t* len;
    int32_t* ctrl;
    int32_t* scratch;
    int P, S, M;
};

static Meta to_meta(const lf_pool_meta* m) {
    return Meta{m->free_queue, m->refcount, m->block_table, m->seq_len, m->ctrl, m->scratch,
                m->num_pages, m->max_seqs, m->max_pages_per_seq};
}

__device__ __forceinline__ int pages_for(int tokens) { return (tokens + LF_PAGE_SIZE - 1) / LF_PAGE_SIZE; }

__device__ __forceinline__ int status_of(const Meta& m) {
    return *reinterpret_cast<volatile int32_t*>(m.ctrl + LF_CTRL_STATUS);
}

// Block-wide exclusive scan (blockDim.x == kMetaThreads).  Returns this thread's exclusive
// prefix; *total receives the block sum.  Reuses `buf` (>= 32 ints of shared memory).
static __device__ int block_excl_scan(int v, int* total, int* buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    __syncthreads();
    if (lane == 31) buf[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = (lane < (kMetaThreads / 32)) ? buf[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += y;
        }
        buf[lane] = w;
    }
    __syncthreads();
    const int warp_excl = warp > 0 ? buf[warp - 1] : 0;
    *total = buf[kMetaThreads / 32 - 1];
    __syncthreads();
    return warp_excl + x - v;
}

static __device__ int block_min(int v, int* buf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, off));
    __syncthreads();
    if (lane == 0) buf[warp] = v;
    __syncthreads();
    int r = buf[0];
    for (int w = 1; w < kMetaThreads / 32; ++w) r = min(r, buf[w]);
    __syncthreads();
    return r;
}

static int check_meta(const lf_pool_meta* m) {
    LF_CHECK_ARG(m != nullptr, "pool: meta is null");
    LF_CHECK_ARG(m->free_queue && m->refcount && m->block_table && m->seq_len && m->ctrl && m->scratch,
                 "pool: meta has a null array");
    LF_CHECK_ARG(m->num_pages > 0 && m->max_seqs > 0 && m->max_pages_per_seq > 0,
                 "pool: sizes must be positive");
    LF_CHECK_ARG(m->page_size == LF_PAGE_SIZE, "pool: page_size must be %d", LF_PAGE_SIZE);
    return LF_OK;
}

static int grid_for(long work, int threads) {
    long b = (work + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148L * 16) b = 148L * 16;
    return (int)b;
}

}  // namespace pool
}  // namespace lf
