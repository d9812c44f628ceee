// Per-session pass of the paged split-KV decode on the warp-level tensor-core MMA
// (mma.sync m16n8k16, bf16 -> fp32).
//
// A CUDA-core formulation (a fused multiply-add per (head, dim, token) plus shuffle reductions)
// costs ~1000 warp instructions per 16-token page of one KV head: measured with ncu, it issues on
// 56% of active cycles and reaches the HBM roofline only with many long sessions.  Here a page
// costs ~100 instructions.  The attention of one page is two small matrix products, with the
// roles chosen so that the page's 16 tokens are the M dimension:
//
//   S^T [16 tokens x 8 heads]  = K_page [16 x D] . Q^T [D x 8]      (D/16 MMAs)
//   O^T [D x 8 heads]         += V_page^T [D x 16] . P^T [16 x 8]   (D/16 MMAs)
//
// The GQA group (G <= 8 query heads of one KV head) fills the N = 8 columns.  CTA = (split, KV
// head, session), four warps taking the split's pages round-robin.  K and V pages are staged in
// shared memory by TMA (three-dimensional tiled loads of the [P*Hkv][16][D] pool with 128-byte
// swizzle, so that ldmatrix reads them without bank conflicts), kStages pages ahead of the page a
// warp computes on; page ids for 32 pages at a time are held one per lane, so no block-table load
// sits between pages.  K fragments come from ldmatrix, V^T fragments from ldmatrix.trans, and the
// probabilities go from the S^T accumulator to the P^T operand with movmatrix.trans.  Scores are
// scaled in fp32 after the product (q stays exactly bf16), the softmax runs online in the log2
// domain with fp32 running sums, and P is rounded to bf16 for the second product.  The warps'
// partials are merged through shared memory into one (o, max, sum) per query head, in the slot
// layout the combine kernel (decode.cu) reads.
//
// Every barrier wait is bounded (site 211 in the device error word when a stage never lands);
// a warp that gives up stops computing and drains its other loads, bounded again, before exit.
//
// Fused append (lf_decode_fwd_append): the CTA that holds a session's last page first stores
// the session's newest token (K and V rows of its KV head) into that page, then loads it.  A
// newest token without a page of its own past the shared prefix, or with a page id out of
// range, is not stored and leaves site 212.
#include "decode_common.cuh"
#include "sm100_primitives.cuh"
#include "tmap.cuh"

#include <math.h>

namespace lf {
namespace decode {
namespace mma {

constexpr uint64_t kWaitNs = 2000000000ull;
// Stages per warp: two pages in flight per warp and three CTAs per SM (64 KB of shared memory
// each at head_dim 128).  Three stages (two CTAs per SM) measured the same or slower.
constexpr int kStages = 2;

__device__ __forceinline__ bool wait_stage(uint32_t bar, uint32_t parity) {
    if (sm100::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = sm100::global_timer_ns();
    while (!sm100::mbar_try_wait(bar, parity))
        if (sm100::global_timer_ns() - t0 > kWaitNs) return false;
    return true;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t r;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
    return r;
}

// D += A . B, m16n8k16, A row-major bf16 (4 regs), B column-major bf16 (2 regs), fp32 D.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Shared-memory byte offset of 16-byte chunk `j` (8 dims) of token row `t` inside one head-page
// staged as D/64 swizzled [16][64] boxes of 2 KB each.
__device__ __forceinline__ uint32_t chunk_off(int t, int j) {
    return (uint32_t)((j >> 3) * 2048 + t * 128 + (((j & 7) ^ (t & 7)) << 4));
}

template <int D, int S>
struct Layout {
    static constexpr int kHeadPageBytes = kPage * D * 2;           // 2 or 4 KB
    static constexpr int kStageBytes = 2 * kHeadPageBytes;          // K then V
    static constexpr int kSmemBytes = kWarps * S * kStageBytes + 1024;   // + alignment slack
};

template <int D, int G, int S>
__global__ void __launch_bounds__(kThreads)
split_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                 const uint16_t* __restrict__ q, const int32_t* __restrict__ bt,
                 const int32_t* __restrict__ seq_lens, float* __restrict__ part_o,
                 float2* __restrict__ part_ml, int Hq, int Hkv, int num_pages, int max_pages,
                 int pages_per_split, int first_page, int n_slots, float qscale,
                 const uint16_t* __restrict__ k_new, const uint16_t* __restrict__ v_new,
                 uint16_t* kp_w, uint16_t* vp_w) {
    static_assert(D == 64 || D == 128, "head_dim 64 or 128");
    static_assert(G >= 1 && G <= 8, "a GQA group fills at most the 8 MMA columns");
    using LY = Layout<D, S>;
    constexpr int KS = D / 16;                                      // k-steps of Q.K^T
    constexpr int MT = D / 16;                                      // m-tiles of V^T.P^T
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bars[kWarps][S];

    const int split = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
    const int L = min(max(seq_lens[n], 0), max_pages * kPage);
    const int npages = (L + kPage - 1) / kPage;
    const int p_begin = first_page + split * pages_per_split;
    if (p_begin >= npages) {
        // fused append: a session whose newest token would not sit in a page of its own (no
        // tokens, or none past the shared prefix) has no CTA to store it -- reported, not stored
        if (k_new != nullptr && split == 0 && threadIdx.x == 0) atomicCAS(&g_device_error, 0, 212);
        return;
    }
    const int n_local = min(p_begin + pages_per_split, npages) - p_begin;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int my_pages = n_local > warp ? (n_local - warp + kWarps - 1) / kWarps : 0;
    const int32_t* bt_row = bt + (size_t)n * max_pages;
    const uint32_t wstage = sm100::smem_addr(smem) + (uint32_t)(warp * S * LY::kStageBytes);
    const uint32_t wbar = sm100::smem_addr(&bars[warp][0]);

    if (lane == 0) {
        sm100::tma_prefetch_desc(&tmk);
        sm100::tma_prefetch_desc(&tmv);
        for (int i = 0; i < S; ++i) sm100::mbar_init(wbar + 8 * i, 1);
        sm100::fence_barrier_init();
    }
    __syncwarp();

    // Fused append (k_new / v_new given): the CTA holding the session's last page first stores
    // the newest token's K and V rows of its KV head at position L - 1, then makes the stores
    // visible to its own TMA page loads (proxy fence, then a CTA barrier before any warp issues).
    // No other CTA reads that page: it is the session's own, past the shared-prefix pages, and
    // other heads' rows of it are other CTAs' rows.
    if (k_new != nullptr && p_begin + n_local == npages) {
        constexpr int kChunks = D / 8;                       // 16-byte pieces of a row
        if (threadIdx.x < 2 * kChunks) {
            const int pos = L - 1;
            const int page = bt_row[pos / kPage];
            if (static_cast<unsigned>(page) < static_cast<unsigned>(num_pages)) {
                const bool isv = threadIdx.x >= kChunks;
                const int c = threadIdx.x - (isv ? kChunks : 0);
                const size_t src = ((size_t)n * Hkv + h) * D;
                const size_t dst = (((size_t)page * Hkv + h) * kPage + pos % kPage) * D;
                reinterpret_cast<uint4*>((isv ? vp_w : kp_w) + dst)[c] =
                    reinterpret_cast<const uint4*>((isv ? v_new : k_new) + src)[c];
                sm100::fence_proxy_async_global();
            } else if (threadIdx.x == 0) {
                atomicCAS(&g_device_error, 0, 212);
            }
        }
        __syncthreads();
    }

    int ids = 0, ids_batch = -1;                   // page ids of 32 pages, one per lane
    // A session's own pages are read once: evicted first from L2, so the split and prefix
    // partials that the combine reads next stay there.
    const uint64_t l2_policy = sm100::l2_evict_first_policy();
    auto issue = [&](int k) {                      // warp-uniform
        if (k >= my_pages) return;
        const int b = k >> 5;
        if (b != ids_batch) {
            const int j = warp + kWarps * ((b << 5) + lane);
            ids = j < n_local ? checked_page(bt_row[p_begin + j], num_pages) : 0;
            ids_batch = b;
        }
        const int page = __shfl_sync(0xffffffffu, ids, k & 31);
        if (lane == 0) {
            const int st = k % S;
            const uint32_t dst = wstage + (uint32_t)(st * LY::kStageBytes);
            const uint32_t bar = wbar + 8 * st;
            const int row = page * Hkv + h;
            sm100::fence_proxy_async_smem();
            sm100::mbar_arrive_expect_tx(bar, LY::kStageBytes);
#pragma unroll
            for (int bx = 0; bx < D / 64; ++bx) {
                sm100::tma_load_3d_hint(dst + bx * 2048, &tmk, bar, 64 * bx, 0, row, l2_policy);
                sm100::tma_load_3d_hint(dst + LY::kHeadPageBytes + bx * 2048, &tmv, bar, 64 * bx, 0,
                                        row, l2_policy);
            }
        }
    };
#pragma unroll
    for (int k = 0; k < S; ++k) issue(k);

    // Q^T fragments: column g is query head h*G + g (zero past the group), rows are dims.
    uint32_t qb[KS][2];
    {
        const uint32_t* qrow = reinterpret_cast<const uint32_t*>(q + ((size_t)n * Hq + h * G + g) * D);
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            qb[kk][0] = g < G ? qrow[(16 * kk + 2 * c) >> 1] : 0u;
            qb[kk][1] = g < G ? qrow[(16 * kk + 2 * c + 8) >> 1] : 0u;
        }
    }
    float o[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY;          // running max of heads 2c, 2c+1 (log2 units)
    float l0 = 0.f, l1 = 0.f;                      // this thread's share of the running sums

    // ldmatrix row addresses: lane l serves matrix l/8, row l%8.
    const int lq = lane >> 3, lr = lane & 7;
    const int k_row = lr + 8 * (lq & 1), k_chunk = lq >> 1;       // K as A (16 tok x 16 dims)
    const int v_row = lr + 8 * (lq >> 1), v_chunk = lq & 1;       // V^T as A via .trans

    int done = 0;
    bool failed = false;
    for (int k = 0; k < my_pages; ++k) {
        const int st = k % S;
        const bool ok = __all_sync(0xffffffffu, wait_stage(wbar + 8 * st, (uint32_t)((k / S) & 1)));
        if (!ok) {
            if (lane == 0) atomicCAS(&g_device_error, 0, 211);
            failed = true;
            break;
        }
        done = k + 1;
        const uint32_t kbase = wstage + (uint32_t)(st * LY::kStageBytes);
        const uint32_t vbase = kbase + LY::kHeadPageBytes;

        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
            uint32_t a[4];
            ldsm_x4(kbase + chunk_off(k_row, 2 * kk + k_chunk), a);
            mma16816(s, a, qb[kk][0], qb[kk][1]);
        }
        const int tok = (p_begin + warp + kWarps * k) * kPage + g;
        s[0] = tok < L ? s[0] * qscale : -INFINITY;
        s[1] = tok < L ? s[1] * qscale : -INFINITY;
        s[2] = tok + 8 < L ? s[2] * qscale : -INFINITY;
        s[3] = tok + 8 < L ? s[3] * qscale : -INFINITY;
        float x0 = fmaxf(s[0], s[2]), x1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, off));
            x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, off));
        }
        // Every page below npages holds a valid token, so the new maxima are finite.
        const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
        const float a0 = fast_exp2(m0 - n0), a1 = fast_exp2(m1 - n1);
        m0 = n0;
        m1 = n1;
        const float e0 = fast_exp2(s[0] - n0), e1 = fast_exp2(s[1] - n1);   // token g
        const float e2 = fast_exp2(s[2] - n0), e3 = fast_exp2(s[3] - n1);   // token g+8
        l0 = l0 * a0 + (e0 + e2);                  // sums in fp32; P.V takes bf16 P
        l1 = l1 * a1 + (e1 + e3);
        const uint32_t p01 = pack_bf16x2(e0, e1), p23 = pack_bf16x2(e2, e3);
        const uint32_t pb0 = movm_t(p01), pb1 = movm_t(p23);        // P^T fragments
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            o[mt][0] *= a0; o[mt][1] *= a1; o[mt][2] *= a0; o[mt][3] *= a1;
            uint32_t a[4];
            ldsm_x4_t(vbase + chunk_off(v_row, 2 * mt + v_chunk), a);
            mma16816(o[mt], a, pb0, pb1);
        }
        __syncwarp();                              // every lane is done with stage st
        issue(k + S);
    }
    if (failed && lane == 0) {                     // let the loads in flight land
        for (int k = done + 1; k < min(my_pages, done + S); ++k)
            wait_stage(wbar + 8 * (k % S), (uint32_t)((k / S) & 1));
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {       // whole-column sums
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }

    // Cross-warp merge through the (now idle) stage memory: per warp, the max and sum of each
    // head and its unnormalised output row.
    __syncthreads();
    float* sm_m = reinterpret_cast<float*>(smem);                 // [kWarps][8]
    float* sm_l = sm_m + kWarps * 8;                              // [kWarps][8]
    float* sm_o = sm_l + kWarps * 8;                              // [kWarps][8][D]
    if (g == 0) {
        sm_m[warp * 8 + 2 * c] = m0;
        sm_m[warp * 8 + 2 * c + 1] = m1;
        sm_l[warp * 8 + 2 * c] = l0;
        sm_l[warp * 8 + 2 * c + 1] = l1;
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        float* r0 = sm_o + (size_t)(warp * 8 + 2 * c) * D + 16 * mt + g;
        float* r1 = r0 + D;
        r0[0] = o[mt][0]; r1[0] = o[mt][1]; r0[8] = o[mt][2]; r1[8] = o[mt][3];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
        const int hd = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w * 8 + hd]);
        float acc = 0.f, l = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float mw = sm_m[w * 8 + hd];
            if (mw == -INFINITY) continue;                         // a warp without pages
            const float sc = fast_exp2(mw - M);
            acc = fmaf(sc, sm_o[(size_t)(w * 8 + hd) * D + d], acc);
            l = fmaf(sc, sm_l[w * 8 + hd], l);
        }
        const size_t slot = ((size_t)n * Hq + h * G + hd) * n_slots + split;
        part_o[slot * D + d] = acc;
        if (d == 0) part_ml[slot] = make_float2(M, l);
    }
}

// Dynamic shared-memory opt-in, once per CUDA context.
template <int D, int G, int S>
int opt_in() {
    static PerContextOnce once;
    return once.run([] {
        LF_CHECK_CUDA(cudaFuncSetAttribute(split_mma_kernel<D, G, S>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Layout<D, S>::kSmemBytes));
        return LF_OK;
    });
}

template <int D, int S>
int launch_d(int G, dim3 grid, cudaStream_t st, const CUtensorMap& mk, const CUtensorMap& mv,
             const uint16_t* q, const int32_t* bt, const int32_t* lens, float* po, float2* pml,
             int Hq, int Hkv, int num_pages, int max_pages, int pps, int first_page, int n_slots,
             float qscale, const uint16_t* k_new, const uint16_t* v_new, uint16_t* kp_w,
             uint16_t* vp_w) {
    int rc = LF_OK;
#define LF_MMA_CASE(GG)                                                                         \
    case GG:                                                                                    \
        rc = opt_in<D, GG, S>();                                                                \
        if (rc != LF_OK) return rc;                                                             \
        split_mma_kernel<D, GG, S><<<grid, kThreads, Layout<D, S>::kSmemBytes, st>>>(           \
            mk, mv, q, bt, lens, po, pml, Hq, Hkv, num_pages, max_pages, pps, first_page,       \
            n_slots, qscale, k_new, v_new, kp_w, vp_w);                                         \
        return LF_OK;
    switch (G) {
        LF_MMA_CASE(1)
        LF_MMA_CASE(2)
        LF_MMA_CASE(4)
        LF_MMA_CASE(8)
        default: return set_error(LF_EINVAL, "decode: Hq/Hkv must be 1, 2, 4 or 8 (got %d)", G);
    }
#undef LF_MMA_CASE
}

}  // namespace mma

// Per-session pages of a paged decode: grid (split, KV head, session); partials into the
// workspace slots [0, max_split) of every (session, query head) row.  With k_new / v_new
// ([N][Hkv][D]) each session's newest token is stored into its last page first (fused append).
int launch_split_mma(dim3 grid, cudaStream_t st, const uint16_t* q, const uint16_t* kp,
                     const uint16_t* vp, const int32_t* bt, const int32_t* lens, float* po,
                     float2* pml, int Hq, int Hkv, int D, int num_pages, int max_pages, int pps,
                     int first_page, int n_slots, float qscale, const uint16_t* k_new,
                     const uint16_t* v_new) {
    uint16_t* kp_w = const_cast<uint16_t*>(kp);
    uint16_t* vp_w = const_cast<uint16_t*>(vp);
    CUtensorMap mk, mv;
    // pages [P*Hkv][16][D]: box = one page of one head, 64 dims (128-byte swizzled rows).
    const cuuint64_t dims[3] = {(cuuint64_t)D, 16, (cuuint64_t)num_pages * Hkv};
    const cuuint64_t str[2] = {(cuuint64_t)D * 2, (cuuint64_t)16 * D * 2};
    const cuuint32_t box[3] = {64, 16, 1};
    int rc = encode_bf16_map(&mk, kp, 3, dims, str, box);
    if (rc) return rc;
    rc = encode_bf16_map(&mv, vp, 3, dims, str, box);
    if (rc) return rc;
    const int G = Hq / Hkv;
    if (D == 128)
        return mma::launch_d<128, mma::kStages>(G, grid, st, mk, mv, q, bt, lens, po, pml, Hq, Hkv,
                                                num_pages, max_pages, pps, first_page, n_slots,
                                                qscale, k_new, v_new, kp_w, vp_w);
    return mma::launch_d<64, mma::kStages>(G, grid, st, mk, mv, q, bt, lens, po, pml, Hq, Hkv,
                                           num_pages, max_pages, pps, first_page, n_slots, qscale,
                                           k_new, v_new, kp_w, vp_w);
}

}  // namespace decode
}  // namespace lf
