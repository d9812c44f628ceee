// Shared-prefix pass of the paged decode.
//
// When every session's block table starts with the same num_prefix_pages pages (a prefix
// forked to all sessions: the KV-fusion case), those pages are read once per group of
// 4-8 sessions rather than once per session.  CTA (chunk, kv_head, group) stages
// each prefix page of its chunk in shared memory (16-byte loads, next page prefetched into
// registers while the current one is used) and each warp applies it to one or two
// sessions with the same lane layout and reductions as the per-session split kernel.  Every
// session is owned by one warp, so its partial (o, max, sum) for the chunk is written
// directly to the slot suffix_splits + chunk; the combine kernel merges it with the
// session's own splits.
//
// The page ids are read from the group's longest session; callers guarantee the prefix
// entries a session holds equal everybody else's (KVPool.fork produces exactly that).  Tokens
// at or past a session's length are masked, so a session shorter than the prefix is exact.
#include "decode_common.cuh"

#include <math.h>

namespace lf {
namespace decode {

// Sessions per warp: two keep the q and accumulator registers of a GQA group of <= 4 heads
// resident; a group of 8 heads takes one.
template <int G>
struct PrefixCfg {
    static constexpr int SPW = G >= 8 ? 1 : 2;
    static constexpr int SPC = kWarps * SPW;
};

template <int D, int G>
__global__ void __launch_bounds__(kThreads)
prefix_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kp,
              const uint16_t* __restrict__ vp, const int32_t* __restrict__ bt,
              const int32_t* __restrict__ seq_lens, float* __restrict__ part_o,
              float2* __restrict__ part_ml, int N, int Hq, int Hkv, int num_pages, int max_pages,
              int n_prefix, int pages_per_chunk, int n_slots, int slot0, float qscale) {
    using C = Cfg<D, G>;
    constexpr int SPW = PrefixCfg<G>::SPW;
    constexpr int kVec = kPage * D / 8;                  // uint4 per page of one head
    constexpr int kPer = (kVec + kThreads - 1) / kThreads;
    const int chunk = blockIdx.x, h = blockIdx.y, grp = blockIdx.z;
    const int p_begin = chunk * pages_per_chunk;
    const int p_end = min(p_begin + pages_per_chunk, n_prefix);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = lane % C::LPT, sub = lane / C::LPT;
    const int hl = head_of_chunk<D, G>(c);

    __shared__ __align__(16) uint4 sk[kVec];
    __shared__ __align__(16) uint4 sv[kVec];

    // Page ids come from the group's longest session: every session's row holds the shared
    // pages it covers, and the longest one covers all the pages any session here needs.
    const int n0 = grp * PrefixCfg<G>::SPC;
    __shared__ int s_src, s_src_pages;
    if (threadIdx.x == 0) {
        int best = n0, best_len = -1;
        for (int n = n0; n < min(n0 + PrefixCfg<G>::SPC, N); ++n) {
            const int L = min(max(seq_lens[n], 0), max_pages * kPage);
            if (L > best_len) { best_len = L; best = n; }
        }
        s_src = best;
        s_src_pages = (max(best_len, 0) + kPage - 1) / kPage;
    }
    __syncthreads();
    const int32_t* bt_row = bt + (size_t)s_src * max_pages;
    const int p_stop = min(p_end, s_src_pages);

    int sess[SPW], len[SPW];
    float qf[SPW][G][8], acc[SPW][G][8], m_run[SPW], l_run[SPW];
#pragma unroll
    for (int i = 0; i < SPW; ++i) {
        const int n = n0 + warp * SPW + i;
        sess[i] = n;
        len[i] = n < N ? min(max(seq_lens[n], 0), max_pages * kPage) : 0;
        m_run[i] = -INFINITY;
        l_run[i] = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (n < N) {
                const uint4 raw =
                    *reinterpret_cast<const uint4*>(q + ((size_t)n * Hq + h * G + g) * D + 8 * c);
                unpack8(raw, qf[i][g]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) qf[i][g][j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                qf[i][g][j] *= qscale;
                acc[i][g][j] = 0.f;
            }
        }
    }

    uint4 nk[kPer], nv[kPer];
    auto fetch = [&](int pi) {
        const size_t base = ((size_t)checked_page(bt_row[pi], num_pages) * Hkv + h) * (size_t)(kPage * D);
        const uint4* kb = reinterpret_cast<const uint4*>(kp + base);
        const uint4* vb = reinterpret_cast<const uint4*>(vp + base);
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            const int idx = threadIdx.x + e * kThreads;
            if (idx < kVec) {
                nk[e] = ldg_stream(kb + idx);
                nv[e] = ldg_stream(vb + idx);
            }
        }
    };
    if (p_begin < p_stop) fetch(p_begin);

    for (int pi = p_begin; pi < p_stop; ++pi) {
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
            const int idx = threadIdx.x + e * kThreads;
            if (idx < kVec) {
                sk[idx] = nk[e];
                sv[idx] = nv[e];
            }
        }
        __syncthreads();
        if (pi + 1 < p_stop) fetch(pi + 1);

#pragma unroll
        for (int i = 0; i < SPW; ++i) {
            const int L = len[i];
            const int tok0 = pi * kPage + sub;
            if (pi * kPage >= L) continue;               // warp-uniform: whole page masked
            float s[C::ROWS];
#pragma unroll
            for (int r = 0; r < C::ROWS; ++r) {
                float kf[8];
                unpack8(sk[(r * C::TPI + sub) * (D / 8) + c], kf);
                float part[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float a = 0.f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) a = fmaf(qf[i][g][j], kf[j], a);
                    part[g] = a;
                }
                const float sc = reduce_scatter_row<D, G>(part, c);
                s[r] = (tok0 + r * C::TPI < L) ? sc : -INFINITY;
            }
            float mx = s[0];
#pragma unroll
            for (int r = 1; r < C::ROWS; ++r) mx = fmaxf(mx, s[r]);
#pragma unroll
            for (int off = C::LPT; off < 32; off <<= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[i], mx);
            const float alpha = fast_exp2(m_run[i] - m_new);
            float p[C::ROWS];
            float ps = 0.f;
#pragma unroll
            for (int r = 0; r < C::ROWS; ++r) {
                p[r] = fast_exp2(s[r] - m_new);
                ps += p[r];
            }
#pragma unroll
            for (int off = C::LPT; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l_run[i] = l_run[i] * alpha + ps;
            m_run[i] = m_new;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float ag = __shfl_sync(0xffffffffu, alpha, chunk_of_head<D, G>(g));
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][g][j] *= ag;
            }
#pragma unroll
            for (int r = 0; r < C::ROWS; ++r) {
                float vf[8];
                unpack8(sv[(r * C::TPI + sub) * (D / 8) + c], vf);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg =
                        __shfl_sync(0xffffffffu, p[r], sub * C::LPT + chunk_of_head<D, G>(g));
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[i][g][j] = fmaf(pg, vf[j], acc[i][g][j]);
                }
            }
        }
        __syncthreads();
    }

    // Prefix slots hold the normalised output O / l as bf16 in the first D * 2 bytes of the
    // slot (half the bytes of fp32; the combine scales it back by l), plus (m, l) in part_ml.
#pragma unroll
    for (int i = 0; i < SPW; ++i) {
        if (sess[i] >= N) continue;
#pragma unroll
        for (int off = C::LPT; off < 32; off <<= 1)
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    acc[i][g][j] += __shfl_xor_sync(0xffffffffu, acc[i][g][j], off);
        float inv_l[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float lg = __shfl_sync(0xffffffffu, l_run[i], chunk_of_head<D, G>(g));
            inv_l[g] = lg > 0.f ? 1.f / lg : 0.f;
        }
        if (sub == 0) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const size_t slot = ((size_t)sess[i] * Hq + h * G + g) * n_slots + slot0 + chunk;
                uint4 pk;
                pk.x = pack_bf16x2(acc[i][g][0] * inv_l[g], acc[i][g][1] * inv_l[g]);
                pk.y = pack_bf16x2(acc[i][g][2] * inv_l[g], acc[i][g][3] * inv_l[g]);
                pk.z = pack_bf16x2(acc[i][g][4] * inv_l[g], acc[i][g][5] * inv_l[g]);
                pk.w = pack_bf16x2(acc[i][g][6] * inv_l[g], acc[i][g][7] * inv_l[g]);
                reinterpret_cast<uint4*>(part_o + slot * D)[c] = pk;
            }
            if (c == chunk_of_head<D, G>(hl)) {
                const size_t slot = ((size_t)sess[i] * Hq + h * G + hl) * n_slots + slot0 + chunk;
                part_ml[slot] = make_float2(m_run[i], l_run[i]);
            }
        }
    }
}

template <int D>
static int dispatch_prefix(int G, dim3 grid, cudaStream_t st, const uint16_t* q,
                           const uint16_t* kp, const uint16_t* vp, const int32_t* bt,
                           const int32_t* lens, float* po, float2* pml, int N, int Hq, int Hkv,
                           int num_pages, int max_pages, int n_prefix, int ppc, int n_slots,
                           int slot0, float qscale) {
#define LF_PREFIX_CASE(GG)                                                                     \
    case GG:                                                                                   \
        prefix_kernel<D, GG><<<grid, kThreads, 0, st>>>(q, kp, vp, bt, lens, po, pml, N, Hq, Hkv, \
                                                        num_pages, max_pages, n_prefix, ppc,      \
                                                        n_slots, slot0, qscale);                 \
        break;
    switch (G) {
        LF_PREFIX_CASE(1)
        LF_PREFIX_CASE(2)
        LF_PREFIX_CASE(4)
        LF_PREFIX_CASE(8)
        default: return set_error(LF_EINVAL, "decode: Hq/Hkv must be 1, 2, 4 or 8 (got %d)", G);
    }
#undef LF_PREFIX_CASE
    return launch_status("decode prefix");
}

// Tensor-core version (head_dim 128), in prefill.cu.
int launch_prefix_tc(const uint16_t* q, const uint16_t* kp, const uint16_t* vp, const int32_t* bt,
                     const int32_t* lens, float* po, float2* pml, int N, int Hq, int Hkv,
                     int num_pages, int max_pages, int n_prefix, int chunk_pages, int n_slots,
                     int slot0, float qscale, cudaStream_t st);

// head_dim 128 runs on the tensor cores; head_dim 64 on the CUDA-core kernel above.
int launch_prefix(const uint16_t* q, const uint16_t* kp, const uint16_t* vp, const int32_t* bt,
                  const int32_t* lens, float* po, float2* pml, int N, int Hq, int Hkv, int D,
                  int num_pages, int max_pages, int n_prefix, int pages_per_chunk, int n_slots,
                  int slot0, float qscale, cudaStream_t st) {
    if (D == 128)
        return launch_prefix_tc(q, kp, vp, bt, lens, po, pml, N, Hq, Hkv, num_pages, max_pages,
                                n_prefix, pages_per_chunk, n_slots, slot0, qscale, st);
    const int G = Hq / Hkv;
    const int spc = G >= 8 ? PrefixCfg<8>::SPC : PrefixCfg<1>::SPC;
    dim3 grid((n_prefix + pages_per_chunk - 1) / pages_per_chunk, Hkv, (N + spc - 1) / spc);
    return D == 128 ? dispatch_prefix<128>(G, grid, st, q, kp, vp, bt, lens, po, pml, N, Hq, Hkv,
                                           num_pages, max_pages, n_prefix, pages_per_chunk, n_slots,
                                           slot0, qscale)
                    : dispatch_prefix<64>(G, grid, st, q, kp, vp, bt, lens, po, pml, N, Hq, Hkv,
                                          num_pages, max_pages, n_prefix, pages_per_chunk, n_slots,
                                          slot0, qscale);
}

}  // namespace decode
}  // namespace lf
