// tcgen05 attention core, two query tiles per CTA ("ping-pong").
//
// Same math and the same two instantiations as attn_tc.cuh (Dense prefill, Prefix decode
// pass), but each CTA owns two 128-row query tiles that share one K/V stream.  While the
// softmax warpgroup of one tile works on its scores, the tensor core runs the other tile's
// QK^T and P.V, so neither the MMA pipe nor the softmax waits on the other.
//
// Roles (384 threads, 12 warps):
//   warp 0        TMA producer: Q of both tiles once, then K and V blocks into a 2-stage ring;
//   warp 1        TMEM owner and MMA issuer (one thread); per key block j, in order:
//                   PV(0, j) [after P_0 ready], QK(0, j+1), PV(1, j) [after P_1 ready], QK(1, j+1);
//                 S_t(j+1) overwrites P_t(j) in TMEM only after PV(t, j) has been issued, and
//                 tcgen05 MMAs of one thread run in issue order;
//   warps 2-3     idle;
//   warps 4-7     softmax + epilogue of tile 0, warps 8-11 of tile 1 (thread = query row =
//                 TMEM lane).  Scores are read from TMEM in two passes of 64 columns (row max,
//                 then exp2 / sum / bf16 pack), and the bf16 P row is written back over the
//                 first 64 columns of the same S buffer, where PV reads it as the A operand.
// TMEM (512 columns): S0/P0 [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512).
// Causal pairing: the two tiles are adjacent query tiles; the upper one needs one more key
// block than the lower one, which skips that block's MMAs and softmax.
#pragma once

#include "lf_common.cuh"
#include "sm100_primitives.cuh"

#include <math.h>

namespace lf {
namespace tc2 {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int HD = 128;
constexpr int kThreads = 384;
constexpr uint32_t kTileBytes = BM * HD * 2;      // 32 KB
constexpr uint32_t kHalfBytes = kTileBytes / 2;   // 16 KB: [128 rows][64 dims]
constexpr uint32_t kPageBoxBytes = 16 * 64 * 2;   // 2 KB: [16 rows][64 dims]
constexpr uint32_t OFF_Q = 0;                            // 2 tiles
constexpr uint32_t OFF_K = OFF_Q + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_V = OFF_K + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_BAR = OFF_V + 2 * kTileBytes;
constexpr uint32_t OFF_LEN = OFF_BAR + 256;              // per-row session lengths (prefix mode)
constexpr uint32_t kSmemBytes = OFF_LEN + 1024 + 1024;
constexpr uint32_t kColS = 0, kColO = 256, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 3, V_FULL = 5, V_EMPTY = 7, S_FULL = 9, P_FULL = 11,
           O_DONE = 13, NUM_BARS = 15 };

enum class Mode { Dense, Prefix };

struct Params {
    float c;
    uint16_t* o;
    float* lse;
    int B, Hq, Hkv, Sq, Sk, n_qt, n_pairs, causal, q_offset;
    const int32_t* bt;
    const int32_t* lens;
    float* part_o;
    float2* part_ml;
    int N, G, num_pages, max_pages, n_prefix, chunk_pages, n_chunks, n_qtiles, n_slots, slot0;
};

template <Mode M>
__global__ void __launch_bounds__(kThreads, 1)
attn2_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
             const __grid_constant__ CUtensorMap tmv, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    auto bar = [&](int i) { return sbase + OFF_BAR + 8u * i; };
    int* abort_flag = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8 * NUM_BARS + 8);
    int* s_misc = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS + 16);
    int* s_len = reinterpret_cast<int*>(smem + OFF_LEN);     // [256]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- tile coordinates (tile t = 0, 1) ----
    int bhq = 0, kvh = 0, q_row0[2] = {0, 0};
    int h = 0, n0 = 0, p_begin = 0, p_end = 0;
    int nb[2] = {0, 0};
    if constexpr (M == Mode::Dense) {
        const int BH = p.B * p.Hq;
        bhq = blockIdx.x % BH;
        const int pair = p.n_pairs - 1 - static_cast<int>(blockIdx.x / BH);   // heavy first
        const int b = bhq / p.Hq, hq = bhq % p.Hq;
        kvh = b * p.Hkv + hq / (p.Hq / p.Hkv);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            q_row0[t] = (2 * pair + t) * BM;
            if (q_row0[t] >= p.Sq) { nb[t] = 0; continue; }
            int kv_end = p.Sk;
            if (p.causal) kv_end = min(p.Sk, q_row0[t] + BM + p.q_offset);
            nb[t] = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
        }
    } else {
        const int qtile = blockIdx.x % p.n_qtiles;             // 2 x 128 rows
        const int rest = blockIdx.x / p.n_qtiles;
        h = rest % p.Hkv;
        const int chunk = rest / p.Hkv;
        const int spt = 2 * BM / p.G;
        n0 = qtile * spt;
        p_begin = chunk * p.chunk_pages;
        p_end = min(p_begin + p.chunk_pages, p.n_prefix);
        if (threadIdx.x < 2 * BM) {
            const int n = n0 + threadIdx.x / p.G;
            s_len[threadIdx.x] = n < p.N ? min(max(p.lens[n], 0), p.max_pages * 16) : 0;
        }
        if (threadIdx.x == 0) {
            int best = n0, best_len = -1;
            for (int n = n0; n < min(n0 + spt, p.N); ++n) {
                const int L = min(max(p.lens[n], 0), p.max_pages * 16);
                if (L > best_len) { best_len = L; best = n; }
            }
            s_misc[0] = best;
            s_misc[1] = (max(best_len, 0) + 15) / 16;
        }
        __syncthreads();
        p_end = min(p_end, s_misc[1]);
        const int n = p_end > p_begin ? (p_end - p_begin + 7) / 8 : 0;
        nb[0] = nb[1] = n;
    }
    const int nbk = max(nb[0], nb[1]);   // key blocks streamed (nb[0] <= nb[1])

    if (threadIdx.x == 0) {
        mbar_init(bar(Q_FULL), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(K_FULL + s), 1);
            mbar_init(bar(K_EMPTY + s), 1);
            mbar_init(bar(V_FULL + s), 1);
            mbar_init(bar(V_EMPTY + s), 1);
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(P_FULL + s), 128);
            mbar_init(bar(O_DONE + s), 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && nbk > 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            mbar_arrive_expect_tx(bar(Q_FULL), 2 * kTileBytes);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint32_t dst = sbase + OFF_Q + t * kTileBytes;
                if constexpr (M == Mode::Dense) {
                    tma_load_3d(dst, &tmq, bar(Q_FULL), 0, q_row0[t], bhq);
                    tma_load_3d(dst + kHalfBytes, &tmq, bar(Q_FULL), 64, q_row0[t], bhq);
                } else {
                    const int nt = n0 + t * (BM / p.G);
                    tma_load_4d(dst, &tmq, bar(Q_FULL), 0, 0, h, nt);
                    tma_load_4d(dst + kHalfBytes, &tmq, bar(Q_FULL), 64, 0, h, nt);
                }
            }
            const int32_t* bt_row = nullptr;
            if constexpr (M == Mode::Prefix) bt_row = p.bt + (size_t)s_misc[0] * p.max_pages;
            auto load_kv = [&](const CUtensorMap* map, uint32_t dst, uint32_t full, int j) {
                if constexpr (M == Mode::Dense) {
                    tma_load_3d(dst, map, full, 0, j * BN, kvh);
                    tma_load_3d(dst + kHalfBytes, map, full, 64, j * BN, kvh);
                } else {
#pragma unroll 1
                    for (int pg = 0; pg < 8; ++pg) {
                        const int pi = p_begin + j * 8 + pg;
                        int row = p.num_pages * p.Hkv;               // out of range: zeros
                        if (pi < p_end) {
                            const int page = bt_row[pi];
                            if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_pages))
                                atomicCAS(&g_device_error, 0, 201);
                            else
                                row = page * p.Hkv + h;
                        }
                        tma_load_3d(dst + pg * kPageBoxBytes, map, full, 0, 0, row);
                        tma_load_3d(dst + kHalfBytes + pg * kPageBoxBytes, map, full, 64, 0, row);
                    }
                }
            };
            for (int j = 0; j < nbk; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(bar(K_EMPTY + st), ph ^ 1, abort_flag, 1)) break;
                mbar_arrive_expect_tx(bar(K_FULL + st), kTileBytes);
                load_kv(&tmk, sbase + OFF_K + st * kTileBytes, bar(K_FULL + st), j);
                if (!mbar_wait(bar(V_EMPTY + st), ph ^ 1, abort_flag, 2)) break;
                mbar_arrive_expect_tx(bar(V_FULL + st), kTileBytes);
                load_kv(&tmv, sbase + OFF_V + st * kTileBytes, bar(V_FULL + st), j);
            }
            for (int j = max(0, nbk - 2); j < nbk; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(bar(K_EMPTY + st), ph, abort_flag, 10)) break;
                if (!mbar_wait(bar(V_EMPTY + st), ph, abort_flag, 11)) break;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && nbk > 0) {
            constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, false);
            constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, HD, true);
            auto qk = [&](int t, int st) {
                const uint32_t d = tmem + kColS + t * 128;
                const uint32_t qa = sbase + OFF_Q + t * kTileBytes, ka = sbase + OFF_K + st * kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
                    mma_ss(d, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024),
                           idesc_qk, kk > 0);
                }
            };
            auto pv = [&](int t, int st, bool acc) {
                const uint32_t va = sbase + OFF_V + st * kTileBytes;
                const uint32_t pa = tmem + kColS + t * 128;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    mma_ts(tmem + kColO + t * 128, pa + kk * 8,
                           sdesc_sw128(va + kk * 2048, kHalfBytes, 1024), idesc_pv,
                           (acc || kk > 0) ? 1u : 0u);
            };
            bool ok = mbar_wait(bar(Q_FULL), 0, abort_flag, 3);
            // block 0 scores for both tiles
            ok = ok && mbar_wait(bar(K_FULL + 0), 0, abort_flag, 4);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < 2; ++t)
                    if (nb[t] > 0) {
                        qk(t, 0);
                        mma_commit(bar(S_FULL + t));
                    }
                mma_commit(bar(K_EMPTY + 0));
            }
            for (int j = 0; ok && j < nbk; ++j) {
                const int st = j & 1;
                const bool next = j + 1 < nbk;
                // V(j) and K(j+1) are awaited lazily, right before their first use, so a load
                // still in flight never holds back an MMA that could already run.
                bool have_v = false, have_k = false;
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (j < nb[t]) {
                        if (!have_v) {
                            if (!mbar_wait(bar(V_FULL + st), (j >> 1) & 1, abort_flag, 6)) { ok = false; break; }
                            have_v = true;
                        }
                        if (!mbar_wait(bar(P_FULL + t), j & 1, abort_flag, 5)) { ok = false; break; }
                        tc_fence_after();
                        pv(t, st, j > 0);
                        mma_commit(bar(O_DONE + t));
                        if (j + 1 < nb[t]) {
                            if (!have_k) {
                                if (!mbar_wait(bar(K_FULL + (st ^ 1)), ((j + 1) >> 1) & 1, abort_flag, 4)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                                have_k = true;
                            }
                            qk(t, st ^ 1);
                            mma_commit(bar(S_FULL + t));
                        }
                    }
                }
                if (!ok) break;
                mma_commit(bar(V_EMPTY + st));
                if (next) mma_commit(bar(K_EMPTY + (st ^ 1)));
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- softmax + epilogue (tile t) ----------------
        const int t = (warp - 4) >> 2;
        const int row = ((warp - 4) & 3) * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t s_col = tmem + lane_off + kColS + t * 128;
        const uint32_t o_col = tmem + lane_off + kColO + t * 128;
        const int n_blk = nb[t];
        int qpos = 0, key_limit = 0;
        if constexpr (M == Mode::Dense) {
            qpos = q_row0[t] + row + p.q_offset;
            key_limit = p.Sk;
        } else {
            key_limit = min(s_len[t * BM + row], p_end * 16) - p_begin * 16;
        }
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_blk; ++j) {
            if (!mbar_wait(bar(S_FULL + t), j & 1, abort_flag, 7)) { ok = false; break; }
            tc_fence_after();
            // Visible keys of this block form a prefix [0, lim) of its columns (ragged end
            // and causal diagonal alike).  Masked blocks are rare (the last and the diagonal
            // ones): their S row is rewritten in TMEM with -inf past lim, so the two passes
            // below stay branch-free and small.
            const int kbase = j * BN;
            int lim = key_limit - kbase;
            if constexpr (M == Mode::Dense)
                if (p.causal) lim = min(lim, qpos - kbase + 1);
            if (__any_sync(0xffffffffu, lim < BN)) {
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t r[32];
                    tmem_ld32(s_col + cc * 32, r);
                    tmem_wait_ld();
                    const int l = lim - cc * 32;
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = (i < l) ? r[i] : 0xff800000u;   // -inf
                    tmem_st32(s_col + cc * 32, r);
                }
                tmem_wait_st();
            }
            // pass 1: row max
            float mxs[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) mxs[i] = -INFINITY;
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t r[32], r2[32];
                tmem_ld32(s_col + hf * 64, r);
                tmem_ld32(s_col + hf * 64 + 32, r2);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    mxs[i & 7] = fmaxf(mxs[i & 7], fmaxf(__uint_as_float(r[i]), __uint_as_float(r2[i])));
            }
            const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                                   fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
            const float m_blk = mx * p.c;
            const float m_new = (m_blk > m_run + kRescaleThreshold) ? m_blk : m_run;
            const float alpha = (m_new == m_run) ? 1.f : fast_exp2(m_run - m_new);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            // pass 2: exp2, row sum, bf16 P over the first 64 columns of this S buffer.  Scale
            // and shift run as packed f32x2 FMAs; a quarter of the exponentials are computed
            // on the FMA pipe (exp2_poly2) so the MUFU unit is not the limit.
            const uint64_t c2 = f2_pack(p.c, p.c), nm2 = f2_pack(-m_use, -m_use);
            uint64_t lsa = f2_pack(0.f, 0.f), lsb = f2_pack(0.f, 0.f);
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t r[32], r2[32], pr[32];
                tmem_ld32(s_col + hf * 64, r);
                tmem_ld32(s_col + hf * 64 + 32, r2);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 a = f2_unpack(ffma2(
                        f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), c2, nm2));
                    const uint64_t b = ffma2(
                        f2_pack(__uint_as_float(r2[2 * i]), __uint_as_float(r2[2 * i + 1])), c2, nm2);
                    const float e0 = fast_exp2(a.x), e1 = fast_exp2(a.y);
                    float2 f;
                    if ((i & 1) == 0) {
                        f = exp2_poly2(b);
                    } else {
                        const float2 bv = f2_unpack(b);
                        f = make_float2(fast_exp2(bv.x), fast_exp2(bv.y));
                    }
                    lsa = fadd2(lsa, f2_pack(e0, e1));
                    lsb = fadd2(lsb, f2_pack(f.x, f.y));
                    pr[i] = pack_bf16x2(e0, e1);
                    pr[16 + i] = pack_bf16x2(f.x, f.y);
                }
                // columns [hf*32, hf*32+32) hold P of score columns [hf*64, hf*64+64): those
                // scores were read above, so the overwrite is safe.
                tmem_st32(s_col + hf * 32, pr);
            }
            const float2 lsv = f2_unpack(fadd2(lsa, lsb));
            const float lsum = lsv.x + lsv.y;
            if (j > 0) {
                if (!mbar_wait(bar(O_DONE + t), (j - 1) & 1, abort_flag, 8)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    uint32_t r[32];
#pragma unroll
                    for (int cc = 0; cc < HD / 32; ++cc) {
                        tmem_ld32(o_col + cc * 32, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                        tmem_st32(o_col + cc * 32, r);
                    }
                }
            }
            l_run = l_run * alpha + lsum;
            m_run = m_new;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(P_FULL + t));
        }

        if (n_blk > 0 && ok) {
            ok = mbar_wait(bar(O_DONE + t), (n_blk - 1) & 1, abort_flag, 9);
            tc_fence_after();
        }
        if constexpr (M == Mode::Dense) {
            const int grow = q_row0[t] + row;
            const size_t orow = static_cast<size_t>(bhq) * p.Sq + grow;
            if (ok && q_row0[t] < p.Sq) {
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t r[32];
                    if (n_blk > 0) {
                        tmem_ld32(o_col + cc * 32, r);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = 0u;
                    }
                    if (grow < p.Sq) {
                        uint4* dst = reinterpret_cast<uint4*>(p.o + orow * HD + cc * 32);
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint4 w;
                            w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
                            w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
                            w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
                            w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
                            dst[v] = w;
                        }
                    }
                }
                if (p.lse != nullptr && grow < p.Sq)
                    p.lse[orow] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
            }
        } else {
            const int rr = t * BM + row;
            const int n = n0 + rr / p.G;
            const int chunk = static_cast<int>(blockIdx.x) / (p.n_qtiles * p.Hkv);
            const size_t slot =
                ((size_t)n * (p.Hkv * p.G) + h * p.G + rr % p.G) * p.n_slots + p.slot0 + chunk;
            if (ok) {
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t r[32];
                    if (n_blk > 0) {
                        tmem_ld32(o_col + cc * 32, r);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = 0u;
                    }
                    if (n < p.N) {
                        float4* dst = reinterpret_cast<float4*>(p.part_o + slot * HD + cc * 32);
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                 __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
                    }
                }
                if (n < p.N) p.part_ml[slot] = make_float2(m_run, l_run);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
    if (threadIdx.x == 0 && *abort_flag != 0) atomicCAS(&g_device_error, 0, 100 + *abort_flag);
}

}  // namespace tc2
}  // namespace lf
