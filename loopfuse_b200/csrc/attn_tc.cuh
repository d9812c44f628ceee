// tcgen05 attention core shared by the prefill op and the decode's shared-prefix pass.
//
// One CTA computes softmax(Q K^T * scale) V for a 128-row query tile against a run of 128-key
// blocks.  Roles (256 threads):
//   warp 0      TMA producer: Q once, then K and V blocks into a 2-stage ring of
//               128-byte-swizzled [rows][64 dims] boxes;
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_j = Q K_j^T   into TMEM S[j%2]   (M=128, N=128, K=128 -> 8 MMAs),
//                 O  += P_j V_j   with P_j read from TMEM P[j%2] (A operand in TMEM);
//               S_{j+2} is issued right after PV_j so the tensor core has work while the
//               softmax warps process block j+1;
//   warps 4-7   softmax, one thread per query row (TMEM lane = row): tcgen05.ld the S row, mask,
//               row max in the log2 domain, exp2, row sum, bf16 P packed into TMEM with
//               tcgen05.st.  The running max is only raised when it grows by more than 8 (a
//               factor 256), so O in TMEM is rescaled rarely; O and the row sum always refer to
//               the same max, so the result is exact.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O [256,384), P0 [384,448), P1 [448,512).
//
// Two instantiations:
//   Dense  (prefill)  Q [B,Hq,Sq,D], K/V [B,Hkv,Sk,D]; causal mask with queries aligned to the
//                     end of the keys; bf16 O normalised + natural-log LSE.
//   Prefix (decode)   128 query rows = 128/G sessions x the G query heads of one KV head (a 4-D
//                     TMA box over q [N][Hkv][G][D]); K/V are pool pages [P][Hkv][16][D] fetched
//                     through the block table, 8 pages (16-row boxes) per 128-key block, pages
//                     past the run read as zeros via out-of-range box coordinates; a key is
//                     visible when it lies inside the chunk and before the row's session length;
//                     the epilogue writes the unnormalised fp32 O and (max, sum) into the decode
//                     workspace slot of the chunk, merged later by the decode combine kernel.
//
// Every mbarrier wait is bounded in time; a timeout aborts all roles of the CTA, frees TMEM
// and leaves a code that lf_device_status() reports.
#pragma once

#include "lf_common.cuh"
#include "sm100_primitives.cuh"

#include <math.h>

namespace lf {
namespace tc {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int HD = 128;
constexpr int kThreads = 256;
constexpr uint32_t kTileBytes = BM * HD * 2;      // 32 KB: one Q, K or V tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;   // 16 KB: [128 rows][64 dims]
constexpr uint32_t kPageBoxBytes = 16 * 64 * 2;   // 2 KB: [16 rows][64 dims]
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + kTileBytes;           // 2 stages
constexpr uint32_t OFF_V = OFF_K + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_BAR = OFF_V + 2 * kTileBytes;     // barriers, TMEM slot, flags
constexpr uint32_t OFF_LEN = OFF_BAR + 256;              // per-row session lengths (prefix mode)
constexpr uint32_t kSmemBytes = OFF_LEN + 512 + 1024;    // + alignment slack
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;                // log2 units

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 3, V_FULL = 5, V_EMPTY = 7, S_FULL = 9, P_FULL = 11,
           O_DONE = 13, NUM_BARS = 14 };

enum class Mode { Dense, Prefix };

struct Params {
    float c;                 // softmax scale * log2(e)
    // dense
    uint16_t* o;
    float* lse;
    int B, Hq, Hkv, Sq, Sk, n_qt, causal, q_offset;
    // prefix
    const int32_t* bt;
    const int32_t* lens;
    float* part_o;
    float2* part_ml;
    int N, G, num_pages, max_pages, n_prefix, chunk_pages, n_chunks, n_qtiles, n_slots, slot0;
};

template <Mode M>
__global__ void __launch_bounds__(kThreads, 1)
attn_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
            const __grid_constant__ CUtensorMap tmv, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    auto bar = [&](int i) { return sbase + OFF_BAR + 8u * i; };
    int* abort_flag = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8 * NUM_BARS + 8);
    int* s_misc = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS + 16);   // [src row, pages]
    int* s_len = reinterpret_cast<int*>(smem + OFF_LEN);                         // [128]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- tile coordinates ----
    int bhq = 0, q_row0 = 0, kvh = 0;          // dense
    int h = 0, n0 = 0, p_begin = 0, p_end = 0; // prefix
    int n_blk = 0;
    if constexpr (M == Mode::Dense) {
        const int BH = p.B * p.Hq;
        bhq = blockIdx.x % BH;
        const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x / BH);   // heavy tiles first
        const int b = bhq / p.Hq, hq = bhq % p.Hq;
        kvh = b * p.Hkv + hq / (p.Hq / p.Hkv);
        q_row0 = qt * BM;
        int kv_end = p.Sk;
        if (p.causal) kv_end = min(p.Sk, q_row0 + BM + p.q_offset);
        n_blk = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
    } else {
        const int qtile = blockIdx.x % p.n_qtiles;
        const int rest = blockIdx.x / p.n_qtiles;
        h = rest % p.Hkv;
        const int chunk = rest / p.Hkv;
        const int spt = BM / p.G;                    // sessions per tile
        n0 = qtile * spt;
        p_begin = chunk * p.chunk_pages;
        p_end = min(p_begin + p.chunk_pages, p.n_prefix);
        if (threadIdx.x < BM) {
            const int n = n0 + threadIdx.x / p.G;
            s_len[threadIdx.x] = n < p.N ? min(max(p.lens[n], 0), p.max_pages * 16) : 0;
        }
        if (threadIdx.x == 0) {
            // Page ids come from the tile's longest session (it covers every page the tile needs).
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
        n_blk = p_end > p_begin ? (p_end - p_begin + 7) / 8 : 0;
    }

    if (threadIdx.x == 0) {
        mbar_init(bar(Q_FULL), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(K_FULL + s), 1);
            mbar_init(bar(K_EMPTY + s), 1);
            mbar_init(bar(V_FULL + s), 1);
            mbar_init(bar(V_EMPTY + s), 1);
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(P_FULL + s), 128);
        }
        mbar_init(bar(O_DONE), 1);
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
        if (lane == 0 && n_blk > 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
            mbar_arrive_expect_tx(bar(Q_FULL), kTileBytes);
            if constexpr (M == Mode::Dense) {
                tma_load_3d(sbase + OFF_Q, &tmq, bar(Q_FULL), 0, q_row0, bhq);
                tma_load_3d(sbase + OFF_Q + kHalfBytes, &tmq, bar(Q_FULL), 64, q_row0, bhq);
            } else {
                tma_load_4d(sbase + OFF_Q, &tmq, bar(Q_FULL), 0, 0, h, n0);
                tma_load_4d(sbase + OFF_Q + kHalfBytes, &tmq, bar(Q_FULL), 64, 0, h, n0);
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
                            int page = bt_row[pi];
                            if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_pages)) {
                                atomicCAS(&g_device_error, 0, 201);
                            } else {
                                row = page * p.Hkv + h;
                            }
                        }
                        tma_load_3d(dst + pg * kPageBoxBytes, map, full, 0, 0, row);
                        tma_load_3d(dst + kHalfBytes + pg * kPageBoxBytes, map, full, 64, 0, row);
                    }
                }
            };
            for (int j = 0; j < n_blk; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(bar(K_EMPTY + st), ph ^ 1, abort_flag, 1)) break;
                mbar_arrive_expect_tx(bar(K_FULL + st), kTileBytes);
                load_kv(&tmk, sbase + OFF_K + st * kTileBytes, bar(K_FULL + st), j);
                if (!mbar_wait(bar(V_EMPTY + st), ph ^ 1, abort_flag, 2)) break;
                mbar_arrive_expect_tx(bar(V_FULL + st), kTileBytes);
                load_kv(&tmv, sbase + OFF_V + st * kTileBytes, bar(V_FULL + st), j);
            }
            // Tail: wait until the MMA commits releasing the last use of each stage have
            // landed, so no barrier arrival reaches this CTA's shared memory after it exits.
            for (int j = max(0, n_blk - 2); j < n_blk; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(bar(K_EMPTY + st), ph, abort_flag, 10)) break;
                if (!mbar_wait(bar(V_EMPTY + st), ph, abort_flag, 11)) break;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && n_blk > 0) {
            constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, false);
            constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, HD, true);
            auto issue_qk = [&](int j) -> bool {
                const int st = j & 1;
                if (!mbar_wait(bar(K_FULL + st), (j >> 1) & 1, abort_flag, 4)) return false;
                tc_fence_after();
                const uint32_t d = tmem + kColS + (j & 1) * 128;
                const uint32_t qa = sbase + OFF_Q, ka = sbase + OFF_K + st * kTileBytes;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
                    mma_ss(d, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024),
                           idesc_qk, kk > 0);
                }
                mma_commit(bar(K_EMPTY + st));
                mma_commit(bar(S_FULL + (j & 1)));
                return true;
            };
            bool ok = mbar_wait(bar(Q_FULL), 0, abort_flag, 3);
            ok = ok && issue_qk(0);
            if (ok && n_blk > 1) ok = issue_qk(1);
            for (int j = 0; ok && j < n_blk; ++j) {
                const int st = j & 1;
                if (!mbar_wait(bar(P_FULL + (j & 1)), (j >> 1) & 1, abort_flag, 5)) break;
                if (!mbar_wait(bar(V_FULL + st), (j >> 1) & 1, abort_flag, 6)) break;
                tc_fence_after();
                const uint32_t va = sbase + OFF_V + st * kTileBytes;
                const uint32_t pa = tmem + kColP + (j & 1) * 64;
#pragma unroll
                for (int kk = 0; kk < BN / 16; ++kk)
                    mma_ts(tmem + kColO, pa + kk * 8, sdesc_sw128(va + kk * 2048, kHalfBytes, 1024),
                           idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
                mma_commit(bar(V_EMPTY + st));
                mma_commit(bar(O_DONE));
                if (j + 2 < n_blk && !issue_qk(j + 2)) break;
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---------------- softmax + epilogue ----------------
        const int row = (warp - 4) * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        // A key k of block j is visible when k < key_limit (and, causal, k <= qpos).
        int qpos = 0, first_q = 0, key_limit = 0;
        if constexpr (M == Mode::Dense) {
            qpos = q_row0 + row + p.q_offset;
            first_q = q_row0 + p.q_offset;
            key_limit = p.Sk;
        } else {
            key_limit = min(s_len[row], p_end * 16) - p_begin * 16;   // relative to the run
        }
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_blk; ++j) {
            if (!mbar_wait(bar(S_FULL + (j & 1)), (j >> 1) & 1, abort_flag, 7)) { ok = false; break; }
            tc_fence_after();
            float s[BN];
            {
                uint32_t r[32];
#pragma unroll
                for (int cc = 0; cc < BN / 32; ++cc) {
                    tmem_ld32(tmem + lane_off + kColS + (j & 1) * 128 + cc * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 32; ++t) s[cc * 32 + t] = __uint_as_float(r[t]);
                }
            }
            const int kbase = j * BN;
            bool need_mask = kbase + BN > key_limit;
            if constexpr (M == Mode::Dense) need_mask = need_mask || (p.causal && kbase + BN - 1 > first_q);
            if (need_mask) {
#pragma unroll
                for (int i = 0; i < BN; ++i) {
                    const int kpos = kbase + i;
                    bool vis = kpos < key_limit;
                    if constexpr (M == Mode::Dense) vis = vis && (!p.causal || kpos <= qpos);
                    s[i] = vis ? s[i] : -INFINITY;
                }
            }
            // Row max as 8 independent chains (one warp per scheduler: ILP hides latency).
            float mxs[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) mxs[t] = s[t];
#pragma unroll
            for (int i = 8; i < BN; i += 8)
#pragma unroll
                for (int t = 0; t < 8; ++t) mxs[t] = fmaxf(mxs[t], s[i + t]);
            const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                                   fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
            const float m_blk = mx * p.c;
            const float m_new = (m_blk > m_run + kRescaleThreshold) ? m_blk : m_run;
            const float alpha = (m_new == m_run) ? 1.f : fast_exp2(m_run - m_new);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            // P_j goes to TMEM P[j%2]; its previous reader PV_{j-2} finished before S_j was
            // committed, so the buffer is free.
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int cc = 0; cc < BN / 64; ++cc) {
                uint32_t pr[32];
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const float p0 = fast_exp2(fmaf(s[cc * 64 + 2 * t], p.c, -m_use));
                    const float p1 = fast_exp2(fmaf(s[cc * 64 + 2 * t + 1], p.c, -m_use));
                    ls[t & 3] += p0 + p1;
                    pr[t] = pack_bf16x2(p0, p1);
                }
                tmem_st32(tmem + lane_off + kColP + (j & 1) * 64 + cc * 32, pr);
            }
            const float lsum = (ls[0] + ls[1]) + (ls[2] + ls[3]);
            // Every O_DONE phase is awaited in order (PV_{j-1} here), which keeps the parity
            // unambiguous and makes O safe to rescale.
            if (j > 0) {
                if (!mbar_wait(bar(O_DONE), (j - 1) & 1, abort_flag, 8)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    uint32_t r[32];
#pragma unroll
                    for (int cc = 0; cc < HD / 32; ++cc) {
                        const uint32_t addr = tmem + lane_off + kColO + cc * 32;
                        tmem_ld32(addr, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int t = 0; t < 32; ++t)
                            r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
                        tmem_st32(addr, r);
                    }
                }
            }
            l_run = l_run * alpha + lsum;
            m_run = m_new;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(P_FULL + (j & 1)));
        }

        if (n_blk > 0 && ok) {
            ok = mbar_wait(bar(O_DONE), (n_blk - 1) & 1, abort_flag, 9);
            tc_fence_after();
        }
        if constexpr (M == Mode::Dense) {
            const int grow = q_row0 + row;
            const size_t orow = static_cast<size_t>(bhq) * p.Sq + grow;
            if (ok) {
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t r[32];
                    if (n_blk > 0) {
                        tmem_ld32(tmem + lane_off + kColO + cc * 32, r);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int t = 0; t < 32; ++t) r[t] = 0u;
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
            const int n = n0 + row / p.G;
            const int chunk = static_cast<int>(blockIdx.x) / (p.n_qtiles * p.Hkv);
            const size_t slot =
                ((size_t)n * (p.Hkv * p.G) + h * p.G + row % p.G) * p.n_slots + p.slot0 + chunk;
            if (ok) {
#pragma unroll
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t r[32];
                    if (n_blk > 0) {
                        tmem_ld32(tmem + lane_off + kColO + cc * 32, r);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int t = 0; t < 32; ++t) r[t] = 0u;
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

}  // namespace tc
}  // namespace lf
