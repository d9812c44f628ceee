// tcgen05 attention core: two query tiles per work item ("ping-pong"), dynamic work list.
//
// The grid has one CTA per work item, items in heavy-first order.  The first wave of CTAs (one
// per SM) keeps running: a CTA that finishes an item takes over the item of a CTA not launched
// yet (cluster launch control, below), so the SMs drain one shared queue.  An item is two
// 128-row query tiles that share one K/V stream.  While the softmax warpgroup of one tile works on its scores, the tensor core runs
// the other tile's QK^T and P.V, and the next item's Q/K loads and first QK^T overlap the
// previous item's epilogue.
//
// Roles (384 threads, 12 warps):
//   warp 0        TMA producer: per item, Q of both tiles (after the previous item's last QK^T
//                 released the Q buffer), then K and V blocks into a 2-stage ring shared by all
//                 items (running block counter g);
//   warp 1        TMEM owner and MMA issuer (the warp waits, one elected lane issues);
//                 per key block j of an item:
//                   PV(0, j) [after P_0 ready], QK(0, j+1), PV(1, j) [after P_1 ready], QK(1, j+1);
//                 S_t(j+1) overwrites P_t(j) in TMEM only after PV(t, j) has been issued, and
//                 tcgen05 MMAs of one thread run in issue order;
//   warps 2-3     idle;
//   warps 4-7     softmax + epilogue of tile 0, warps 8-11 of tile 1 (thread = query row =
//                 TMEM lane).  The whole 128-column S row comes into registers with one TMEM
//                 round trip; masked blocks (ragged end, causal diagonal) get -inf past the
//                 visible prefix of columns there.  Row max (three-input max), then exp2 / sum /
//                 bf16 pack, and the bf16 P row is written over the first 64 columns of the same
//                 S buffer, where P.V reads it as the A operand.  Scale-and-shift and row sums
//                 use packed f32x2 math, and two exponential pairs in eight run on the FMA pipe
//                 (exp2_poly2) to relieve the MUFU unit.  The first
//                 half of P is stored and signalled (P_HALF) before the second half is computed,
//                 so its P.V overlaps the rest of the softmax.  The running max is raised only when it
//                 grows by more than 8 (log2 units), so O is rarely rescaled; O and the row sum
//                 always refer to the same max, so the result is exact.
// TMEM (512 columns): S0/P0 [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512).
//
// Barrier phases are running counters across items, so each barrier's waiters see its phases
// strictly in order.  A tcgen05 commit signals completion of every earlier MMA of the issuing
// thread, so S_FULL(t) for block j+1 also tells softmax t that P.V(t, j) is done (O_t may be
// rescaled); O_DONE(t) is committed once per item, after the tile's last P.V.  The next item's
// first P.V (which overwrites O_t) is issued only after the softmax warps of tile t signalled P
// for that item, which they do after their epilogue has read O_t.
//
// Two instantiations:
//   Dense  (prefill)  Q [B,Hq,Sq,D], K/V [B,Hkv,Sk,D]; an item = query tiles (2i, 2i+1) of one
//                     (batch, head); causal mask with queries aligned to the end of the keys;
//                     bf16 O normalised + natural-log LSE.
//   Paged  (append)   varlen queries q [T_total, Hq, D] (session n owns rows cu_q[n]..cu_q[n+1])
//                     over that session's pool pages (its block-table row, lk[n] tokens including
//                     the new ones); an item = query tiles (2i, 2i+1) of one (session, query head);
//                     causal mask with the queries at the end of the session; bf16 O + LSE.
//   Prefix (decode)   an item = 2 x 128 query rows = 256/G sessions x G heads of one KV head and
//                     one chunk of shared-prefix pages; q via 4-D TMA boxes over [N][Hkv][G][D];
//                     K/V pages [P][Hkv][16][D] via 16-row boxes through the block table of the
//                     item's longest session (pages past the run read zeros); epilogue writes
//                     partials into the decode workspace: O / l as bf16, (max, sum) as fp32.
//
// Every mbarrier wait is bounded in time; a timeout aborts all roles, frees TMEM and leaves a
// code that lf_device_status() reports.
#pragma once

#include "lf_common.cuh"
#include "sm100_primitives.cuh"

#include <math.h>

namespace lf {
namespace tc2 {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kMaxHD = 128;                       // buffers are sized for head_dim 128
constexpr int kThreads = 384;
constexpr uint32_t kRegsControl = 88, kRegsSoftmax = 208;   // per thread, after the split
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * 168, "register split");
constexpr uint32_t kTileBytes = BM * kMaxHD * 2;  // 32 KB
constexpr uint32_t kHalfBytes = kTileBytes / 2;   // 16 KB: [128 rows][64 dims]
constexpr uint32_t kPageBoxBytes = 16 * 64 * 2;   // 2 KB: [16 rows][64 dims]
constexpr uint32_t OFF_Q = 0;                            // 2 tiles
constexpr uint32_t OFF_K = OFF_Q + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_V = OFF_K + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_EPI = OFF_V + 2 * kTileBytes;     // epilogue staging, 4 KB per softmax warp
constexpr uint32_t kEpiWarpBytes = 4096;
constexpr uint32_t OFF_BAR = OFF_EPI + 8 * kEpiWarpBytes;
constexpr uint32_t OFF_RESP = OFF_BAR + 256;               // work-ring responses, 16 B each
constexpr int kRing = 4;                                    // work-ring depth (a power of two)
constexpr uint32_t kSmemBytes = OFF_RESP + 16 * kRing + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");
constexpr uint32_t kColS = 0, kColO = 256, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;

enum Bar { Q_FULL = 0, Q_EMPTY = 1, K_FULL = 2, K_EMPTY = 4, V_FULL = 6, V_EMPTY = 8, S_FULL = 10,
           P_FULL = 12, O_DONE = 14, P_HALF = 16, ITEM_FULL = 18, ITEM_EMPTY = 22, NUM_BARS = 26 };
static_assert(8 * NUM_BARS + 16 <= 256, "barriers, abort flag and TMEM slot fit before OFF_RESP");
// Consumers of a work-ring slot: the producer, the MMA warp and the 8 softmax warps.
constexpr int kRingConsumers = 10;

enum class Mode { Dense, Paged, Prefix };

// Which exp2 pairs of each group of 8 run as a polynomial on the FMA pipe (bit i: pair i % 8);
// the rest use the MUFU unit.  A/B on one box: two in eight is best for the dense prefill (over
// 1/8 to 4/8), one in eight for paged appends (962 against 933 TFLOP/s at 2/8).  Which pair of
// the eight matters only to register allocation: pair 3 compiles without spills, pair 7 spills.
// A paged prefill over a contiguous context therefore differs from the dense prefill in the
// last bits of some probabilities.
template <Mode M>
constexpr unsigned poly_mask() { return M == Mode::Paged ? 0x08u : 0x88u; }

struct Params {
    float c;
    int n_items;
    uint16_t* o;
    float* lse;
    int B, Hq, Hkv, Sq, Sk, n_qt, n_pairs, causal, q_offset;
    const int32_t* bt;
    const int32_t* lens;
    float* part_o;
    float2* part_ml;
    int N, G, num_pages, max_pages, n_prefix, chunk_pages, n_chunks, n_qtiles, n_slots, slot0;
    // G: prefix mode -- the GQA group; paged mode -- query heads packed per work item
    const int32_t* cu_q;     // paged: [N+1] query row offsets
    int max_pairs;           // paged: tile pairs of the longest packed query run
    int o_align32;           // dense / paged: o is 32-byte aligned (32-byte output stores)
    int part_align32;        // prefix: part_o is 32-byte aligned (32-byte partial stores)
};

struct Item {
    int bhq, kvh, q_row0[2];                 // dense / paged
    int sess, q_tok0, lq, lk;                // paged
    int h, n0, chunk, p_begin, p_end, src;   // prefix
    int nb[2];
    int nbk;
};

// Coordinates of work item w.  Every role computes them (no shared state), with all 32 lanes
// of a warp (prefix mode may reduce over the tile's sessions with shuffles).
template <Mode M>
__device__ __forceinline__ Item item_coords(const Params& p, int w, int lane) {
    Item it;
    it.bhq = it.kvh = it.h = it.n0 = it.chunk = it.p_begin = it.p_end = it.src = 0;
    it.q_row0[0] = it.q_row0[1] = 0;
    it.sess = it.q_tok0 = it.lq = it.lk = 0;
    if constexpr (M == Mode::Paged) {
        // GQA packing: the p.G query heads of a group share one K/V stream; packed row r of a
        // (session, group) is token r / p.G, head group * p.G + r % p.G.
        const int NG = p.Hq / p.G;
        const int pair = p.max_pairs - 1 - w / (p.N * NG);      // heavy pairs first
        const int rest = w % (p.N * NG);
        it.sess = rest / NG;
        it.bhq = rest % NG;                                     // query group
        it.kvh = it.bhq * p.G / (p.Hq / p.Hkv);
        it.q_tok0 = p.cu_q[it.sess];
        it.lq = p.cu_q[it.sess + 1] - it.q_tok0;
        it.lk = min(max(p.lens[it.sess], 0), p.max_pages * 16);
        it.p_end = (it.lk + 15) / 16;
        const int rows = it.lq * p.G;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            it.q_row0[t] = (2 * pair + t) * BM;
            int n = 0;
            if (it.q_row0[t] < rows) {
                int kv_end = it.lk;
                if (p.causal) kv_end = min(it.lk, (it.q_row0[t] + BM) / p.G + (it.lk - it.lq));
                n = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
            }
            it.nb[t] = n;
        }
    } else if constexpr (M == Mode::Dense) {
        const int BH = p.B * p.Hq;
        it.bhq = w % BH;
        const int pair = p.n_pairs - 1 - w / BH;   // heavy pairs first
        const int b = it.bhq / p.Hq, hq = it.bhq % p.Hq;
        it.kvh = b * p.Hkv + hq / (p.Hq / p.Hkv);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            it.q_row0[t] = (2 * pair + t) * BM;
            int n = 0;
            if (it.q_row0[t] < p.Sq) {
                int kv_end = p.Sk;
                if (p.causal) kv_end = min(p.Sk, it.q_row0[t] + BM + p.q_offset);
                n = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
            }
            it.nb[t] = n;
        }
    } else {
        // The item's pages come from one session's block-table row (src).  Fast path: the tile's
        // first session n0 covers the whole chunk (one length read).  Otherwise the longest
        // session of the tile is taken (a lane-parallel scan) and the chunk is cut at its
        // length; rows shorter than the chunk are masked per row by the softmax (key_limit).
        const int qtile = w % p.n_qtiles;
        const int rest = w / p.n_qtiles;
        it.h = rest % p.Hkv;
        it.chunk = rest / p.Hkv;
        const int spt = 2 * BM / p.G;
        it.n0 = qtile * spt;
        it.p_begin = it.chunk * p.chunk_pages;
        it.p_end = min(it.p_begin + p.chunk_pages, p.n_prefix);
        const int L0 = min(max(p.lens[it.n0], 0), p.max_pages * 16);
        if ((L0 + 15) / 16 >= it.p_end) {
            it.src = it.n0;
        } else {
            int best_len = -1, best = it.n0;
            for (int k = lane; k < spt; k += 32) {
                const int n = it.n0 + k;
                if (n < p.N) {
                    const int L = min(max(p.lens[n], 0), p.max_pages * 16);
                    if (L > best_len) { best_len = L; best = n; }
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const int ol = __shfl_xor_sync(0xffffffffu, best_len, off);
                const int on = __shfl_xor_sync(0xffffffffu, best, off);
                if (ol > best_len || (ol == best_len && on < best)) { best_len = ol; best = on; }
            }
            it.src = best;
            it.p_end = min(it.p_end, (max(best_len, 0) + 15) / 16);
        }
        const int n = it.p_end > it.p_begin ? (it.p_end - it.p_begin + 7) / 8 : 0;
        it.nb[0] = it.nb[1] = n;
    }
    it.nbk = max(it.nb[0], it.nb[1]);
    return it;
}

// Work distribution (all modes): the grid has one CTA per work item, ordered heavy first, and
// a CTA that has finished its item takes over the item of a CTA that has not been launched yet
// (cluster launch control: the hardware cancels that CTA's launch and reports its index).  So
// the first wave of CTAs keeps working until the queue is empty, like a persistent kernel, but
// with dynamic load balance: ragged items (paged prefill) no longer leave SMs idle at the end.
// The producer requests the next item one item ahead; every role reads the answer from a ring
// of kRing slots in shared memory (mbarrier-signalled) and releases the slot after reading it.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
    asm volatile(
        "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 "
        "[%0], [%1];" ::"r"(resp),
        "r"(bar)
        : "memory");
}
// The item index a response names, or -1 when no launch was cancelled (no work left).
__device__ __forceinline__ int clc_item(uint32_t resp) {
    uint32_t cancelled;
    asm volatile(
        "{\n\t.reg .b128 h;\n\t.reg .pred p;\n\t"
        "ld.shared.b128 h, [%1];\n\t"
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, h;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(cancelled)
        : "r"(resp)
        : "memory");
    if (!cancelled) return -1;
    uint32_t x;
    asm volatile(
        "{\n\t.reg .b128 h;\n\t"
        "ld.shared.b128 h, [%1];\n\t"
        "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, h;\n\t}"
        : "=r"(x)
        : "r"(resp)
        : "memory");
    return static_cast<int>(x);
}

// HDIM: head_dim, 128 or 64.  At 64 a tile is a single 128-byte-swizzled [rows][64] box and the
// MMAs run with K = 64 (QK^T) and N = 64 (P.V).
template <Mode M, int HDIM>
__global__ void __launch_bounds__(kThreads, 1)
attn2_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
             const __grid_constant__ CUtensorMap tmv, const Params p) {
    static_assert(HDIM == 128 || HDIM == 64, "head_dim must be 64 or 128");
    constexpr int HD = HDIM;
    constexpr uint32_t kLoadBytes = BM * HD * 2;      // bytes of one Q, K or V tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    auto bar = [&](int i) { return sbase + OFF_BAR + 8u * i; };
    int* abort_flag = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8 * NUM_BARS + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(bar(Q_FULL), 1);
        mbar_init(bar(Q_EMPTY), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar(K_FULL + s), 1);
            mbar_init(bar(K_EMPTY + s), 1);
            mbar_init(bar(V_FULL + s), 1);
            mbar_init(bar(V_EMPTY + s), 1);
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(P_FULL + s), 4);           // one arrival per softmax warp
            mbar_init(bar(P_HALF + s), 4);
            mbar_init(bar(O_DONE + s), 1);
        }
        for (int r = 0; r < kRing; ++r) {
            mbar_init(bar(ITEM_FULL + r), 1);
            mbar_init(bar(ITEM_EMPTY + r), kRingConsumers);
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
    auto resp = [&](int r) { return sbase + OFF_RESP + 16u * r; };
    // Item k >= 1 of this CTA (all 32 lanes call it): -1 when the queue is empty or a wait gave
    // up (then ok is false).
    auto next_item = [&](int k, bool& ok) -> int {
        const int r = (k - 1) & (kRing - 1);
        ok = __all_sync(0xffffffffu, mbar_wait(bar(ITEM_FULL + r), ((k - 1) / kRing) & 1, abort_flag, 14));
        if (!ok) return -1;
        const int w = clc_item(resp(r));
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(ITEM_EMPTY + r));
        return w;
    };

    // Registers move from warpgroup 0 (TMA, MMA and two idle warps) to the two softmax
    // warpgroups, whose whole-row S registers otherwise spill: 128 x 88 + 256 x 208 = 64512, within
    // the 384 x 168 = 64512 the block is launched with.
    // Each role adjusts its own budget at the top of its branch.
    static_assert(kThreads == 384, "register split sized for 384 threads");

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        setmaxnreg_dec<kRegsControl>();
        if (lane == 0) {
            tma_prefetch_desc(&tmq);
            tma_prefetch_desc(&tmk);
            tma_prefetch_desc(&tmv);
        }
        int g = 0, qi = 0, requested = 0;
        bool ok = true;
        for (int k = 0, w = blockIdx.x; ok && w >= 0 && w < p.n_items; w = next_item(++k, ok)) {
            // ask for the item after this one (a request follows only a successful answer)
            if (lane == 0) {
                const int r = k & (kRing - 1);
                if (k >= kRing) ok = mbar_wait(bar(ITEM_EMPTY + r), ((k / kRing) - 1) & 1, abort_flag, 15);
                if (ok) {
                    mbar_arrive_expect_tx(bar(ITEM_FULL + r), 16);
                    clc_try_cancel(resp(r), bar(ITEM_FULL + r));
                    requested = k + 1;
                }
            }
            if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
            // Paged modes: a 128-key tile is 8 pages x (HD / 64) boxes of [16 rows][64 dims].
            // Lane 2 * page + half issues one box of K and one of V, so the whole tile's boxes go
            // out at once; its page id is fetched one block ahead.  Prefix mode reads the first
            // block's ids from the tile's first session before the item's coordinates are known
            // (the usual source row), so the two reads overlap.
            const int pg = lane >> 1, hf = lane & 1;
            const bool loader = lane < 16 && hf < HD / 64;
            int spec_src = -1, spec_page = -1;
            if constexpr (M == Mode::Prefix) {
                const int rest = w / p.n_qtiles;
                spec_src = (w % p.n_qtiles) * (2 * BM / p.G);
                const int pb = (rest / p.Hkv) * p.chunk_pages;
                const int pi = pb + pg;
                if (loader && pi < min(pb + p.chunk_pages, p.n_prefix))
                    spec_page = __ldg(p.bt + (size_t)spec_src * p.max_pages + pi);
            }
            // Prefix mode: Q's coordinates need no loads, so its load goes out first; an item that
            // turns out empty (every session of the tile ends before the chunk) leaves this Q
            // phase to the MMA warp, which takes it without MMAs.
            bool q_early = false;
            if constexpr (M == Mode::Prefix) {
                if (lane == 0) {
                    if (qi > 0) ok = mbar_wait(bar(Q_EMPTY), (qi - 1) & 1, abort_flag, 12);
                    if (ok) {
                        mbar_arrive_expect_tx(bar(Q_FULL), 2 * kLoadBytes);
                        const int h = (w / p.n_qtiles) % p.Hkv;
#pragma unroll
                        for (int t = 0; t < 2; ++t)
#pragma unroll
                            for (int hf = 0; hf < HD / 64; ++hf)
                                tma_load_4d(sbase + OFF_Q + t * kTileBytes + hf * kHalfBytes, &tmq,
                                            bar(Q_FULL), hf * 64, 0, h, spec_src + t * (BM / p.G));
                    }
                }
                if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
                q_early = true;
            }
            const Item it = item_coords<M>(p, w, lane);
            if (it.nbk == 0) {
                if (q_early) ++qi;
                continue;
            }
            const int32_t* bt_row = (M == Mode::Dense) ? nullptr
                                    : (M == Mode::Prefix) ? p.bt + (size_t)it.src * p.max_pages
                                                          : p.bt + (size_t)it.sess * p.max_pages;
            const int kv_head = (M == Mode::Paged) ? it.kvh : it.h;
            auto to_row = [&](int page) -> int {
                if (static_cast<unsigned>(page) >= static_cast<unsigned>(p.num_pages)) {
                    atomicCAS(&g_device_error, 0, 201);
                    return p.num_pages * p.Hkv;                  // out of range: zeros
                }
                return page * p.Hkv + kv_head;
            };
            auto page_row = [&](int j) -> int {
                const int pi = it.p_begin + j * 8 + pg;
                return (loader && pi < it.p_end) ? to_row(__ldg(bt_row + pi)) : p.num_pages * p.Hkv;
            };
            int row = 0;
            if constexpr (M == Mode::Prefix) {
                if (it.src == spec_src) {
                    const int pi = it.p_begin + pg;
                    row = (loader && pi < it.p_end) ? to_row(spec_page) : p.num_pages * p.Hkv;
                } else {
                    row = page_row(0);
                }
            }
            if (lane == 0 && !q_early) {
                if (qi > 0) ok = mbar_wait(bar(Q_EMPTY), (qi - 1) & 1, abort_flag, 12);
                if (ok) {
                    mbar_arrive_expect_tx(bar(Q_FULL), 2 * kLoadBytes);
#pragma unroll
                    for (int t = 0; t < 2; ++t) {
#pragma unroll
                        for (int hf = 0; hf < HD / 64; ++hf) {
                            const uint32_t dst = sbase + OFF_Q + t * kTileBytes + hf * kHalfBytes;
                            if constexpr (M == Mode::Dense) {
                                tma_load_3d(dst, &tmq, bar(Q_FULL), hf * 64, it.q_row0[t], it.bhq);
                            } else if constexpr (M == Mode::Paged) {
                                tma_load_4d(dst, &tmq, bar(Q_FULL), hf * 64, 0, it.bhq,
                                            it.q_tok0 + it.q_row0[t] / p.G);
                            } else {
                                tma_load_4d(dst, &tmq, bar(Q_FULL), hf * 64, 0, it.h,
                                            it.n0 + t * (BM / p.G));
                            }
                        }
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if constexpr (M == Mode::Dense) {
                if (lane == 0) {
                    for (int j = 0; ok && j < it.nbk; ++j) {
                        const int gj = g + j, st = gj & 1;
                        const uint32_t ph = (gj >> 1) & 1;
                        if (!(ok = mbar_wait(bar(K_EMPTY + st), ph ^ 1, abort_flag, 1))) break;
                        mbar_arrive_expect_tx(bar(K_FULL + st), kLoadBytes);
#pragma unroll
                        for (int hf = 0; hf < HD / 64; ++hf)
                            tma_load_3d(sbase + OFF_K + st * kTileBytes + hf * kHalfBytes, &tmk,
                                        bar(K_FULL + st), hf * 64, j * BN, it.kvh);
                        if (!(ok = mbar_wait(bar(V_EMPTY + st), ph ^ 1, abort_flag, 2))) break;
                        mbar_arrive_expect_tx(bar(V_FULL + st), kLoadBytes);
#pragma unroll
                        for (int hf = 0; hf < HD / 64; ++hf)
                            tma_load_3d(sbase + OFF_V + st * kTileBytes + hf * kHalfBytes, &tmv,
                                        bar(V_FULL + st), hf * 64, j * BN, it.kvh);
                    }
                }
            } else if (ok) {
                // Lane 0 waits for the free stage and posts the tile's byte count before the
                // boxes are issued (the shuffle orders it).
                if constexpr (M == Mode::Paged) row = page_row(0);
                const uint32_t box = hf * kHalfBytes + pg * kPageBoxBytes;
                for (int j = 0; j < it.nbk; ++j) {
                    const int gj = g + j, st = gj & 1;
                    const uint32_t ph = (gj >> 1) & 1;
                    if (lane == 0) {
                        ok = mbar_wait(bar(K_EMPTY + st), ph ^ 1, abort_flag, 1);
                        if (ok) mbar_arrive_expect_tx(bar(K_FULL + st), kLoadBytes);
                    }
                    if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
                    if (loader)
                        tma_load_3d(sbase + OFF_K + st * kTileBytes + box, &tmk, bar(K_FULL + st),
                                    hf * 64, 0, row);
                    if (lane == 0) {
                        ok = mbar_wait(bar(V_EMPTY + st), ph ^ 1, abort_flag, 2);
                        if (ok) mbar_arrive_expect_tx(bar(V_FULL + st), kLoadBytes);
                    }
                    if (!(ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0)) break;
                    if (loader)
                        tma_load_3d(sbase + OFF_V + st * kTileBytes + box, &tmv, bar(V_FULL + st),
                                    hf * 64, 0, row);
                    if (j + 1 < it.nbk) row = page_row(j + 1);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            g += it.nbk;
            ++qi;
        }
        // Tail: wait until the commits releasing the last K/V stages and Q have landed, so no
        // barrier arrival reaches this CTA's shared memory after it exits.
        if (lane == 0 && ok) {
            for (int gj = max(0, g - 2); gj < g && ok; ++gj) {
                const int st = gj & 1;
                const uint32_t ph = (gj >> 1) & 1;
                ok = mbar_wait(bar(K_EMPTY + st), ph, abort_flag, 10) &&
                     mbar_wait(bar(V_EMPTY + st), ph, abort_flag, 11);
            }
            if (ok && qi > 0) mbar_wait(bar(Q_EMPTY), (qi - 1) & 1, abort_flag, 13);
        }
        // The answer to the last request must land before the CTA exits (it is normally read
        // already; after a give-up it may still be in flight).
        if (lane == 0 && requested > 0) {
            const int r = (requested - 1) & (kRing - 1);
            const uint32_t par = ((requested - 1) / kRing) & 1;
            if (!mbar_try_wait(bar(ITEM_FULL + r), par)) {
                const uint64_t t0 = global_timer_ns();
                while (!mbar_try_wait(bar(ITEM_FULL + r), par) && global_timer_ns() - t0 < 100000000ull) {
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        setmaxnreg_dec<kRegsControl>();
        constexpr uint32_t idesc_qk = idesc_bf16_f32(BM, BN, false);
        constexpr uint32_t idesc_pv = idesc_bf16_f32(BM, HD, true);
        auto qk = [&](int t, int st) {
            const uint32_t d = tmem + kColS + t * 128;
            const uint32_t qa = sbase + OFF_Q + t * kTileBytes, ka = sbase + OFF_K + st * kTileBytes;
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
                mma_ss(d, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), idesc_qk,
                       kk > 0);
            }
        };
        // P.V over keys [k0 * 16, k0 * 16 + BN / 2): the first half of a block runs as soon as
        // the softmax warps have stored the first half of P.
        auto pv = [&](int t, int st, bool acc, int k0) {
            const uint32_t va = sbase + OFF_V + st * kTileBytes;
            const uint32_t pa = tmem + kColS + t * 128;
#pragma unroll
            for (int kk = k0; kk < k0 + BN / 32; ++kk)
                mma_ts(tmem + kColO + t * 128, pa + kk * 8, sdesc_sw128(va + kk * 2048, kHalfBytes, 1024),
                       idesc_pv, (acc || kk > 0) ? 1u : 0u);
        };
        // The whole warp runs this loop and every wait (each wait's result is voted, so control
        // flow stays warp-uniform); one elected lane issues the MMAs and their commits.  Keeping
        // the loop converged keeps the MMA operands in the uniform datapath: the same loop run
        // by one divergent lane issued tcgen05.mma about 25% slower.
        auto vote = [&](bool v) { return __all_sync(0xffffffffu, v); };
        int g = 0, qi = 0, pc[2] = {0, 0};
        bool ok = true;
        for (int k = 0, w = blockIdx.x; ok && w >= 0 && w < p.n_items; w = next_item(++k, ok)) {
            const Item it = item_coords<M>(p, w, lane);
            if (it.nbk == 0) {
                if constexpr (M == Mode::Prefix) {
                    // the producer loaded this item's Q before it knew the item was empty
                    const uint32_t b1[1] = {bar(Q_FULL)};
                    const uint32_t p1[1] = {static_cast<uint32_t>(qi & 1)};
                    if (!(ok = vote(mbar_wait_all(b1, p1, abort_flag, 3)))) break;
                    if (lane == 0) mbar_arrive(bar(Q_EMPTY));
                    ++qi;
                }
                continue;
            }
            {
                const uint32_t bs[2] = {bar(Q_FULL), bar(K_FULL + (g & 1))};
                const uint32_t ps[2] = {static_cast<uint32_t>(qi & 1), static_cast<uint32_t>((g >> 1) & 1)};
                if (!(ok = vote(mbar_wait_all(bs, ps, abort_flag, 3)))) break;
            }
            tc_fence_after();
            if (elect_one()) {
#pragma unroll
                for (int t = 0; t < 2; ++t)
                    if (it.nb[t] > 0) {
                        qk(t, g & 1);
                        mma_commit(bar(S_FULL + t));
                    }
                mma_commit(bar(K_EMPTY + (g & 1)));
                if (it.nbk == 1) mma_commit(bar(Q_EMPTY));
            }
            __syncwarp();
            for (int j = 0; j < it.nbk; ++j) {
                const int gj = g + j, st = gj & 1;
                const bool next = j + 1 < it.nbk;
                bool have_v = false, have_k = false;
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    if (j >= it.nb[t]) continue;
                    const bool more = j + 1 < it.nb[t];
                    // One wait point per half of P_t; the first also covers V(j) and K(j+1) when
                    // not yet awaited (unused slots repeat the P barrier).  Keeping the waits
                    // together keeps the issue gaps short: the MMA queue holds only a few MMAs.
                    const uint32_t pbar = bar(P_HALF + t), ppar = pc[t] & 1;
                    const uint32_t bs[3] = {pbar, have_v ? pbar : bar(V_FULL + st),
                                            (more && !have_k) ? bar(K_FULL + (st ^ 1)) : pbar};
                    const uint32_t ps[3] = {ppar, have_v ? ppar : static_cast<uint32_t>((gj >> 1) & 1),
                                            (more && !have_k) ? static_cast<uint32_t>(((gj + 1) >> 1) & 1) : ppar};
                    if (!(ok = vote(mbar_wait_all(bs, ps, abort_flag, 5)))) break;
                    have_v = true;
                    have_k = have_k || more;
                    tc_fence_after();
                    if (elect_one()) pv(t, st, j > 0, 0);
                    __syncwarp();
                    {
                        const uint32_t b1[1] = {bar(P_FULL + t)};
                        const uint32_t p1[1] = {ppar};
                        if (!(ok = vote(mbar_wait_all(b1, p1, abort_flag, 5)))) break;
                    }
                    ++pc[t];
                    tc_fence_after();
                    if (elect_one()) {
                        pv(t, st, true, BN / 32);
                        if (more) {
                            qk(t, st ^ 1);
                            mma_commit(bar(S_FULL + t));
                        } else {
                            mma_commit(bar(O_DONE + t));   // O_t final
                        }
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (elect_one()) {
                    mma_commit(bar(V_EMPTY + st));
                    if (next) mma_commit(bar(K_EMPTY + (st ^ 1)));
                    if (j + 2 == it.nbk) mma_commit(bar(Q_EMPTY));   // last QK^T of the item issued
                }
                __syncwarp();
            }
            g += it.nbk;
            ++qi;
        }
        __syncwarp();
    } else if (warp < 4) {
        setmaxnreg_dec<kRegsControl>();                  // idle warps of warpgroup 0
    } else {
        // ---------------- softmax + epilogue (tile t) ----------------
        setmaxnreg_inc<kRegsSoftmax>();
        const int t = (warp - 4) >> 2;
        const int row = ((warp - 4) & 3) * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const uint32_t s_col = tmem + lane_off + kColS + t * 128;
        const uint32_t o_col = tmem + lane_off + kColO + t * 128;
        int cnt = 0;        // blocks this tile has processed, across items
        int ocnt = 0;       // items with blocks this tile has finished (O_DONE phases)
        bool ok = true;
        // The next item is fetched at the end of the body: fetching it at the top keeps one more
        // value live across the loop and made these warps spill.
        for (int k = 1, w = blockIdx.x; ok && w >= 0 && w < p.n_items; w = next_item(k++, ok)) {
            const Item it = item_coords<M>(p, w, lane);
            const int n_blk = it.nb[t];
            int qpos = 0, key_limit = 0, n = 0;
            if constexpr (M == Mode::Dense) {
                qpos = it.q_row0[t] + row + p.q_offset;
                key_limit = p.Sk;
            } else if constexpr (M == Mode::Paged) {
                qpos = (it.q_row0[t] + row) / p.G + (it.lk - it.lq);
                key_limit = it.lk;
            } else {
                const int rr = t * BM + row;
                n = it.n0 + rr / p.G;
                const int L_row = n < p.N ? min(max(p.lens[n], 0), p.max_pages * 16) : 0;
                key_limit = min(L_row, it.p_end * 16) - it.p_begin * 16;
            }
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_blk; ++j) {
                ok = __all_sync(0xffffffffu, mbar_wait(bar(S_FULL + t), cnt & 1, abort_flag, 7));
                if (!ok) break;
                tc_fence_after();
                // Visible keys of this block form a prefix [0, lim) of its columns (ragged end
                // and causal diagonal alike).  The whole 128-column S row comes into registers
                // with one TMEM round trip; masked blocks (rare) get -inf past lim there.
                const int kbase = j * BN;
                int lim = key_limit - kbase;
                if constexpr (M != Mode::Prefix)
                    if (p.causal) lim = min(lim, qpos - kbase + 1);
                uint32_t r[BN];
                using Chunk = uint32_t[32];
                auto chunk = [&](int c) -> Chunk& { return *reinterpret_cast<Chunk*>(r + 32 * c); };
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_col + c * 32, chunk(c));
                tmem_wait_ld();
                if (__any_sync(0xffffffffu, lim < BN)) {
#pragma unroll
                    for (int i = 0; i < BN; ++i) r[i] = (i < lim) ? r[i] : 0xff800000u;   // -inf
                }
                // row max: eight chains of three-input max over the 128 columns
                static_assert(BN == 128, "row max unrolled for 128 columns");
                auto sv = [&](int i) { return __uint_as_float(r[i]); };
                float mxs[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) mxs[k] = fmax3(sv(k), sv(k + 8), sv(k + 16));
#pragma unroll
                for (int i = 24; i < 120; i += 16)
#pragma unroll
                    for (int k = 0; k < 8; ++k) mxs[k] = fmax3(mxs[k], sv(i + k), sv(i + 8 + k));
#pragma unroll
                for (int k = 0; k < 8; ++k) mxs[k] = fmaxf(mxs[k], sv(120 + k));
                const float mx = fmax3(fmax3(mxs[0], mxs[1], mxs[2]), fmax3(mxs[3], mxs[4], mxs[5]),
                                       fmaxf(mxs[6], mxs[7]));
                const float m_blk = mx * p.c;
                const float m_new = (m_blk > m_run + kRescaleThreshold) ? m_blk : m_run;
                const float alpha = (m_new == m_run) ? 1.f : fast_exp2(m_run - m_new);
                const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
                if (j > 0) {
                    // PV(t, j-1) has finished: it was issued before QK(t, j), whose S_FULL
                    // commit this warp has waited on, so O_t is safe to scale -- before this
                    // block's first P.V, which the P_HALF arrival below releases.
                    if (__any_sync(0xffffffffu, alpha != 1.f)) {
                        // 8 columns at a time: the S row is live in registers here
                        uint32_t o8[8];
#pragma unroll 1
                        for (int cc = 0; cc < HD / 8; ++cc) {
                            tmem_ld8(o_col + cc * 8, o8);
                            tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                o8[i] = __float_as_uint(__uint_as_float(o8[i]) * alpha);
                            tmem_st8(o_col + cc * 8, o8);
                        }
                    }
                }
                // exp2, row sum and bf16 P, packed in place: pair i (columns 2i, 2i+1) becomes
                // r[i], so P of score columns [0, 128) lands in TMEM columns [0, 64) of this
                // S buffer.  The pairs poly_mask<M>() selects run on the FMA pipe.  The first half
                // of P is stored and signalled (P_HALF) before the second half is computed, so
                // its P.V overlaps the rest of this softmax.
                const uint64_t c2 = f2_pack(p.c, p.c), nm2 = f2_pack(-m_use, -m_use);
                uint64_t lsa = f2_pack(0.f, 0.f), lsb = f2_pack(0.f, 0.f);
                auto pair = [&](int i) {
                    const uint64_t a = ffma2(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                             c2, nm2);
                    float2 e;
                    if ((poly_mask<M>() >> (i & 7)) & 1u) {
                        e = exp2_poly2(a);
                    } else {
                        const float2 av = f2_unpack(a);
                        e = make_float2(fast_exp2(av.x), fast_exp2(av.y));
                    }
                    if (i & 1) lsb = fadd2(lsb, f2_pack(e.x, e.y));
                    else lsa = fadd2(lsa, f2_pack(e.x, e.y));
                    r[i] = pack_bf16x2(e.x, e.y);
                };
#pragma unroll
                for (int i = 0; i < BN / 4; ++i) pair(i);
                tmem_st32(s_col, chunk(0));
                tmem_wait_st();                      // also orders any O rescale above
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(P_HALF + t));
#pragma unroll
                for (int i = BN / 4; i < BN / 2; ++i) pair(i);
                tmem_st32(s_col + 32, chunk(1));
                const float2 lsv = f2_unpack(fadd2(lsa, lsb));
                const float lsum = lsv.x + lsv.y;
                l_run = l_run * alpha + lsum;
                m_run = m_new;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();                        // the warp's P rows are all in TMEM
                if (lane == 0) mbar_arrive(bar(P_FULL + t));
                ++cnt;
            }
            if (!ok) break;
            if (n_blk > 0) {
                // one O_DONE phase per item with blocks: the commit after its last P.V
                ok = __all_sync(0xffffffffu, mbar_wait(bar(O_DONE + t), ocnt & 1, abort_flag, 9));
                if (!ok) break;
                ++ocnt;
                tc_fence_after();
            }
            // ---- epilogue: read O_t (the next item's first P.V may then overwrite it) ----
            if constexpr (M != Mode::Prefix) {
                // dense: o [B*Hq][Sq][D]; paged: o [T_total][Hq][D] from packed rows; lse alike
                // without D.
                const int grow = it.q_row0[t] + row;
                const int rows = (M == Mode::Dense) ? p.Sq : it.lq * p.G;
                const size_t orow = (M == Mode::Dense)
                                        ? static_cast<size_t>(it.bhq) * p.Sq + grow
                                        : (static_cast<size_t>(it.q_tok0) + grow / p.G) * p.Hq +
                                              static_cast<size_t>(it.bhq) * p.G + grow % p.G;
                if (it.q_row0[t] < rows) {
                    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll 1
                    for (int cc = 0; cc < HD / 32; ++cc) {
                        uint32_t r[32];
                        if (n_blk > 0) {
                            tmem_ld32(o_col + cc * 32, r);
                            tmem_wait_ld();
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i) r[i] = 0u;
                        }
                        if (grow < rows) {
                            // 32-byte stores when o is 32-byte aligned (rows are 2 * HD bytes):
                            // half the store instructions of 16-byte ones
                            uint16_t* dst = p.o + orow * HD + cc * 32;
                            if (p.o_align32) {
#pragma unroll
                                for (int v = 0; v < 2; ++v) {
                                    uint32_t w[8];
#pragma unroll
                                    for (int i = 0; i < 8; ++i)
                                        w[i] = pack_bf16x2(__uint_as_float(r[16 * v + 2 * i]) * inv,
                                                           __uint_as_float(r[16 * v + 2 * i + 1]) * inv);
                                    st_global_v8(dst + 16 * v, w);
                                }
                            } else {
#pragma unroll
                                for (int v = 0; v < 4; ++v) {
                                    uint4 wv;
                                    wv.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
                                    wv.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
                                    wv.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
                                    wv.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
                                    reinterpret_cast<uint4*>(dst)[v] = wv;
                                }
                            }
                        }
                    }
                    if (p.lse != nullptr && grow < rows)
                        p.lse[orow] = l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
                }
            } else {
                // prefix partials: slot (n, hq, slot0 + chunk) of part_o [N][Hq][n_slots][D] fp32
                // holds O / l as bf16 in its first D * 2 bytes (the epilogue is bound by the SM's
                // store bandwidth: half the bytes of fp32), (m, l) go to part_ml.  TMEM gives each
                // thread one row and consecutive rows live in different slots, so the rows go out
                // through this warp's staging tile in shared memory: each lane writes its row's
                // 16-byte pieces at XOR-swizzled positions (no bank conflicts), then groups of 4
                // lanes store one row's 64 contiguous bytes (8 rows per store).
                auto slot_of = [&](int rr) -> size_t {
                    const int nn = it.n0 + rr / p.G;
                    return ((size_t)nn * (p.Hkv * p.G) + it.h * p.G + rr % p.G) * p.n_slots +
                           p.slot0 + it.chunk;
                };
                const int rr = t * BM + row;
                const int n_row = it.n0 + rr / p.G;
                const int g0 = ((warp - 4) & 3) * 32;     // tile row of this warp's lane 0
                const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
                uint4* stage = reinterpret_cast<uint4*>(smem + OFF_EPI + (warp - 4) * kEpiWarpBytes);
#pragma unroll 1
                for (int cc = 0; cc < HD / 32; ++cc) {
                    uint32_t r[32];
                    if (n_blk > 0) {
                        tmem_ld32(o_col + cc * 32, r);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = 0u;
                    }
                    __syncwarp();                      // the previous chunk's reads are done
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint4 wv;
                        wv.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
                        wv.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
                        wv.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
                        wv.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
                        stage[lane * 4 + (v ^ ((lane >> 1) & 3))] = wv;
                    }
                    __syncwarp();
                    if (p.part_align32) {
                        // 64 bytes of a row per 2 lanes (32-byte stores), 16 rows per store
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const int rl = i * 16 + (lane >> 1), hf = lane & 1, sw = (rl >> 1) & 3;
                            const uint4 a = stage[rl * 4 + ((2 * hf) ^ sw)];
                            const uint4 b = stage[rl * 4 + ((2 * hf + 1) ^ sw)];
                            const int rr2 = t * BM + g0 + rl;
                            if (it.n0 + rr2 / p.G < p.N) {
                                const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                                st_global_v8(reinterpret_cast<uint8_t*>(p.part_o + slot_of(rr2) * HD) +
                                                 cc * 64 + hf * 32, w);
                            }
                        }
                    } else {
                        // 64 bytes of a row per 4 lanes, 8 rows per store
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int rl = i * 8 + (lane >> 2), q = lane & 3;
                            const uint4 v = stage[rl * 4 + (q ^ ((rl >> 1) & 3))];
                            const int rr2 = t * BM + g0 + rl;
                            if (it.n0 + rr2 / p.G < p.N)
                                reinterpret_cast<uint4*>(p.part_o + slot_of(rr2) * HD)[cc * 4 + q] = v;
                        }
                    }
                }
                if (n_row < p.N) p.part_ml[slot_of(rr)] = make_float2(m_run, l_run);
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
