// y[M, N] = x[M, K] . W[K, N] for decode-sized batches (M <= 128): a weight-streaming,
// persistent tcgen05 GEMM.
//
// At M = 64 a projection does 64 multiply-adds per weight element it reads, far below what the
// tensor cores could do per byte of HBM, so the kernel's job is to keep every SM streaming
// weights.  Library GEMMs tile the 64 x N output into a few dozen 128-wide blocks (48 for a
// 6144-wide QKV projection) and leave most of the 148 SMs idle.  Here the work is cut into
// units of one 128-column block x 64 rows of K (16 KB of W), the units are numbered block-major,
// and each of G persistent CTAs (G = the SM count) takes one contiguous run of U / G of them
// (stream-K).  A run covers a few whole column blocks plus at most two partial ones, at its
// ends; whole blocks are written as bf16 directly, partial ones as fp32 partials that a second
// kernel sums in a fixed order (deterministic: no atomics).
//
// The product is computed transposed, y^T = W^T . x^T, so that the weight block is the 128-row
// A operand of tcgen05.mma (M = 128) and the batch is its N (MT = 64 or 128):
//   A  W[k0:k0+64, n0:n0+128], stored N-contiguous: two [64 k][64 n] 128-byte-swizzled TMA boxes,
//      described MN-major (the layout the prefill kernel uses for V, here as the A operand);
//   B  x[0:MT, k0:k0+64], K-contiguous: one [MT][64 k] swizzled box (rows past M read zeros);
//   D  TMEM, 128 lanes (output columns) x MT columns (batch rows), fp32, double-buffered so the
//      epilogue of one column block overlaps the MMAs of the next.
// Warp roles (192 threads): warp 0 issues the TMA loads through a ring of kStages stages, warp 1
// issues the MMAs (the whole warp runs the loop and votes on every wait, one elected lane
// issues), warps 2-5 drain TMEM (thread = output column) and store.  Every barrier wait is
// bounded (sites 220-223 in the device error word); a CTA that gives up stores nothing further,
// waits (bounded) for its own copies and MMAs in flight, frees its TMEM and exits.
#include "lf_common.cuh"
#include "sm100_primitives.cuh"
#include "tmap.cuh"

namespace lf {
namespace gemm {

using namespace sm100;

constexpr int BN = 128;                        // output columns per unit (MMA M)
constexpr int BK = 64;                         // K rows per unit
constexpr int kThreads = 192;

template <int MT>
struct Cfg {
    static constexpr int kStages = MT == 64 ? 8 : 6;
    static constexpr uint32_t kWBytes = BK * BN * 2;              // 16 KB: two [64][64] boxes
    static constexpr uint32_t kXBytes = MT * BK * 2;              // 8 or 16 KB
    static constexpr uint32_t kStageBytes = kWBytes + kXBytes;
    static constexpr uint32_t kSmemBytes = kStages * kStageBytes + 1024;
    static constexpr uint32_t kTmemCols = 2 * MT;
};

// Units [unit_begin(c), unit_begin(c + 1)) belong to CTA c; cta_of(u) is the CTA holding unit u.
__host__ __device__ __forceinline__ long long unit_begin(long long c, long long U, long long G) {
    return c * U / G;
}
__host__ __device__ __forceinline__ long long cta_of(long long u, long long U, long long G) {
    return ((u + 1) * G - 1) / U;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1)
skinny_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
              uint16_t* __restrict__ y, float* __restrict__ part, int M, int N, int nc,
              long long U) {
    using C = Cfg<MT>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[S], empty[S], tfull[2], tempty[2], drained;
    __shared__ uint32_t tmem_slot;
    __shared__ int err;
    const uint32_t sbase = smem_addr(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long G = gridDim.x;
    const long long u0 = unit_begin(blockIdx.x, U, G), u1 = unit_begin(blockIdx.x + 1, U, G);
    const int n_units = (int)(u1 - u0);
    const int nb_first = (int)(u0 / nc), nb_last = (int)((u1 - 1) / nc);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(smem_addr(&full[i]), 1);
            mbar_init(smem_addr(&empty[i]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_addr(&tfull[b]), 1);
            mbar_init(smem_addr(&tempty[b]), 4);
        }
        mbar_init(smem_addr(&drained), 1);
        err = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(&tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    auto stage = [&](int st) { return sbase + (uint32_t)st * C::kStageBytes; };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            tma_prefetch_desc(&tmw);
            tma_prefetch_desc(&tmx);
            int issued = 0;
            for (int i = 0; i < n_units; ++i) {
                const int st = i % S;
                if (i >= S && !mbar_wait(smem_addr(&empty[st]), ((i / S) - 1) & 1, &err, 220)) break;
                const long long u = u0 + i;
                const int n0 = (int)(u / nc) * BN, k0 = (int)(u % nc) * BK;
                const uint32_t bar = smem_addr(&full[st]);
                mbar_arrive_expect_tx(bar, C::kStageBytes);
                tma_load_2d(stage(st), &tmw, bar, n0, k0);
                tma_load_2d(stage(st) + C::kWBytes / 2, &tmw, bar, n0 + 64, k0);
                tma_load_2d(stage(st) + C::kWBytes, &tmx, bar, k0, 0);
                issued = i + 1;
            }
            // After a give-up, copies still in flight must land before the CTA exits.
            if (*reinterpret_cast<volatile int*>(&err) != 0)
                for (int i = max(0, issued - S); i < issued; ++i)
                    if (!mbar_try_wait(smem_addr(&full[i % S]), (i / S) & 1)) {
                        const uint64_t t0 = global_timer_ns();
                        while (!mbar_try_wait(smem_addr(&full[i % S]), (i / S) & 1) &&
                               global_timer_ns() - t0 < 100000000ull) {
                        }
                    }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        // A (W block), MN-major: the 16-row k slice kk starts kk * 2 KB into each [64 k][64 n]
        // box, the two boxes are 8 KB apart (leading offset), 8-row groups 1 KB apart.
        // B (x), K-major: the 16-wide k slice kk starts kk * 32 bytes into the swizzled rows.
        constexpr uint32_t idesc = idesc_bf16_f32(BN, MT, false) | (1u << 15);
        bool ok = true;
        int i = 0;
        for (int nb = nb_first, seg = 0; nb <= nb_last && ok; ++nb, ++seg) {
            const long long base = (long long)nb * nc;
            const int ca = (int)(max(u0, base) - base), cb = (int)(min(u1, base + nc) - base);
            const int buf = seg & 1;
            if (seg >= 2) {
                ok = __all_sync(0xffffffffu, mbar_wait(smem_addr(&tempty[buf]), ((seg >> 1) - 1) & 1,
                                                       &err, 221));
                if (!ok) break;
                tc_fence_after();
            }
            const uint32_t d = tmem + (uint32_t)(buf * MT);
            for (int ch = ca; ch < cb; ++ch, ++i) {
                const int st = i % S;
                ok = __all_sync(0xffffffffu,
                                mbar_wait(smem_addr(&full[st]), (i / S) & 1, &err, 222));
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t wa = stage(st), xa = stage(st) + C::kWBytes;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_ss(d, sdesc_sw128(wa + kk * 2048, C::kWBytes / 2, 1024),
                               sdesc_sw128(xa + kk * 32, 16, 1024), idesc,
                               (ch > ca || kk > 0) ? 1u : 0u);
                    mma_commit(smem_addr(&empty[st]));
                    if (ch == cb - 1) mma_commit(smem_addr(&tfull[buf]));
                }
                __syncwarp();
            }
        }
        if (!ok) {
            // Let every MMA already issued finish before TMEM is released.
            if (elect_one()) mma_commit(smem_addr(&drained));
            __syncwarp();
            if (lane == 0 && !mbar_try_wait(smem_addr(&drained), 0)) {
                const uint64_t t0 = global_timer_ns();
                while (!mbar_try_wait(smem_addr(&drained), 0) &&
                       global_timer_ns() - t0 < 100000000ull) {
                }
            }
            __syncwarp();
        }
    } else {
        // ---------------- epilogue: thread = output column ----------------
        const int q = warp & 3;                                    // TMEM lanes 32q .. 32q + 31
        const int j = q * 32 + lane;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        for (int nb = nb_first, seg = 0; nb <= nb_last; ++nb, ++seg) {
            const long long base = (long long)nb * nc;
            const bool whole = u0 <= base && u1 >= base + nc;
            const int buf = seg & 1;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(smem_addr(&tfull[buf]), (seg >> 1) & 1, &err, 223)))
                break;
            tc_fence_after();
            const int n = nb * BN + j;
            float* pdst = part + ((size_t)blockIdx.x * 2 + (seg == 0 ? 0 : 1)) * M * BN + j;
#pragma unroll 1
            for (int c0 = 0; c0 < MT && c0 < M; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + lane_base + (uint32_t)(buf * MT + c0), r);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const int m = c0 + t;
                    if (m < M) {
                        const float v = __uint_as_float(r[t]);
                        if (whole) {
                            if (n < N) y[(size_t)m * N + n] = f32_to_bf16_rn(v);
                        } else {
                            pdst[(size_t)m * BN] = v;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&tempty[buf]));
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, C::kTmemCols);
    if (threadIdx.x == 0 && err != 0) atomicCAS(&g_device_error, 0, err);
}

// Column blocks that several CTAs shared: y = bf16(sum of their fp32 partials, in CTA order).
// Block (b, my) looks at the run boundary of CTA c = b + 1: the column block holding unit
// unit_begin(c) is summed here if the boundary falls inside it and is the first one that does
// (c - 1 is the block's first contributor).  Thread = column; kRows rows per block, their loads
// independent so that they overlap.
constexpr int kRows = 8;
__global__ void __launch_bounds__(BN)
reduce_kernel(const float* __restrict__ part, uint16_t* __restrict__ y, int M, int N, int nc,
              long long U, long long G) {
    const long long c = blockIdx.x + 1;
    const long long ub = unit_begin(c, U, G);
    if (ub % nc == 0) return;                                  // boundary on a block edge
    const long long nb = ub / nc, base = nb * nc;
    const long long c_first = cta_of(base, U, G);
    if (c != c_first + 1) return;                              // not the block's first boundary
    const long long c_last = cta_of(base + nc - 1, U, G);
    const int j = threadIdx.x, n = (int)nb * BN + j;
    if (n >= N) return;
    const int m0 = blockIdx.y * kRows;
    float acc[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
    for (long long cc = c_first; cc <= c_last; ++cc) {
        // Only the first contributor can have started before this block (its slot 1).
        const int slot = (cc == c_first && unit_begin(cc, U, G) < base) ? 1 : 0;
        const float* src = part + (((size_t)cc * 2 + slot) * M + m0) * BN + j;
#pragma unroll
        for (int r = 0; r < kRows; ++r)
            if (m0 + r < M) acc[r] += src[(size_t)r * BN];
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
        if (m0 + r < M) y[(size_t)(m0 + r) * N + n] = f32_to_bf16_rn(acc[r]);
}

// Dynamic shared-memory opt-in, once per CUDA context.
template <int MT>
int opt_in() {
    static PerContextOnce once;
    return once.run([] {
        LF_CHECK_CUDA(cudaFuncSetAttribute(skinny_kernel<MT>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)Cfg<MT>::kSmemBytes));
        return LF_OK;
    });
}

inline long long grid_size(long long U, int sm_count) { return U < sm_count ? U : sm_count; }

}  // namespace gemm
}  // namespace lf

using namespace lf;

extern "C" int lf_gemm_skinny_workspace_size(int M, int N, int K, int sm_count, size_t* bytes) {
    LF_CHECK_ARG(bytes != nullptr && M > 0 && N > 0 && K > 0 && sm_count > 0,
                 "gemm_skinny: bad workspace arguments");
    const long long U = (long long)((N + gemm::BN - 1) / gemm::BN) * ((K + gemm::BK - 1) / gemm::BK);
    *bytes = (size_t)gemm::grid_size(U, sm_count) * 2 * M * gemm::BN * sizeof(float);
    clear_error();
    return LF_OK;
}

extern "C" int lf_gemm_skinny(const lf_bf16* x, const lf_bf16* w, lf_bf16* y, int M, int N, int K,
                              void* workspace, size_t workspace_bytes, int sm_count, void* stream) {
    LF_CHECK_ARG(x && w && y && workspace, "gemm_skinny: null pointer argument");
    LF_CHECK_ARG(M >= 1 && M <= 128 && N > 0 && K > 0, "gemm_skinny: need 1 <= M <= 128 (got %d)", M);
    LF_CHECK_ARG(N % 8 == 0 && K % 8 == 0, "gemm_skinny: N and K must be multiples of 8");
    LF_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(y) && aligned16(workspace),
                 "gemm_skinny: buffers must be 16-byte aligned");
    LF_CHECK_ARG(sm_count > 0, "gemm_skinny: sm_count must be positive");
    const int nc = (K + gemm::BK - 1) / gemm::BK;
    const long long U = (long long)((N + gemm::BN - 1) / gemm::BN) * nc;
    const long long G = gemm::grid_size(U, sm_count);
    LF_CHECK_ARG(workspace_bytes >= (size_t)G * 2 * M * gemm::BN * sizeof(float),
                 "gemm_skinny: workspace too small (see lf_gemm_skinny_workspace_size)");
    const int MT = M <= 64 ? 64 : 128;
    // W [K][N]: boxes of [64 k rows][64 n]; x [M][K]: boxes of [MT rows][64 k].
    CUtensorMap mw, mx;
    const cuuint64_t wdims[2] = {(cuuint64_t)N, (cuuint64_t)K};
    const cuuint64_t wstr[1] = {(cuuint64_t)N * 2};
    const cuuint32_t wbox[2] = {64, 64};
    int rc = encode_bf16_map(&mw, w, 2, wdims, wstr, wbox);
    if (rc) return rc;
    const cuuint64_t xdims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t xstr[1] = {(cuuint64_t)K * 2};
    const cuuint32_t xbox[2] = {64, (cuuint32_t)MT};
    rc = encode_bf16_map(&mx, x, 2, xdims, xstr, xbox);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint16_t* yo = reinterpret_cast<uint16_t*>(y);
    float* part = static_cast<float*>(workspace);
    if (MT == 64) {
        rc = gemm::opt_in<64>();
        if (rc) return rc;
        gemm::skinny_kernel<64><<<(unsigned)G, gemm::kThreads, gemm::Cfg<64>::kSmemBytes, st>>>(
            mw, mx, yo, part, M, N, nc, U);
    } else {
        rc = gemm::opt_in<128>();
        if (rc) return rc;
        gemm::skinny_kernel<128><<<(unsigned)G, gemm::kThreads, gemm::Cfg<128>::kSmemBytes, st>>>(
            mw, mx, yo, part, M, N, nc, U);
    }
    rc = launch_status("gemm_skinny");
    if (rc != LF_OK) return rc;
    bool split = false;                       // does any CTA's run start inside a column block?
    for (long long c = 1; c < G && !split; ++c) split = gemm::unit_begin(c, U, G) % nc != 0;
    if (!split) return LF_OK;
    const dim3 rgrid((unsigned)(G - 1), (M + gemm::kRows - 1) / gemm::kRows);
    gemm::reduce_kernel<<<rgrid, gemm::BN, 0, st>>>(part, yo, M, N, nc, U, G);
    return launch_status("gemm_skinny reduce");
}
