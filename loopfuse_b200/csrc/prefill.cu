// Causal GQA prefill attention for sm_100a: tcgen05 MMA, TMEM accumulators, TMA tiles.
//
// Replaces prefill_attention_fwd (kernels/triton/prefill_attn.py:127-168, an FA2-style
// Triton kernel, MHA/fp16 only) and the reference's sm_80 agent_prefill_kernel
// (kernels/cuda/async_prefill.cu:56-236, wmma QK^T only, no softmax or P.V).
//
// One CTA computes a 128-row query tile of one (batch, query head) against the key blocks
// its causal mask reaches, 128 keys at a time.  Roles (256 threads):
//   warp 0      TMA producer: Q once, then K and V blocks into a 2-stage ring
//               (128-byte-swizzled [128 rows][64 dims] boxes, two per 128-dim tile);
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_j = Q K_j^T   into TMEM S[j%2]   (M=128, N=128, K=128 -> 8 MMAs),
//                 O  += P_j V_j   with P_j read from TMEM P[j%2] (A operand in TMEM);
//               S_{j+2} is issued right after PV_j so the tensor core always has work
//               while the softmax warps process block j+1;
//   warps 4-7   softmax, one thread per query row (TMEM lane = row): tcgen05.ld the S row,
//               causal/ragged mask, row max in the log2 domain, exp2, row sum, bf16 P packed
//               into TMEM with tcgen05.st.  The running max is only raised when it grows by
//               more than 8 (a factor 256), so O in TMEM is rescaled rarely; O and the row sum
//               always refer to the same stale max, so the result is exact.
// TMEM (512 columns): S0 [0,128), S1 [128,256), O [256,384), P0 [384,448), P1 [448,512).
// Epilogue: O row / row sum -> bf16 -> global; natural-log LSE per row.
//
// Every mbarrier wait is bounded in time; a timeout aborts all roles of the CTA, frees TMEM
// and leaves a code that lf_device_status() reports.
#include "lf_common.cuh"
#include "sm100_primitives.cuh"

#include <cudaTypedefs.h>
#include <math.h>

namespace lf {

__device__ int g_device_error = 0;

namespace prefill {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int HD = 128;
constexpr int kThreads = 256;
constexpr uint32_t kTileBytes = BM * HD * 2;      // 32 KB: one Q, K or V tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;   // 16 KB: [128 rows][64 dims]
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + kTileBytes;           // 2 stages
constexpr uint32_t OFF_V = OFF_K + 2 * kTileBytes;       // 2 stages
constexpr uint32_t OFF_BAR = OFF_V + 2 * kTileBytes;     // barriers, TMEM slot, abort flag
constexpr uint32_t kSmemBytes = OFF_BAR + 256 + 1024;    // + alignment slack
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384, kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;                // log2 units

enum Bar { Q_FULL = 0, K_FULL = 1, K_EMPTY = 3, V_FULL = 5, V_EMPTY = 7, S_FULL = 9, P_FULL = 11,
           O_DONE = 13, NUM_BARS = 14 };

struct Params {
    uint16_t* o;
    float* lse;
    int B, Hq, Hkv, Sq, Sk;
    int n_qt;
    int causal;
    int q_offset;   // Sk - Sq: query i sits at key position i + q_offset
    float c;        // softmax scale * log2(e)
};

__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
               const __grid_constant__ CUtensorMap tmv, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);
    auto bar = [&](int i) { return sbase + OFF_BAR + 8u * i; };
    int* abort_flag = reinterpret_cast<int*>(smem + OFF_BAR + 8 * NUM_BARS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_BAR + 8 * NUM_BARS + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BH = p.B * p.Hq;
    const int bhq = blockIdx.x % BH;
    const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x / BH);   // heavy tiles first
    const int b = bhq / p.Hq, hq = bhq % p.Hq;
    const int hkv = hq / (p.Hq / p.Hkv);
    const int q_row0 = qt * BM;

    int kv_end = p.Sk;
    if (p.causal) kv_end = min(p.Sk, q_row0 + BM + p.q_offset);
    const int n_blk = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;

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
            tma_load_3d(sbase + OFF_Q, &tmq, bar(Q_FULL), 0, q_row0, bhq);
            tma_load_3d(sbase + OFF_Q + kHalfBytes, &tmq, bar(Q_FULL), 64, q_row0, bhq);
            const int kvh = b * p.Hkv + hkv;
            for (int j = 0; j < n_blk; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(bar(K_EMPTY + st), ph ^ 1, abort_flag, 1)) break;
                mbar_arrive_expect_tx(bar(K_FULL + st), kTileBytes);
                tma_load_3d(sbase + OFF_K + st * kTileBytes, &tmk, bar(K_FULL + st), 0, j * BN, kvh);
                tma_load_3d(sbase + OFF_K + st * kTileBytes + kHalfBytes, &tmk, bar(K_FULL + st), 64,
                            j * BN, kvh);
                if (!mbar_wait(bar(V_EMPTY + st), ph ^ 1, abort_flag, 2)) break;
                mbar_arrive_expect_tx(bar(V_FULL + st), kTileBytes);
                tma_load_3d(sbase + OFF_V + st * kTileBytes, &tmv, bar(V_FULL + st), 0, j * BN, kvh);
                tma_load_3d(sbase + OFF_V + st * kTileBytes + kHalfBytes, &tmv, bar(V_FULL + st), 64,
                            j * BN, kvh);
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
        const int qpos = q_row0 + row + p.q_offset;
        const int first_q = q_row0 + p.q_offset;
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
            const bool need_mask = (kbase + BN > p.Sk) || (p.causal && kbase + BN - 1 > first_q);
            if (need_mask) {
#pragma unroll
                for (int i = 0; i < BN; ++i) {
                    const int kpos = kbase + i;
                    const bool vis = kpos < p.Sk && (!p.causal || kpos <= qpos);
                    s[i] = vis ? s[i] : -INFINITY;
                }
            }
            float mx = s[0];
#pragma unroll
            for (int i = 1; i < BN; ++i) mx = fmaxf(mx, s[i]);
            const float m_blk = mx * p.c;
            const float m_new = (m_blk > m_run + kRescaleThreshold) ? m_blk : m_run;
            const float alpha = (m_new == m_run) ? 1.f : fast_exp2(m_run - m_new);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            // P_j goes to TMEM P[j%2]; its previous reader PV_{j-2} finished before S_j was
            // committed, so the buffer is free.
            float lsum = 0.f;
#pragma unroll
            for (int cc = 0; cc < BN / 64; ++cc) {
                uint32_t pr[32];
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const float p0 = fast_exp2(fmaf(s[cc * 64 + 2 * t], p.c, -m_use));
                    const float p1 = fast_exp2(fmaf(s[cc * 64 + 2 * t + 1], p.c, -m_use));
                    lsum += p0 + p1;
                    pr[t] = pack_bf16x2(p0, p1);
                }
                tmem_st32(tmem + lane_off + kColP + (j & 1) * 64 + cc * 32, pr);
            }
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

        const int grow = q_row0 + row;
        const size_t orow = (static_cast<size_t>(bhq) * p.Sq + grow);
        if (n_blk > 0 && ok) {
            ok = mbar_wait(bar(O_DONE), (n_blk - 1) & 1, abort_flag, 9);
            tc_fence_after();
        }
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
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
    if (threadIdx.x == 0 && *abort_flag != 0) atomicCAS(&g_device_error, 0, 100 + *abort_flag);
}

// ---- host side ------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// [rows = BH][seq][128 dims] bf16 tensor, 128-byte swizzled boxes of [128 rows][64 dims].
static int make_map(CUtensorMap* map, const void* base, int seq, int bh) {
    auto fn = encode_fn();
    if (fn == nullptr) return set_error(LF_ECUDA, "prefill: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)seq, (cuuint64_t)bh};
    cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)seq * HD * 2};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LF_ECUDA, "prefill: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LF_OK;
}

}  // namespace prefill
}  // namespace lf

using namespace lf;

extern "C" int lf_prefill_fwd(const lf_bf16* q, const lf_bf16* k, const lf_bf16* v, lf_bf16* o,
                              float* lse, int batch, int num_q_heads, int num_kv_heads, int seq_q,
                              int seq_k, int head_dim, float scale, int causal, void* stream) {
    using namespace lf::prefill;
    LF_CHECK_ARG(q && k && v && o, "prefill: null pointer argument");
    LF_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o),
                 "prefill: q, k, v, o must be 16-byte aligned");
    LF_CHECK_ARG(head_dim == HD, "prefill: head_dim must be %d (got %d)", HD, head_dim);
    LF_CHECK_ARG(batch > 0 && num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                 "prefill: need Hq a positive multiple of Hkv");
    LF_CHECK_ARG(seq_q > 0 && seq_k > 0, "prefill: sequence lengths must be positive");
    const long n_qt = (seq_q + BM - 1) / BM;
    const long grid = n_qt * batch * num_q_heads;
    LF_CHECK_ARG(grid < 2147483647L, "prefill: grid too large");

    CUtensorMap mq, mk, mv;
    int rc = make_map(&mq, q, seq_q, batch * num_q_heads);
    if (rc) return rc;
    rc = make_map(&mk, k, seq_k, batch * num_kv_heads);
    if (rc) return rc;
    rc = make_map(&mv, v, seq_k, batch * num_kv_heads);
    if (rc) return rc;

    static bool attr_set = false;
    if (!attr_set) {
        LF_CHECK_CUDA(cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemBytes));
        attr_set = true;
    }
    Params p;
    p.o = o;
    p.lse = lse;
    p.B = batch;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.Sq = seq_q;
    p.Sk = seq_k;
    p.n_qt = (int)n_qt;
    p.causal = causal ? 1 : 0;
    p.q_offset = seq_k - seq_q;
    p.c = scale * kLog2e;
    prefill_kernel<<<(unsigned)grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(mq, mk, mv, p);
    return launch_status("prefill");
}

extern "C" int lf_device_status(int* out) {
    LF_CHECK_ARG(out != nullptr, "device_status: out is null");
    int v = 0;
    LF_CHECK_CUDA(cudaMemcpyFromSymbol(&v, lf::g_device_error, sizeof(int)));
    const int zero = 0;
    LF_CHECK_CUDA(cudaMemcpyToSymbol(lf::g_device_error, &zero, sizeof(int)));
    *out = v;
    clear_error();
    return LF_OK;
}
