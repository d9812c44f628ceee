// Fused QKV epilogue: split one layer's QKV projection output, rotate q and k (RoPE), write q
// contiguous for the attention kernels and scatter k and v into the session's pages.
//
// Replaces the reference's ring-buffer append (kernels/cuda/ring_kv_cache.cu:69-109, which
// writes one dense slot and applies no rotation) and the separate split / rotate / cast / copy
// steps a torch model runs between its QKV GEMM and the pool.  One read of qkv and one write of
// q, k, v per token: HBM-bound, 16-byte vectors.
//
// Rotation is the "rotate half" form: for pair i < D/2 of a head,
//   out[i]       = x[i] * cos[pos][i] - x[i + D/2] * sin[pos][i]
//   out[i + D/2] = x[i + D/2] * cos[pos][i] + x[i] * sin[pos][i]
// in fp32 with every product and sum rounded separately (no FMA contraction), then rounded to
// bf16 -- the same arithmetic as an eager fp32 torch evaluation of that formula, so the result
// is bit-identical to it.  cos/sin come from a caller-built [rope_rows][D/2] fp32 table.
#include "pool_common.cuh"

#include <cuda_bf16.h>

namespace lf {
namespace pool {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);      // one packed conversion
    return *reinterpret_cast<const uint32_t*>(&v);
}

// One CTA per token (grid-stride over tokens); its threads walk (head, vector) pairs with heads
// ordered q (Hq), k (Hkv), v (Hkv).  A vector is 8 dims of the first half of a head together with
// the matching 8 dims of the second half.  vph = D / 16 vectors per head is a power of two.
__global__ void qkv_rope_append_kernel(Meta m, const int32_t* __restrict__ seq_ids,
                                       const int32_t* __restrict__ start_pos,
                                       const int32_t* __restrict__ cu_tokens, int n, int total_tokens,
                                       const uint16_t* __restrict__ qkv, long row_stride,
                                       const float* __restrict__ rope_cos,
                                       const float* __restrict__ rope_sin, int rope_rows,
                                       uint16_t* __restrict__ q_out, uint16_t* __restrict__ kp,
                                       uint16_t* __restrict__ vp, int Hq, int Hkv, int D,
                                       int vph_shift) {
    if (status_of(m) != LF_OK) return;
    const int half = D / 2, vph_mask = (1 << vph_shift) - 1;
    const int H = Hq + 2 * Hkv;
    const int units = H << vph_shift;
    for (int t = blockIdx.x; t < total_tokens; t += gridDim.x) {
        int lo = 0, hi = n - 1;                      // session i with cu[i] <= t < cu[i+1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (cu_tokens[mid] <= t) lo = mid; else hi = mid - 1;
        }
        const int pos = start_pos[lo] + (t - cu_tokens[lo]);
        const int s = seq_ids[lo];
        const bool pos_ok = rope_cos == nullptr || (pos >= 0 && pos < rope_rows);
        const uint16_t* src_row = qkv + (long)t * row_stride;
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
            const int v = u & vph_mask;
            const int h = u >> vph_shift;
            const uint16_t* src = src_row + h * D + v * 8;
            uint4 a = *reinterpret_cast<const uint4*>(src);
            uint4 b = *reinterpret_cast<const uint4*>(src + half);
            if (rope_cos != nullptr && h < Hq + Hkv) {
                if (!pos_ok) {
                    atomicCAS(m.ctrl + LF_CTRL_STATUS, LF_OK, LF_EINVAL);
                    continue;
                }
                const float4* cp = reinterpret_cast<const float4*>(rope_cos + (long)pos * half + v * 8);
                const float4* sp = reinterpret_cast<const float4*>(rope_sin + (long)pos * half + v * 8);
                const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
                const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                uint32_t* aw = reinterpret_cast<uint32_t*>(&a);
                uint32_t* bw = reinterpret_cast<uint32_t*>(&b);
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const float x1l = bf16_lo(aw[w]), x1h = bf16_hi(aw[w]);
                    const float x2l = bf16_lo(bw[w]), x2h = bf16_hi(bw[w]);
                    const float cl = cs[2 * w], ch = cs[2 * w + 1], sl = sn[2 * w], sh = sn[2 * w + 1];
                    const float o1l = __fsub_rn(__fmul_rn(x1l, cl), __fmul_rn(x2l, sl));
                    const float o1h = __fsub_rn(__fmul_rn(x1h, ch), __fmul_rn(x2h, sh));
                    const float o2l = __fadd_rn(__fmul_rn(x2l, cl), __fmul_rn(x1l, sl));
                    const float o2h = __fadd_rn(__fmul_rn(x2h, ch), __fmul_rn(x1h, sh));
                    aw[w] = pack_bf16(o1l, o1h);
                    bw[w] = pack_bf16(o2l, o2h);
                }
            }
            uint16_t* dst;
            if (h < Hq) {
                dst = q_out + ((long)t * Hq + h) * D + v * 8;
            } else {
                const bool is_k = h < Hq + Hkv;
                const int kh = is_k ? h - Hq : h - Hq - Hkv;
                const int page = m.bt[(long)s * m.M + pos / LF_PAGE_SIZE];
                if (static_cast<unsigned>(page) >= static_cast<unsigned>(m.P)) {
                    atomicCAS(m.ctrl + LF_CTRL_STATUS, LF_OK, LF_EINVAL);
                    continue;
                }
                dst = (is_k ? kp : vp) + (((long)page * Hkv + kh) * LF_PAGE_SIZE + pos % LF_PAGE_SIZE) * D + v * 8;
            }
            *reinterpret_cast<uint4*>(dst) = a;
            *reinterpret_cast<uint4*>(dst + half) = b;
        }
    }
}

}  // namespace pool
}  // namespace lf

using namespace lf;
using namespace lf::pool;

extern "C" int lf_pool_write_qkv(const lf_pool_meta* m, const int32_t* seq_ids,
                                 const int32_t* start_pos, const int32_t* cu_tokens, int n,
                                 int total_tokens, const void* qkv, int64_t qkv_row_stride,
                                 const float* rope_cos, const float* rope_sin, int rope_rows,
                                 void* q_out, void* k_pages, void* v_pages, int num_q_heads,
                                 int num_kv_heads, int head_dim, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && total_tokens >= 0, "pool write_qkv: negative sizes");
    if (n == 0 || total_tokens == 0) { clear_error(); return LF_OK; }
    LF_CHECK_ARG(seq_ids && start_pos && cu_tokens && qkv && q_out && k_pages && v_pages,
                 "pool write_qkv: null pointer argument");
    LF_CHECK_ARG(head_dim % 16 == 0 && head_dim > 0 && num_q_heads > 0 && num_kv_heads > 0,
                 "pool write_qkv: head_dim must be a multiple of 16");
    LF_CHECK_ARG(qkv_row_stride >= (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim &&
                     qkv_row_stride % 8 == 0,
                 "pool write_qkv: qkv rows must hold (Hq + 2 Hkv) * D elements, 16-byte aligned");
    LF_CHECK_ARG(aligned16(qkv) && aligned16(q_out) && aligned16(k_pages) && aligned16(v_pages),
                 "pool write_qkv: buffers must be 16-byte aligned");
    LF_CHECK_ARG((rope_cos == nullptr) == (rope_sin == nullptr), "pool write_qkv: give cos and sin");
    if (rope_cos) {
        LF_CHECK_ARG(rope_rows > 0 && aligned16(rope_cos) && aligned16(rope_sin),
                     "pool write_qkv: rope table must be 16-byte aligned with rows > 0");
    }
    int vph_shift = 0;
    while ((1 << vph_shift) < head_dim / 16) ++vph_shift;
    LF_CHECK_ARG((1 << vph_shift) == head_dim / 16, "pool write_qkv: head_dim / 16 must be a power of two");
    const int units = (num_q_heads + 2 * num_kv_heads) << vph_shift;
    const int threads = units < 512 ? ((units + 31) / 32) * 32 : 512;
    const int blocks = total_tokens < 148 * 32 ? total_tokens : 148 * 32;
    qkv_rope_append_kernel<<<blocks, threads, 0, (cudaStream_t)stream>>>(
        to_meta(m), seq_ids, start_pos, cu_tokens, n, total_tokens,
        static_cast<const uint16_t*>(qkv), (long)qkv_row_stride, rope_cos, rope_sin, rope_rows,
        static_cast<uint16_t*>(q_out), static_cast<uint16_t*>(k_pages),
        static_cast<uint16_t*>(v_pages), num_q_heads, num_kv_heads, head_dim, vph_shift);
    return launch_status("pool write_qkv");
}
