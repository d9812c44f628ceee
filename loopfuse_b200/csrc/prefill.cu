// Causal GQA prefill attention for sm_100a: tcgen05 MMA, TMEM accumulators, TMA tiles.
//
// Replaces prefill_attention_fwd (kernels/triton/prefill_attn.py:127-168, an FA2-style
// Triton kernel, MHA/fp16 only) and the reference's sm_80 agent_prefill_kernel
// (kernels/cuda/async_prefill.cu:56-236, wmma QK^T only, no softmax or P.V).  The kernel is the
// dense instantiation of the tcgen05 attention core in attn_tc2.cuh: CTAs that stay resident
// (one per SM) take pairs of adjacent 128-row query tiles of one (batch, query head) from a
// heavy-first queue.
//
// This file also launches the core's Prefix instantiation for the decode's shared-prefix pass.

#include "attn_tc2.cuh"
#include "tmap.cuh"

using namespace lf;

namespace {

// The dynamic shared-memory opt-in is a setting of the kernel in one CUDA context, so it is made
// once for each context this process launches in (setting it twice is harmless).
template <lf::tc2::Mode M, int HD>
int set_smem_attr() {
    static lf::PerContextOnce once;
    return once.run([] {
        LF_CHECK_CUDA(cudaFuncSetAttribute(lf::tc2::attn2_kernel<M, HD>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)lf::tc2::kSmemBytes));
        return LF_OK;
    });
}

template <int HD>
int launch_dense(const lf_bf16* q, const lf_bf16* k, const lf_bf16* v, lf::tc2::Params p,
                 long n_items, cudaStream_t st) {
    using namespace lf::tc2;
    // [B*H][S][HD] bf16 views; [128 rows][64 dims] boxes.
    CUtensorMap mq, mk, mv;
    const cuuint32_t box[3] = {64, 128, 1};
    const cuuint64_t qdims[3] = {(cuuint64_t)HD, (cuuint64_t)p.Sq, (cuuint64_t)p.B * p.Hq};
    const cuuint64_t qstr[2] = {(cuuint64_t)HD * 2, (cuuint64_t)p.Sq * HD * 2};
    const cuuint64_t kdims[3] = {(cuuint64_t)HD, (cuuint64_t)p.Sk, (cuuint64_t)p.B * p.Hkv};
    const cuuint64_t kstr[2] = {(cuuint64_t)HD * 2, (cuuint64_t)p.Sk * HD * 2};
    int rc = lf::encode_bf16_map(&mq, q, 3, qdims, qstr, box);
    if (rc) return rc;
    rc = lf::encode_bf16_map(&mk, k, 3, kdims, kstr, box);
    if (rc) return rc;
    rc = lf::encode_bf16_map(&mv, v, 3, kdims, kstr, box);
    if (rc) return rc;
    rc = set_smem_attr<Mode::Dense, HD>();
    if (rc) return rc;
    // One CTA per item: CTAs of the first wave take over the items of CTAs not yet launched
    // (cluster launch control), so the grid behaves like a persistent one with dynamic balance.
    LF_CHECK_ARG(n_items <= 2147483647L, "prefill: too many work items");
    attn2_kernel<Mode::Dense, HD><<<(unsigned)n_items, kThreads, kSmemBytes, st>>>(mq, mk, mv, p);
    return lf::launch_status("prefill");
}

template <int HD>
int launch_paged(const lf_bf16* q, const lf_bf16* kp, const lf_bf16* vp, int total_q, lf::tc2::Params p,
                 long n_items, cudaStream_t st) {
    using namespace lf::tc2;
    CUtensorMap mq, mk, mv;
    // q [total_q][Hq / G][G][HD]: one box = 128 / G tokens x the G heads of one group.
    const cuuint64_t qdims[4] = {(cuuint64_t)HD, (cuuint64_t)p.G, (cuuint64_t)(p.Hq / p.G),
                                 (cuuint64_t)total_q};
    const cuuint64_t qstr[3] = {(cuuint64_t)HD * 2, (cuuint64_t)p.G * HD * 2, (cuuint64_t)p.Hq * HD * 2};
    const cuuint32_t qbox[4] = {64, (cuuint32_t)p.G, 1, (cuuint32_t)(BM / p.G)};
    const cuuint64_t pdims[3] = {(cuuint64_t)HD, 16, (cuuint64_t)p.num_pages * p.Hkv};
    const cuuint64_t pstr[2] = {(cuuint64_t)HD * 2, (cuuint64_t)16 * HD * 2};
    const cuuint32_t pbox[3] = {64, 16, 1};
    int rc = lf::encode_bf16_map(&mq, q, 4, qdims, qstr, qbox);
    if (rc) return rc;
    rc = lf::encode_bf16_map(&mk, kp, 3, pdims, pstr, pbox);
    if (rc) return rc;
    rc = lf::encode_bf16_map(&mv, vp, 3, pdims, pstr, pbox);
    if (rc) return rc;
    rc = set_smem_attr<Mode::Paged, HD>();
    if (rc) return rc;
    LF_CHECK_ARG(n_items <= 2147483647L, "prefill paged: too many work items");
    attn2_kernel<Mode::Paged, HD><<<(unsigned)n_items, kThreads, kSmemBytes, st>>>(mq, mk, mv, p);
    return lf::launch_status("prefill paged");
}

}  // namespace

extern "C" int lf_prefill_fwd(const lf_bf16* q, const lf_bf16* k, const lf_bf16* v, lf_bf16* o,
                              float* lse, int batch, int num_q_heads, int num_kv_heads, int seq_q,
                              int seq_k, int head_dim, float scale, int causal, void* stream) {
    using namespace lf::tc2;
    LF_CHECK_ARG(q && k && v && o, "prefill: null pointer argument");
    LF_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o),
                 "prefill: q, k, v, o must be 16-byte aligned");
    LF_CHECK_ARG(head_dim == 128 || head_dim == 64, "prefill: head_dim must be 64 or 128 (got %d)",
                 head_dim);
    LF_CHECK_ARG(batch > 0 && num_q_heads > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                 "prefill: need Hq a positive multiple of Hkv");
    LF_CHECK_ARG(seq_q > 0 && seq_k > 0, "prefill: sequence lengths must be positive");
    const long n_qt = (seq_q + BM - 1) / BM;
    const long n_pairs = (n_qt + 1) / 2;
    const long n_items = n_pairs * batch * num_q_heads;
    LF_CHECK_ARG(n_items < 2147483647L, "prefill: too many query tiles");
    Params p{};
    p.c = scale * kLog2e;
    p.o = o;
    p.o_align32 = (reinterpret_cast<uintptr_t>(o) & 31u) == 0 ? 1 : 0;
    p.lse = lse;
    p.B = batch;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.Sq = seq_q;
    p.Sk = seq_k;
    p.n_qt = (int)n_qt;
    p.n_pairs = (int)n_pairs;
    p.n_items = (int)n_items;
    p.causal = causal ? 1 : 0;
    p.q_offset = seq_k - seq_q;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return head_dim == 128 ? launch_dense<128>(q, k, v, p, n_items, st)
                           : launch_dense<64>(q, k, v, p, n_items, st);
}

extern "C" int lf_prefill_paged_fwd(const lf_bf16* q, const lf_bf16* k_pages,
                                    const lf_bf16* v_pages, const int32_t* block_table,
                                    const int32_t* cu_seqlens_q, const int32_t* seqlens_k,
                                    lf_bf16* o, float* lse, int num_seqs, int total_q,
                                    int max_seqlen_q, int num_q_heads, int num_kv_heads,
                                    int head_dim, int num_pages, int max_pages, float scale,
                                    int causal, void* stream) {
    using namespace lf::tc2;
    LF_CHECK_ARG(q && k_pages && v_pages && block_table && cu_seqlens_q && seqlens_k && o,
                 "prefill paged: null pointer argument");
    LF_CHECK_ARG(aligned16(q) && aligned16(k_pages) && aligned16(v_pages) && aligned16(o),
                 "prefill paged: q, pages and o must be 16-byte aligned");
    LF_CHECK_ARG(head_dim == 128 || head_dim == 64,
                 "prefill paged: head_dim must be 64 or 128 (got %d)", head_dim);
    LF_CHECK_ARG(num_seqs > 0 && total_q > 0 && max_seqlen_q > 0 && num_kv_heads > 0 &&
                     num_q_heads % num_kv_heads == 0 && num_pages > 0 && max_pages > 0,
                 "prefill paged: bad sizes");
    // GQA packing: the query heads of a KV group share a work item (and its K/V stream) when
    // the group size divides the 128-row tile; otherwise every head is its own group.
    const int group = num_q_heads / num_kv_heads;
    const int pack = (BM % group == 0) ? group : 1;
    const long max_pairs = (((long)max_seqlen_q * pack + BM - 1) / BM + 1) / 2;
    const long n_items = max_pairs * num_seqs * (num_q_heads / pack);
    LF_CHECK_ARG(n_items < 2147483647L, "prefill paged: too many work items");
    Params p{};
    p.c = scale * kLog2e;
    p.o = o;
    p.o_align32 = (reinterpret_cast<uintptr_t>(o) & 31u) == 0 ? 1 : 0;
    p.lse = lse;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.causal = causal ? 1 : 0;
    p.bt = block_table;
    p.lens = seqlens_k;
    p.cu_q = cu_seqlens_q;
    p.N = num_seqs;
    p.G = pack;
    p.num_pages = num_pages;
    p.max_pages = max_pages;
    p.max_pairs = (int)max_pairs;
    p.n_items = (int)n_items;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return head_dim == 128 ? launch_paged<128>(q, k_pages, v_pages, total_q, p, n_items, st)
                           : launch_paged<64>(q, k_pages, v_pages, total_q, p, n_items, st);
}

namespace lf {
namespace decode {

// Shared-prefix partials on the tensor cores (head_dim 128): the Prefix instantiation of the
// attention core.  Each CTA takes 2 x 128 query rows = 256/G sessions x G heads of one KV head
// and one chunk of prefix pages, and writes fp32 partials to workspace slots slot0 + chunk.
int launch_prefix_tc(const uint16_t* q, const uint16_t* kp, const uint16_t* vp, const int32_t* bt,
                     const int32_t* lens, float* po, float2* pml, int N, int Hq, int Hkv,
                     int num_pages, int max_pages, int n_prefix, int chunk_pages, int n_slots,
                     int slot0, float qscale, cudaStream_t st) {
    using namespace lf::tc2;
    const int G = Hq / Hkv;
    LF_CHECK_ARG(G >= 1 && G <= 8 && (G & (G - 1)) == 0, "decode prefix: Hq/Hkv must be 1, 2, 4 or 8");
    CUtensorMap mq, mk, mv;
    // q [N][Hkv][G][D]: box = 128/G sessions x G heads x 64 dims of one KV head.
    constexpr int HD = 128;
    const cuuint64_t qdims[4] = {(cuuint64_t)HD, (cuuint64_t)G, (cuuint64_t)Hkv, (cuuint64_t)N};
    const cuuint64_t qstr[3] = {(cuuint64_t)HD * 2, (cuuint64_t)G * HD * 2, (cuuint64_t)Hq * HD * 2};
    const cuuint32_t qbox[4] = {64, (cuuint32_t)G, 1, (cuuint32_t)(BM / G)};
    // pages [P*Hkv][16][D]: box = one page of one head, 64 dims.
    const cuuint64_t pdims[3] = {(cuuint64_t)HD, 16, (cuuint64_t)num_pages * Hkv};
    const cuuint64_t pstr[2] = {(cuuint64_t)HD * 2, (cuuint64_t)16 * HD * 2};
    const cuuint32_t pbox[3] = {64, 16, 1};
    int rc = encode_bf16_map(&mq, q, 4, qdims, qstr, qbox);
    if (rc) return rc;
    rc = encode_bf16_map(&mk, kp, 3, pdims, pstr, pbox);
    if (rc) return rc;
    rc = encode_bf16_map(&mv, vp, 3, pdims, pstr, pbox);
    if (rc) return rc;

    int rc0 = set_smem_attr<Mode::Prefix, 128>();
    if (rc0) return rc0;
    Params p{};
    p.c = qscale;
    p.Hkv = Hkv;
    p.bt = bt;
    p.lens = lens;
    p.part_o = po;
    p.part_align32 = (reinterpret_cast<uintptr_t>(po) & 31u) == 0 ? 1 : 0;
    p.part_ml = pml;
    p.N = N;
    p.G = G;
    p.num_pages = num_pages;
    p.max_pages = max_pages;
    p.n_prefix = n_prefix;
    p.chunk_pages = chunk_pages;
    p.n_chunks = (n_prefix + chunk_pages - 1) / chunk_pages;
    p.n_qtiles = (N * G + 2 * BM - 1) / (2 * BM);
    p.n_slots = n_slots;
    p.slot0 = slot0;
    const long n_items = (long)p.n_qtiles * Hkv * p.n_chunks;
    LF_CHECK_ARG(n_items < 2147483647L, "decode prefix: too many work items");
    p.n_items = (int)n_items;
    attn2_kernel<Mode::Prefix, 128><<<(unsigned)n_items, kThreads, kSmemBytes, st>>>(mq, mk, mv, p);
    return launch_status("decode prefix (tensor cores)");
}

}  // namespace decode
}  // namespace lf

