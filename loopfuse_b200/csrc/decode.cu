// Paged split-KV decode attention for sm_100a: entry points, the combine kernel and the
// launch sequence.
//
// Replaces the reference's decode_attention_fwd (kernels/triton/decode_attn.py:133-171,
// one program per (batch, head) over a contiguous cache) and the non-compiling
// ring_kv_decode_kernel (kernels/cuda/ring_kv_cache.cu:120-248).
//
// A decode is up to three launches on the caller's stream:
//   split    CTA (split, kv_head, session) applies pages_per_split consecutive pages of the
//            session's own block-table row to the Hq/Hkv query heads of kv_head (GQA: every K/V
//            byte is read once for the whole group) and writes one unnormalised partial
//            (o, max, sum) per query head.  Warp-level tensor-core kernel (decode_mma.cu).
//   prefix   when the first num_prefix_pages table entries are a prefix shared by every
//            session, those pages are applied once per group of sessions (tcgen05 kernel in
//            prefill.cu for head_dim 128, decode_prefix.cu for 64), on a side stream forked
//            next to the split launch; its partials go to their own slots.
//   combine  one warp per (session, query head) merges the row's partials by log-sum-exp.
#include "decode_common.cuh"

#include <math.h>

#include <mutex>

namespace lf {
namespace decode {

// Partial slots: part_o [N, Hq, n_slots, D] fp32 (unnormalised), part_ml [N, Hq, n_slots]
// (max in log2 units of the scaled scores, sum).

// Where combine puts a finished row.  n_peers == 0: o [N][Hq][D] of this call.  n_peers > 0
// (head-tensor-parallel decode): row (n, hq) of every output peers[k] [N][hq_total][D] at head
// head0 + hq -- the all-gather of the heads' outputs, done by the kernel that finishes them
// (peer-memory stores over NVLink).
struct CombineOut {
    uint16_t* o;
    uint16_t* const* peers;
    int n_peers, head0, hq_total;
};

// One warp per (session, query head) row, four rows per CTA.  The row's used slots (its own
// splits, then the shared-prefix chunks) are merged by log-sum-exp.  A split slot holds its
// unnormalised output in fp32; a prefix slot holds O / l in bf16 (first D * 2 bytes of the
// slot), scaled back by its l here.  Only the session length is read before the slots'
// addresses are known; then every lane loads its slot's (max, sum) pair and the first kPrefetch
// slots' output vectors (4 dims per lane) at once, so a row costs two dependent memory round
// trips, not one per batch of slots.  Rows with more slots take the rest in a loop.
constexpr int kCombineRows = 4;
constexpr int kPrefetch = 12;

template <int D>
__global__ void __launch_bounds__(32 * kCombineRows)
combine_kernel(const float* __restrict__ part_o, const float2* __restrict__ part_ml,
               const int32_t* __restrict__ seq_lens, const CombineOut out,
               float* __restrict__ lse, int Hq, int max_pages, int pages_per_split,
               int first_page, int n_slots, int prefix_slot0, int n_prefix_chunks,
               int prefix_chunk_pages) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hq = blockIdx.x * kCombineRows + warp, n = blockIdx.y;
    if (hq >= Hq) return;
    const int L = min(max(seq_lens[n], 0), max_pages * kPage);
    const int npages = (L + kPage - 1) / kPage;
    const int rem = npages - first_page;
    const int nsplit = rem > 0 ? (rem + pages_per_split - 1) / pages_per_split : 0;
    // shared-prefix chunks that hold some of this session's keys (a session shorter than the
    // prefix uses only the first ones; the prefix pass may skip the rest for its whole tile)
    const int pre_pages = min(first_page, npages);
    const int nchunk = n_prefix_chunks > 0
                           ? min(n_prefix_chunks, (pre_pages + prefix_chunk_pages - 1) / prefix_chunk_pages)
                           : 0;
    const int total = nsplit + nchunk;
    const size_t row = (size_t)n * Hq + hq;
    const float2* ml = part_ml + row * n_slots;
    const float* po = part_o + row * n_slots * D;
    auto slot = [&](int j) { return j < nsplit ? j : prefix_slot0 + (j - nsplit); };

    constexpr int kLanes = D / 4;                          // lanes that own 4 output dims
    const int d0 = 4 * lane;
    const bool owner = lane < kLanes;
    auto load = [&](int j) -> float4 {                     // slot j's 4 dims of this lane
        const float* base = po + (size_t)slot(j) * D;
        if (j < nsplit) return *reinterpret_cast<const float4*>(base + d0);
        const uint2 b = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + d0);
        return make_float4(bf16lo_to_f32(b.x), bf16hi_to_f32(b.x), bf16lo_to_f32(b.y), bf16hi_to_f32(b.y));
    };
    float2 e = make_float2(-INFINITY, 0.f);
    if (lane < total) e = ml[slot(lane)];
    float4 v[kPrefetch];
#pragma unroll
    for (int t = 0; t < kPrefetch; ++t)
        v[t] = (t < total && owner) ? load(t) : make_float4(0.f, 0.f, 0.f, 0.f);

    float M = e.x;
    for (int j = lane + 32; j < total; j += 32) M = fmaxf(M, ml[slot(j)].x);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
    float w = lane < total ? fast_exp2(e.x - M) : 0.f;
    if (lane < total) l = w * e.y;
    // weight of slot j's vector: w for a split slot, w * l for a (normalised) prefix slot
    float wv = lane >= nsplit ? w * e.y : w;
#pragma unroll
    for (int t = 0; t < kPrefetch; ++t) {
        const float wt = __shfl_sync(0xffffffffu, wv, t);
        acc.x = fmaf(wt, v[t].x, acc.x); acc.y = fmaf(wt, v[t].y, acc.y);
        acc.z = fmaf(wt, v[t].z, acc.z); acc.w = fmaf(wt, v[t].w, acc.w);
    }
    for (int j0 = 0; j0 < total; j0 += 32) {
        if (j0 > 0) {
            wv = 0.f;
            if (j0 + lane < total) {
                const float2 ej = ml[slot(j0 + lane)];
                const float wj = fast_exp2(ej.x - M);
                l = fmaf(wj, ej.y, l);
                wv = j0 + lane >= nsplit ? wj * ej.y : wj;
            }
        }
        const int t_end = min(32, total - j0);
#pragma unroll 4
        for (int t = (j0 == 0 ? kPrefetch : 0); t < t_end; ++t) {
            const float wt = __shfl_sync(0xffffffffu, wv, t);
            if (owner) {
                const float4 vt = load(j0 + t);
                acc.x = fmaf(wt, vt.x, acc.x); acc.y = fmaf(wt, vt.y, acc.y);
                acc.z = fmaf(wt, vt.z, acc.z); acc.w = fmaf(wt, vt.w, acc.w);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);

    if (lane < kLanes) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint2 packed;
        packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
        packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
        if (out.n_peers == 0) {
            *reinterpret_cast<uint2*>(out.o + row * D + d0) = packed;
        } else {
            const size_t grow = ((size_t)n * out.hq_total + out.head0 + hq) * D + d0;
            for (int k = 0; k < out.n_peers; ++k) *reinterpret_cast<uint2*>(out.peers[k] + grow) = packed;
            __threadfence_system();                  // visible to the peers before the kernel ends
        }
    }
    if (lse != nullptr && lane == 0) lse[row] = l > 0.f ? (M + log2f(l)) * kLn2 : -INFINITY;
}

// Slots [0, suffix_splits) hold the per-session splits after the prefix; slots
// [suffix_splits, suffix_splits + prefix_chunks) hold the shared-prefix chunks.
inline int suffix_splits(int max_pages, int pps, int n_prefix) {
    return (max_pages - n_prefix + pps - 1) / pps;
}
// Shared-prefix pages are cut into chunks; a tensor-core work item is one (pair of 128-row query
// tiles, KV head, chunk).  Longer chunks amortise an item's fixed cost (start-up loads, epilogue)
// and leave fewer partials for the combine; shorter ones make more items, which matters when the
// prefix pass is the critical path (few sessions, short private runs).  The chunk starts at 32
// pages and doubles while the pass keeps at least 8 items per KV head (64 at 8 KV heads).
// Measured on B200 with a 4096-token prefix and 600-1600 private tokens per session: 64
// sessions -> 32 pages, 96-128 -> 64, 256 -> 128, 512 -> 256, each the fastest of 16..256 pages
// or within 3% of it.  Counting per KV head makes the chunk -- and with it the order in which
// partials are merged -- depend on the sessions only, not on how many KV heads one call holds:
// a head-parallel decode over a share of the heads reproduces the one-GPU result bit for bit.
constexpr int kMinPrefixChunk = 32;
inline int prefix_chunk_pages(int N, int G, int n_prefix) {
    const long tiles = ((long)N * G + 255) / 256;
    int c = kMinPrefixChunk;
    while (c < n_prefix && tiles * ((n_prefix + 2L * c - 1) / (2L * c)) >= 8) c *= 2;
    return c;
}
inline int prefix_chunks(int chunk_pages, int n_prefix) {
    return (n_prefix + chunk_pages - 1) / chunk_pages;
}
// chunk_pages = kMinPrefixChunk gives the most slots any launch can use (workspace sizing).
inline int num_slots(int max_pages, int pages_per_split, int num_prefix_pages, int chunk_pages) {
    return suffix_splits(max_pages, pages_per_split, num_prefix_pages) +
           prefix_chunks(chunk_pages, num_prefix_pages);
}

}  // namespace decode
}  // namespace lf

using namespace lf;

extern "C" int lf_decode_workspace_size(int num_seqs, int num_q_heads, int head_dim,
                                        int max_pages, int pages_per_split, int num_prefix_pages,
                                        size_t* bytes) {
    LF_CHECK_ARG(bytes != nullptr, "decode: bytes is null");
    LF_CHECK_ARG(num_seqs >= 0 && num_q_heads > 0 && head_dim > 0 && max_pages > 0 &&
                     pages_per_split > 0 && num_prefix_pages >= 0,
                 "decode: bad workspace arguments");
    const size_t slots = (size_t)decode::num_slots(max_pages, pages_per_split, num_prefix_pages,
                                                   decode::kMinPrefixChunk);
    *bytes = (size_t)num_seqs * num_q_heads * slots * ((size_t)head_dim * sizeof(float) + sizeof(float2));
    clear_error();
    return LF_OK;
}

namespace lf {
namespace decode {

// SM count of the current device, looked up once per device ordinal.
static int device_sm_count(int* out) {
    static std::mutex mu;
    static int cached[128] = {0};
    int dev = 0;
    LF_CHECK_CUDA(cudaGetDevice(&dev));
    LF_CHECK_ARG(dev >= 0 && dev < 128, "decode: device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int sms = 0;
        LF_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        cached[dev] = sms;
    }
    *out = cached[dev];
    return LF_OK;
}

// Default split size: enough CTAs for several waves of three split CTAs per SM (eight waves of
// the table's capacity, with sessions taken to be half full), 32 to 128 pages per split.  The
// floor of 32 keeps small batches from launching many short or empty splits.
static int default_split(int num_seqs, int num_kv_heads, int max_pages, int num_prefix_pages,
                         int sm_count) {
    const long target_ctas = (long)sm_count * 3 * 8;
    const long own = max(1, (max_pages - num_prefix_pages) / 2);
    const long per = max(1L, ((long)num_seqs * num_kv_heads * own) / target_ctas);
    int pps = 32;
    while (pps < per && pps < 128) pps *= 2;
    return pps;
}

}  // namespace decode
}  // namespace lf

extern "C" int lf_decode_default_split(int num_seqs, int num_kv_heads, int max_pages,
                                       int num_prefix_pages, int sm_count, int* pages_per_split) {
    LF_CHECK_ARG(pages_per_split != nullptr, "decode split: out pointer is null");
    LF_CHECK_ARG(num_seqs >= 0 && num_kv_heads > 0 && max_pages > 0 && num_prefix_pages >= 0 &&
                     num_prefix_pages <= max_pages,
                 "decode split: bad arguments");
    if (sm_count <= 0) {
        const int rc = decode::device_sm_count(&sm_count);
        if (rc != LF_OK) return rc;
    }
    *pages_per_split = decode::default_split(num_seqs, num_kv_heads, max_pages, num_prefix_pages,
                                             sm_count);
    clear_error();
    return LF_OK;
}

// Defined in decode_mma.cu: the per-session split pass on the warp-level tensor-core MMA.
namespace lf { namespace decode {
int launch_split_mma(dim3 grid, cudaStream_t st, const uint16_t* q, const uint16_t* kp,
                     const uint16_t* vp, const int32_t* bt, const int32_t* lens, float* po,
                     float2* pml, int Hq, int Hkv, int D, int num_pages, int max_pages, int pps,
                     int first_page, int n_slots, float qscale,
                     const uint16_t* k_new, const uint16_t* v_new);
}}

// Defined in decode_prefix.cu: shared-prefix partials, one pass over the prefix pages per
// group of sessions.
namespace lf { namespace decode {
int launch_prefix(const uint16_t* q, const uint16_t* kp, const uint16_t* vp, const int32_t* bt,
                  const int32_t* lens, float* po, float2* pml, int N, int Hq, int Hkv, int D,
                  int num_pages, int max_pages, int n_prefix, int pages_per_chunk, int n_slots,
                  int slot0, float qscale, cudaStream_t st);
}}

static cudaEvent_t g_prof_begin = nullptr, g_prof_end = nullptr;

extern "C" int lf_decode_set_profile_events(void* ev_begin, void* ev_end) {
    g_prof_begin = static_cast<cudaEvent_t>(ev_begin);
    g_prof_end = static_cast<cudaEvent_t>(ev_end);
    clear_error();
    return LF_OK;
}

// The shared-prefix partial pass is latency-bound (a few tensor-core work items) while the split
// kernel is bandwidth-bound, and they write disjoint partial slots: the prefix pass runs on a
// library-owned stream forked from the caller's (event record / wait, the pattern stream capture
// supports) and joins back before the combine.  One side stream and its two events per CUDA
// context, created the first time the context decodes (streams and events belong to a context,
// so they are keyed on its id, not on the device ordinal: after a device reset or with another
// context current a new set is made); a mutex keeps concurrent callers' fork/join pairs from
// interleaving.
namespace {
struct SideStream {
    unsigned long long ctx = 0;
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mu;
constexpr int kSideStreams = 64;
SideStream g_side[kSideStreams];
int g_side_next = 0;

int side_stream(SideStream** out) {                  // caller holds g_side_mu
    unsigned long long id = 0;
    int rc = current_context_id(&id);
    if (rc != LF_OK) return rc;
    for (SideStream& ss : g_side)
        if (ss.s != nullptr && ss.ctx == id) {
            *out = &ss;
            return LF_OK;
        }
    // A new context takes the next entry.  Past kSideStreams contexts the oldest entry is
    // reused; its handles are left alone (they may belong to a context that no longer exists).
    SideStream& ss = g_side[g_side_next];
    SideStream fresh;
    fresh.ctx = id;
    LF_CHECK_CUDA(cudaStreamCreateWithFlags(&fresh.s, cudaStreamNonBlocking));
    LF_CHECK_CUDA(cudaEventCreateWithFlags(&fresh.fork, cudaEventDisableTiming));
    LF_CHECK_CUDA(cudaEventCreateWithFlags(&fresh.join, cudaEventDisableTiming));
    ss = fresh;
    g_side_next = (g_side_next + 1) % kSideStreams;
    *out = &ss;
    return LF_OK;
}
}  // namespace

static int decode_impl(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                       const int32_t* block_table, const int32_t* seq_lens, int num_prefix_pages,
                       const decode::CombineOut& out, float* lse, void* workspace,
                       size_t workspace_bytes, int num_seqs, int num_q_heads, int num_kv_heads,
                       int head_dim, int num_pages, int max_pages, int pages_per_split,
                       float scale, void* stream, const lf_bf16* k_new = nullptr,
                       const lf_bf16* v_new = nullptr) {
    LF_CHECK_ARG(q && k_pages && v_pages && block_table && seq_lens && workspace,
                 "decode: null pointer argument");
    LF_CHECK_ARG(aligned16(q) && aligned16(k_pages) && aligned16(v_pages) && aligned16(workspace),
                 "decode: q, pages and workspace must be 16-byte aligned");
    LF_CHECK_ARG(head_dim == 128 || head_dim == 64, "decode: head_dim must be 64 or 128 (got %d)",
                 head_dim);
    LF_CHECK_ARG(num_seqs > 0 && num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
                 "decode: need num_seqs > 0 and Hq a multiple of Hkv");
    LF_CHECK_ARG(num_pages > 0 && max_pages > 0 && pages_per_split > 0,
                 "decode: num_pages, max_pages and pages_per_split must be > 0");
    LF_CHECK_ARG(num_prefix_pages >= 0 && num_prefix_pages <= max_pages,
                 "decode: num_prefix_pages out of range");
    LF_CHECK_ARG(num_seqs <= 65535 && num_kv_heads <= 65535, "decode: grid limits exceeded");
    size_t need = 0;
    lf_decode_workspace_size(num_seqs, num_q_heads, head_dim, max_pages, pages_per_split,
                             num_prefix_pages, &need);
    LF_CHECK_ARG(workspace_bytes >= need, "decode: workspace too small (%zu < %zu bytes)",
                 workspace_bytes, need);

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int G = num_q_heads / num_kv_heads;
    const int chunk = decode::prefix_chunk_pages(num_seqs, G, num_prefix_pages);
    const int n_slots = decode::num_slots(max_pages, pages_per_split, num_prefix_pages, chunk);
    const int max_split = decode::suffix_splits(max_pages, pages_per_split, num_prefix_pages);
    const int n_prefix_chunks = decode::prefix_chunks(chunk, num_prefix_pages);
    float* po = static_cast<float*>(workspace);
    float2* pml = reinterpret_cast<float2*>(po + (size_t)num_seqs * num_q_heads * n_slots * head_dim);
    const float qscale = scale * kLog2e;
    const uint16_t* q16 = q;

    const bool overlap = num_prefix_pages > 0 && max_split > 0;
    std::unique_lock<std::mutex> side_lock(g_side_mu, std::defer_lock);
    SideStream* side = nullptr;
    // With both passes, the prefix pass forks onto the side stream and is launched first: its
    // few persistent CTAs need a whole SM's shared memory each, and launched first they get SMs
    // at once while the split's small CTAs fill the rest.  (Launched second, they waited for SMs
    // to drain of split CTAs: 53.4 against 41.7 us per call at 64 sessions x 600 private tokens,
    // the same at 256 sessions x 16k tokens.)
    if (overlap) {
        side_lock.lock();
        int rc = side_stream(&side);
        if (rc != LF_OK) return rc;
        LF_CHECK_CUDA(cudaEventRecord(side->fork, st));
        LF_CHECK_CUDA(cudaStreamWaitEvent(side->s, side->fork, 0));
    }
    auto prefix_pass = [&](cudaStream_t pst) {
        return decode::launch_prefix(q16, k_pages, v_pages, block_table, seq_lens, po, pml,
                                     num_seqs, num_q_heads, num_kv_heads, head_dim, num_pages,
                                     max_pages, num_prefix_pages,
                                     chunk, n_slots,
                                     max_split, qscale, pst);
    };
    if (num_prefix_pages > 0 && !overlap) {
        int rc = prefix_pass(st);
        if (rc != LF_OK) return rc;
    }
    if (overlap) {
        const int rc = prefix_pass(side->s);
        cudaEventRecord(side->join, side->s);
        if (rc != LF_OK) {
            cudaStreamWaitEvent(st, side->join, 0);           // keep the fork closed
            return rc;
        }
    }
    const bool prof = g_prof_begin != nullptr && g_prof_end != nullptr;
    if (prof) LF_CHECK_CUDA(cudaEventRecord(g_prof_begin, st));
    if (max_split > 0) {
        dim3 grid(max_split, num_kv_heads, num_seqs);
        LF_CHECK_ARG(max_split <= 2147483647, "decode: too many splits");
        int rc = decode::launch_split_mma(grid, st, q16, k_pages, v_pages, block_table, seq_lens,
                                          po, pml, num_q_heads, num_kv_heads, head_dim, num_pages,
                                          max_pages, pages_per_split, num_prefix_pages, n_slots,
                                          qscale, k_new, v_new);
        if (rc == LF_OK) rc = launch_status("decode split");
        if (rc != LF_OK) {
            if (overlap) {                                    // keep the fork closed
                cudaEventRecord(side->join, side->s);
                cudaStreamWaitEvent(st, side->join, 0);
            }
            return rc;
        }
    }
    if (prof) LF_CHECK_CUDA(cudaEventRecord(g_prof_end, st));
    if (overlap) LF_CHECK_CUDA(cudaStreamWaitEvent(st, side->join, 0));   // prefix partials ready
    dim3 cgrid((num_q_heads + decode::kCombineRows - 1) / decode::kCombineRows, num_seqs);
    constexpr int cthreads = 32 * decode::kCombineRows;
    if (head_dim == 128)
        decode::combine_kernel<128><<<cgrid, cthreads, 0, st>>>(po, pml, seq_lens, out, lse, num_q_heads,
                                                                max_pages, pages_per_split, num_prefix_pages,
                                                                n_slots, max_split, n_prefix_chunks, chunk);
    else
        decode::combine_kernel<64><<<cgrid, cthreads, 0, st>>>(po, pml, seq_lens, out, lse, num_q_heads,
                                                               max_pages, pages_per_split, num_prefix_pages,
                                                               n_slots, max_split, n_prefix_chunks, chunk);
    return launch_status("decode combine");
}

extern "C" int lf_decode_fwd(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                             const int32_t* block_table, const int32_t* seq_lens,
                             int num_prefix_pages, lf_bf16* o, float* lse, void* workspace,
                             size_t workspace_bytes, int num_seqs, int num_q_heads,
                             int num_kv_heads, int head_dim, int num_pages, int max_pages,
                             int pages_per_split, float scale, void* stream) {
    LF_CHECK_ARG(o != nullptr && aligned16(o), "decode: o must be a 16-byte aligned pointer");
    const decode::CombineOut out{o, nullptr, 0, 0, num_q_heads};
    return decode_impl(q, k_pages, v_pages, block_table, seq_lens, num_prefix_pages, out, lse,
                       workspace, workspace_bytes, num_seqs, num_q_heads, num_kv_heads, head_dim,
                       num_pages, max_pages, pages_per_split, scale, stream);
}

extern "C" int lf_decode_fwd_append(const lf_bf16* q, lf_bf16* k_pages, lf_bf16* v_pages,
                                    const int32_t* block_table, const int32_t* seq_lens,
                                    int num_prefix_pages, const lf_bf16* k_new,
                                    const lf_bf16* v_new, lf_bf16* o, float* lse, void* workspace,
                                    size_t workspace_bytes, int num_seqs, int num_q_heads,
                                    int num_kv_heads, int head_dim, int num_pages, int max_pages,
                                    int pages_per_split, float scale, void* stream) {
    LF_CHECK_ARG(o != nullptr && aligned16(o), "decode append: o must be a 16-byte aligned pointer");
    LF_CHECK_ARG(k_new != nullptr && v_new != nullptr && aligned16(k_new) && aligned16(v_new),
                 "decode append: k_new and v_new must be 16-byte aligned pointers");
    // The newest token of every session must lie in a page of its own (past the shared-prefix
    // pages), which the split pass reads: a table wide enough to hold own pages is required.
    LF_CHECK_ARG(max_pages > num_prefix_pages,
                 "decode append: the newest tokens must lie past the %d shared-prefix pages",
                 num_prefix_pages);
    const decode::CombineOut out{o, nullptr, 0, 0, num_q_heads};
    return decode_impl(q, k_pages, v_pages, block_table, seq_lens, num_prefix_pages, out, lse,
                       workspace, workspace_bytes, num_seqs, num_q_heads, num_kv_heads, head_dim,
                       num_pages, max_pages, pages_per_split, scale, stream, k_new, v_new);
}

extern "C" int lf_decode_fwd_gather(const lf_bf16* q, const lf_bf16* k_pages,
                                    const lf_bf16* v_pages, const int32_t* block_table,
                                    const int32_t* seq_lens, int num_prefix_pages,
                                    lf_bf16* const* out_peers, int n_peers, int head_offset,
                                    int num_q_heads_total, float* lse, void* workspace,
                                    size_t workspace_bytes, int num_seqs, int num_q_heads,
                                    int num_kv_heads, int head_dim, int num_pages, int max_pages,
                                    int pages_per_split, float scale, void* stream) {
    LF_CHECK_ARG(out_peers != nullptr && n_peers > 0 && n_peers <= 64,
                 "decode gather: need 1..64 output pointers (a device array)");
    LF_CHECK_ARG(head_offset >= 0 && head_offset + num_q_heads <= num_q_heads_total,
                 "decode gather: heads [%d, %d) outside the %d output heads", head_offset,
                 head_offset + num_q_heads, num_q_heads_total);
    const decode::CombineOut out{nullptr, out_peers, n_peers, head_offset, num_q_heads_total};
    return decode_impl(q, k_pages, v_pages, block_table, seq_lens, num_prefix_pages, out, lse,
                       workspace, workspace_bytes, num_seqs, num_q_heads, num_kv_heads, head_dim,
                       num_pages, max_pages, pages_per_split, scale, stream);
}

// ---- decode without device allocation ------------------------------------------------------
//
// lf_decode_fwd needs a caller-provided workspace for the split partials.  Some callers have
// no way to provide one: a binding from another language with no device allocator of its own,
// or a serving loop whose caching allocator has already reserved nearly all of HBM for the KV
// pool, where a cudaMalloc would fail or synchronise the device.  lf_decode_fwd_noalloc runs
// the same kernels with the partials kept in the fixed array below, which is part of the
// library image: every GPU that loads the library holds these bytes until the process exits.
//
// The split size is chosen here (the smallest power-of-two page count, from the default
// heuristic upward, whose partials fit); a request whose partials do not fit even with one
// split per session is rejected with LF_EINVAL.  Every slot the combine kernel reads is written
// earlier in the same call, so nothing in the array needs clearing between calls.  All calls
// share the array: two calls whose kernels overlap on the GPU (different streams, or different
// host threads on one device) race on it and must be serialised by the caller.

static __device__ __align__(256) unsigned char g_noalloc_scratch[LF_DECODE_NOALLOC_SCRATCH_BYTES];


namespace lf {
namespace decode {

// Device address of g_noalloc_scratch in the current context.  The symbol's host-side name is
// only a stand-in, so the address is looked up with cudaGetSymbolAddress, with the device
// current, the first time a context calls, and kept for that context.  The cache is keyed on the
// driver's context id, which is unique for the life of the process: a device reset or a
// different context current on the same device gets a fresh lookup, never a stale address.
static int noalloc_scratch(void** out) {
    static std::mutex mu;
    constexpr int kEntries = 128;
    static unsigned long long ids[kEntries] = {0};
    static void* addr[kEntries] = {nullptr};
    static int next = 0;
    unsigned long long id = 0;
    int rc = lf::current_context_id(&id);
    if (rc != LF_OK) return rc;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < kEntries; ++i)
        if (addr[i] != nullptr && ids[i] == id) {
            *out = addr[i];
            return LF_OK;
        }
    void* p = nullptr;
    LF_CHECK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    ids[next] = id;
    addr[next] = p;
    next = (next + 1) % kEntries;
    *out = p;
    return LF_OK;
}

static size_t partial_bytes(int N, int Hq, int D, int max_pages, int pps, int n_prefix,
                            int chunk) {
    return (size_t)N * Hq * (size_t)num_slots(max_pages, pps, n_prefix, chunk) *
           ((size_t)D * sizeof(float) + sizeof(float2));
}

}  // namespace decode
}  // namespace lf

extern "C" int lf_decode_fwd_noalloc(const lf_bf16* q, const lf_bf16* k_pages,
                                     const lf_bf16* v_pages, const int32_t* block_table,
                                     const int32_t* seq_lens, int num_prefix_pages, lf_bf16* o,
                                     float* lse, int num_seqs, int num_q_heads, int num_kv_heads,
                                     int head_dim, int num_pages, int max_pages, float scale,
                                     void* stream) {
    LF_CHECK_ARG(q && k_pages && v_pages && block_table && seq_lens && o,
                 "decode noalloc: null pointer argument");
    LF_CHECK_ARG(aligned16(q) && aligned16(k_pages) && aligned16(v_pages) && aligned16(o),
                 "decode noalloc: q, pages and o must be 16-byte aligned");
    LF_CHECK_ARG(head_dim == 128 || head_dim == 64, "decode noalloc: head_dim must be 64 or 128");
    LF_CHECK_ARG(num_seqs > 0 && num_seqs <= 65535 && num_kv_heads > 0 && num_kv_heads <= 65535 &&
                     num_q_heads % num_kv_heads == 0,
                 "decode noalloc: need 0 < num_seqs <= 65535 and Hq a multiple of Hkv");
    LF_CHECK_ARG(num_pages > 0 && max_pages > 0 && num_prefix_pages >= 0 &&
                     num_prefix_pages <= max_pages,
                 "decode noalloc: bad page counts");

    // Split size: the default (lf_decode_default_split on this device), doubled until the
    // partials fit the fixed scratch.
    int sms = 0;
    int rc = decode::device_sm_count(&sms);
    if (rc != LF_OK) return rc;
    int pps = decode::default_split(num_seqs, num_kv_heads, max_pages, num_prefix_pages, sms);
    const int chunk = decode::prefix_chunk_pages(num_seqs, num_q_heads / num_kv_heads, num_prefix_pages);
    while (decode::partial_bytes(num_seqs, num_q_heads, head_dim, max_pages, pps, num_prefix_pages,
                                 chunk) >
               (size_t)LF_DECODE_NOALLOC_SCRATCH_BYTES &&
           pps < max_pages)
        pps = pps * 2 < max_pages ? pps * 2 : max_pages;
    const size_t need =
        decode::partial_bytes(num_seqs, num_q_heads, head_dim, max_pages, pps, num_prefix_pages, chunk);
    LF_CHECK_ARG(need <= (size_t)LF_DECODE_NOALLOC_SCRATCH_BYTES,
                 "decode noalloc: %d sessions x %d heads need %zu bytes of partials even with one "
                 "split per session; the fixed scratch holds %u bytes (use lf_decode_fwd with a "
                 "workspace)",
                 num_seqs, num_q_heads, need, (unsigned)LF_DECODE_NOALLOC_SCRATCH_BYTES);

    void* scratch = nullptr;
    rc = decode::noalloc_scratch(&scratch);
    if (rc != LF_OK) return rc;

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int n_slots = decode::num_slots(max_pages, pps, num_prefix_pages, chunk);
    const int max_split = decode::suffix_splits(max_pages, pps, num_prefix_pages);
    const int n_prefix_chunks = decode::prefix_chunks(chunk, num_prefix_pages);
    float* po = static_cast<float*>(scratch);
    float2* pml = reinterpret_cast<float2*>(po + (size_t)num_seqs * num_q_heads * n_slots * head_dim);
    const float qscale = scale * kLog2e;

    if (num_prefix_pages > 0) {
        rc = decode::launch_prefix(q, k_pages, v_pages, block_table, seq_lens, po, pml, num_seqs,
                                   num_q_heads, num_kv_heads, head_dim, num_pages, max_pages,
                                   num_prefix_pages, chunk, n_slots, max_split,
                                   qscale, st);
        if (rc != LF_OK) return rc;
    }
    if (max_split > 0) {
        dim3 grid(max_split, num_kv_heads, num_seqs);
        rc = decode::launch_split_mma(grid, st, q, k_pages, v_pages, block_table, seq_lens, po,
                                      pml, num_q_heads, num_kv_heads, head_dim, num_pages,
                                      max_pages, pps, num_prefix_pages, n_slots, qscale, nullptr,
                                      nullptr);
        if (rc != LF_OK) return rc;
        rc = launch_status("decode noalloc split");
        if (rc != LF_OK) return rc;
    }
    dim3 cgrid((num_q_heads + decode::kCombineRows - 1) / decode::kCombineRows, num_seqs);
    if (head_dim == 128)
        decode::combine_kernel<128><<<cgrid, 32 * decode::kCombineRows, 0, st>>>(po, pml, seq_lens,
                                                          decode::CombineOut{o, nullptr, 0, 0, num_q_heads},
                                                          lse, num_q_heads,
                                                          max_pages, pps, num_prefix_pages,
                                                          n_slots, max_split, n_prefix_chunks, chunk);
    else
        decode::combine_kernel<64><<<cgrid, 32 * decode::kCombineRows, 0, st>>>(po, pml, seq_lens,
                                                         decode::CombineOut{o, nullptr, 0, 0, num_q_heads},
                                                         lse, num_q_heads,
                                                         max_pages, pps, num_prefix_pages,
                                                         n_slots, max_split, n_prefix_chunks, chunk);
    return launch_status("decode noalloc combine");
}
