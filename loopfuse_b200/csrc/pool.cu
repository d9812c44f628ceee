// Device kernels of the paged, refcounted KV pool.
//
// Replaces the dense slot pool of the reference (runtime/kv_pool.py:28-235: per-slot
// [L, H, max_seq, D] strips, FIFO slots, append at current_len) and its ring-buffer write
// kernel (kernels/cuda/ring_kv_cache.cu:69-109).  Metadata lives in device arrays owned by
// the caller (lf_pool_meta); every operation is a stream-ordered kernel, so a decode step can
// follow an append without a host round trip.  The pool oracle fixes the exact order in which
// pages leave and re-enter the FIFO free queue; these kernels reproduce it:
//   reserve  sessions in call order take ceil-page deltas from the queue head
//            (exclusive scan over the requests), all or nothing;
//   fork     shared full pages get refcount += n_dst; a partial page is copied to one fresh
//            page per destination, in destination order;
//   free     refcounts drop once per (session, page) occurrence; pages at zero re-enter the
//            queue tail once, at their first occurrence (session order, then page order),
//            found with an atomicMin on a per-page scratch word.
// Errors detected on the device go to the sticky ctrl[LF_CTRL_STATUS]; every kernel is a
// no-op while it is set, so a failed reserve never lets a later write scatter data.
#include "pool_common.cuh"

namespace lf {
namespace pool {

__global__ void init_kernel(Meta m) {
    const long total = max((long)m.P, (long)m.S * m.M);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        if (i < m.P) {
            m.fq[i] = (int)i;
            m.rc[i] = 0;
            m.scratch[i] = INT_MAX;
        }
        if (i < (long)m.S * m.M) m.bt[i] = -1;
        if (i < m.S) m.len[i] = 0;
        if (i < LF_CTRL_WORDS) m.ctrl[i] = 0;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) m.ctrl[LF_CTRL_COUNT] = m.P;
}

__global__ void clear_status_kernel(Meta m) { m.ctrl[LF_CTRL_STATUS] = LF_OK; }

// Error precedence follows the oracle: the first offending session (in call order) decides
// between EINVAL and EOVERFLOW; ENOPAGES is checked only when every session is valid.
__global__ void __launch_bounds__(kMetaThreads)
reserve_kernel(Meta m, const int32_t* __restrict__ seq_ids, const int32_t* __restrict__ n_new,
               int n, int32_t* __restrict__ start_pos) {
    __shared__ int buf[32];
    __shared__ unsigned seen[kDupBits / 32];
    if (status_of(m) != LF_OK) return;
    // A session that grows appears once: the page deltas are computed from each session's
    // length before the call, so a repeated id would take pages twice (and its entries would
    // race on its length).  Entries of zero tokens change nothing and may repeat -- padding rows
    // of a fixed-size batch -- unless their session also grows in this call.  A bitmap of the
    // growing sessions finds whether any entry conflicts; only then does the exact scan name
    // the first conflicting entry in call order.
    int dup = 0;
    if (m.S <= kDupBits) {
        for (int w = threadIdx.x; w < (m.S + 31) / 32; w += kMetaThreads) seen[w] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += kMetaThreads) {
            const int s = seq_ids[i];
            if (s < 0 || s >= m.S || n_new[i] == 0) continue;
            const unsigned bit = 1u << (s & 31);
            if (atomicOr(&seen[s >> 5], bit) & bit) dup = 1;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += kMetaThreads) {
            const int s = seq_ids[i];
            if (s < 0 || s >= m.S || n_new[i] != 0) continue;
            if (seen[s >> 5] & (1u << (s & 31))) dup = 1;
        }
        dup = -block_min(-dup, buf);
    } else {
        dup = 1;
    }
    int first_bad = INT_MAX;
    long need_total = 0;
    for (int i = threadIdx.x; i < n; i += kMetaThreads) {
        const int s = seq_ids[i];
        const int t = n_new[i];
        bool repeat = false;
        if (dup)
            for (int j = 0; j < i && !repeat; ++j)
                repeat = seq_ids[j] == s && (t != 0 || n_new[j] != 0);
        if (s < 0 || s >= m.S || t < 0 || repeat) {
            first_bad = min(first_bad, i * 8 + LF_EINVAL);
            continue;
        }
        const int L = m.len[s];
        if ((long)L + t > (long)m.M * LF_PAGE_SIZE) {
            first_bad = min(first_bad, i * 8 + LF_EOVERFLOW);
            continue;
        }
        need_total += pages_for(L + t) - pages_for(L);
    }
    first_bad = block_min(first_bad, buf);
    // need_total fits in int: it is bounded by S * M page slots.
    int total = 0;
    block_excl_scan((int)need_total, &total, buf);
    const int head = m.ctrl[LF_CTRL_HEAD];
    const int count = m.ctrl[LF_CTRL_COUNT];
    __syncthreads();
    if (first_bad != INT_MAX || total > count) {
        if (threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = first_bad != INT_MAX ? (first_bad & 7) : LF_ENOPAGES;
        return;
    }
    int carry = 0;
    for (int base = 0; base < n; base += kMetaThreads) {
        const int i = base + threadIdx.x;
        int need = 0, L = 0, s = 0;
        if (i < n) {
            s = seq_ids[i];
            L = m.len[s];
            need = pages_for(L + n_new[i]) - pages_for(L);
        }
        int round_total = 0;
        const int off = carry + block_excl_scan(need, &round_total, buf);
        if (i < n) {
            const int old_pages = pages_for(L);
            for (int j = 0; j < need; ++j) {
                const int p = m.fq[(int)(((long)head + off + j) % m.P)];
                m.bt[(long)s * m.M + old_pages + j] = p;
                m.rc[p] = 1;
            }
            if (start_pos) start_pos[i] = L;
            m.len[s] = L + n_new[i];
        }
        carry += round_total;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        m.ctrl[LF_CTRL_HEAD] = (int)(((long)head + total) % m.P);
        m.ctrl[LF_CTRL_COUNT] = count - total;
    }
}

// Token rows of the new K/V go to their pages with 16-byte vector copies.  grid.x walks
// (token, head, vector) triples of one layer, grid.y is the layer.
__global__ void write_kv_kernel(Meta m, const int32_t* __restrict__ seq_ids,
                                const int32_t* __restrict__ start_pos,
                                const int32_t* __restrict__ cu_tokens, int n, int total_tokens,
                                const uint16_t* __restrict__ k_new,
                                const uint16_t* __restrict__ v_new, long sl, long st, long sh,
                                uint16_t* __restrict__ kp, uint16_t* __restrict__ vp, int Hkv,
                                int D) {
    if (status_of(m) != LF_OK) return;
    const int vecs = D / 8;
    const long per_layer = (long)total_tokens * Hkv * vecs;
    const int l = blockIdx.y;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < per_layer;
         idx += (long)gridDim.x * blockDim.x) {
        const int vec = (int)(idx % vecs);
        const int h = (int)((idx / vecs) % Hkv);
        const int t = (int)(idx / ((long)vecs * Hkv));
        int lo = 0, hi = n - 1;                      // session i with cu[i] <= t < cu[i+1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (cu_tokens[mid] <= t) lo = mid; else hi = mid - 1;
        }
        const int s = seq_ids[lo];
        const int pos = start_pos[lo] + (t - cu_tokens[lo]);
        // A row without a reserved page (stale start_pos, a session that was not reserved, a
        // bad id) is not stored: the sticky status says so and the other rows still land.
        if (s < 0 || s >= m.S || pos < 0 || pos / LF_PAGE_SIZE >= m.M) {
            atomicCAS(m.ctrl + LF_CTRL_STATUS, LF_OK, LF_EINVAL);
            continue;
        }
        const int page = m.bt[(long)s * m.M + pos / LF_PAGE_SIZE];
        if (static_cast<unsigned>(page) >= static_cast<unsigned>(m.P)) {
            atomicCAS(m.ctrl + LF_CTRL_STATUS, LF_OK, LF_EINVAL);
            continue;
        }
        const long src = l * sl + (long)t * st + (long)h * sh + vec * 8;
        const long dst = ((((long)l * m.P + page) * Hkv + h) * LF_PAGE_SIZE + pos % LF_PAGE_SIZE) * D + vec * 8;
        *reinterpret_cast<uint4*>(kp + dst) = *reinterpret_cast<const uint4*>(k_new + src);
        *reinterpret_cast<uint4*>(vp + dst) = *reinterpret_cast<const uint4*>(v_new + src);
    }
}

__global__ void __launch_bounds__(kMetaThreads)
fork_kernel(Meta m, int src, const int32_t* __restrict__ dsts, int n, int prefix_len) {
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    int bad = 0;
    if (src < 0 || src >= m.S || prefix_len < 0 || prefix_len > m.len[src]) bad = 1;
    for (int i = threadIdx.x; i < n; i += kMetaThreads) {
        const int d = dsts[i];
        if (d < 0 || d >= m.S || d == src || m.len[d] != 0) bad = 1;
    }
    bad = -block_min(-bad, buf);
    const int full = prefix_len / LF_PAGE_SIZE, part = prefix_len % LF_PAGE_SIZE;
    const int head = m.ctrl[LF_CTRL_HEAD];
    const int count = m.ctrl[LF_CTRL_COUNT];
    __syncthreads();
    if (bad || (part && n > count)) {
        if (threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = bad ? LF_EINVAL : LF_ENOPAGES;
        return;
    }
    const long srow = (long)src * m.M;
    for (long idx = threadIdx.x; idx < (long)n * full; idx += kMetaThreads) {
        const int i = (int)(idx / full), j = (int)(idx % full);
        m.bt[(long)dsts[i] * m.M + j] = m.bt[srow + j];
    }
    for (int j = threadIdx.x; j < full; j += kMetaThreads) m.rc[m.bt[srow + j]] += n;
    for (int i = threadIdx.x; i < n; i += kMetaThreads) {
        if (part) {
            const int p = m.fq[(int)(((long)head + i) % m.P)];
            m.rc[p] = 1;
            m.bt[(long)dsts[i] * m.M + full] = p;
        }
        m.len[dsts[i]] = prefix_len;
    }
    __syncthreads();
    if (threadIdx.x == 0 && part) {
        m.ctrl[LF_CTRL_HEAD] = (int)(((long)head + n) % m.P);
        m.ctrl[LF_CTRL_COUNT] = count - n;
    }
}

// Copies the first `part` rows of the source's partial page into each destination's fresh
// page.  grid = (destination, layer); threads walk (kv head, row, vector).
__global__ void fork_copy_kernel(Meta m, int src, const int32_t* __restrict__ dsts, int full,
                                 int part, uint16_t* __restrict__ kp, uint16_t* __restrict__ vp,
                                 int Hkv, int D) {
    if (status_of(m) != LF_OK) return;
    const int i = blockIdx.x, l = blockIdx.y;
    const int sp = m.bt[(long)src * m.M + full];
    const int dp = m.bt[(long)dsts[i] * m.M + full];
    const int vecs = D / 8;
    for (int idx = threadIdx.x; idx < Hkv * part * vecs; idx += blockDim.x) {
        const int vec = idx % vecs, r = (idx / vecs) % part, h = idx / (vecs * part);
        const long so = ((((long)l * m.P + sp) * Hkv + h) * LF_PAGE_SIZE + r) * D + vec * 8;
        const long dof = ((((long)l * m.P + dp) * Hkv + h) * LF_PAGE_SIZE + r) * D + vec * 8;
        *reinterpret_cast<uint4*>(kp + dof) = *reinterpret_cast<const uint4*>(kp + so);
        *reinterpret_cast<uint4*>(vp + dof) = *reinterpret_cast<const uint4*>(vp + so);
    }
}

__global__ void __launch_bounds__(kMetaThreads)
free_kernel(Meta m, const int32_t* __restrict__ seq_ids, int n) {
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    int bad = 0;
    for (int i = threadIdx.x; i < n; i += kMetaThreads) {
        const int s = seq_ids[i];
        if (s < 0 || s >= m.S) bad = 1;
    }
    bad = -block_min(-bad, buf);
    if (bad) {
        if (threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = LF_EINVAL;
        return;
    }
    // Pass A: one decrement per occurrence; remember each page's first occurrence index.
    int carry = 0;
    for (int base = 0; base < n; base += kMetaThreads) {
        const int i = base + threadIdx.x;
        const int np = i < n ? pages_for(m.len[seq_ids[i]]) : 0;
        int round_total = 0;
        const int off = carry + block_excl_scan(np, &round_total, buf);
        if (i < n) {
            const long row = (long)seq_ids[i] * m.M;
            for (int j = 0; j < np; ++j) {
                const int p = m.bt[row + j];
                atomicSub(m.rc + p, 1);
                atomicMin(m.scratch + p, off + j);
            }
        }
        carry += round_total;
    }
    __threadfence();
    __syncthreads();
    // Pass B: pages at zero re-enter the queue tail at their first occurrence.
    const int head = m.ctrl[LF_CTRL_HEAD];
    const int count = m.ctrl[LF_CTRL_COUNT];
    int occ_carry = 0, freed_carry = 0;
    for (int base = 0; base < n; base += kMetaThreads) {
        const int i = base + threadIdx.x;
        const int np = i < n ? pages_for(m.len[seq_ids[i]]) : 0;
        int round_occ = 0;
        const int off = occ_carry + block_excl_scan(np, &round_occ, buf);
        int nfree = 0;
        const long row = i < n ? (long)seq_ids[i] * m.M : 0;
        for (int j = 0; j < np; ++j) {
            const int p = m.bt[row + j];
            if (__ldcg(m.rc + p) == 0 && __ldcg(m.scratch + p) == off + j) ++nfree;
        }
        int round_freed = 0;
        int pos = freed_carry + block_excl_scan(nfree, &round_freed, buf);
        for (int j = 0; j < np; ++j) {
            const int p = m.bt[row + j];
            if (__ldcg(m.rc + p) == 0 && __ldcg(m.scratch + p) == off + j) {
                m.fq[(int)(((long)head + count + pos) % m.P)] = p;
                ++pos;
            }
        }
        occ_carry += round_occ;
        freed_carry += round_freed;
    }
    __syncthreads();
    // Pass C: restore scratch, clear the rows.
    for (int base = 0; base < n; base += kMetaThreads) {
        const int i = base + threadIdx.x;
        if (i < n) {
            const long row = (long)seq_ids[i] * m.M;
            const int np = pages_for(m.len[seq_ids[i]]);
            for (int j = 0; j < np; ++j) {
                m.scratch[m.bt[row + j]] = INT_MAX;
                m.bt[row + j] = -1;
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kMetaThreads) m.len[seq_ids[i]] = 0;
    if (threadIdx.x == 0) m.ctrl[LF_CTRL_COUNT] = count + freed_carry;
}

__global__ void gather_kernel(Meta m, const int32_t* __restrict__ seq_ids, int n,
                              int32_t* __restrict__ out, int stride, int32_t* __restrict__ lens) {
    const int i = blockIdx.x;
    const int s = seq_ids[i];
    const bool ok = s >= 0 && s < m.S;
    for (int j = threadIdx.x; j < stride; j += blockDim.x)
        out[(long)i * stride + j] = (ok && j < m.M) ? m.bt[(long)s * m.M + j] : -1;
    if (threadIdx.x == 0 && lens) lens[i] = ok ? m.len[s] : 0;
}

__global__ void read_kernel(Meta m, int s, int layer, int start, int count,
                            const uint16_t* __restrict__ kp, const uint16_t* __restrict__ vp,
                            uint16_t* __restrict__ ko, uint16_t* __restrict__ vo, int Hkv, int D) {
    const int vecs = D / 8;
    const long total = (long)Hkv * count * vecs;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < total;
         idx += (long)gridDim.x * blockDim.x) {
        const int vec = (int)(idx % vecs);
        const int t = (int)((idx / vecs) % count);
        const int h = (int)(idx / ((long)vecs * count));
        const int pos = start + t;
        const int page = m.bt[(long)s * m.M + pos / LF_PAGE_SIZE];
        if (page < 0 || page >= m.P) {           // past the session's pages: zeros, as the dense pool
            *reinterpret_cast<uint4*>(ko + idx * 8) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vo + idx * 8) = make_uint4(0, 0, 0, 0);
            continue;
        }
        const long so = ((((long)layer * m.P + page) * Hkv + h) * LF_PAGE_SIZE + pos % LF_PAGE_SIZE) * D + vec * 8;
        *reinterpret_cast<uint4*>(ko + idx * 8) = *reinterpret_cast<const uint4*>(kp + so);
        *reinterpret_cast<uint4*>(vo + idx * 8) = *reinterpret_cast<const uint4*>(vp + so);
    }
}

}  // namespace pool
}  // namespace lf

using namespace lf;
using namespace lf::pool;

extern "C" int lf_pool_init(const lf_pool_meta* m, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    const Meta mm = to_meta(m);
    const long work = mm.P > (long)mm.S * mm.M ? (long)mm.P : (long)mm.S * mm.M;
    init_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(mm);
    return launch_status("pool init");
}

extern "C" int lf_pool_clear_status(const lf_pool_meta* m, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    clear_status_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(to_meta(m));
    return launch_status("pool clear_status");
}

extern "C" int lf_pool_reserve(const lf_pool_meta* m, const int32_t* seq_ids, const int32_t* n_new,
                               int n, int32_t* start_pos, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && (n == 0 || (seq_ids && n_new)), "pool reserve: bad arguments");
    if (n == 0) { clear_error(); return LF_OK; }
    reserve_kernel<<<1, kMetaThreads, 0, (cudaStream_t)stream>>>(to_meta(m), seq_ids, n_new, n, start_pos);
    return launch_status("pool reserve");
}

extern "C" int lf_pool_write_kv(const lf_pool_meta* m, const int32_t* seq_ids,
                                const int32_t* start_pos, const int32_t* cu_tokens, int n,
                                int total_tokens, const void* k_new, const void* v_new,
                                int64_t stride_layer, int64_t stride_token, int64_t stride_head,
                                void* k_pages, void* v_pages, int num_layers, int num_kv_heads,
                                int head_dim, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && total_tokens >= 0, "pool write: negative sizes");
    if (n == 0 || total_tokens == 0) { clear_error(); return LF_OK; }
    LF_CHECK_ARG(seq_ids && start_pos && cu_tokens && k_new && v_new && k_pages && v_pages,
                 "pool write: null pointer argument");
    LF_CHECK_ARG(head_dim % 8 == 0 && num_layers > 0 && num_kv_heads > 0, "pool write: bad shape");
    LF_CHECK_ARG(aligned16(k_new) && aligned16(v_new) && aligned16(k_pages) && aligned16(v_pages) &&
                     stride_layer % 8 == 0 && stride_token % 8 == 0 && stride_head % 8 == 0,
                 "pool write: rows must be 16-byte aligned");
    LF_CHECK_ARG(num_layers <= 65535, "pool write: too many layers");
    const long work = (long)total_tokens * num_kv_heads * (head_dim / 8);
    dim3 grid(grid_for(work, 256), num_layers);
    write_kv_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        to_meta(m), seq_ids, start_pos, cu_tokens, n, total_tokens,
        static_cast<const uint16_t*>(k_new), static_cast<const uint16_t*>(v_new), stride_layer,
        stride_token, stride_head, static_cast<uint16_t*>(k_pages), static_cast<uint16_t*>(v_pages),
        num_kv_heads, head_dim);
    return launch_status("pool write_kv");
}

extern "C" int lf_pool_fork(const lf_pool_meta* m, int src_seq, const int32_t* dst_seqs, int n,
                            int prefix_len, void* k_pages, void* v_pages, int num_layers,
                            int num_kv_heads, int head_dim, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && (n == 0 || dst_seqs), "pool fork: bad arguments");
    if (n == 0) { clear_error(); return LF_OK; }
    cudaStream_t st = (cudaStream_t)stream;
    const Meta mm = to_meta(m);
    fork_kernel<<<1, kMetaThreads, 0, st>>>(mm, src_seq, dst_seqs, n, prefix_len);
    rc = launch_status("pool fork");
    if (rc) return rc;
    const int part = prefix_len % LF_PAGE_SIZE;
    if (part && k_pages && v_pages && num_layers > 0) {
        LF_CHECK_ARG(head_dim % 8 == 0 && aligned16(k_pages) && aligned16(v_pages) && n <= 2147483647 &&
                         num_layers <= 65535,
                     "pool fork: bad data arguments");
        fork_copy_kernel<<<dim3(n, num_layers), 256, 0, st>>>(mm, src_seq, dst_seqs,
                                                               prefix_len / LF_PAGE_SIZE, part,
                                                               static_cast<uint16_t*>(k_pages),
                                                               static_cast<uint16_t*>(v_pages),
                                                               num_kv_heads, head_dim);
        return launch_status("pool fork copy");
    }
    return LF_OK;
}

extern "C" int lf_pool_free(const lf_pool_meta* m, const int32_t* seq_ids, int n, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && (n == 0 || seq_ids), "pool free: bad arguments");
    if (n == 0) { clear_error(); return LF_OK; }
    free_kernel<<<1, kMetaThreads, 0, (cudaStream_t)stream>>>(to_meta(m), seq_ids, n);
    return launch_status("pool free");
}

extern "C" int lf_pool_gather(const lf_pool_meta* m, const int32_t* seq_ids, int n,
                              int32_t* out_table, int out_stride, int32_t* out_lens, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(n >= 0 && out_stride > 0 && (n == 0 || (seq_ids && out_table)),
                 "pool gather: bad arguments");
    if (n == 0) { clear_error(); return LF_OK; }
    gather_kernel<<<n, 128, 0, (cudaStream_t)stream>>>(to_meta(m), seq_ids, n, out_table, out_stride,
                                                       out_lens);
    return launch_status("pool gather");
}

extern "C" int lf_pool_read(const lf_pool_meta* m, int seq, int layer, int start, int end,
                            const void* k_pages, const void* v_pages, void* k_out, void* v_out,
                            int num_layers, int num_kv_heads, int head_dim, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    LF_CHECK_ARG(seq >= 0 && seq < m->max_seqs && layer >= 0 && layer < num_layers && start >= 0 &&
                     end >= start && end <= m->max_pages_per_seq * LF_PAGE_SIZE,
                 "pool read: bad range");
    LF_CHECK_ARG(k_pages && v_pages && k_out && v_out && head_dim % 8 == 0 && aligned16(k_out) &&
                     aligned16(v_out) && aligned16(k_pages) && aligned16(v_pages),
                 "pool read: bad buffers");
    if (end == start) { clear_error(); return LF_OK; }
    const long work = (long)num_kv_heads * (end - start) * (head_dim / 8);
    read_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(
        to_meta(m), seq, layer, start, end - start, static_cast<const uint16_t*>(k_pages),
        static_cast<const uint16_t*>(v_pages), static_cast<uint16_t*>(k_out),
        static_cast<uint16_t*>(v_out), num_kv_heads, head_dim);
    return launch_status("pool read");
}
