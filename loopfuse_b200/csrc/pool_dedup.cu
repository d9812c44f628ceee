// Prefix-hash dedup of the paged pool: sessions whose leading token pages are identical share
// the pages by content, found through a device hash registry.
//
// The reference's only KV fusion is a compile-time pass keyed on IR positions
// (passes/kv_fusion.py:80-107) over a pool without sharing (runtime/kv_pool.py:28-235); this is
// the runtime, content-addressed form of it.  A full page is named by a chained hash:
//   local_j = FNV-1a-64 over the little-endian bytes of its 16 int32 token ids  (parallel),
//   h_j     = fmix64(h_{j-1} ^ local_j), h_{-1} = 0, 0 mapped to 1               (serial, cheap)
// (FNV-1a: Fowler-Noll-Vo; fmix64: MurmurHash3's 64-bit finaliser).  The registry is an
// open-addressing table with linear probing, key 0 meaning empty, kept at most half full so
// every probe sequence ends at an empty slot; it holds one refcount on each registered page.
// Order rules shared with the pool oracle: register is all or nothing against the half-full
// limit; dedup validates every destination before any is touched; unregister returns the
// pages reaching refcount 0 to the queue tail in ascending page-id order.
#include "pool_common.cuh"

namespace lf {
namespace pool {

constexpr unsigned long long kFnvOffset = 0xCBF29CE484222325ull;
constexpr unsigned long long kFnvPrime = 0x100000001B3ull;

struct Reg {
    unsigned long long* keys;
    int32_t* pages;
    int32_t* used;
    int cap;
};

static Reg to_reg(const lf_prefix_registry* r) {
    return Reg{r->keys, r->pages, r->used, r->capacity};
}

__device__ __forceinline__ unsigned long long fmix64(unsigned long long h) {
    h ^= h >> 33;
    h *= 0xFF51AFD7ED558CCDull;
    h ^= h >> 33;
    h *= 0xC4CEB9FE1A85EC53ull;
    h ^= h >> 33;
    return h;
}

__device__ __forceinline__ unsigned long long local_hash(const int32_t* tok) {
    unsigned long long h = kFnvOffset;
#pragma unroll
    for (int t = 0; t < LF_PAGE_SIZE; ++t) {
        const uint32_t v = static_cast<uint32_t>(tok[t]);
#pragma unroll
        for (int b = 0; b < 4; ++b) h = (h ^ ((v >> (8 * b)) & 0xFFu)) * kFnvPrime;
    }
    return h;
}

// Chained hashes of the first `np` (<= LF_MAX_DEDUP_PAGES) pages of `tok` into sh[0, np).
// Called by every thread of the block.
__device__ void block_page_hashes(const int32_t* tok, int np, unsigned long long* sh) {
    for (int j = threadIdx.x; j < np; j += blockDim.x) sh[j] = local_hash(tok + (long)j * LF_PAGE_SIZE);
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long h = 0;
        for (int j = 0; j < np; ++j) {
            h = fmix64(h ^ sh[j]);
            if (h == 0) h = 1;
            sh[j] = h;
        }
    }
    __syncthreads();
}

__device__ int reg_find(const Reg& r, unsigned long long h) {
    const unsigned mask = static_cast<unsigned>(r.cap) - 1u;
    unsigned i = static_cast<unsigned>(h) & mask;
    for (int probe = 0; probe < r.cap; ++probe) {
        const unsigned long long k = r.keys[i];
        if (k == h) return r.pages[i];
        if (k == 0) return -1;
        i = (i + 1u) & mask;
    }
    return -1;
}

// True if this call added the key (false: already present, or no empty slot).
__device__ bool reg_insert(const Reg& r, unsigned long long h, int page) {
    const unsigned mask = static_cast<unsigned>(r.cap) - 1u;
    unsigned i = static_cast<unsigned>(h) & mask;
    for (int probe = 0; probe < r.cap; ++probe) {
        const unsigned long long prev = atomicCAS(r.keys + i, 0ull, h);
        if (prev == 0) {
            r.pages[i] = page;
            return true;
        }
        if (prev == h) return false;
        i = (i + 1u) & mask;
    }
    return false;
}

__global__ void registry_init_kernel(Reg r) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < r.cap; i += (long)gridDim.x * blockDim.x) {
        r.keys[i] = 0;
        r.pages[i] = -1;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *r.used = 0;
}

__global__ void __launch_bounds__(kMetaThreads)
hashes_kernel(const int32_t* __restrict__ tokens, int np, unsigned long long* __restrict__ out) {
    __shared__ unsigned long long sh[LF_MAX_DEDUP_PAGES];
    block_page_hashes(tokens, np, sh);
    for (int j = threadIdx.x; j < np; j += blockDim.x) out[j] = sh[j];
}

__global__ void __launch_bounds__(kMetaThreads)
register_kernel(Meta m, Reg r, int seq, const int32_t* __restrict__ tokens, int n_tokens,
                int32_t* __restrict__ added) {
    __shared__ unsigned long long sh[LF_MAX_DEDUP_PAGES];
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    if (seq < 0 || seq >= m.S) {
        if (threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = LF_EINVAL;
        return;
    }
    const int np = min(min(n_tokens, m.len[seq]) / LF_PAGE_SIZE, min(m.M, LF_MAX_DEDUP_PAGES));
    block_page_hashes(tokens, np, sh);
    int missing = 0;
    for (int j = threadIdx.x; j < np; j += kMetaThreads) missing += reg_find(r, sh[j]) < 0;
    int total = 0;
    block_excl_scan(missing, &total, buf);
    const int used = *r.used;
    if (used + total > r.cap / 2) {
        if (threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = LF_ENOPAGES;
        return;
    }
    int mine = 0;
    const long row = (long)seq * m.M;
    for (int j = threadIdx.x; j < np; j += kMetaThreads) {
        const int page = m.bt[row + j];
        if (reg_insert(r, sh[j], page)) {
            atomicAdd(m.rc + page, 1);
            ++mine;
        }
    }
    int n_added = 0;
    block_excl_scan(mine, &n_added, buf);
    if (threadIdx.x == 0) {
        *r.used = used + n_added;
        if (added) *added = n_added;
    }
}

__global__ void __launch_bounds__(kMetaThreads)
dedup_check_kernel(Meta m, const int32_t* __restrict__ seq_ids, int n) {
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    int bad = 0;
    for (int i = threadIdx.x; i < n; i += kMetaThreads) {
        const int s = seq_ids[i];
        if (s < 0 || s >= m.S || m.len[s] != 0) {
            bad = 1;
            continue;
        }
        for (int k = i + 1; k < n; ++k) bad |= seq_ids[k] == s;
    }
    bad = -block_min(-bad, buf);
    if (bad && threadIdx.x == 0) m.ctrl[LF_CTRL_STATUS] = LF_EINVAL;
}

// One CTA per destination session.
__global__ void __launch_bounds__(kMetaThreads)
dedup_kernel(Meta m, Reg r, const int32_t* __restrict__ seq_ids, const int32_t* __restrict__ tokens,
             const int32_t* __restrict__ cu_tokens, int32_t* __restrict__ covered) {
    __shared__ unsigned long long sh[LF_MAX_DEDUP_PAGES];
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    const int i = blockIdx.x;
    const int s = seq_ids[i];
    const int t0 = cu_tokens[i];
    const int nt = max(cu_tokens[i + 1] - t0, 0);
    const int np = min(nt / LF_PAGE_SIZE, min(m.M, LF_MAX_DEDUP_PAGES));
    block_page_hashes(tokens + t0, np, sh);
    int first_miss = INT_MAX;
    for (int j = threadIdx.x; j < np; j += kMetaThreads) {
        const int page = reg_find(r, sh[j]);
        if (page < 0 || page >= m.P) first_miss = min(first_miss, j);
        sh[j] = static_cast<unsigned long long>(static_cast<long long>(page));
    }
    const int n_shared = min(block_min(first_miss, buf), np);
    const long row = (long)s * m.M;
    for (int j = threadIdx.x; j < n_shared; j += kMetaThreads) {
        const int page = static_cast<int>(static_cast<long long>(sh[j]));
        m.bt[row + j] = page;
        atomicAdd(m.rc + page, 1);
    }
    if (threadIdx.x == 0) {
        m.len[s] = n_shared * LF_PAGE_SIZE;
        if (covered) covered[i] = n_shared * LF_PAGE_SIZE;
    }
}

__global__ void __launch_bounds__(kMetaThreads) unregister_kernel(Meta m, Reg r) {
    __shared__ int buf[32];
    if (status_of(m) != LF_OK) return;
    for (int i = threadIdx.x; i < r.cap; i += kMetaThreads) {
        if (r.keys[i] == 0) continue;
        const int p = r.pages[i];
        if (static_cast<unsigned>(p) < static_cast<unsigned>(m.P) && atomicSub(m.rc + p, 1) == 1)
            m.scratch[p] = 0;                        // mark: reached zero (scratch rests at INT_MAX)
        r.keys[i] = 0;
        r.pages[i] = -1;
    }
    __threadfence();
    __syncthreads();
    const int head = m.ctrl[LF_CTRL_HEAD];
    const int count = m.ctrl[LF_CTRL_COUNT];
    int carry = 0;
    for (int base = 0; base < m.P; base += kMetaThreads) {
        const int p = base + threadIdx.x;
        const int flag = (p < m.P && __ldcg(m.scratch + p) == 0) ? 1 : 0;
        int round_total = 0;
        const int pos = carry + block_excl_scan(flag, &round_total, buf);
        if (flag) {
            m.fq[(int)(((long)head + count + pos) % m.P)] = p;
            m.scratch[p] = INT_MAX;
        }
        carry += round_total;
    }
    if (threadIdx.x == 0) {
        m.ctrl[LF_CTRL_COUNT] = count + carry;
        *r.used = 0;
    }
}

static int check_reg(const lf_prefix_registry* r) {
    LF_CHECK_ARG(r != nullptr && r->keys && r->pages && r->used, "registry: null pointer");
    LF_CHECK_ARG(r->capacity >= 2 && r->capacity <= (1 << 30) && (r->capacity & (r->capacity - 1)) == 0,
                 "registry: capacity must be a power of two in [2, 2^30] (got %d)", r->capacity);
    return LF_OK;
}

}  // namespace pool
}  // namespace lf

using namespace lf;
using namespace lf::pool;

extern "C" int lf_registry_init(const lf_prefix_registry* r, void* stream) {
    int rc = check_reg(r);
    if (rc) return rc;
    registry_init_kernel<<<grid_for(r->capacity, 256), 256, 0, (cudaStream_t)stream>>>(to_reg(r));
    return launch_status("registry init");
}

extern "C" int lf_prefix_hashes(const int32_t* tokens, int n_tokens, unsigned long long* out,
                                void* stream) {
    LF_CHECK_ARG(n_tokens >= 0, "prefix hashes: negative length");
    const int np = n_tokens / LF_PAGE_SIZE < LF_MAX_DEDUP_PAGES ? n_tokens / LF_PAGE_SIZE : LF_MAX_DEDUP_PAGES;
    if (np == 0) { clear_error(); return LF_OK; }
    LF_CHECK_ARG(tokens && out, "prefix hashes: null pointer");
    hashes_kernel<<<1, kMetaThreads, 0, (cudaStream_t)stream>>>(tokens, np, out);
    return launch_status("prefix hashes");
}

extern "C" int lf_pool_register_prefix(const lf_pool_meta* m, const lf_prefix_registry* r, int seq,
                                       const int32_t* tokens, int n_tokens, int32_t* added,
                                       void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    if ((rc = check_reg(r))) return rc;
    LF_CHECK_ARG(n_tokens >= 0 && (n_tokens < LF_PAGE_SIZE || tokens), "register: bad tokens");
    register_kernel<<<1, kMetaThreads, 0, (cudaStream_t)stream>>>(to_meta(m), to_reg(r), seq, tokens,
                                                                   n_tokens, added);
    return launch_status("pool register_prefix");
}

extern "C" int lf_pool_dedup_prefix(const lf_pool_meta* m, const lf_prefix_registry* r,
                                    const int32_t* seq_ids, const int32_t* tokens,
                                    const int32_t* cu_tokens, int n, int32_t* covered, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    if ((rc = check_reg(r))) return rc;
    LF_CHECK_ARG(n >= 0 && (n == 0 || (seq_ids && cu_tokens)), "dedup: bad arguments");
    if (n == 0) { clear_error(); return LF_OK; }
    cudaStream_t st = (cudaStream_t)stream;
    const Meta mm = to_meta(m);
    dedup_check_kernel<<<1, kMetaThreads, 0, st>>>(mm, seq_ids, n);
    if ((rc = launch_status("pool dedup check"))) return rc;
    dedup_kernel<<<n, kMetaThreads, 0, st>>>(mm, to_reg(r), seq_ids, tokens, cu_tokens, covered);
    return launch_status("pool dedup_prefix");
}

extern "C" int lf_pool_unregister_all(const lf_pool_meta* m, const lf_prefix_registry* r, void* stream) {
    int rc = check_meta(m);
    if (rc) return rc;
    if ((rc = check_reg(r))) return rc;
    unregister_kernel<<<1, kMetaThreads, 0, (cudaStream_t)stream>>>(to_meta(m), to_reg(r));
    return launch_status("pool unregister_all");
}
