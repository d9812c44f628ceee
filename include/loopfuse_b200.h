/*
 * loopfuse_b200.h -- C ABI of the sm_100a attention hot path.
 *
 * One shared library, liblf_sm100.so, exports these symbols.  Signatures use
 * plain pointers and sizes only: every device buffer is allocated by the caller
 * (PyTorch's caching allocator in the Python host layer) and passed as a raw
 * device pointer; `stream` is a cudaStream_t passed as void*.  Every call is
 * asynchronous on that stream and returns a status code (LF_OK == 0) after
 * validating its arguments on the host; lf_last_error() gives the message.
 *
 * Element types: K/V/Q/O are bf16 bit patterns (uint16_t).  Pool data copies
 * (write / fork) move raw 2-byte elements and also serve fp16 pools.
 *
 * Reference interfaces replaced (paths inside the loopfuse repository):
 *   prefill   kernels/triton/prefill_attn.py:127-168  prefill_attention_fwd
 *             kernels/cuda/async_prefill.cu:56-236     agent_prefill_kernel,
 *                                                      loopfuse_agent_prefill
 *   decode    kernels/triton/decode_attn.py:133-171    decode_attention_fwd
 *             kernels/cuda/ring_kv_cache.cu:120-248    ring_kv_decode_kernel
 *   pool      runtime/kv_pool.py:103-198               KVPool.allocate_slot/
 *                                                      write/release/read
 *             kernels/cuda/ring_kv_cache.cu:69-109,282-297 ring_kv_write
 *             kernels/cuda/_cuda_ext.py:60-116          ring_kv_write /
 *                                                      async_zero_slot bindings
 */
#ifndef LOOPFUSE_B200_H
#define LOOPFUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define LF_OK        0
#define LF_EINVAL    1   /* bad shape, pointer, alignment or argument        */
#define LF_ENOPAGES  2   /* pool has fewer free pages than requested         */
#define LF_EOVERFLOW 3   /* a session would exceed max_pages_per_seq         */
#define LF_ETIMEOUT  4   /* a bounded device-side wait gave up               */
#define LF_ECUDA     5   /* a CUDA runtime call failed                       */

#define LF_PAGE_SIZE 16  /* tokens per KV page */

typedef uint16_t lf_bf16;

/* Library version string and the message of the last failing call on this
 * host thread (empty when the last call succeeded). */
const char* lf_version(void);
const char* lf_last_error(void);

/* Reads and clears the library's device-side error report (synchronous).  A
 * kernel whose bounded wait gave up (a pipeline barrier that never completed)
 * or that met a bad page id records a non-zero site code instead of hanging or
 * faulting; *out == 0 means no kernel has reported a failure since the last
 * call.  Each source file of the library keeps its own error word: one call
 * returns and clears one report, so a caller that wants them all calls until
 * *out == 0.  No reference counterpart: the reference kernels have no
 * device-side error reporting. */
int lf_device_status(int* out);

/* Runs, on the given stream, the bounded barrier wait that every pipelined kernel here uses,
 * on a barrier that nothing arrives at, giving up after timeout_us (1..100000).  The expiry is
 * recorded in the device error word exactly like a kernel's (site code 177), so a caller can
 * check the failure path: lf_device_status() then reports it, and the context stays usable.
 * No reference counterpart (diagnostic). */
int lf_selftest_bounded_wait(unsigned timeout_us, void* stream);

/* ---- prefill attention --------------------------------------------------
 * Replaces prefill_attention_fwd (kernels/triton/prefill_attn.py:127-168) and
 * the host launcher loopfuse_agent_prefill (kernels/cuda/async_prefill.cu:220-236).
 *
 * o = softmax(scale * q k^T + mask) v for q [B,Hq,Sq,D], k/v [B,Hkv,Sk,D],
 * o [B,Hq,Sq,D]; query head h reads KV head h / (Hq/Hkv).  causal != 0 masks
 * key j for query i when j > i + (Sk - Sq) (the reference's q >= k mask when
 * Sq == Sk, prefill_attn.py:97-99).  lse [B,Hq,Sq] (nullable) receives the
 * natural-log log-sum-exp of each row.  D must be 128 or 64; all pointers
 * 16-byte aligned.  tcgen05 MMA with TMEM accumulators, TMA-loaded tiles. */
int lf_prefill_fwd(const lf_bf16* q, const lf_bf16* k, const lf_bf16* v, lf_bf16* o,
                   float* lse, int batch, int num_q_heads, int num_kv_heads, int seq_q,
                   int seq_k, int head_dim, float scale, int causal, void* stream);

/* Prefill over cached paged context (tool-output appends).  Extends the same
 * reference entry points to queries appended after a session's cached KV:
 * q [total_q, Hq, D] holds the new tokens of num_seqs sessions back to back
 * (session n owns rows cu_seqlens_q[n] .. cu_seqlens_q[n+1]-1, at most
 * max_seqlen_q of them); its keys and values are the first seqlens_k[n] tokens
 * of its block-table row in the pool pages [P, Hkv, 16, D] (the new tokens
 * already written).  causal != 0 puts query i of session n at key position
 * seqlens_k[n] - (its query count) + i.  o [total_q, Hq, D]; lse [total_q, Hq]
 * (nullable).  The reference's causal mask assumes seq_q == seq_k
 * (kernels/triton/prefill_attn.py:98) and has no cached-prefix prefill. */
int lf_prefill_paged_fwd(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                         const int32_t* block_table, const int32_t* cu_seqlens_q,
                         const int32_t* seqlens_k, lf_bf16* o, float* lse, int num_seqs,
                         int total_q, int max_seqlen_q, int num_q_heads, int num_kv_heads,
                         int head_dim, int num_pages, int max_pages, float scale, int causal,
                         void* stream);

/* ---- paged split-KV decode ----------------------------------------------
 * Replaces decode_attention_fwd (kernels/triton/decode_attn.py:133-171) and
 * ring_kv_decode_kernel (kernels/cuda/ring_kv_cache.cu:120-248).
 *
 * One query token per session: q [N,Hq,D]; K/V pages [P,Hkv,16,D];
 * block_table [N,max_pages] int32 page ids in token order; seq_lens [N] >= 1;
 * o [N,Hq,D]; lse [N,Hq] (nullable, natural log).  Each session's pages are
 * split into chunks of pages_per_split pages, processed by independent CTAs
 * (GQA group of Hq/Hkv heads per CTA, pages staged by TMA, warp-level
 * tensor-core MMA) and merged by log-sum-exp.  num_prefix_pages > 0 says
 * the first num_prefix_pages block-table entries are the same pages for every
 * session (a forked shared prefix): they are read once per group of sessions
 * instead of once per session.  workspace holds the split partials; its size
 * comes from lf_decode_workspace_size.  D must be 128 (or 64).  A length
 * past max_pages*16 is clamped and a page id outside [0, num_pages) is
 * replaced by page 0; either is reported through lf_device_status(). */
int lf_decode_workspace_size(int num_seqs, int num_q_heads, int head_dim, int max_pages,
                             int pages_per_split, int num_prefix_pages, size_t* bytes);

/* Default pages_per_split for lf_decode_fwd: enough split CTAs for several waves
 * on sm_count SMs (sm_count <= 0: the current device's count), with sessions
 * taken to be half full, 32 to 128 pages per split.  Host-only when sm_count >
 * 0.  The reference's decode has no split (one program per (batch, head),
 * kernels/triton/decode_attn.py:159-171); this is the grid choice that
 * replaces it. */
int lf_decode_default_split(int num_seqs, int num_kv_heads, int max_pages, int num_prefix_pages,
                            int sm_count, int* pages_per_split);
int lf_decode_fwd(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                  const int32_t* block_table, const int32_t* seq_lens, int num_prefix_pages,
                  lf_bf16* o, float* lse, void* workspace, size_t workspace_bytes,
                  int num_seqs, int num_q_heads, int num_kv_heads, int head_dim,
                  int num_pages, int max_pages, int pages_per_split, float scale,
                  void* stream);

/* lf_decode_fwd with the K/V append fused in: replaces ring_kv_write_kernel followed by the
 * decode (kernels/cuda/ring_kv_cache.cu:69-109, then :120-248).  k_new, v_new [N,Hkv,D] are
 * each session's newest token, at position seq_lens[n] - 1, whose page the caller has already
 * reserved in block_table (past the num_prefix_pages shared pages, in a page of the session's
 * own).  The split CTA that holds that page stores the token's rows into k_pages / v_pages
 * before loading the page, so the pages are written and the launch sequence is one kernel
 * shorter than a separate append.  Pages afterwards hold what lf_pool_write_kv would have
 * written.  A page id of the newest token outside [0, num_pages) stores nothing and is
 * reported through lf_device_status(). */
int lf_decode_fwd_append(const lf_bf16* q, lf_bf16* k_pages, lf_bf16* v_pages,
                         const int32_t* block_table, const int32_t* seq_lens, int num_prefix_pages,
                         const lf_bf16* k_new, const lf_bf16* v_new, lf_bf16* o, float* lse,
                         void* workspace, size_t workspace_bytes, int num_seqs, int num_q_heads,
                         int num_kv_heads, int head_dim, int num_pages, int max_pages,
                         int pages_per_split, float scale, void* stream);

/* Head-tensor-parallel decode with the all-gather of the outputs fused into the combine
 * step (the reference has no multi-GPU path).  This rank holds num_kv_heads of the model's KV
 * heads and computes num_q_heads query heads (all arguments as in lf_decode_fwd for that
 * slice); each finished row (n, h) is stored into every one of the n_peers outputs
 * out_peers[k] ([num_seqs][num_q_heads_total][head_dim] bf16, one per rank, this rank's
 * included) at head head_offset + h, with peer-memory stores, followed by a system-scope
 * fence.  out_peers is a DEVICE array of pointers (from lf_ipc_import).  The caller orders
 * readers after every rank's call (e.g. a collective on the same stream). */
int lf_decode_fwd_gather(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                         const int32_t* block_table, const int32_t* seq_lens,
                         int num_prefix_pages, lf_bf16* const* out_peers, int n_peers,
                         int head_offset, int num_q_heads_total, float* lse, void* workspace,
                         size_t workspace_bytes, int num_seqs, int num_q_heads, int num_kv_heads,
                         int head_dim, int num_pages, int max_pages, int pages_per_split,
                         float scale, void* stream);

/* Cross-process sharing of one device buffer within a node (no reference counterpart):
 * lf_ipc_export writes the 64-byte IPC handle of the allocation holding `ptr` and ptr's
 * offset inside it; lf_ipc_import opens a handle from another process (peer access enabled
 * on demand) and returns that allocation's base in this process; lf_ipc_close unmaps it. */
int lf_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
int lf_ipc_import(const void* handle, void** base_out);
int lf_ipc_close(void* base);

/* Decode without any device allocation.  Same computation as lf_decode_fwd,
 * but the split partials live in a fixed array inside the library
 * (LF_DECODE_NOALLOC_SCRATCH_BYTES on every GPU that loads it, held until
 * exit), so callers that cannot allocate device memory -- a foreign-language
 * binding without a device allocator, or a loop whose allocator has reserved
 * nearly all of HBM for the KV pool -- need pass only inputs and outputs.
 * No counterpart in the reference.  The split size starts from
 * lf_decode_default_split and doubles until the partials fit the array; a
 * request that does not fit even with one split per session returns
 * LF_EINVAL.  The first call in a CUDA context looks up the array's device
 * address (with that context's device current) and keeps it for that
 * context, so make the first call before any stream capture.  Calls share the
 * array: calls whose kernels overlap on the GPU race and must be serialised
 * by the caller. */
#define LF_DECODE_NOALLOC_SCRATCH_BYTES (32u << 20)
int lf_decode_fwd_noalloc(const lf_bf16* q, const lf_bf16* k_pages, const lf_bf16* v_pages,
                          const int32_t* block_table, const int32_t* seq_lens,
                          int num_prefix_pages, lf_bf16* o, float* lse, int num_seqs,
                          int num_q_heads, int num_kv_heads, int head_dim, int num_pages,
                          int max_pages, float scale, void* stream);

/* Instrumentation for timing the dominant decode kernel: while both events
 * are non-null, every lf_decode_fwd records ev_begin right before and ev_end
 * right after its per-session split kernel, on the call's stream (events are
 * cudaEvent_t passed as void*).  Pass two nulls to stop.  No work is skipped
 * or changed.  No reference counterpart (the reference has no decode launch
 * to time). */
int lf_decode_set_profile_events(void* ev_begin, void* ev_end);

/* ---- paged KV pool --------------------------------------------------------
 * Device-resident metadata of a paged, refcounted KV pool.  Replaces the
 * dense slot pool of runtime/kv_pool.py:28-235 (allocate_slot :103, release
 * :117, write :123, read :151) and the ring-buffer write of
 * kernels/cuda/ring_kv_cache.cu:69-109.  All arrays are device memory owned
 * by the caller.  Semantics (FIFO free queue, all-or-nothing allocation,
 * refcounted sharing, free order) are specified by the pool oracle and
 * reproduced bit for bit.
 *
 * Errors found on the device (ENOPAGES, EOVERFLOW) are written to
 * ctrl[LF_CTRL_STATUS]; the status is sticky: every later pool call is a no-op
 * until lf_pool_clear_status.  Reading it is the caller's one host sync. */
#define LF_CTRL_HEAD   0   /* queue index of the first free page           */
#define LF_CTRL_COUNT  1   /* number of free pages                         */
#define LF_CTRL_STATUS 2   /* sticky device status (LF_OK when fine)       */
#define LF_CTRL_WORDS  8

typedef struct lf_pool_meta {
    int32_t* free_queue;    /* [num_pages] ring of free page ids             */
    int32_t* refcount;      /* [num_pages]                                   */
    int32_t* block_table;   /* [max_seqs * max_pages_per_seq], -1 = no page  */
    int32_t* seq_len;       /* [max_seqs] tokens held per session            */
    int32_t* ctrl;          /* [LF_CTRL_WORDS]                               */
    int32_t* scratch;       /* [num_pages] kept at INT32_MAX between calls   */
    int32_t num_pages;
    int32_t max_seqs;
    int32_t max_pages_per_seq;
    int32_t page_size;      /* must be LF_PAGE_SIZE                          */
} lf_pool_meta;

/* Reset to: queue 0..P-1, refcounts 0, tables -1, lengths 0, status OK. */
int lf_pool_init(const lf_pool_meta* m, void* stream);
int lf_pool_clear_status(const lf_pool_meta* m, void* stream);

/* Allocation step of append: session seq_ids[i] grows by n_new[i] tokens,
 * taking ceil-page deltas from the queue head in order; start_pos[i] receives
 * its old length.  All or nothing.  A session that grows (n_new > 0) must
 * appear once; zero-count entries (padding rows) may repeat.  A conflicting
 * entry is rejected with LF_EINVAL in the sticky status (nothing changes). */
int lf_pool_reserve(const lf_pool_meta* m, const int32_t* seq_ids, const int32_t* n_new, int n,
                    int32_t* start_pos, void* stream);

/* Data step of append: token t of session i (rows cu_tokens[i] ..
 * cu_tokens[i+1]-1 of k_new/v_new) goes to position start_pos[i] + t.
 * k_new element (layer l, token t, head h, dim d) is at
 * l*stride_layer + t*stride_token + h*stride_head + d (elements).  Pages are
 * [num_layers][num_pages][Hkv][16][D].  A row whose position has no reserved
 * page (or an out-of-range session id) is not stored and sets the sticky
 * status to LF_EINVAL; the other rows are stored. */
int lf_pool_write_kv(const lf_pool_meta* m, const int32_t* seq_ids, const int32_t* start_pos,
                     const int32_t* cu_tokens, int n, int total_tokens, const void* k_new,
                     const void* v_new,
                     int64_t stride_layer, int64_t stride_token, int64_t stride_head,
                     void* k_pages, void* v_pages, int num_layers, int num_kv_heads,
                     int head_dim, void* stream);

/* Share src's first prefix_len tokens with each (empty) dst: full pages by
 * reference (refcount += 1 each), a partial last page copied into a fresh
 * page per destination. */
int lf_pool_fork(const lf_pool_meta* m, int src_seq, const int32_t* dst_seqs, int n,
                 int prefix_len, void* k_pages, void* v_pages, int num_layers,
                 int num_kv_heads, int head_dim, void* stream);

/* Release sessions: refcount -1 per page occurrence; pages reaching zero go to
 * the queue tail in first-occurrence order; rows reset. */
int lf_pool_free(const lf_pool_meta* m, const int32_t* seq_ids, int n, void* stream);

/* Batch block table: out_table[i*out_stride + j] = table row of seq_ids[i]
 * (j < out_stride), out_lens[i] = its length. */
int lf_pool_gather(const lf_pool_meta* m, const int32_t* seq_ids, int n, int32_t* out_table,
                   int out_stride, int32_t* out_lens, void* stream);

/* Copy one session's tokens [start, end) of one layer out of the pages into
 * dense k_out/v_out [Hkv][end-start][D] (the reference's read(), :151-165). */
int lf_pool_read(const lf_pool_meta* m, int seq, int layer, int start, int end,
                 const void* k_pages, const void* v_pages, void* k_out, void* v_out,
                 int num_layers, int num_kv_heads, int head_dim, void* stream);

/* Fused QKV epilogue of one layer (replaces kernels/cuda/ring_kv_cache.cu:69-109
 * ring_kv_write_kernel plus the model's split / rotate / copy steps).  `qkv` is the QKV
 * projection output, [total_tokens] rows of `qkv_row_stride` bf16 elements, each row q heads
 * (num_q_heads x head_dim), then k heads, then v heads (num_kv_heads x head_dim each); sessions
 * back to back as in lf_pool_write_kv (seq_ids, start_pos from lf_pool_reserve, cu_tokens).
 * q and k are rotated ("rotate half" RoPE, out[i] = x[i]c - x[i+D/2]s, out[i+D/2] =
 * x[i+D/2]c + x[i]s, fp32 without FMA contraction, rounded to bf16) with c, s =
 * rope_cos/rope_sin[pos][i] from [rope_rows][head_dim/2] fp32 tables, pos = the token's
 * position in its session; NULL tables skip the rotation.  q goes to q_out [total_tokens,
 * num_q_heads, head_dim]; k and v go to this layer's pages (k_pages, v_pages: [P, Hkv, 16, D]).
 * head_dim a multiple of 16; all buffers 16-byte aligned.  A position past the table or a
 * missing page sets the pool's sticky status to LF_EINVAL. */
int lf_pool_write_qkv(const lf_pool_meta* m, const int32_t* seq_ids, const int32_t* start_pos,
                      const int32_t* cu_tokens, int n, int total_tokens, const void* qkv,
                      int64_t qkv_row_stride, const float* rope_cos, const float* rope_sin,
                      int rope_rows, void* q_out, void* k_pages, void* v_pages, int num_q_heads,
                      int num_kv_heads, int head_dim, void* stream);

/* ---- decoder elementwise ops around the attention path ---------------------------------
 * Residual add + RMSNorm, one CTA per row (the norm half of kernels/triton/fused_ln_qkv.py:27-72,
 * whose LayerNorm stays in registers ahead of the QKV product; here the norm is RMSNorm and the
 * residual add is fused in instead).  For each of `rows` contiguous rows of `dim` bf16:
 * if delta != NULL, x = bf16(x + delta) in place; then if w != NULL,
 * out = bf16(bf16(x * r) * w) with r = 1 / sqrt(mean(x^2) + eps).  dim a multiple of 8, at most
 * 8192; buffers 16-byte aligned. */
int lf_add_rmsnorm(lf_bf16* x, const lf_bf16* delta, const lf_bf16* w, lf_bf16* out, int rows,
                   int dim, float eps, void* stream);

/* SwiGLU gate of a fused gate|up projection gu [rows, 2*ffn] bf16:
 * out[r][j] = bf16(bf16(silu(gu[r][j])) * gu[r][ffn + j]), out [rows, ffn].  No reference
 * counterpart (the reference models are GPT-style). */
int lf_swiglu(const lf_bf16* gu, lf_bf16* out, int rows, int ffn, void* stream);

/* Decode-batch projection y[M, N] = x[M, K] . w[K, N] (bf16 in and out, fp32 accumulation),
 * for 1 <= M <= 128: the weight-streaming tcgen05 GEMM the decoder's decode steps use for their
 * dense projections (the projection half of kernels/triton/fused_ln_qkv.py:64-72, which computes
 * a row's QKV output one weight column at a time; here for any projection, the whole batch
 * sharing each weight tile).  Persistent: min(sm_count,
 * units) CTAs split the 128-column x 64-row weight units evenly; column blocks shared by two or
 * more CTAs are summed from fp32 partials in a fixed order, so results are deterministic.
 * x [M][K], w [K][N], y [M][N] contiguous; N and K multiples of 8; buffers 16-byte aligned.
 * workspace: lf_gemm_skinny_workspace_size bytes (same M, N, K, sm_count). */
int lf_gemm_skinny_workspace_size(int M, int N, int K, int sm_count, size_t* bytes);
int lf_gemm_skinny(const lf_bf16* x, const lf_bf16* w, lf_bf16* y, int M, int N, int K,
                   void* workspace, size_t workspace_bytes, int sm_count, void* stream);

/* ---- prefix-hash dedup (KV fusion by content) ------------------------------------------
 * The reference's KV fusion is a compile-time pass keyed on IR positions
 * (passes/kv_fusion.py:80-107) and its pool has no sharing (runtime/kv_pool.py:28-235), so
 * these have no reference counterpart; they are the device side of the pool's dedup path.
 * A full page of 16 tokens is named by a chained 64-bit hash,
 *   local_j = FNV-1a-64 over the little-endian bytes of its 16 int32 token ids,
 *   h_j     = fmix64(h_{j-1} ^ local_j)   (h_{-1} = 0; a result of 0 becomes 1),
 * so a page's hash covers every token before it.  The registry is an open-addressing table
 * (linear probing, key 0 = empty) of `capacity` (a power of two) entries in device memory,
 * filled to at most capacity / 2; it holds one refcount on every registered page.  At most
 * LF_MAX_DEDUP_PAGES pages of a session are hashed.  Errors go to the pool's sticky status
 * (LF_EINVAL bad session / non-empty dedup destination, LF_ENOPAGES registry full). */
#define LF_MAX_DEDUP_PAGES 4096

typedef struct lf_prefix_registry {
    unsigned long long* keys; /* [capacity]; 0 = empty */
    int32_t* pages;           /* [capacity] page id of each key */
    int32_t* used;            /* [1] entries in use */
    int capacity;             /* power of two */
} lf_prefix_registry;

/* Empty the table (no refcounts are touched: use lf_pool_unregister_all first). */
int lf_registry_init(const lf_prefix_registry* r, void* stream);

/* Chained page hashes of `n_tokens` token ids: out[j] for the n_tokens / 16 full pages
 * (at most LF_MAX_DEDUP_PAGES). */
int lf_prefix_hashes(const int32_t* tokens, int n_tokens, unsigned long long* out, void* stream);

/* Register the full pages of session `seq` whose token ids are `tokens` (the first
 * min(n_tokens, len(seq)) tokens count): every page whose hash is not yet in the registry is
 * added with one more reference.  All or nothing on LF_ENOPAGES.  *added (device, nullable)
 * receives the number of pages added. */
int lf_pool_register_prefix(const lf_pool_meta* m, const lf_prefix_registry* r, int seq,
                            const int32_t* tokens, int n_tokens, int32_t* added, void* stream);

/* For each of `n` distinct empty sessions, map the longest run of leading full pages whose
 * hashes are registered (session i's tokens are tokens[cu_tokens[i] .. cu_tokens[i+1]]) onto
 * the registered pages (refcount += 1) and set its length to the tokens covered, also written
 * to covered[i] (device, nullable).  One CTA per session. */
int lf_pool_dedup_prefix(const lf_pool_meta* m, const lf_prefix_registry* r,
                         const int32_t* seq_ids, const int32_t* tokens, const int32_t* cu_tokens,
                         int n, int32_t* covered, void* stream);

/* Drop the registry's references and empty it; pages reaching refcount 0 re-enter the free
 * queue tail in ascending page-id order. */
int lf_pool_unregister_all(const lf_pool_meta* m, const lf_prefix_registry* r, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LOOPFUSE_B200_H */
