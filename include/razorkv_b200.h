/*
 * razorkv_b200 -- C ABI of the B200 (sm_100a) RazorKV decode path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, enqueues its
 * work on the given CUDA stream (passed as void*, a cudaStream_t; NULL = legacy default
 * stream) and returns an rkv_status.  Nothing here allocates, frees or synchronises: the
 * caller owns every buffer, including the workspaces whose sizes the *_workspace_size
 * queries report, and all sizes needed for a launch are host-known.  Calls are
 * stream-ordered; the library keeps no per-call state, so calls from several host threads
 * on different streams are independent.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   rkv_decode_attention      razorkv/kernels/triton_paged_sparse.py:105-174
 *                             (triton_paged_sparse_attention) and, with page_table == NULL,
 *                             razorkv/kernels/torch_sparse.py:15-61 (compacted_paged_sdpa)
 *   rkv_page_salience_pool    razorkv/kernels/torch_sparse.py:64-93 (compute_page_salience_pool)
 *   rkv_append                razorkv/cache.py:239-247 (_init_salience) and :369-390
 *                             (the append half of RazorKVCache.update)
 *   rkv_score                 razorkv/cache.py:249-287 (update_salience_with_query)
 *   rkv_decode_fused          razorkv/cache.py:392-393 followed by the attention call of a
 *                             non-compacting decode step (score and attend in one K pass)
 *   rkv_decode_scored         razorkv/engine.py:119-126 (the q_proj hook's
 *                             update_salience_with_query with the pre-RoPE query, before the
 *                             layer's update) and the layer's attention after it, in one K pass
 *   rkv_page_scores           razorkv/cache.py:322-331 (haystack page max-pool)
 *   rkv_select_pages          razorkv/cache.py:333-341 (batch mean, top-k, ascending sort)
 *   rkv_compact_pages         razorkv/cache.py:343-359 when the sink is page aligned
 *                             (page-table rewrite + free-list push, no data movement)
 *   rkv_compact_tokens        razorkv/cache.py:310-320 and :343-359 in general (token copy)
 *   rkv_release_pages         the storage release implied by razorkv/cache.py:356-358
 *   rkv_gather_tokens         materialises the contiguous key_cache/value_cache tensors of
 *                             razorkv/cache.py:89-91 from the paged layout
 *   rkv_reindex_batch         razorkv/cache.py:198-229 (batch_repeat_interleave,
 *                             batch_select_indices, reorder_cache) on the live pages only
 *   rkv_append_score_pool     razorkv/cache.py:361-393 and :322-331 (append, score, page
 *                             max-pool of a compacting decode step, one pass over K)
 *   rkv_select_compact_pages  razorkv/cache.py:333-359 (selection and pointer-only
 *                             compaction in one launch)
 *   rkv_append_decode_peer,   the head-sharded step with the exchange by peer stores over
 *   rkv_salience_apply_peer   NVLink instead of a collective (same reference lines)
 *   rkv_append_partial,       the same steps (razorkv/cache.py:239-287, 361-393) for a rank
 *   rkv_score_partial,        that holds only some kv heads of a layer: each writes its share
 *   rkv_append_decode_partial of the salience update to an exchange block, and
 *   rkv_salience_apply        rkv_salience_apply finishes it after an all-reduce MAX
 */
#ifndef RAZORKV_B200_H
#define RAZORKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum rkv_status {
    RKV_OK = 0,
    RKV_ERR_INVALID_ARGUMENT = 1,   /* null pointer, negative or inconsistent size */
    RKV_ERR_UNSUPPORTED = 2,        /* shape / dtype combination not implemented */
    RKV_ERR_WORKSPACE_TOO_SMALL = 3,
    RKV_ERR_FREE_LIST_EXHAUSTED = 4,
    RKV_ERR_ALIGNMENT = 5,          /* pointer or stride misaligned for the vector path */
    RKV_ERR_CUDA = 6,               /* launch or runtime error */
    RKV_ERR_PAGE_OUT_OF_RANGE = 7   /* host-visible page index outside the pool */
} rkv_status;

typedef enum rkv_dtype { RKV_F32 = 0, RKV_F16 = 1, RKV_BF16 = 2 } rkv_dtype;

typedef enum rkv_pool { RKV_POOL_MAX = 0, RKV_POOL_MEAN = 1 } rkv_pool;

typedef enum rkv_salience_init { RKV_SAL_NORM = 0, RKV_SAL_UNIFORM = 1 } rkv_salience_init;

/* Key/value storage of one layer.  Row (b, h, t) -- D contiguous elements -- starts at
 *   base + b*stride_b + h*stride_h + page_table[b*pt_stride_b + t/page_size]*stride_p
 *        + (t % page_size)*stride_t
 * or, with page_table == NULL, at base + b*stride_b + h*stride_h + t*stride_t.
 * Strides are in elements.  For the reference's paged operator the storage is
 * [B, Hkv, MAXP, P, D]; for the cache pool it is [slots, B, Hkv, P, D] with one page table
 * shared by all sequences (pt_stride_b = 0).
 * row_map (optional; pool storage with a shared page table, not read without a page table):
 * int32 [num_slots][batch].  Sequence b's rows of the page in slot s are stored in the pool's
 * sequence row row_map[s*batch + b] instead of row b, so sequences can share a page (beam
 * search: rkv_reindex_batch rewrites the map instead of moving K/V).  Rows are only written
 * through identity entries: an appended token's page must map b -> b, and a slot taken from
 * the free stack has its entries reset to identity by the call that takes it. */
typedef struct rkv_kv_layout {
    const void* k;
    const void* v;               /* may be NULL for score-only calls */
    int32_t dtype;               /* rkv_dtype of k and v */
    int32_t head_dim;            /* D */
    int64_t batch;               /* B */
    int64_t num_kv_heads;        /* Hkv */
    int64_t stride_b, stride_h, stride_p, stride_t;
    int64_t page_size;           /* tokens per physical page */
    int64_t num_slots;           /* physical pages in the storage */
    const int64_t* page_table;   /* NULL = contiguous tokens */
    int64_t pt_stride_b;         /* 0 = table shared by every sequence */
    int64_t num_tokens;          /* valid tokens per sequence */
    int32_t* row_map;            /* NULL = sequence b in row b (see above) */
} rkv_kv_layout;

/* Query rows [B, Hq, QL, D]: element (b, h, t, d) at q + b*stride_b + h*stride_h + t*stride_t + d. */
typedef struct rkv_query {
    const void* q;
    int32_t dtype;
    int32_t num_heads;           /* Hq, a multiple of Hkv */
    int64_t q_len;               /* QL */
    int64_t stride_b, stride_h, stride_t;
} rkv_query;

/* Attention output [B, Hq, QL, D], same addressing as rkv_query. */
typedef struct rkv_output {
    void* out;
    int32_t dtype;
    int32_t reserved;
    int64_t stride_b, stride_h, stride_t;
} rkv_output;

/* fp32 token salience.  Score of (b, t) at
 *   s + page_table[t/page_size]*stride_p + b*stride_b + t % page_size      (paged), or
 *   s + b*stride_b + t                                                   (page_table NULL),
 * using the page table and page size of the rkv_kv_layout it is passed with. */
typedef struct rkv_salience {
    float* s;
    int64_t stride_b;
    int64_t stride_p;
} rkv_salience;

const char* rkv_status_string(int status);
int rkv_abi_version(void);

/* Number of kernels this library has launched in this process (all threads, all devices);
 * lets a caller count the launches inside a timed region. */
unsigned long long rkv_launch_count(void);

/* Every workspace passed to this library must start with RKV_WORKSPACE_HEADER_BYTES of
 * zeros before its first use.  The decode kernels keep an error flag there; the rest of the
 * header is reserved for cross-CTA counters, which every launch leaves at zero.  All other
 * workspace use starts after the header.  The *_workspace_size queries include the header. */
#define RKV_WORKSPACE_HEADER_BYTES 65536

/* Reads nothing on the device: returns the byte offset, inside a workspace, of the int32
 * flag the decode kernels set when a bounded wait gives up (0 = no error). */
size_t rkv_workspace_error_flag_offset(void);

/* Self-test of the bounded waits (no reference counterpart).  One CTA waits on a barrier
 * that nothing arrives on, with a limit of limit_cycles SM cycles (1 .. 1e10): the wait gives
 * up and sets result[0] to 1, as the decode kernels set the workspace error flag; result[1]
 * is 1 if any wait reported success (expected 0); result[2] is 1 if a second wait after the
 * abort returned at once (expected 1).  result: 3 device int32 zeroed by the caller.  The
 * kernel ends normally and the context stays usable. */
int rkv_selftest_wait_timeout(int* result, long long limit_cycles, void* stream);

/* ---- attention --------------------------------------------------------------------------
 * out = softmax(q.k * scale) . v over the num_tokens tokens of each (b, kv-head), GQA head
 * h reading kv head h / (Hq/Hkv).  causal != 0 masks key t > query row (upper-left aligned).
 * scale <= 0 selects 1/sqrt(D).  fp32 accumulation; the output is rounded to out->dtype. */
size_t rkv_decode_attention_workspace_size(const rkv_query* q, const rkv_kv_layout* kv);
int rkv_decode_attention(const rkv_query* q, const rkv_kv_layout* kv, float scale, int causal,
                         const rkv_output* out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* rkv_decode_attention without a caller workspace.  No counterpart in the reference: it
 * serves callers that cannot allocate device memory when they call (a host framework that
 * owns the whole device heap, or a decode loop that must not enter the driver's allocator).
 * Its scratch is a fixed RKV_NOALLOC_SCRATCH_BYTES array built into the library, held on
 * every device that loads it; calls needing more return RKV_ERR_WORKSPACE_TOO_SMALL without
 * launching.  The first call on a device looks up the array's device address, so make it
 * before any stream capture.  All calls share the array: calls that overlap on the GPU race.
 * Device-side errors (a bounded wait that gave up, a page id outside the storage) are not
 * reported by this entry point: they land in an error flag inside the array that nothing
 * reads back; use rkv_decode_attention with a readable workspace when they matter. */
#define RKV_NOALLOC_SCRATCH_BYTES (16u << 20)
int rkv_decode_attention_noalloc(const rkv_query* q, const rkv_kv_layout* kv, float scale,
                                 int causal, const rkv_output* out, void* stream);

/* ---- page pooling -----------------------------------------------------------------------
 * out[b, p] = max (or mean) of sal[b*stride_b + p*page_size + i], i < page_size, for
 * p < S / page_size (when S < page_size: out[b, 0] = max over the row). */
int rkv_page_salience_pool(const float* sal, int64_t batch, int64_t seq_len, int64_t stride_b,
                           int64_t page_size, int pool_type, float* out, void* stream);

/* ---- cache: append ------------------------------------------------------------------------
 * Writes n_new tokens (rows k_new/v_new [B, Hkv, n_new, D] with the given element strides)
 * at logical positions [pos, pos + n_new) of the layer described by kv (k and v are written),
 * and their initial salience (||k||_2 averaged over kv heads, or 1.0).  Every logical page
 * that starts inside the range takes the physical page free_stack[free_top - 1 - i] (i-th
 * new page) and records it in page_table (writable, shared by all sequences); the caller
 * then lowers its free-stack top by the number of new pages. */
int rkv_append(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
               const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
               int64_t new_stride_t, int64_t n_new, int64_t pos, int64_t* page_table,
               const int64_t* free_stack, int64_t free_top, int salience_init, void* stream);

/* ---- cache: salience --------------------------------------------------------------------
 * R[b, t] = max over query rows (h, r) of the canonical fp32 dot fl(q*scale_r) . k[b, h/G, t];
 * then S = fl(fl(decay*S) + fl(one_minus_decay*R)) when ewma != 0, else S = R.
 * scale_r = 1/sqrt(D) rounded to fp32 (the reference's fixed resonance scale). */
int rkv_score(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
              float decay, float one_minus_decay, int ewma, void* stream);

/* Score (as rkv_score with ewma = 1, q_len = 1) and attention (as rkv_decode_attention,
 * causal = 0) from one pass over K. */
size_t rkv_decode_fused_workspace_size(const rkv_query* q, const rkv_kv_layout* kv);
int rkv_decode_fused(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
                     float decay, float one_minus_decay, float scale, const rkv_output* out,
                     void* workspace, size_t workspace_bytes, void* stream);

/* One non-compacting decode step of a layer in a single call: rkv_append of the single new
 * token (k_new / v_new [B, Hkv, 1, D]) at position kv->num_tokens, then rkv_decode_fused over
 * the kv->num_tokens + 1 tokens.  The caller lowers its free-stack top by one when
 * kv->num_tokens % page_size == 0 (a page was taken).  Replaces the append half of
 * razorkv/cache.py:361-390, the scoring call at :392-393 and the attention over the returned
 * cache, for steps that do not cross the hysteresis threshold (:409-412). */
int rkv_append_decode(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
                      const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                      int64_t* page_table, const int64_t* free_stack, int64_t free_top,
                      int salience_init, const rkv_query* q, float decay, float one_minus_decay,
                      float scale, const rkv_output* out, void* workspace, size_t workspace_bytes,
                      void* stream);

/* The HF decode step of the hooked model in one pass over K: the salience of the tokens
 * before score_tokens is updated as by rkv_score (ewma = 1) with q_score -- the q_proj hook's
 * pre-RoPE query, which scores the cache before the layer appends its new token -- and the
 * output is the attention of q_attn (the post-RoPE query) over all kv->num_tokens tokens, as
 * rkv_decode_attention with causal = 0.  Tokens at or past score_tokens keep their salience.
 * 0 <= score_tokens <= kv->num_tokens; q_score and q_attn have the same heads, q_len 1. */
size_t rkv_decode_scored_workspace_size(const rkv_query* q_attn, const rkv_kv_layout* kv);
int rkv_decode_scored(const rkv_query* q_score, const rkv_query* q_attn, const rkv_kv_layout* kv,
                      const rkv_salience* sal, int64_t score_tokens, float decay,
                      float one_minus_decay, float scale, const rkv_output* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- cache: selection --------------------------------------------------------------------
 * scores[b, p] = max over i < sel_page_size of S(b, first_token + p*sel_page_size + i),
 * p < num_pages, written with row stride num_pages. */
int rkv_page_scores(const rkv_kv_layout* kv, const rkv_salience* sal, int64_t first_token,
                    int64_t num_pages, int64_t sel_page_size, float* scores, void* stream);

/* kept[0..k) = the k pages with the largest batch mean of scores[b, p] (sequential fp32
 * sum over b = 0..batch-1, then one division; batch == 1 uses the row itself), exact ties to
 * the lower page index, in ascending page order.  margin (optional, one float) receives
 * mean[k-th] - mean[(k+1)-th] in selection order (+inf when k == num_pages). */
size_t rkv_select_pages_workspace_size(int64_t num_pages);
int rkv_select_pages(const float* scores, int64_t batch, int64_t num_pages, int64_t k,
                     int64_t* kept, float* margin, void* workspace, size_t workspace_bytes,
                     void* stream);

/* The score half of a compacting decode step in one pass over K (razorkv/cache.py:361-393
 * and :322-331): append the new token (as rkv_append, position kv->num_tokens), score every
 * token of the grown layer (as rkv_score, ewma = 1, q_len 1) and write the max-pooled page
 * scores of the num_pages pages starting at token first_token to scores [B][num_pages]
 * (as rkv_page_scores with sel_page_size = page_size).  The caller lowers its free-stack top
 * by one when kv->num_tokens % page_size == 0. */
int rkv_append_score_pool(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
                          const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                          int64_t* page_table, const int64_t* free_stack, int64_t free_top,
                          int salience_init, const rkv_query* q, float decay,
                          float one_minus_decay, int64_t first_token, int64_t num_pages,
                          float* scores, void* stream);

/* rkv_select_pages followed by rkv_compact_pages in one launch (razorkv/cache.py:333-359):
 * select the k pages with the largest batch mean of scores, then rewrite the shared page
 * table and push the dropped pages (arguments as in the two calls; workspace as in
 * rkv_select_pages).  kept[0..k) and margin receive the selection as rkv_select_pages. */
int rkv_select_compact_pages(const float* scores, int64_t batch, int64_t num_pages, int64_t k,
                             int64_t* page_table, int64_t sink_pages, int64_t tail_first_page,
                             int64_t n_pages_total, int64_t* free_stack, int64_t free_top,
                             int64_t* kept, float* margin, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- cache: compaction -------------------------------------------------------------------
 * Pointer-only compaction of a shared page table whose haystack pages are
 * [sink_pages, sink_pages + num_pages): the table becomes
 *   table[0:sink_pages] ++ table[sink_pages + kept[i]] ++ table[tail_first_page:n_pages_total]
 * and the dropped haystack pages are pushed, in ascending logical order, at
 * free_stack[free_top ...]; the caller raises its free-stack top by num_pages - k. */
int rkv_compact_pages(int64_t* page_table, int64_t sink_pages, int64_t num_pages,
                      const int64_t* kept, int64_t k, int64_t tail_first_page,
                      int64_t n_pages_total, int64_t* free_stack, int64_t free_top,
                      void* stream);

/* Copying compaction.  New logical token i < new_len takes old token
 *   i                                          for i < sink,
 *   hay_start + kept[j / P]*P + j % P          for j = i - sink < k*P  (P = sel_page_size),
 *   tail_src_start + (i - sink - k*P)          otherwise,
 * of the layer kv (old table), written through new_page_table whose pages are popped as
 * new_page_table[i] = free_stack[free_top - 1 - i].  K, V and salience move together. */
int rkv_compact_tokens(const rkv_kv_layout* kv, const rkv_salience* sal,
                       int64_t* new_page_table, const int64_t* free_stack, int64_t free_top,
                       int64_t new_len, int64_t sink, const int64_t* kept, int64_t k,
                       int64_t sel_page_size, int64_t hay_start, int64_t tail_src_start,
                       void* stream);

/* free_stack[free_top + i] = pages[i], i < n. */
int rkv_release_pages(const int64_t* pages, int64_t n, int64_t* free_stack, int64_t free_top,
                      void* stream);

/* ---- KV-head sharding ---------------------------------------------------------------------
 * When the kv heads of a layer are spread over the ranks of a head group, no rank can finish
 * a token's salience alone: the resonance is a max over every query head and the initial
 * salience a mean over every kv head (razorkv/cache.py:239-247, :274-287).  The partial calls
 * write this rank's share into an exchange block instead of updating the salience; the caller
 * takes the element-wise int32 MAX of the blocks over the head group (an all-reduce MAX:
 * exact and independent of the order of the ranks) and rkv_salience_apply then updates the
 * salience, bit for bit as one rank holding every head would.
 *
 * Exchange block: int32 x[b * stride_b + ...] per sequence b.  Entry t < num_tokens holds the
 * signed key of token t's resonance over this rank's query heads; entry
 * norm_off + i * num_kv_heads_total + h holds the signed key of ||k|| of global kv head h of
 * the i-th token the call appends (INT32_MIN where this rank does not hold head h).  The
 * signed key of an fp32 value is its order-preserving uint32 key with the top bit flipped, so
 * int32 order is the fp32 order.  The layout's kv heads are global heads head0 ..
 * head0 + kv->num_kv_heads - 1. */
typedef struct rkv_exchange {
    int32_t* x;
    int64_t stride_b;
    int64_t norm_off;
    int32_t head0;
    int32_t num_kv_heads_total;
} rkv_exchange;

/* rkv_append that leaves the salience alone and writes the new tokens' norms (salience_init
 * == RKV_SAL_NORM) to the exchange block (razorkv/cache.py:239-247, 369-390, one rank's heads). */
int rkv_append_partial(const rkv_kv_layout* kv, const void* k_new, const void* v_new,
                       int64_t new_stride_b, int64_t new_stride_h, int64_t new_stride_t,
                       int64_t n_new, int64_t pos, int64_t* page_table, const int64_t* free_stack,
                       int64_t free_top, int salience_init, const rkv_exchange* xc, void* stream);

/* The resonance keys of every token of kv over this rank's query heads (q holds the query
 * heads of the layout's kv heads only), written to the exchange block
 * (razorkv/cache.py:249-280, one rank's heads). */
int rkv_score_partial(const rkv_query* q, const rkv_kv_layout* kv, const rkv_exchange* xc,
                      void* stream);

/* rkv_append_decode whose scoring is partial: the appended token's norms and every token's
 * resonance key go to the exchange block (nothing is written to the salience); the attention
 * output covers this rank's query heads.  Follow with the all-reduce MAX and
 * rkv_salience_apply(score_tokens = num_tokens + 1, new_first = num_tokens, n_new = 1). */
int rkv_append_decode_partial(const rkv_kv_layout* kv,
                              const void* k_new, const void* v_new, int64_t new_stride_b,
                              int64_t new_stride_h, int64_t* page_table,
                              const int64_t* free_stack, int64_t free_top, int salience_init,
                              const rkv_query* q, float scale, const rkv_output* out,
                              const rkv_exchange* xc, void* workspace, size_t workspace_bytes,
                              void* stream);

/* The salience update from a reduced exchange block (razorkv/cache.py:282-287 with the
 * initial salience of :239-247): tokens [new_first, new_first + n_new) start from their mean
 * norm (salience_init == RKV_SAL_NORM, sequential fp32 sum over the kv heads then one
 * division) or 1.0; tokens t < score_tokens take S = fl(fl(decay S) + fl(one_minus_decay R)). */
int rkv_salience_apply(const rkv_kv_layout* kv, const rkv_salience* sal, const rkv_exchange* xc,
                       int64_t score_tokens, int64_t new_first, int64_t n_new,
                       int salience_init, float decay, float one_minus_decay, void* stream);

/* The exchange without a collective (no reference counterpart; ranks on one node with peer
 * access over NVLink).  Every rank owns a region of two buffers x nranks sub-blocks of `sub`
 * int32 (a sub-block laid out as the rkv_exchange block: rows of stride_b per sequence) and
 * nranks uint32 flags, and every rank can address every other rank's region and flags
 * (CUDA IPC).  rkv_append_decode_peer stores this rank's share into sub-block `rank` of
 * buffer buf_off of every rank's region -- plain stores into peer memory, no multicast --
 * and its last CTA then releases flags[r][rank] = epoch on every rank r.
 * rkv_salience_apply_peer waits (bounded, about a second; on timeout it sets the workspace
 * error flag to 1 and leaves the salience alone) until every flag of this rank has reached
 * the epoch and applies the update from the MAX over the sub-blocks.  The caller advances the
 * epoch by one per exchange and alternates the two buffers (buf_off = (epoch & 1) * nranks *
 * sub), so a rank never overwrites a sub-block a peer may still be reading. */
typedef struct rkv_peer_exchange {
    int32_t* const* regions;     /* device array [nranks]: each rank's region, as seen here */
    uint32_t* const* flags;      /* device array [nranks]: each rank's flags, as seen here */
    const int32_t* my_region;    /* this rank's region */
    const uint32_t* my_flags;    /* this rank's flags */
    int32_t rank, nranks;
    int64_t sub;                 /* int32 elements per sub-block */
    int64_t buf_off;             /* int32 elements to the buffer of this exchange */
    uint32_t epoch;              /* 1, 2, 3, ... */
    uint32_t reserved;
} rkv_peer_exchange;

/* CUDA IPC of an exchange region between the ranks' processes.  rkv_ipc_export returns the
 * handle (RKV_IPC_HANDLE_BYTES bytes) of the device allocation holding ptr and ptr's offset in
 * it; rkv_ipc_import maps a peer's allocation into the CURRENT device's context (peer access
 * enabled as needed) and returns the address of the exported pointer; rkv_ipc_release unmaps
 * it.  Call import with the device that will run the kernels current. */
#define RKV_IPC_HANDLE_BYTES 64
int rkv_ipc_export(const void* ptr, void* handle, int64_t* offset);
int rkv_ipc_import(const void* handle, int64_t offset, void** ptr);
int rkv_ipc_release(void* ptr, int64_t offset);

/* rkv_append_decode_partial with the share stored to every rank (xc gives the block layout:
 * stride_b, norm_off, head0, num_kv_heads_total; xc->x is not used).  Fused decode shapes
 * only (RKV_ERR_UNSUPPORTED otherwise; use the collective path then). */
int rkv_append_decode_peer(const rkv_kv_layout* kv, const void* k_new, const void* v_new,
                           int64_t new_stride_b, int64_t new_stride_h, int64_t* page_table,
                           const int64_t* free_stack, int64_t free_top, int salience_init,
                           const rkv_query* q, float scale, const rkv_output* out,
                           const rkv_exchange* xc, const rkv_peer_exchange* px, void* workspace,
                           size_t workspace_bytes, void* stream);

/* rkv_salience_apply on the MAX over the sub-blocks of this rank's region, after the wait. */
int rkv_salience_apply_peer(const rkv_kv_layout* kv, const rkv_salience* sal,
                            const rkv_exchange* xc, const rkv_peer_exchange* px,
                            int64_t score_tokens, int64_t new_first, int64_t n_new,
                            int salience_init, float decay, float one_minus_decay,
                            void* workspace, size_t workspace_bytes, void* stream);

/* dst[b, h, t, :] = row (b, h, t) of kv (K when which == 0, V when 1), t < num_tokens;
 * dst is contiguous [B, Hkv, num_tokens, D] of kv->dtype.  sal_dst (optional, [B, num_tokens])
 * receives the salience. */
int rkv_gather_tokens(const rkv_kv_layout* kv, int which, void* dst, const rkv_salience* sal,
                      float* sal_dst, void* stream);

/* Batch reindex of a cache pool's live pages: the index_select along the batch dimension
 * behind razorkv/cache.py:198-206 (batch_repeat_interleave), :208-218 (batch_select_indices)
 * and :220-229 (reorder_cache).  Sequence b of dst becomes sequence index[b] of src on every
 * slot in slots[0 .. num_listed), for K, V (when both layouts have one) and the salience (when
 * both salience pointers are given).  src and dst are pools [slots, B, Hkv, P, D]: each
 * (slot, sequence) plane must be contiguous (stride_t == D, stride_h == P*D); their
 * page_table and num_tokens are not used.  index holds dst->batch device entries in
 * [0, src->batch).
 * Out of place (dst is another pool, any batch): every listed slot's rows are gathered
 * through src->row_map (when set) and dst holds sequence b in row b (dst->row_map NULL).
 * In place (dst == src, same batch and strides): the salience rows are permuted.  Without a
 * row map the K/V rows are too.  With src->row_map set, only the first num_moved listed
 * slots move their K/V rows (to identity rows: use it for every page that will still be
 * written, i.e. each layer's last page); the other slots keep their K/V and their row map
 * entries are rewritten, row_map[s][b] <- row_map[s][index[b]]: a page-table update, not a
 * copy.  A row that would copy onto itself is neither read nor written.  List each slot at
 * most once, and only slots whose contents matter (the pages of the layers' page tables):
 * unlisted slots are left as they are.  err (optional device int32, e.g. a workspace's error
 * flag) is set to 2 when a listed slot is outside the pools or an index is outside
 * [0, src->batch); such a slot or row is left unchanged.  Batches above about 1500 rows
 * return RKV_ERR_UNSUPPORTED. */
int rkv_reindex_batch(const rkv_kv_layout* src, const rkv_salience* src_sal,
                      const rkv_kv_layout* dst, const rkv_salience* dst_sal,
                      const int64_t* index, const int64_t* slots, int64_t num_listed,
                      int64_t num_moved, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RAZORKV_B200_H */
