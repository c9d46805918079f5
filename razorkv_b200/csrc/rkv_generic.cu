// Shape-general kernels of the RazorKV decode path: any head_dim <= 256, any page size,
// fp32 / fp16 / bf16, any query length.  They define the semantics the specialised sm_100a
// decode kernel (rkv_decode_sm100.cu) must reproduce, and serve every shape it does not
// cover.  All of them are HBM- or latency-bound scans; none is GEMM-shaped.
#include <math.h>

#include "rkv_common.cuh"
#include "rkv_kernels.h"

namespace rkv {

// ------------------------------------------------------------------------------------------
// Salience score (razorkv/cache.py:249-287)
// ------------------------------------------------------------------------------------------
// CTA = (token block of kScoreTokens tokens, sequence b).  256 threads = 32 groups of 8
// lanes; group g handles tokens t0 + g + 32*i.  The query rows of one kv head are staged in
// shared memory as fl(q * scale) (fp32); every group walks its tokens, loads the K row once
// per kv head (lane j keeps the elements of chunks j, j+8, ...) and takes the canonical dot
// with every query row of that head.
constexpr int kScoreThreads = 256;
constexpr int kScoreTokens = 128;   // 4 tokens per group
constexpr int kScoreTPG = kScoreTokens / 32;
constexpr int kLaneElts = 32;       // max elements one lane owns (D <= 256)

__device__ __forceinline__ int lane_elements(int D, int ch, int j, int* idx) {
    int n = 0;
    for (int c = j; c * ch < D; c += 8)
        for (int e = c * ch; e < min(D, c * ch + ch); ++e) idx[n++] = e;
    return n;
}

__global__ void __launch_bounds__(kScoreThreads)
score_kernel(ScoreParams p) {
    extern __shared__ float qs[];   // [rows_per_chunk][D]
    const int b = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int group = threadIdx.x >> 3;   // 0..31
    const int j = lane & 7;
    const int D = p.D;
    const int ch = 16 / elt_bytes(p.kv_dtype);
    const int G = p.Hq / p.Hkv;
    const int64_t t0 = (int64_t)blockIdx.x * kScoreTokens;

    int idx[kLaneElts];
    const int ne = lane_elements(D, ch, j, idx);

    uint32_t best[kScoreTPG];
#pragma unroll
    for (int i = 0; i < kScoreTPG; ++i) best[i] = 0u;   // below every ordered key

    const int rows_per_head = G * p.QL;
    const int chunk_rows = p.rows_per_chunk;
    const float scale = p.scale_r;
    TokenMap tm{p.page_table ? p.page_table + (int64_t)b * p.pt_stride_b : nullptr,
                p.page_size, p.stride_p, p.stride_t};
    tm.row_map = p.row_map; tm.batch = p.B; tm.seq = b; tm.stride_b = p.stride_b;

    for (int h = 0; h < p.Hkv; ++h) {
        for (int r0 = 0; r0 < rows_per_head; r0 += chunk_rows) {
            const int nr = min(chunk_rows, rows_per_head - r0);
            __syncthreads();
            for (int i = threadIdx.x; i < nr * D; i += blockDim.x) {
                int r = r0 + i / D, d = i % D;
                int hq = h * G + r / p.QL, tq = r % p.QL;
                float qv = load_elt(p.q, (int64_t)b * p.q_stride_b + (int64_t)hq * p.q_stride_h +
                                             (int64_t)tq * p.q_stride_t + d, p.q_dtype);
                qs[i] = __fmul_rn(qv, scale);
            }
            __syncthreads();
            // every lane runs the same number of group8_sum shuffles; tokens past N are
            // computed on zeros and discarded
            for (int it = 0; it < kScoreTPG; ++it) {
                const int64_t t = t0 + group + 32 * it;
                const bool valid = t < p.N;
                float kr[kLaneElts];
                if (valid) {
                    const int64_t row = (int64_t)b * p.stride_b + (int64_t)h * p.stride_h + tm.offset(t);
                    for (int e = 0; e < ne; ++e) kr[e] = load_elt(p.k, row + idx[e], p.kv_dtype);
                } else {
                    for (int e = 0; e < ne; ++e) kr[e] = 0.0f;
                }
                for (int r = 0; r < nr; ++r) {
                    float ev = 0.0f, od = 0.0f;   // even / odd positions of the lane's elements
                    const float* qr = qs + r * D;
                    for (int e = 0; e < ne; ++e) {
                        if (e & 1) od = __fmaf_rn(qr[idx[e]], kr[e], od);
                        else ev = __fmaf_rn(qr[idx[e]], kr[e], ev);
                    }
                    const float s = group8_sum(__fadd_rn(ev, od));
                    if (valid) best[it] = max(best[it], ordered_key(s));
                }
            }
        }
    }
    if (j == 0) {
        for (int it = 0; it < kScoreTPG; ++it) {
            int64_t t = t0 + group + 32 * it;
            if (t >= p.N) break;
            if (p.xc.x) {   // head-sharded: this rank's key; the salience waits for the MAX
                p.xc.x[(int64_t)b * p.xc.stride_b + t] = signed_key_of(best[it]);
                continue;
            }
            float R = key_to_float(best[it]);
            float* sp = p.sal + (p.page_table ? tm.page_table[t / p.page_size] * p.sal_stride_p +
                                                    (int64_t)b * p.sal_stride_b + t % p.page_size
                                              : (int64_t)b * p.sal_stride_b + t);
            *sp = p.ewma ? __fadd_rn(__fmul_rn(p.decay, *sp), __fmul_rn(p.one_minus_decay, R)) : R;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Attention, split over tokens (razorkv/kernels/triton_paged_sparse.py:23-102 semantics:
// online softmax over the pages of the table; razorkv/kernels/torch_sparse.py:15-61 for the
// contiguous case).  CTA = (split, b*Hkv + kvh, block of 4 query rows); one warp per query
// row; lanes split D (element e = lane + 32*i).  Partials (m, l, acc[D]) go to the workspace
// and merge_kernel combines them.
// ------------------------------------------------------------------------------------------
constexpr int kAttnWarps = 4;

__global__ void __launch_bounds__(kAttnWarps * 32)
attn_split_kernel(AttnParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y;
    const int b = bh / p.Hkv, kvh = bh % p.Hkv;
    const int G = p.Hq / p.Hkv;
    const int row = blockIdx.z * kAttnWarps + warp;      // 0 .. G*QL-1
    if (row >= G * p.QL) return;
    const int hq = kvh * G + row / p.QL, tq = row % p.QL;
    const int D = p.D;
    const int split = blockIdx.x;
    const int64_t per = (p.N + p.num_splits - 1) / p.num_splits;
    const int64_t s0 = split * per;
    int64_t s1 = (p.N < s0 + per ? p.N : s0 + per);
    if (p.causal) { const int64_t lim = (int64_t)tq + 1; s1 = s1 < lim ? s1 : lim; };

    float q[8], acc[8];
    const int ne = (D + 31) / 32;
    for (int i = 0; i < 8; ++i) {
        int e = lane + 32 * i;
        q[i] = (i < ne && e < D)
                   ? load_elt(p.q, (int64_t)b * p.q_stride_b + (int64_t)hq * p.q_stride_h +
                                       (int64_t)tq * p.q_stride_t + e, p.q_dtype)
                   : 0.0f;
        acc[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    TokenMap tm{p.page_table ? p.page_table + (int64_t)b * p.pt_stride_b : nullptr,
                p.page_size, p.stride_p, p.stride_t, p.num_slots};
    tm.row_map = p.row_map; tm.batch = p.B; tm.seq = b; tm.stride_b = p.stride_b;
    const int64_t base = (int64_t)b * p.stride_b + (int64_t)kvh * p.stride_h;
    for (int64_t t = s0; t < s1; ++t) {
        const int64_t off = base + tm.offset(t);
        float part = 0.0f;
        for (int i = 0; i < ne; ++i) {
            int e = lane + 32 * i;
            if (e < D) part = fmaf(q[i], load_elt(p.k, off + e, p.kv_dtype), part);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float s = part * p.scale;
        const float mn = fmaxf(m, s);
        const float alpha = __expf(m - mn);
        const float pw = __expf(s - mn);
        l = l * alpha + pw;
        for (int i = 0; i < ne; ++i) {
            int e = lane + 32 * i;
            float v = e < D ? load_elt(p.v, off + e, p.kv_dtype) : 0.0f;
            acc[i] = acc[i] * alpha + pw * v;
        }
        m = mn;
    }
    // workspace layout: [split][b][hq][tq] -> {m, l, acc[D]}
    const int64_t slot = (((int64_t)split * p.B + b) * p.Hq + hq) * p.QL + tq;
    float* w = p.workspace + slot * (D + 2);
    if (lane == 0) { w[0] = m; w[1] = l; }
    for (int i = 0; i < ne; ++i) {
        int e = lane + 32 * i;
        if (e < D) w[2 + e] = acc[i];
    }
}

__global__ void merge_kernel(AttnParams p) {
    // one CTA per (b, hq, tq); threads over D
    const int64_t r = blockIdx.x;
    const int tq = r % p.QL;
    const int hq = (r / p.QL) % p.Hq;
    const int b = r / ((int64_t)p.QL * p.Hq);
    const int D = p.D;
    float M = -INFINITY;
    for (int s = 0; s < p.num_splits; ++s) {
        const float* w = p.workspace + ((((int64_t)s * p.B + b) * p.Hq + hq) * p.QL + tq) * (D + 2);
        M = fmaxf(M, w[0]);
    }
    float L = 0.0f;
    for (int s = 0; s < p.num_splits; ++s) {
        const float* w = p.workspace + ((((int64_t)s * p.B + b) * p.Hq + hq) * p.QL + tq) * (D + 2);
        if (w[0] != -INFINITY) L += w[1] * __expf(w[0] - M);
    }
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.0f;
        for (int s = 0; s < p.num_splits; ++s) {
            const float* w =
                p.workspace + ((((int64_t)s * p.B + b) * p.Hq + hq) * p.QL + tq) * (D + 2);
            if (w[0] != -INFINITY) o += w[2 + d] * __expf(w[0] - M);
        }
        store_elt(p.out, (int64_t)b * p.o_stride_b + (int64_t)hq * p.o_stride_h +
                             (int64_t)tq * p.o_stride_t + d, p.out_dtype, L > 0.0f ? o / L : 0.0f);
    }
}

// ------------------------------------------------------------------------------------------
// Page pooling (razorkv/kernels/torch_sparse.py:64-93) and haystack page scores
// (razorkv/cache.py:322-331).  NaN propagates like torch.amax.
// ------------------------------------------------------------------------------------------
__global__ void pool_kernel(const float* sal, int64_t B, int64_t S, int64_t stride_b, int64_t P,
                            int64_t n_pages, int mean, float* out) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= B * n_pages) return;
    int64_t b = i / n_pages, pg = i % n_pages;
    const float* row = sal + b * stride_b;
    if (S < P) {   // fewer tokens than one page: the reference returns the row max
        uint32_t best = 0u;
        for (int64_t t = 0; t < S; ++t) best = max(best, ordered_key(row[t]));
        out[i] = key_to_float(best);
        return;
    }
    if (mean) {
        float acc = 0.0f;
        for (int64_t t = 0; t < P; ++t) acc = __fadd_rn(acc, row[pg * P + t]);
        out[i] = __fdiv_rn(acc, (float)P);
    } else {
        uint32_t best = 0u;
        for (int64_t t = 0; t < P; ++t) best = max(best, ordered_key(row[pg * P + t]));
        out[i] = key_to_float(best);
    }
}

__global__ void page_scores_kernel(PageScoreParams p) {
    int64_t pg = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int b = blockIdx.y;
    if (pg >= p.num_pages) return;
    uint32_t best = 0u;
    for (int64_t i = 0; i < p.sel_page_size; ++i) {
        int64_t t = p.first_token + pg * p.sel_page_size + i;
        const float* sp = p.sal + (p.page_table ? p.page_table[t / p.page_size] * p.sal_stride_p +
                                                     (int64_t)b * p.sal_stride_b + t % p.page_size
                                               : (int64_t)b * p.sal_stride_b + t);
        best = max(best, ordered_key(*sp));
    }
    p.scores[(int64_t)b * p.num_pages + pg] = key_to_float(best);
}

// ------------------------------------------------------------------------------------------
// Top-k page selection (razorkv/cache.py:333-341) -- one CTA.
// mean[p] = (sum_b scores[b, p] in ascending b) / B; radix select of the k-th largest
// ordered key over four 8-bit digits; keys equal to the threshold are taken lowest index
// first; kept pages are emitted in ascending order by a block scan.
// ------------------------------------------------------------------------------------------
constexpr int kSelThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        warp_sums[lane] = w;   // inclusive
    }
    __syncthreads();
    int res = x - v + (warp > 0 ? warp_sums[warp - 1] : 0);
    if (total) *total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return res;
}

constexpr int kSelSmemKeys = 11264;   // keys kept in shared memory up to this many pages (44 KiB)

// Warp 0 picks the radix digit holding the rem-th largest key: lane l owns bins 8l..8l+7,
// a suffix scan over lanes (highest digits first) finds the owning lane, which walks its 8
// bins.  Writes the digit and the count still to take among keys with that digit.
__device__ __forceinline__ void select_digit(const int* hist, int rem, uint32_t prefix, int shift,
                                             uint32_t* s_prefix, int* s_remaining) {
    const int lane = threadIdx.x & 31;
    int c[8];
    int mine = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) { c[i] = hist[8 * lane + i]; mine += c[i]; }
    // inclusive sum over lanes >= lane (digits from the top)
    int above = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_down_sync(0xffffffffu, above, o);
        if (lane + o < 32) above += y;
    }
    const int before = above - mine;   // keys in higher lanes' bins
    const bool here = before < rem && above >= rem;
    if (here) {
        int cum = before;
#pragma unroll
        for (int i = 7; i >= 0; --i) {
            if (cum + c[i] >= rem) {
                *s_prefix = prefix | ((uint32_t)(8 * lane + i) << shift);
                *s_remaining = rem - cum;
                break;
            }
            cum += c[i];
        }
    }
}

// The selection of one CTA (select_kernel, select_compact_kernel).
__device__ __forceinline__ void select_body(const float* scores, int64_t B, int64_t n, int64_t k,
                                            int64_t* kept, float* margin, uint32_t* gkeys) {
    __shared__ int hist[256];
    __shared__ int warp_sums[32];
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining;
    __shared__ uint32_t s_best_out;
    __shared__ uint32_t s_keys[kSelSmemKeys];
    uint32_t* keys = n <= kSelSmemKeys ? s_keys : gkeys;   // uniform over the CTA
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float acc = scores[i];
        if (B > 1) {
            for (int64_t b = 1; b < B; ++b) acc = __fadd_rn(acc, scores[b * n + i]);
            acc = __fdiv_rn(acc, (float)B);
        }
        keys[i] = ordered_key(acc);
    }
    if (threadIdx.x == 0) { s_prefix = 0u; s_remaining = (int)k; s_best_out = 0u; }
    __syncthreads();
    uint32_t mask = 0u;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        const int rem = s_remaining;
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
            uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
        }
        __syncthreads();
        if (threadIdx.x < 32) select_digit(hist, rem, prefix, shift, &s_prefix, &s_remaining);
        mask |= 255u << shift;
        __syncthreads();
    }
    const uint32_t thr = s_prefix;
    const int need_eq = s_remaining;   // how many keys equal to thr are kept (lowest index first)
    int eq_base = 0, out_base = 0;
    for (int64_t c = 0; c < n; c += blockDim.x) {
        int64_t i = c + threadIdx.x;
        uint32_t key = i < n ? keys[i] : 0u;
        int is_eq = (i < n && key == thr) ? 1 : 0;
        int eq_total;
        int eq_rank = eq_base + block_exclusive_scan(is_eq, warp_sums, &eq_total);
        int take = (i < n) && (key > thr || (is_eq && eq_rank < need_eq)) ? 1 : 0;
        if (i < n && !take) atomicMax(&s_best_out, key);
        int out_total;
        int pos = out_base + block_exclusive_scan(take, warp_sums, &out_total);
        if (take && pos < k) kept[pos] = i;
        eq_base += eq_total;
        out_base += out_total;
    }
    __syncthreads();
    if (margin && threadIdx.x == 0) {
        *margin = (k >= n) ? INFINITY : __fsub_rn(key_to_float(thr), key_to_float(s_best_out));
    }
}

__global__ void __launch_bounds__(kSelThreads)
select_kernel(const float* scores, int64_t B, int64_t n, int64_t k, int64_t* kept, float* margin,
              uint32_t* gkeys) {
    select_body(scores, B, n, k, kept, margin, gkeys);
}

// ------------------------------------------------------------------------------------------
// Pointer-only compaction (razorkv/cache.py:343-359 for a page-aligned sink).  One CTA.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ int64_t lower_bound(const int64_t* a, int64_t n, int64_t x) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if (a[mid] < x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

__device__ __forceinline__ void compact_body(int64_t* pt, int64_t sink_pages, int64_t num_pages,
                                             const int64_t* kept, int64_t k, int64_t tail_first,
                                             int64_t n_total, int64_t* free_stack,
                                             int64_t free_top) {
    // 1. push dropped haystack pages in ascending logical order
    for (int64_t j = threadIdx.x; j < num_pages; j += blockDim.x) {
        int64_t lb = lower_bound(kept, k, j);
        bool is_kept = lb < k && kept[lb] == j;
        if (!is_kept) free_stack[free_top + (j - lb)] = pt[sink_pages + j];
    }
    __syncthreads();
    // 2. rewrite in place; destination index <= source index, chunk by chunk
    const int64_t n_tail = n_total - tail_first;
    const int64_t n_out = k + n_tail;
    for (int64_t c = 0; c < n_out; c += blockDim.x) {
        int64_t i = c + threadIdx.x;
        int64_t v = 0;
        if (i < n_out) v = i < k ? pt[sink_pages + kept[i]] : pt[tail_first + (i - k)];
        __syncthreads();
        if (i < n_out) pt[sink_pages + i] = v;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(1024)
compact_pages_kernel(int64_t* pt, int64_t sink_pages, int64_t num_pages, const int64_t* kept,
                     int64_t k, int64_t tail_first, int64_t n_total, int64_t* free_stack,
                     int64_t free_top) {
    compact_body(pt, sink_pages, num_pages, kept, k, tail_first, n_total, free_stack, free_top);
}

// Selection and pointer-only compaction in one launch (razorkv/cache.py:333-359): the CTA
// selects, then -- after a barrier that makes its writes of the kept pages visible to every
// thread of the CTA -- rewrites the page table and pushes the dropped pages.
__global__ void __launch_bounds__(kSelThreads)
select_compact_kernel(const float* scores, int64_t B, int64_t num_pages, int64_t k,
                      int64_t* kept, float* margin, uint32_t* gkeys, int64_t* pt,
                      int64_t sink_pages, int64_t tail_first, int64_t n_total,
                      int64_t* free_stack, int64_t free_top) {
    select_body(scores, B, num_pages, k, kept, margin, gkeys);
    __syncthreads();
    compact_body(pt, sink_pages, num_pages, kept, k, tail_first, n_total, free_stack, free_top);
}

// ------------------------------------------------------------------------------------------
// Append (razorkv/cache.py:239-247, 369-390): write rows, initial salience, new page ids.
// Work item = (sequence b, new token i); 256 threads = 32 groups of 8 lanes.  With Hkv <= 32
// a CTA takes 32 / Hkv items and group g serves kv head g % Hkv of item g / Hkv; with more
// heads a CTA takes one item and its groups stride over the heads.  A group copies its K and
// V rows (16-byte vectors when aligned), computes sqrt(canonical k.k) and leaves it in
// shared memory; one thread per item then sums the heads in ascending order and divides.
// ------------------------------------------------------------------------------------------
constexpr int kAppendThreads = 256;
constexpr int kAppendGroups = kAppendThreads / 8;

__device__ __forceinline__ int64_t append_phys(const AppendParams& p, int64_t t) {
    const int64_t P = p.page_size;
    const int64_t first_new_page = (p.pos + P - 1) / P;
    const int64_t lp = t / P;
    return lp < first_new_page ? p.page_table[lp]
                               : p.free_stack[p.free_top - 1 - (lp - first_new_page)];
}

__global__ void __launch_bounds__(kAppendThreads)
append_kernel(AppendParams p) {
    extern __shared__ float nrm[];   // [items per CTA][Hkv]
    const int lane = threadIdx.x & 31, j = lane & 7, grp = threadIdx.x >> 3;
    const int hk = p.Hkv;
    const int ipc = hk >= kAppendGroups ? 1 : kAppendGroups / hk;   // items per CTA
    const int li = hk >= kAppendGroups ? 0 : grp / hk;              // local item
    const int h0 = hk >= kAppendGroups ? grp : grp % hk;
    const int hstep = hk >= kAppendGroups ? kAppendGroups : hk;
    const int64_t item = (int64_t)blockIdx.x * ipc + li;
    const bool active = li < ipc && item < p.n_new * p.B;
    const int64_t b = active ? item / p.n_new : 0;
    const int64_t i = active ? item % p.n_new : 0;
    const int64_t t = p.pos + i;
    const int64_t P = p.page_size;
    const int64_t phys = active ? append_phys(p, t) : 0;
    if (active && h0 == 0 && j == 0 && b == 0 && t % P == 0) {
        const int64_t lp = t / P;
        if (lp >= (p.pos + P - 1) / P) {
            p.page_table[lp] = phys;
            // a page from the free stack starts with every sequence in its own row
            if (p.row_map)
                for (int64_t bb = 0; bb < p.B; ++bb) p.row_map[phys * p.B + bb] = (int32_t)bb;
        }
    }
    const int eb = elt_bytes(p.dtype);
    const int ch = 16 / eb;
    // 16-byte vector path: every row start 16-byte aligned and D a whole number of chunks
    const bool vec = p.vec_ok;
    for (int h = h0; h < hk; h += hstep) {
        float ev = 0.0f, od = 0.0f;   // canonical even / odd sub-chains of k.k
        if (active) {
            const int64_t src = b * p.new_stride_b + (int64_t)h * p.new_stride_h + i * p.new_stride_t;
            const int64_t dst = b * p.stride_b + (int64_t)h * p.stride_h + phys * p.stride_p +
                                (t % P) * p.stride_t;
            if (vec) {
                int pos = 0;
                for (int c = j; c * ch < p.D; c += 8) {
                    const uint4 kw = *reinterpret_cast<const uint4*>(
                        static_cast<const char*>(p.k_new) + (src + (int64_t)c * ch) * eb);
                    const uint4 vw = *reinterpret_cast<const uint4*>(
                        static_cast<const char*>(p.v_new) + (src + (int64_t)c * ch) * eb);
                    *reinterpret_cast<uint4*>(static_cast<char*>(p.k) + (dst + (int64_t)c * ch) * eb) = kw;
                    *reinterpret_cast<uint4*>(static_cast<char*>(p.v) + (dst + (int64_t)c * ch) * eb) = vw;
                    const uint32_t u[4] = {kw.x, kw.y, kw.z, kw.w};
                    for (int e = 0; e < ch; ++e, ++pos) {
                        float kv;
                        if (eb == 4) kv = __uint_as_float(u[e]);
                        else if (p.dtype == RKV_BF16)
                            kv = __uint_as_float((e & 1) ? (u[e >> 1] & 0xffff0000u) : (u[e >> 1] << 16));
                        else {
                            const __half2 hv = *reinterpret_cast<const __half2*>(&u[e >> 1]);
                            kv = (e & 1) ? __high2float(hv) : __low2float(hv);
                        }
                        if (pos & 1) od = __fmaf_rn(kv, kv, od);
                        else ev = __fmaf_rn(kv, kv, ev);
                    }
                }
            } else {
                int idx[kLaneElts];
                const int ne = lane_elements(p.D, ch, j, idx);
                for (int e = 0; e < ne; ++e) {
                    const float kv = load_elt(p.k_new, src + idx[e], p.dtype);
                    store_elt(p.k, dst + idx[e], p.dtype, kv);
                    store_elt(p.v, dst + idx[e], p.dtype, load_elt(p.v_new, src + idx[e], p.dtype));
                    if (e & 1) od = __fmaf_rn(kv, kv, od);
                    else ev = __fmaf_rn(kv, kv, ev);
                }
            }
        }
        const float ss = group8_sum(__fadd_rn(ev, od));
        if (active && j == 0) nrm[li * hk + h] = __fsqrt_rn(ss);
    }
    __syncthreads();
    if (active && h0 == 0 && j == 0 && p.xc.x) {
        // head-sharded: this item's kv-head norms at their global head positions (others
        // absent); the initial salience is set by rkv_salience_apply after the MAX
        if (p.salience_init == RKV_SAL_NORM) {
            int32_t* xr = p.xc.x + b * p.xc.stride_b + p.xc.norm_off + i * p.xc.htot;
            for (int hh = 0; hh < p.xc.htot; ++hh) {
                const int lh = hh - p.xc.h0;
                xr[hh] = (lh >= 0 && lh < hk) ? signed_key_of(ordered_key(nrm[li * hk + lh])) : INT32_MIN;
            }
        }
    } else if (active && h0 == 0 && j == 0) {
        float s0 = 1.0f;
        if (p.salience_init == RKV_SAL_NORM) {
            float acc = 0.0f;
            for (int h = 0; h < hk; ++h) acc = __fadd_rn(acc, nrm[li * hk + h]);
            s0 = __fdiv_rn(acc, (float)hk);
        }
        p.sal[phys * p.sal_stride_p + b * p.sal_stride_b + t % P] = s0;
    }
}

// ------------------------------------------------------------------------------------------
// Copying compaction (razorkv/cache.py:310-320, 343-359 in general).
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ int64_t compact_source(const CompactTokensParams& p, int64_t i) {
    if (i < p.sink) return i;
    int64_t j = i - p.sink;
    int64_t P = p.sel_page_size;
    if (j < p.n_kept * P) return p.hay_start + p.kept[j / P] * P + j % P;
    return p.tail_src_start + (j - p.n_kept * P);
}

__global__ void compact_tokens_kernel(CompactTokensParams p) {
    // one thread per (b, h, new token, element-chunk of 4)
    const int64_t D = p.D;
    const int64_t nd = (D + 3) / 4;
    int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t total = p.new_len * p.B * p.Hkv * nd;
    if (gid >= total) return;
    const int64_t dq = gid % nd;
    int64_t r = gid / nd;
    const int64_t i = r % p.new_len; r /= p.new_len;
    const int64_t h = r % p.Hkv;
    const int64_t b = r / p.Hkv;
    const int64_t P = p.page_size;
    const int64_t src_t = compact_source(p, i);
    const int64_t src_pg = p.old_pt[src_t / P];
    const int64_t dst_pg = p.free_stack[p.free_top - 1 - i / P];
    if (b == 0 && h == 0 && dq == 0 && i % P == 0) {
        p.new_pt[i / P] = dst_pg;
        // the new pages (from the free stack) hold every sequence in its own row
        if (p.row_map)
            for (int64_t bb = 0; bb < p.B; ++bb) p.row_map[dst_pg * p.B + bb] = (int32_t)bb;
    }
    int64_t src_row = b;
    if (p.row_map) {
        const int64_t r = p.row_map[src_pg * p.B + b];
        if (r >= 0 && r < p.B) src_row = r;
    }
    const int64_t so = src_row * p.stride_b + h * p.stride_h + src_pg * p.stride_p + (src_t % P) * p.stride_t;
    const int64_t dof = b * p.stride_b + h * p.stride_h + dst_pg * p.stride_p + (i % P) * p.stride_t;
    const int eb = elt_bytes(p.dtype);
    for (int64_t e = dq * 4; e < min(D, dq * 4 + 4); ++e) {
        if (eb == 4) {
            static_cast<float*>(p.k)[dof + e] = static_cast<const float*>(p.k)[so + e];
            static_cast<float*>(p.v)[dof + e] = static_cast<const float*>(p.v)[so + e];
        } else {
            static_cast<uint16_t*>(p.k)[dof + e] = static_cast<const uint16_t*>(p.k)[so + e];
            static_cast<uint16_t*>(p.v)[dof + e] = static_cast<const uint16_t*>(p.v)[so + e];
        }
    }
    if (h == 0 && dq == 0) {
        p.sal[dst_pg * p.sal_stride_p + b * p.sal_stride_b + i % P] =
            p.sal[src_pg * p.sal_stride_p + b * p.sal_stride_b + src_t % P];
    }
}

__global__ void release_kernel(const int64_t* pages, int64_t n, int64_t* free_stack, int64_t top) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < n) free_stack[top + i] = pages[i];
}

// ------------------------------------------------------------------------------------------
// Materialise contiguous [B, Hkv, N, D] rows (and [B, N] salience) from the paged layout.
// ------------------------------------------------------------------------------------------
__global__ void gather_kernel(GatherParams p) {
    int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t total = p.B * p.Hkv * p.N * p.D;
    if (gid >= total) return;
    const int64_t d = gid % p.D;
    int64_t r = gid / p.D;
    const int64_t t = r % p.N; r /= p.N;
    const int64_t h = r % p.Hkv;
    const int64_t b = r / p.Hkv;
    TokenMap tm{p.page_table ? p.page_table + b * p.pt_stride_b : nullptr, p.page_size,
                p.stride_p, p.stride_t};
    tm.row_map = p.row_map; tm.batch = p.B; tm.seq = b; tm.stride_b = p.stride_b;
    const int64_t off = b * p.stride_b + h * p.stride_h + tm.offset(t) + d;
    if (elt_bytes(p.dtype) == 4)
        static_cast<float*>(p.dst)[gid] = static_cast<const float*>(p.src)[off];
    else
        static_cast<uint16_t*>(p.dst)[gid] = static_cast<const uint16_t*>(p.src)[off];
    if (p.sal_dst && h == 0 && d == 0) {
        const float* sp = p.sal + (p.page_table ? tm.page_table[t / p.page_size] * p.sal_stride_p +
                                                     b * p.sal_stride_b + t % p.page_size
                                               : b * p.sal_stride_b + t);
        p.sal_dst[b * p.N + t] = *sp;
    }
}

// ------------------------------------------------------------------------------------------
// Batch reindex of the pool's live slots (razorkv/cache.py:198-229: batch_repeat_interleave,
// batch_select_indices and reorder_cache index_select the batch dimension of every layer's
// K, V and salience).  Only the slots the page tables reference are listed, so the bytes
// moved are those of the retained pages, not of the whole pool.  A work item is (listed slot,
// chunk of one pool's row); each CTA walks items with a grid stride.  For an item it reads
// the chunk of source row index[b] of every moving destination row b into shared memory and
// then writes the staged chunks, so with src == dst the rows are permuted in place.  In
// place, a row whose index is its own does not move: a beam that keeps its own history costs
// nothing, and a call whose rows all stay returns at once.
// ------------------------------------------------------------------------------------------
constexpr int kReindexThreads = 256;
constexpr int kReindexSmem = 48 * 1024;   // per CTA: moving-row lists + staged chunks

// two (destination, source) row lists: the salience's, and the K/V rows of a moved slot
__host__ __device__ inline int64_t reindex_list_bytes(int64_t dst_B) {
    return ((dst_B * 16 + 15) / 16) * 16;
}

// Moving rows in ascending destination order: act_dst[j] <- act_src[j]; returns their count
// (the same in every thread; all threads must call it).  slot < 0: rows index[b] (the
// salience, or K and V without a row map); slot >= 0: the physical K/V rows of that slot,
// row_map[slot][index[b]].  In place, a row that would copy onto itself is left out.
__device__ int reindex_lists(const ReindexParams& p, int64_t slot, int* act_dst, int* act_src,
                             int* warp_count, bool report) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int n = 0;
    for (int b0 = 0; b0 < p.dst_B; b0 += kReindexThreads) {
        const int b = b0 + threadIdx.x;
        int src = -1;
        if (b < p.dst_B) {
            int64_t s = p.index[b];
            const bool bad = s < 0 || s >= p.src_B;
            if (bad && report) atomicExch(p.err, 2);
            // a bad index leaves the sequence as it was: through a row map its own row moves
            // into row b (the slot's map becomes identity), without one nothing moves
            const bool keep = bad && slot >= 0 && b < p.src_B;
            if (keep) s = b;
            if (!bad || keep) {
                int64_t r = s;
                if (slot >= 0) {
                    const int64_t m = p.row_map[slot * p.src_B + s];
                    if (m >= 0 && m < p.src_B) r = m;
                }
                if (!(p.in_place && r == b)) src = (int)r;
            }
        }
        const unsigned ballot = __ballot_sync(0xffffffffu, src >= 0);
        if (lane == 0) warp_count[warp] = __popc(ballot);
        __syncthreads();
        int before = 0, all = 0;
        for (int w = 0; w < kReindexThreads / 32; ++w) {
            before += w < warp ? warp_count[w] : 0;
            all += warp_count[w];
        }
        if (src >= 0) {
            const int pos = n + before + __popc(ballot & ((1u << lane) - 1u));
            act_dst[pos] = b;
            act_src[pos] = src;
        }
        n += all;
        __syncthreads();
    }
    return n;
}

// Threads split into rows_per_pass groups of lanes_per_row lanes; lane e of a group handles
// vectors e, e + lanes_per_row, ... of its rows, so no element index needs a division.
template <typename T>
__device__ __forceinline__ void reindex_rows(const ReindexParams& p, int which, int64_t slot,
                                             int64_t off, int len, const int* act_dst,
                                             const int* act_src, int n_act, T* stage) {
    const int nv = len / (int)sizeof(T);
    const int cv = (int)(p.chunk / (int64_t)sizeof(T));
    const int lpr = nv < kReindexThreads ? nv : kReindexThreads;
    const int rpp = kReindexThreads / lpr;
    const int my_r = threadIdx.x / lpr;
    const int my_e = threadIdx.x - my_r * lpr;
    const bool on = my_r < rpp;
    const char* sbase = p.src[which] + slot * p.src_slot_stride[which] + off;
    constexpr int U = 8;
    if (on) {
        for (int j0 = my_r; j0 < n_act; j0 += U * rpp) {
            for (int e = my_e; e < nv; e += lpr) {
                T r[U];
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int j = j0 + u * rpp;
                    if (j < n_act)
                        r[u] = reinterpret_cast<const T*>(sbase + act_src[j] * p.src_b_stride[which])[e];
                }
                #pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int j = j0 + u * rpp;
                    if (j < n_act) stage[j * cv + e] = r[u];
                }
            }
        }
    }
    __syncthreads();
    char* dbase = p.dst[which] + slot * p.dst_slot_stride[which] + off;
    if (on) {
        for (int j = my_r; j < n_act; j += rpp) {
            T* drow = reinterpret_cast<T*>(dbase + act_dst[j] * p.dst_b_stride[which]);
            for (int e = my_e; e < nv; e += lpr) drow[e] = stage[j * cv + e];
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kReindexThreads, 4) reindex_kernel(ReindexParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int warp_count[kReindexThreads / 32];
    int* lst_dst = reinterpret_cast<int*>(smem);      // rows by index (salience; K/V unmapped)
    int* lst_src = lst_dst + p.dst_B;
    int* map_dst = lst_src + p.dst_B;                 // K/V rows of one slot through the map
    int* map_src = map_dst + p.dst_B;
    unsigned char* stage = smem + reindex_list_bytes(p.dst_B);
    const int n_lst = reindex_lists(p, -1, lst_dst, lst_src, warp_count, blockIdx.x == 0 && p.err);
    if (n_lst == 0 && (p.row_map == nullptr || p.n_moved == 0)) return;
    // items: every chunk of the first n_moved slots, then the salience chunks of the others
    // (their K/V stay; the row map is rewritten)
    const int64_t ych = p.chunks[0] + p.chunks[1] + p.chunks[2];
    const int64_t items_kv = p.n_moved * ych;
    const int64_t items = items_kv + (p.n_listed - p.n_moved) * p.chunks[2];
    int64_t mapped_slot = -1;   // slot whose mapped lists are in map_dst / map_src
    int n_map = 0;
    for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
        int64_t li, c;
        if (it < items_kv) {
            li = it / ych;
            c = it - li * ych;
        } else {
            const int64_t r = it - items_kv;
            li = p.n_moved + r / p.chunks[2];
            c = p.chunks[0] + p.chunks[1] + r % p.chunks[2];
        }
        const int64_t slot = p.slots[li];
        if (slot < 0 || slot >= p.num_slots) {
            if (threadIdx.x == 0 && p.err) atomicExch(p.err, 2);
            continue;
        }
        int which = 0;
        while (which < 2 && c >= p.chunks[which]) { c -= p.chunks[which]; ++which; }
        const int* ad = lst_dst;
        const int* as = lst_src;
        int n = n_lst;
        if (which < 2 && p.row_map) {
            if (slot != mapped_slot) {
                n_map = reindex_lists(p, slot, map_dst, map_src, warp_count, false);
                mapped_slot = slot;
            }
            ad = map_dst; as = map_src; n = n_map;
        }
        if (n == 0) continue;
        const int64_t off = c * p.chunk;
        const int len = (int)min(p.chunk, p.row_bytes[which] - off);
        reindex_rows<T>(p, which, slot, off, len, ad, as, n, reinterpret_cast<T*>(stage));
        __syncthreads();   // the next item restages
    }
}

// In-place rewrite of the listed slots' row map after their rows were reindexed: moved slots
// (the first n_moved) now hold sequence b in row b; the others keep their K/V and map
// sequence b to the row sequence index[b] used.  A CTA takes a slot at a time, reads all of
// its new entries before writing any.
__global__ void __launch_bounds__(256) row_map_compose_kernel(int32_t* row_map, int64_t B,
                                                               const int64_t* index,
                                                               const int64_t* slots,
                                                               int64_t n_listed, int64_t n_moved,
                                                               int64_t num_slots) {
    extern __shared__ int32_t nrow[];
    for (int64_t li = blockIdx.x; li < n_listed; li += gridDim.x) {
        const int64_t slot = slots[li];
        if (slot < 0 || slot >= num_slots) continue;
        int32_t* m = row_map + slot * B;
        for (int64_t b = threadIdx.x; b < B; b += blockDim.x) {
            const int64_t s = index[b];
            nrow[b] = li < n_moved ? (int32_t)b : (s >= 0 && s < B) ? m[s] : m[b];
        }
        __syncthreads();
        for (int64_t b = threadIdx.x; b < B; b += blockDim.x) m[b] = nrow[b];
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------
// Salience update of a head-sharded step (razorkv/cache.py:239-247 and :282-287 once the
// ranks' partial results are combined): the exchange block holds, after the MAX over the
// ranks of the head group, every token's resonance key (max over all query heads) and the
// appended tokens' norms of every kv head.  New tokens start from the mean norm (sequential
// fp32 sum over kv heads, one division) or 1.0; scored tokens take the EWMA.
// ------------------------------------------------------------------------------------------
__global__ void apply_kernel(ApplyParams p) {
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t b = blockIdx.y;
    const int64_t end = max(p.score_tokens, p.new_first + p.n_new);
    if (t >= end) return;
    const int32_t* xr = p.xc.x + b * p.xc.stride_b;
    float* sp = p.sal + (p.page_table ? p.page_table[t / p.page_size] * p.sal_stride_p +
                                            b * p.sal_stride_b + t % p.page_size
                                      : b * p.sal_stride_b + t);
    const bool is_new = t >= p.new_first && t < p.new_first + p.n_new;
    float old;
    if (is_new) {
        old = 1.0f;
        if (p.norm_init) {
            const int32_t* nr = xr + p.xc.norm_off + (t - p.new_first) * p.xc.htot;
            float acc = 0.0f;
            for (int h = 0; h < p.xc.htot; ++h) acc = __fadd_rn(acc, key_to_float(ordered_of(nr[h])));
            old = __fdiv_rn(acc, (float)p.xc.htot);
        }
    } else {
        old = *sp;
    }
    if (t < p.score_tokens) {
        const float R = key_to_float(ordered_of(xr[t]));
        *sp = __fadd_rn(__fmul_rn(p.decay, old), __fmul_rn(p.one_minus_decay, R));
    } else if (is_new) {
        *sp = old;
    }
}

// ------------------------------------------------------------------------------------------
// The same update when the ranks' shares arrived by peer stores (KV-head sharding over
// NVLink): this rank's region holds one sub-block per rank, and every rank's decode kernel
// releases its flag here once its stores are out.  Thread 0 of each CTA waits (bounded) for
// every flag to reach the epoch; then every thread acquires the flags itself and reads the
// MAX over the sub-blocks.  On timeout the CTA records error 1 and leaves the salience alone.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void apply_peer_kernel(PeerApplyParams p) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        bool ok = true;
        const long long t0 = clock64();
        for (int r = 0; r < p.nranks && ok; ++r) {
            while ((int32_t)(ld_acquire_sys_u32(p.flags + r) - p.epoch) < 0) {
                if (clock64() - t0 > p.wait_limit) { ok = false; break; }
            }
        }
        if (!ok && p.err) atomicExch(p.err, 1);
        s_ok = ok ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok) return;
    for (int r = 0; r < p.nranks; ++r) (void)ld_acquire_sys_u32(p.flags + r);
    const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t b = blockIdx.y;
    const int64_t end = max(p.score_tokens, p.new_first + p.n_new);
    if (t >= end) return;
    const int32_t* base = p.region + p.buf_off + b * p.stride_b;
    float* sp = p.sal + (p.page_table ? p.page_table[t / p.page_size] * p.sal_stride_p +
                                            b * p.sal_stride_b + t % p.page_size
                                      : b * p.sal_stride_b + t);
    const bool is_new = t >= p.new_first && t < p.new_first + p.n_new;
    float old;
    if (is_new) {
        old = 1.0f;
        if (p.norm_init) {
            const int64_t nb = p.norm_off + (t - p.new_first) * p.htot;
            float acc = 0.0f;
            for (int h = 0; h < p.htot; ++h) {
                int32_t k = INT32_MIN;
                for (int r = 0; r < p.nranks; ++r) k = max(k, base[r * p.sub + nb + h]);
                acc = __fadd_rn(acc, key_to_float(ordered_of(k)));
            }
            old = __fdiv_rn(acc, (float)p.htot);
        }
    } else {
        old = *sp;
    }
    if (t < p.score_tokens) {
        int32_t k = INT32_MIN;
        for (int r = 0; r < p.nranks; ++r) k = max(k, base[r * p.sub + t]);
        *sp = __fadd_rn(__fmul_rn(p.decay, old), __fmul_rn(p.one_minus_decay, key_to_float(ordered_of(k))));
    } else if (is_new) {
        *sp = old;
    }
}

// ------------------------------------------------------------------------------------------
// launchers
// ------------------------------------------------------------------------------------------
cudaError_t launch_apply_peer(const PeerApplyParams& p, cudaStream_t st) {
    const int64_t end = p.score_tokens > p.new_first + p.n_new ? p.score_tokens : p.new_first + p.n_new;
    if (end <= 0 || p.B <= 0) return cudaSuccess;
    dim3 grid((unsigned)((end + 255) / 256), (unsigned)p.B);
    apply_peer_kernel<<<grid, 256, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_apply(const ApplyParams& p, cudaStream_t st) {
    const int64_t end = p.score_tokens > p.new_first + p.n_new ? p.score_tokens : p.new_first + p.n_new;
    if (end <= 0 || p.B <= 0) return cudaSuccess;
    dim3 grid((unsigned)((end + 255) / 256), (unsigned)p.B);
    apply_kernel<<<grid, 256, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}
cudaError_t launch_score(const ScoreParams& p, cudaStream_t st) {
    ScoreParams q = p;
    const int rows = (q.Hq / q.Hkv) * q.QL;
    const int max_rows = (48 * 1024) / (q.D * 4);
    q.rows_per_chunk = rows < max_rows ? rows : max_rows;
    dim3 grid((unsigned)((q.N + kScoreTokens - 1) / kScoreTokens), (unsigned)q.B);
    if (q.N == 0) return cudaSuccess;
    score_kernel<<<grid, kScoreThreads, q.rows_per_chunk * q.D * sizeof(float), st>>>(q);
    return counted(cudaGetLastError(), 1);
}

int attn_num_splits(int64_t N, int64_t B, int64_t Hkv, int64_t rows) {
    // aim for ~4 CTAs per SM over 148 SMs; at least 16 tokens per split
    int64_t ctas = B * Hkv * ((rows + kAttnWarps - 1) / kAttnWarps);
    if (ctas <= 0) return 1;
    int64_t want = (148 * 4 + ctas - 1) / ctas;
    int64_t maxs = (N + 15) / 16;
    if (want > maxs) want = maxs;
    if (want < 1) want = 1;
    if (want > 256) want = 256;
    return (int)want;
}

size_t attn_workspace_floats(int64_t B, int64_t Hq, int64_t QL, int64_t D, int splits) {
    return (size_t)splits * B * Hq * QL * (D + 2);
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t st) {
    const int rows = (p.Hq / p.Hkv) * p.QL;
    dim3 grid((unsigned)p.num_splits, (unsigned)(p.B * p.Hkv),
              (unsigned)((rows + kAttnWarps - 1) / kAttnWarps));
    attn_split_kernel<<<grid, kAttnWarps * 32, 0, st>>>(p);
    cudaError_t e = counted(cudaGetLastError(), 1);
    if (e != cudaSuccess) return e;
    merge_kernel<<<(unsigned)(p.B * p.Hq * p.QL), 128, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_pool(const float* sal, int64_t B, int64_t S, int64_t stride_b, int64_t P,
                        int mean, float* out, cudaStream_t st) {
    int64_t n_pages = S / P;
    if (n_pages == 0) n_pages = 1;
    int64_t total = B * n_pages;
    if (total == 0) return cudaSuccess;
    pool_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(sal, B, S, stride_b, P, n_pages,
                                                                 mean, out);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_page_scores(const PageScoreParams& p, cudaStream_t st) {
    if (p.num_pages == 0 || p.B == 0) return cudaSuccess;
    dim3 grid((unsigned)((p.num_pages + 255) / 256), (unsigned)p.B);
    page_scores_kernel<<<grid, 256, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_select(const float* scores, int64_t B, int64_t n, int64_t k, int64_t* kept,
                          float* margin, uint32_t* keys, cudaStream_t st) {
    select_kernel<<<1, kSelThreads, 0, st>>>(scores, B, n, k, kept, margin, keys);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_select_compact(const float* scores, int64_t B, int64_t num_pages, int64_t k,
                                  int64_t* kept, float* margin, uint32_t* keys, int64_t* pt,
                                  int64_t sink_pages, int64_t tail_first, int64_t n_total,
                                  int64_t* free_stack, int64_t free_top, cudaStream_t st) {
    select_compact_kernel<<<1, kSelThreads, 0, st>>>(scores, B, num_pages, k, kept, margin, keys,
                                                       pt, sink_pages, tail_first, n_total,
                                                       free_stack, free_top);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_compact_pages(int64_t* pt, int64_t sink_pages, int64_t num_pages,
                                 const int64_t* kept, int64_t k, int64_t tail_first,
                                 int64_t n_total, int64_t* free_stack, int64_t free_top,
                                 cudaStream_t st) {
    compact_pages_kernel<<<1, 1024, 0, st>>>(pt, sink_pages, num_pages, kept, k, tail_first,
                                             n_total, free_stack, free_top);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_append(const AppendParams& p, cudaStream_t st) {
    const int64_t items = p.n_new * p.B;
    if (items == 0) return cudaSuccess;
    const int ipc = p.Hkv >= kAppendGroups ? 1 : kAppendGroups / p.Hkv;
    const size_t smem = (size_t)ipc * p.Hkv * sizeof(float);
    append_kernel<<<(unsigned)((items + ipc - 1) / ipc), kAppendThreads, smem, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_compact_tokens(const CompactTokensParams& p, cudaStream_t st) {
    int64_t total = p.new_len * p.B * p.Hkv * ((p.D + 3) / 4);
    if (total == 0) return cudaSuccess;
    compact_tokens_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_release(const int64_t* pages, int64_t n, int64_t* free_stack, int64_t top,
                           cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    release_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(pages, n, free_stack, top);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_gather(const GatherParams& p, cudaStream_t st) {
    int64_t total = p.B * p.Hkv * p.N * p.D;
    if (total == 0) return cudaSuccess;
    gather_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

int64_t reindex_chunk_bytes(int64_t dst_B, int64_t max_row_bytes, int vec) {
    if (dst_B < 1) return 0;
    const int64_t avail = (kReindexSmem - reindex_list_bytes(dst_B)) / dst_B;
    if (avail < vec) return 0;
    int64_t chunk = vec;
    while (chunk * 2 <= avail) chunk *= 2;
    const int64_t row = (max_row_bytes + vec - 1) / vec * vec;
    return chunk < row ? chunk : row;
}

cudaError_t launch_row_map_compose(int32_t* row_map, int64_t B, const int64_t* index,
                                   const int64_t* slots, int64_t n_listed, int64_t n_moved,
                                   int64_t num_slots, cudaStream_t st) {
    if (n_listed == 0 || B == 0) return cudaSuccess;
    const int64_t ctas = n_listed < 4096 ? n_listed : 4096;
    row_map_compose_kernel<<<(unsigned)ctas, 256, (size_t)(B * 4), st>>>(
        row_map, B, index, slots, n_listed, n_moved, num_slots);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_reindex(const ReindexParams& p, cudaStream_t st) {
    const int64_t items = p.n_moved * (p.chunks[0] + p.chunks[1] + p.chunks[2]) +
                          (p.n_listed - p.n_moved) * p.chunks[2];
    if (items == 0 || p.dst_B == 0) return cudaSuccess;
    const size_t smem = (size_t)(reindex_list_bytes(p.dst_B) + p.dst_B * p.chunk);
    void (*kern)(ReindexParams) = p.vec == 16 ? reindex_kernel<uint4>
                                  : p.vec == 4 ? reindex_kernel<uint32_t>
                                               : reindex_kernel<uint16_t>;
    // one resident wave: every CTA walks its items until the list ends
    int dev = 0, sms = 148, per_sm = 1;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kReindexThreads, smem) !=
            cudaSuccess || per_sm < 1)
        per_sm = 1;
    int64_t ctas = (int64_t)sms * per_sm;
    if (ctas > items) ctas = items;
    kern<<<(unsigned)ctas, kReindexThreads, smem, st>>>(p);
    return counted(cudaGetLastError(), 1);
}

}  // namespace rkv
