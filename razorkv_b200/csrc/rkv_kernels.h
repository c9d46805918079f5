// Kernel parameter blocks and launchers shared by the C-ABI layer (rkv_capi.cu) and the
// kernel translation units.  Internal to the library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rkv {

// Library-wide count of kernel launches (reported by rkv_launch_count()).
void count_launches(int n);
inline cudaError_t counted(cudaError_t e, int n) {
    if (e == cudaSuccess) count_launches(n);
    return e;
}

// Exchange block of head-sharded scoring (see rkv_exchange in the public header): signed
// keys x[b * stride_b + t] of the resonance, x[b * stride_b + norm_off + i * htot + h] of the
// kv-head norms of the i-th appended token.  x == nullptr: the salience is updated in place.
struct Exchange {
    int32_t* x; int64_t stride_b, norm_off; int h0, htot;
    // peer exchange (regions != nullptr): instead of x, write into region r + buf_off +
    // rank * sub of every rank r (peer memory over NVLink; r == rank is local), then the last
    // CTA releases flags[r][rank] = epoch on every rank
    int32_t* const* regions; uint32_t* const* flags;
    int rank, nranks; int64_t sub, buf_off; uint32_t epoch;
};

// rkv_salience_apply_peer: as ApplyParams, the exchange block being the max over the nranks
// sub-blocks of this rank's region once every rank's flag has reached the epoch.
struct PeerApplyParams {
    float* sal; int64_t sal_stride_b, sal_stride_p;
    const int64_t* page_table; int64_t page_size; int64_t B;
    const int32_t* region; const uint32_t* flags; int nranks; int64_t sub, buf_off;
    uint32_t epoch; int64_t stride_b, norm_off; int htot;
    int64_t score_tokens, new_first, n_new;
    int norm_init; float decay, one_minus_decay;
    int* err; long long wait_limit;
};

// Signed key of an fp32 value: the order-preserving uint32 key with its top bit flipped, so
// that int32 MAX (an all-reduce MAX over ranks) orders like the floats.  INT32_MIN = absent.
__host__ __device__ inline int32_t signed_key_of(uint32_t ordered) {
    return (int32_t)(ordered ^ 0x80000000u);
}
__host__ __device__ inline uint32_t ordered_of(int32_t signed_key) {
    return (uint32_t)signed_key ^ 0x80000000u;
}

struct ScoreParams {
    const void* q; int q_dtype; int64_t q_stride_b, q_stride_h, q_stride_t;
    int Hq, QL;
    const void* k; int kv_dtype; int D; int Hkv; int64_t B, N;
    int64_t stride_b, stride_h, stride_p, stride_t, page_size;
    const int64_t* page_table; int64_t pt_stride_b;
    float* sal; int64_t sal_stride_b, sal_stride_p;
    float scale_r, decay, one_minus_decay; int ewma;
    int rows_per_chunk;
    Exchange xc;   // x != nullptr: write keys, leave the salience
    const int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map)
};

struct AttnParams {
    const void* q; int q_dtype; int64_t q_stride_b, q_stride_h, q_stride_t;
    int Hq, QL;
    const void* k; const void* v; int kv_dtype; int D; int Hkv; int64_t B, N;
    int64_t stride_b, stride_h, stride_p, stride_t, page_size;
    const int64_t* page_table; int64_t pt_stride_b; int64_t num_slots;
    float scale; int causal;
    void* out; int out_dtype; int64_t o_stride_b, o_stride_h, o_stride_t;
    float* workspace; int num_splits;
    const int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map)
};

struct PageScoreParams {
    const float* sal; int64_t sal_stride_b, sal_stride_p;
    const int64_t* page_table; int64_t page_size;
    int64_t B, first_token, num_pages, sel_page_size;
    float* scores;
};

struct AppendParams {
    void* k; void* v; int dtype; int D; int Hkv; int64_t B;
    int64_t stride_b, stride_h, stride_p, stride_t, page_size;
    float* sal; int64_t sal_stride_b, sal_stride_p;
    const void* k_new; const void* v_new; int64_t new_stride_b, new_stride_h, new_stride_t;
    int64_t n_new, pos;
    int64_t* page_table; const int64_t* free_stack; int64_t free_top;
    int salience_init;
    int vec_ok;   // every row 16-byte aligned and D a whole number of 16-byte chunks
    Exchange xc;  // x != nullptr: write the new tokens' kv-head norms, leave the salience
    int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map); slots taken
                        // from the free stack get identity entries
};

// rkv_salience_apply: the salience update of a head-sharded step from the reduced exchange.
struct ApplyParams {
    float* sal; int64_t sal_stride_b, sal_stride_p;
    const int64_t* page_table; int64_t page_size; int64_t B;
    Exchange xc;
    int64_t score_tokens, new_first, n_new;
    int norm_init; float decay, one_minus_decay;
};

struct CompactTokensParams {
    void* k; void* v; int dtype; int64_t D, Hkv, B;
    int64_t stride_b, stride_h, stride_p, stride_t, page_size;
    float* sal; int64_t sal_stride_b, sal_stride_p;
    const int64_t* old_pt; int64_t* new_pt; const int64_t* free_stack; int64_t free_top;
    int64_t new_len, sink, n_kept, sel_page_size, hay_start, tail_src_start;
    const int64_t* kept;
    int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map); slots taken
                        // from the free stack get identity entries
};

struct GatherParams {
    const void* src; void* dst; int dtype; int64_t B, Hkv, N, D;
    int64_t stride_b, stride_h, stride_p, stride_t, page_size;
    const int64_t* page_table; int64_t pt_stride_b;
    const float* sal; int64_t sal_stride_b, sal_stride_p; float* sal_dst;
    const int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map)
};

// Batch reindex of listed pool slots (K, V, salience): row b of dst <- row index[b] of src.
// A "row" is the bytes of one (slot, sequence) plane of a pool; strides are in bytes.
struct ReindexParams {
    const char* src[3]; char* dst[3];
    int64_t src_slot_stride[3], src_b_stride[3];
    int64_t dst_slot_stride[3], dst_b_stride[3];
    int64_t row_bytes[3];
    int64_t chunks[3];          // chunks of `chunk` bytes per row of each pool
    int64_t chunk;
    int64_t src_B, dst_B, num_slots;
    const int64_t* index;       // [dst_B]
    const int64_t* slots; int64_t n_listed;
    int* err;                   // optional: 2 on a slot or index out of range
    int in_place;               // src == dst: rows that would copy onto themselves are skipped
    int vec;                    // bytes per access: 16, 4 or 2
    // source row map ([slots][src_B] int32, nullptr = identity): row b of dst <- physical row
    // row_map[slot][index[b]] of src.  Only the first n_moved listed slots move their K and V;
    // the salience of every listed slot moves.
    const int32_t* row_map;
    int64_t n_moved;
};

// Fused score + attention for the sm_100a fast path (rkv_decode_sm100.cu).
struct FusedParams {
    const void* q; int64_t q_stride_b, q_stride_h;
    int Hq, Hkv, D, dtype; int64_t B, N;
    const void* k; const void* v;
    int64_t stride_b, stride_h, stride_p, stride_t, num_slots;
    const int64_t* page_table; int64_t pt_stride_b;
    float* sal; int64_t sal_stride_b, sal_stride_p;   // nullptr: attention only
    float scale_r, logit_mul, decay, one_minus_decay;
    int attend;                                        // 0: score only (no V, no output)
    void* out; int64_t o_stride_b, o_stride_h;
    float* partials; int* counters; int* err;   // workspace body / header (nullptr: score only)
    // fused append of one new token at position N - 1 (k_new == nullptr: no append)
    const void* k_new; const void* v_new; int64_t new_stride_b, new_stride_h;
    int64_t* pt_w; const int64_t* free_stack; int64_t free_top; int sal_init_norm;
    // a second (attention) query: q scores, q2 attends (q2 == nullptr: q does both)
    const void* q2; int64_t q2_stride_b, q2_stride_h;
    // tokens at or past score_n keep their salience (has_score_n == 0: all are scored)
    int has_score_n; int64_t score_n;
    // head-sharded (partial) scoring: instead of updating the salience, write the signed
    // resonance keys of the local heads and the appended token's kv-head norms here
    Exchange xc;
    // score-only pass of a compacting step: page scores [B][pool_num] (row stride pool_num)
    // of logical pages pool_first .. pool_first + pool_num - 1 (pool == nullptr: none)
    float* pool; int64_t pool_first, pool_num;
    int32_t* row_map;   // optional pool row map (rkv_kv_layout.row_map); slots taken
                        // from the free stack get identity entries
};

cudaError_t launch_score(const ScoreParams& p, cudaStream_t st);
int attn_num_splits(int64_t N, int64_t B, int64_t Hkv, int64_t rows);
size_t attn_workspace_floats(int64_t B, int64_t Hq, int64_t QL, int64_t D, int splits);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t st);
cudaError_t launch_pool(const float* sal, int64_t B, int64_t S, int64_t stride_b, int64_t P,
                        int mean, float* out, cudaStream_t st);
cudaError_t launch_page_scores(const PageScoreParams& p, cudaStream_t st);
cudaError_t launch_select(const float* scores, int64_t B, int64_t n, int64_t k, int64_t* kept,
                          float* margin, uint32_t* keys, cudaStream_t st);
cudaError_t launch_select_compact(const float* scores, int64_t B, int64_t num_pages, int64_t k,
                                  int64_t* kept, float* margin, uint32_t* keys, int64_t* pt,
                                  int64_t sink_pages, int64_t tail_first, int64_t n_total,
                                  int64_t* free_stack, int64_t free_top, cudaStream_t st);
cudaError_t launch_compact_pages(int64_t* pt, int64_t sink_pages, int64_t num_pages,
                                 const int64_t* kept, int64_t k, int64_t tail_first,
                                 int64_t n_total, int64_t* free_stack, int64_t free_top,
                                 cudaStream_t st);
cudaError_t launch_append(const AppendParams& p, cudaStream_t st);
cudaError_t launch_compact_tokens(const CompactTokensParams& p, cudaStream_t st);
cudaError_t launch_release(const int64_t* pages, int64_t n, int64_t* free_stack, int64_t top,
                           cudaStream_t st);
cudaError_t launch_gather(const GatherParams& p, cudaStream_t st);
// chunk size for a reindex into dst_B rows (0: dst_B too large for the staging buffer)
int64_t reindex_chunk_bytes(int64_t dst_B, int64_t max_row_bytes, int vec);
cudaError_t launch_reindex(const ReindexParams& p, cudaStream_t st);
// rewrites the row map of listed slots in place: the first n_moved get identity entries,
// the rest row_map[s][b] <- row_map[s][index[b]] (entries with an index outside [0, B) stay)
cudaError_t launch_row_map_compose(int32_t* row_map, int64_t B, const int64_t* index,
                                   const int64_t* slots, int64_t n_listed, int64_t n_moved,
                                   int64_t num_slots, cudaStream_t st);
cudaError_t launch_apply(const ApplyParams& p, cudaStream_t st);
cudaError_t launch_apply_peer(const PeerApplyParams& p, cudaStream_t st);

// fast path: returns cudaErrorNotSupported when the shape is outside its coverage
bool fused_supported(int dtype, int D, int Hkv, int Hq, int64_t page_size, int64_t stride_t,
                     int64_t stride_h, int64_t stride_b, int64_t stride_p, const void* k,
                     const void* v);
size_t fused_workspace_bytes(int64_t B, int Hq, int Hkv, int D, int64_t N);
cudaError_t launch_fused(const FusedParams& p, cudaStream_t st);
cudaError_t launch_wait_selftest(int* result, long long limit, cudaStream_t st);

}  // namespace rkv
