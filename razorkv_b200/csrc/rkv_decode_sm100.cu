// sm_100a decode kernel: salience scoring and split-K paged attention in one pass over K.
//
// Work decomposition (stream-K over pages).  A *tile* is one 16-token page of one sequence
// across all kv heads.  The B * ceil(N/16) tiles, sequence-major, are cut into equal
// contiguous ranges, one per CTA (at most one CTA per SM, so every SM streams the same
// number of bytes whatever B and N are).  A range that crosses a sequence boundary is
// processed as one *segment* per sequence.
//
// CTA = 8 compute warps + 1 producer warp + 1 salience finisher warp (when scoring).
//   producer : one lane walks the CTA's tiles, reads the page table and issues 5-D TMA tile
//              loads (128-byte swizzle, no multicast) of K and V for all kv heads of up to
//              8/Hkv tiles per pipeline stage into an NS-deep shared-memory ring.
//   finisher : folds the compute warps' per-token maxima over the kv heads, applies the
//              EWMA and stores the salience; the stage is released once it is done too.
//   compute  : warp w serves kv head h = w % Hkv of tile slot s = w / Hkv of every stage,
//              i.e. GQA packing: each K/V page is read from HBM once and used by the G query
//              heads of its kv head.
//
// Per tile a compute warp
//   1. computes the 16 x G scores q.k in fp32 on CUDA cores in the canonical order shared
//      with the CPU oracle (lane j of an 8-lane group owns the 16-byte chunks j, j+8 of the K
//      row; fused multiply-adds from +0.0f; xor-4/2/1 butterfly), so salience is bit-exact;
//   2. (score) takes the max over its heads per token and stores it as an ordered key in
//      shared memory (plain stores, no atomics); the finisher takes the max over the Hkv
//      keys of each token and applies S = fl(fl(d*S) + fl((1-d)*R)) to its salience in HBM;
//   3. (attend) runs the online softmax in the log2 domain with warp shuffles, stores the
//      probabilities as bf16/fp16 and accumulates P.V with mma.sync m16n8k16 (Vt as the A
//      operand straight from the swizzled stage via ldmatrix.trans, P^T as B).
// At the end of a segment every warp writes its (m, l, acc) partial; merge_kernel, launched
// right after on the same stream, combines the partials of each (sequence, head) by
// log-sum-exp with one CTA per row, so no SM sits in a serial merge tail.  Tokens past N in
// the last page are masked and their V rows zeroed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <math.h>

#include <mutex>
#include <type_traits>

#include "rkv_common.cuh"
#include "rkv_kernels.h"
#include "rkv_sm100.cuh"

namespace rkv {
namespace sm100 {

constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = kComputeWarps * 32;
// Three warpgroups: two of compute warps and one whose first warp is the producer.  The
// launch gives every thread 168 registers (384 x 168 = 64512); setmaxnreg then moves them to
// the compute warpgroups: 256 x 224 + 128 x 56 = 64512, and per SM sub-partition (one warp
// of each warpgroup) 2 x 32 x 224 + 32 x 56 = 16128 <= 16384.
constexpr int kThreads = kComputeThreads + 128;
constexpr int kComputeRegs = 224;
constexpr int kProducerRegs = 56;
constexpr int kTileTokens = 16;
constexpr int kMaxStages = 6;
constexpr int kSmemBudget = 192 * 1024;   // stage ring (3 x 64 KB or 6 x 32 KB stages)
constexpr float kRescaleLog2 = 8.0f;      // lazy softmax rescale threshold (log2 units)
constexpr int kQRowPitch = 128;           // elements between the query rows staged in smem

struct DevArgs {
    const void* q; int64_t q_stride_b, q_stride_h;
    int Hq, Hkv, G, wph;
    // stream-K positions: sequence b owns positions [b * seq_pos, (b + 1) * seq_pos); the
    // first lead of them are empty (they stand for the fixed cost of starting a sequence in a
    // CTA), tile t of b sits at b * seq_pos + lead + t
    int64_t B, N, n_tiles, total, W, maxc, seq_pos, lead;
    // partials per CTA and row: wph, or 1 when the tile slots' partials are folded inside
    // the CTA first (one-sequence launches of the tensor-core-logit instances)
    int pw;
    const int64_t* pt; int64_t pt_stride_b; int64_t num_slots;
    // pool row map [num_slots][B] (nullptr: sequence b in row b); the appended token's page
    // maps every sequence to its own row
    int32_t* row_map;
    float* sal; int64_t sal_stride_b, sal_stride_p;
    float scale_r, logit_log2, decay, omd;
    int attend, score, sal_bulk;
    void* out; int64_t o_stride_b, o_stride_h;
    float* partials; int* counters; int* err;
    int stages, stage_bytes, tile_bytes, kv_tile_bytes, half_bytes;
    int role[3];   // tensor-map dims 2..4 in stride order: 0 = kv head, 1 = sequence, 2 = page slot
    // fused append of the token at position N - 1 (k_new == nullptr: none)
    const void* k_new; const void* v_new; int64_t new_stride_b, new_stride_h;
    int64_t* pt_w; const int64_t* free_stack; int64_t free_top; int sal_init_norm;
    void* kpool; void* vpool; int64_t stride_b, stride_h, stride_p, stride_t;
    // MODE 1 / 2: attention query (tensor-core logits) and its log2-domain logit scale;
    // tokens at or past score_n keep their salience (MODE 2 scores the tokens before it)
    const void* q2; int64_t q2_stride_b, q2_stride_h;
    float attn_log2; int64_t score_n;
    Exchange xc;   // head-sharded scoring: keys and norms go here, the salience is left alone
    // MODE 4: page scores [B][pool_num] of logical pages pool_first .. pool_first + pool_num - 1
    float* pool; int64_t pool_first, pool_num;
};

struct SmemTail {             // placed after the stage ring
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t scored[kMaxStages];   // every compute warp has stored its resonance keys
    int32_t phys[kMaxStages][kComputeWarps];
    // per compute warp (tile slot s, kv head h) = warp s * Hkv + h: the token's max score
    // over the warp's query heads as an ordered key
    uint32_t red[kMaxStages][kComputeWarps][kTileTokens];
    uint16_t ps[kComputeWarps][8][kTileTokens];   // P (bf16/fp16) per warp: [head][token]
    float alpha[kComputeWarps][8];
    alignas(16) float sal_old[kMaxStages][kComputeWarps][kTileTokens];   // bulk-copied salience rows
    float new_norm[kMaxStages][kComputeWarps][8];   // ||k_h|| of the appended token, per kv head
    int abort;
};

// Screened instances only, after the tail: each compute warp's copy of its kv head's query
// rows (the scoring query, in its own 16-bit type), read by the canonical recompute of
// candidate heads.  The other instances do not allocate it.
struct QRows {
    alignas(16) uint16_t q[kComputeWarps][8][kQRowPitch];
};
// ring + tail + alignment slack within the 227 KB a CTA may use
static_assert(kSmemBudget + sizeof(SmemTail) + sizeof(QRows) + 1024 <= 227 * 1024,
              "shared memory over budget");

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// 8 consecutive 16-bit elements of a 128-bit word -> fp32 (exact).
template <typename T>
__device__ __forceinline__ void unpack8(uint4 w, float* f);
template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(uint4 w, float* f) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(u[i] << 16);
        f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void unpack8<__half>(uint4 w, float* f) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// The same 8 elements as 4 packed (even, odd) fp32 pairs for fma.rn.f32x2.
template <typename T>
__device__ __forceinline__ void unpack8_pairs(uint4 w, uint64_t* p);
template <>
__device__ __forceinline__ void unpack8_pairs<__nv_bfloat16>(uint4 w, uint64_t* p) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
        p[i] = pack2(__uint_as_float(u[i] << 16), __uint_as_float(u[i] & 0xffff0000u));
}
template <>
__device__ __forceinline__ void unpack8_pairs<__half>(uint4 w, uint64_t* p) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        p[i] = pack2(t.x, t.y);
    }
}

// Two 16-bit elements as one 32-bit mma operand register (lo in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack_elems(T lo, T hi) {
    return (uint32_t)*reinterpret_cast<const uint16_t*>(&lo) |
           ((uint32_t)*reinterpret_cast<const uint16_t*>(&hi) << 16);
}

template <typename T>
__device__ __forceinline__ uint16_t to_bits(float x) {
    T v = from_f<T>(x);
    return *reinterpret_cast<uint16_t*>(&v);
}

// Two fp32 values rounded to T and packed (lo in the low half), as to_bits on each.
template <typename T>
__device__ __forceinline__ uint32_t pack_bits(float lo, float hi) {
    return (uint32_t)to_bits<T>(lo) | ((uint32_t)to_bits<T>(hi) << 16);
}

// Transpose-reduce GP per-lane partials over the 8 lanes of a group in the canonical
// xor-4 / xor-2 / xor-1 order.  Returns the full dot of head (j >> (3 - log2 GP)).
template <int GP>
__device__ __forceinline__ float group_transpose_reduce(float (&v)[GP], int j) {
    int n = GP;
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) {
        const bool upper = (j & m) != 0;
        if (n >= 2) {
#pragma unroll
            for (int i = 0; i < GP / 2; ++i) {
                if (i < n / 2) {
                    const float send = upper ? v[i] : v[i + n / 2];
                    const float keep = upper ? v[i + n / 2] : v[i];
                    const float recv = __shfl_xor_sync(0xffffffffu, send, m);
                    v[i] = __fadd_rn(keep, recv);
                }
            }
            n >>= 1;
        } else {
            v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], m));
        }
    }
    return v[0];
}

template <int GP>
__device__ __forceinline__ int head_of_lane(int j) {
    return GP == 8 ? j : GP == 4 ? (j >> 1) : GP == 2 ? (j >> 2) : 0;
}

// Screened resonance (instances with 5-8 query heads per kv head).  The resonance of a token
// is the max over its G query heads of the canonical fp32 dot fl(q*scale_r).k; only the max
// matters.  Every head's dot is first taken on tensor cores (x_h, fp32 accumulate, order not
// specified) together with A_h = |q_h|.|k| from a second mma on the magnitudes.  With
//   E_h = kScreenTol * scale_r * A_h,   kScreenTol = 2^-14,
// |scale_r * x_h - canonical_h| <= E_h holds with a wide margin: the canonical chains round
// at most ~14 times (<= 2^-19.8 relative to scale_r * A_h) and a tensor-core fp32 sum of
// exact bf16/fp16 products stays within a few ulps of its largest partial sum (<= 2^-19
// relative to A_h for 128 terms).  A head h whose upper bound scale_r * x_h + E_h lies below
// LB = max_j (scale_r * x_j - E_j) cannot hold the maximum, since its canonical value is
// below that of the head attaining LB; the canonical dot is computed only for the remaining
// candidates (usually one head), so the resonance is the same bit pattern as the full
// canonical max over all heads.  Non-finite values keep a head a candidate.
constexpr float kScreenTol = 6.103515625e-05f;   // 2^-14
constexpr uint32_t kAbsMask2 = 0x7fff7fffu;       // clears the sign of both bf16/fp16 halves

// Canonical-order dots of four (K row, query head) pairs of the staged page, one per 8-lane
// group (in round r, group g takes K row t[r] and query row hd[r]): lane j of each group owns
// chunk j of every 64-element half of the K row (128-byte swizzled halves at kb) and of the
// query row (rows of kQRowPitch 16-bit elements at qb, scaled to fl(q * scale) here, exactly
// as the canonical order defines); two FMA chains (even / odd
// element positions) from +0.0f; xor-4/2/1 butterfly.  All loads of the four rounds are
// issued first and the four chains and butterflies are interleaved, so the rounds overlap.
// Every lane of a group returns its round's value in v[r].
template <typename T, int D>
__device__ __forceinline__ void canon_dots4(uint32_t kb, int half_bytes, const int (&t)[4],
                                            uint32_t qb, const int (&hd)[4], int j, float scale,
                                            float (&v)[4]) {
    constexpr int HALVES = D / 64;
    uint4 kw[4][HALVES], qw[4][HALVES];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int hf = 0; hf < HALVES; ++hf) {
            kw[r][hf] = lds128(kb + hf * half_bytes + t[r] * 128 + ((j ^ (t[r] & 7)) << 4));
            qw[r][hf] = lds128(qb + (uint32_t)((hd[r] * kQRowPitch + hf * 64 + 8 * j) * 2));
        }
    }
    const uint64_t sc2 = pack2(scale, scale);
    float part[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        uint64_t x = 0ull;   // (+0.0f, +0.0f)
#pragma unroll
        for (int hf = 0; hf < HALVES; ++hf) {
            uint64_t kp[4], qp[4];
            unpack8_pairs<T>(kw[r][hf], kp);
            unpack8_pairs<T>(qw[r][hf], qp);
#pragma unroll
            for (int i = 0; i < 4; ++i) ffma2(x, fmul2(qp[i], sc2), kp[i]);
        }
        part[r] = sum_pair(x);
    }
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) {
#pragma unroll
        for (int r = 0; r < 4; ++r) part[r] = __fadd_rn(part[r], __shfl_xor_sync(0xffffffffu, part[r], m));
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = part[r];
}

// Row of sequence b in the page in slot v: the row map's entry, or b (no map, an id outside
// the pool, or an entry outside [0, B)).
__device__ __forceinline__ int map_row(const DevArgs& a, int64_t v, int64_t b) {
    if (a.row_map == nullptr || v < 0 || v >= a.num_slots) return (int)b;
    const int r = __ldg(a.row_map + v * a.B + b);
    return (r >= 0 && r < a.B) ? r : (int)b;
}

// MODE 0: one query; its canonical-order scores give the resonance and the attention logits.
// MODE 1: attention only; the logits come from mma.sync (K tile x q^T, fp32 accumulate).
// MODE 2: two queries: the canonical-order scores of q (resonance, tokens before score_n)
//         and the mma.sync logits of q2 (attention over all tokens) -- the HF hook path,
//         where the hook scores with the pre-RoPE query and attention uses the post-RoPE one.
// MODE 3: MODE 0 for a rank holding some kv heads of the layer: the resonance keys and the
//         appended token's kv-head norms go to the exchange block, the salience is untouched.
template <typename T, int D, int GP, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
              const DevArgs a) {
    constexpr int HALVES = D / 64;      // 128-byte swizzle boxes per row
    constexpr int EPL = D / 8;          // K elements a lane owns per row
    constexpr int MT = D / 16;          // 16-dim mma row tiles
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    // MODE 3 is MODE 0 whose scoring is partial (head-sharded): the finisher writes the
    // exchange block instead of the salience.  Everything else follows MODE 0.
    constexpr bool XCH = MODE == 3;
    // MODE 4 is MODE 0's score-only pass (no attention) of a compacting decode step: it also
    // appends the new token and its finisher writes the max-pooled page scores of the
    // haystack pages, so selection can follow at once.
    constexpr bool POOL = MODE == 4;
    constexpr int M = (XCH || POOL) ? 0 : MODE;
    // 5-8 query heads per kv head: resonance by the tensor-core screen (see kScreenTol) and
    // attention logits on tensor cores, as in MODE 1
    constexpr bool SCREEN = GP == 8 && M != 1;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    const int NS = a.stages;
    SmemTail& sm = *reinterpret_cast<SmemTail*>(smem + NS * a.stage_bytes);
    QRows& qrows = *reinterpret_cast<QRows*>(smem + NS * a.stage_bytes + sizeof(SmemTail));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&sm.full[s], 1);
            // a stage is free once every compute warp and, when scoring, the salience
            // finisher are done with it
            mbar_init(&sm.empty[s], kComputeWarps + (a.score ? 1 : 0));
            mbar_init(&sm.scored[s], kComputeWarps);
        }
        fence_mbar_init();
    }
    for (int i = threadIdx.x; i < kComputeWarps * 8 * kTileTokens; i += blockDim.x)
        (&sm.ps[0][0][0])[i] = 0;
    for (int i = threadIdx.x; i < kComputeWarps * 8; i += blockDim.x) (&sm.alpha[0][0])[i] = 0.f;
    if (threadIdx.x == 0) sm.abort = 0;

    const int64_t c = blockIdx.x;
    const int64_t r0 = c * a.W;
    const int64_t r1 = min(a.total, r0 + a.W);
    const int wph = a.wph;
    const int Hkv = a.Hkv;

    // Before the wait on the previous kernel: fetch the tensor maps and warm L2 with the
    // pages of the first stage.  Page ids read here may be stale (the previous kernel may
    // still rewrite the table), which only makes a prefetch useless; they bypass L1, and
    // every load that feeds the computation happens after the wait.  Only the first stage:
    // prefetching all NS stages (28 MB over the grid) kept DRAM busy through the wait
    // release, and the page-table and q loads that gate the first TMA queued behind it
    // (first tile ~1 us later per launch).
    if (warp == kComputeWarps && lane == 0) {
        prefetch_tensormap(&tmk);
        if (a.attend) prefetch_tensormap(&tmv);
        if (r0 < r1) {
            const int64_t b = r0 / a.seq_pos;
            const int64_t t_begin = max(r0 - b * a.seq_pos - a.lead, (int64_t)0);
            const int64_t t_seg = max(min(r1, (b + 1) * a.seq_pos) - b * a.seq_pos - a.lead, (int64_t)0);
            const int64_t t_end = min(t_seg, t_begin + (int64_t)wph);
            for (int64_t t = t_begin; t < t_end; ++t) {
                const int64_t v = __ldcg(a.pt + b * a.pt_stride_b + t);
                if (v < 0 || v >= a.num_slots) continue;
                int cc[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) cc[k] = a.role[k] == 0 ? 0 : a.role[k] == 1 ? (int)b : (int)v;
                for (int hf = 0; hf < D / 64; ++hf) {
                    tma_prefetch_l2_5d(&tmk, hf * 64, 0, cc[0], cc[1], cc[2]);
                    if (a.attend) tma_prefetch_l2_5d(&tmv, hf * 64, 0, cc[0], cc[1], cc[2]);
                }
            }
        }
    }
    __syncthreads();
    // Launched with programmatic stream serialization: everything above overlaps the previous
    // kernel's tail; from here on global memory written by earlier work is read, so wait for
    // it.  This kernel never triggers its dependents early: the merge grid then launches only
    // as CTAs exit and spreads over the whole GPU (triggered early, its CTAs piled onto the
    // few SMs the decode grid leaves free and the merge ran on one or two SMs).
    grid_dependency_wait();
    // fused append: the token at position N - 1 is written by this kernel (tile new_tile,
    // row new_row); when new_row == 0 its page is taken from the free stack here
    const bool append = a.k_new != nullptr;
    const int new_tile = (int)((a.N - 1) / kTileTokens);
    const int new_row = (int)((a.N - 1) % kTileTokens);
    const bool app_new_page = append && new_row == 0;

    // ------------------------------------------------------------------- producer warp
    // The whole warp walks the schedule; lanes fetch the page ids of the next 32 tiles
    // together and lane 0 issues the copies of each stage: the K (and V) boxes of every
    // tile and, when scoring, the tile's 16 salience values (one 64-byte bulk copy) so the
    // EWMA update never waits on a global load.
    if (warp >= kComputeWarps) {
        set_max_regs_dec<kProducerRegs>();
        if (warp == kComputeWarps + 1 && a.score) {
            // ---- salience finisher --------------------------------------------------------
            // Folds the compute warps' per-token keys over the kv heads, applies the EWMA
            // and stores the salience, then releases the stage.  Doing this here keeps the
            // cross-warp fold off the compute warps' path: they only store their keys.
            int slot = 0;
            uint32_t par = 0;
            for (int64_t pos = r0; pos < r1;) {
                const int64_t b = pos / a.seq_pos;
                const int64_t seg_end = min(r1, (b + 1) * a.seq_pos);
                const int64_t tb0 = max(pos - b * a.seq_pos - a.lead, (int64_t)0);
                const int64_t tb1 = max(seg_end - b * a.seq_pos - a.lead, (int64_t)0);
                for (int64_t t0 = tb0; t0 < tb1; t0 += wph) {
                    const int ntile = (int)(tb1 - t0 < wph ? tb1 - t0 : wph);
                    if constexpr (POOL) {
                        // every lane takes part in every round (the page max is a shuffle
                        // reduction over the 16 lanes of a tile)
                        const bool ok = mbar_wait(&sm.scored[slot], par, a.err, &sm.abort);
                        for (int i0 = 0; i0 < ntile * kTileTokens; i0 += 32) {
                            const int i = i0 + lane;
                            const bool in = ok && i < ntile * kTileTokens;
                            const int s = in ? i / kTileTokens : 0, t = i % kTileTokens;
                            const int64_t tile = t0 + s;
                            const int64_t nv = a.N - tile * kTileTokens;
                            const int phys = sm.phys[slot][s];
                            uint32_t pk = 0u;   // ordered key of the token's new salience
                            if (in && t < nv && phys >= 0) {
                                uint32_t key = 0u;
                                for (int hh = 0; hh < Hkv; ++hh) key = max(key, sm.red[slot][s * Hkv + hh][t]);
                                const float R = key_to_float(key);
                                float old;
                                if (append && tile == new_tile && t == new_row) {
                                    old = 1.0f;
                                    if (a.sal_init_norm) {
                                        float acc = 0.0f;
                                        for (int hh = 0; hh < Hkv; ++hh)
                                            acc = __fadd_rn(acc, sm.new_norm[slot][s][hh]);
                                        old = __fdiv_rn(acc, (float)Hkv);
                                    }
                                } else {
                                    old = a.sal_bulk ? sm.sal_old[slot][s][t]
                                                     : a.sal[(int64_t)phys * a.sal_stride_p + b * a.sal_stride_b + t];
                                }
                                const float sn = __fadd_rn(__fmul_rn(a.decay, old), __fmul_rn(a.omd, R));
                                a.sal[(int64_t)phys * a.sal_stride_p + b * a.sal_stride_b + t] = sn;
                                pk = ordered_key(sn);
                            }
                            // page score = max over the tile's 16 tokens (NaN propagates, as
                            // in torch.amax), for the haystack pages only
#pragma unroll
                            for (int o = 8; o >= 1; o >>= 1) pk = max(pk, __shfl_xor_sync(0xffffffffu, pk, o));
                            if (in && t == 0) {
                                const int64_t pg = tile - a.pool_first;
                                if (pg >= 0 && pg < a.pool_num) a.pool[b * a.pool_num + pg] = key_to_float(pk);
                            }
                        }
                    } else if (mbar_wait(&sm.scored[slot], par, a.err, &sm.abort)) {
                        for (int i = lane; i < ntile * kTileTokens; i += 32) {
                            const int s = i / kTileTokens, t = i % kTileTokens;
                            const int64_t tile = t0 + s;
                            const int64_t nv = a.N - tile * kTileTokens;
                            const int phys = sm.phys[slot][s];
                            if (t >= nv || phys < 0) continue;
                            if constexpr (XCH) {
                                // head-sharded: the signed key of this rank's heads and the
                                // appended token's kv-head norms go to the exchange block; the
                                // salience is updated after the MAX over the ranks
                                const int64_t tt = tile * kTileTokens + t;
                                // the local block, or this rank's sub-block of every rank's
                                // region (peer stores over NVLink)
                                const int nr = a.xc.regions ? a.xc.nranks : 1;
                                const int64_t off = a.xc.buf_off + (int64_t)a.xc.rank * a.xc.sub +
                                                    b * a.xc.stride_b;
                                if (tt < a.score_n) {
                                    uint32_t key = 0u;
                                    for (int hh = 0; hh < Hkv; ++hh) key = max(key, sm.red[slot][s * Hkv + hh][t]);
                                    const int32_t sk = signed_key_of(key);
                                    for (int r = 0; r < nr; ++r) {
                                        int32_t* xr = a.xc.regions ? a.xc.regions[r] + off : a.xc.x + b * a.xc.stride_b;
                                        xr[tt] = sk;
                                    }
                                }
                                if (append && tile == new_tile && t == new_row) {
                                    for (int r = 0; r < nr; ++r) {
                                        int32_t* xr = a.xc.regions ? a.xc.regions[r] + off : a.xc.x + b * a.xc.stride_b;
                                        for (int hh = 0; hh < a.xc.htot; ++hh) {
                                            const int lh = hh - a.xc.h0;
                                            xr[a.xc.norm_off + hh] =
                                                (lh >= 0 && lh < Hkv) ? signed_key_of(ordered_key(sm.new_norm[slot][s][lh]))
                                                                      : INT32_MIN;
                                        }
                                    }
                                }
                                continue;
                            }
                            if (tile * kTileTokens + t >= a.score_n) {
                                // not scored this step; only a token appended here gets its
                                // initial salience
                                if (append && tile == new_tile && t == new_row) {
                                    float init = 1.0f;
                                    if (a.sal_init_norm) {
                                        float acc = 0.0f;
                                        for (int hh = 0; hh < Hkv; ++hh)
                                            acc = __fadd_rn(acc, sm.new_norm[slot][s][hh]);
                                        init = __fdiv_rn(acc, (float)Hkv);
                                    }
                                    a.sal[(int64_t)phys * a.sal_stride_p + b * a.sal_stride_b + t] = init;
                                }
                                continue;
                            }
                            uint32_t key = 0u;
                            for (int hh = 0; hh < Hkv; ++hh) key = max(key, sm.red[slot][s * Hkv + hh][t]);
                            const float R = key_to_float(key);
                            float old;
                            if (append && tile == new_tile && t == new_row) {
                                // initial salience of the appended token (mean ||k_h||)
                                old = 1.0f;
                                if (a.sal_init_norm) {
                                    float acc = 0.0f;
                                    for (int hh = 0; hh < Hkv; ++hh)
                                        acc = __fadd_rn(acc, sm.new_norm[slot][s][hh]);
                                    old = __fdiv_rn(acc, (float)Hkv);
                                }
                            } else {
                                old = a.sal_bulk ? sm.sal_old[slot][s][t]
                                                 : a.sal[(int64_t)phys * a.sal_stride_p + b * a.sal_stride_b + t];
                            }
                            a.sal[(int64_t)phys * a.sal_stride_p + b * a.sal_stride_b + t] =
                                __fadd_rn(__fmul_rn(a.decay, old), __fmul_rn(a.omd, R));
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sm.empty[slot]);
                    if (++slot == NS) { slot = 0; par ^= 1u; }
                }
                pos = seg_end;
            }
            if constexpr (XCH) {
                if (a.xc.regions) {
                    // peer exchange: once every CTA's stores are out, the last CTA releases
                    // this rank's flag on every rank (the ticket returns to zero)
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_system();
                        const int ticket = atomicAdd(a.counters, 1);
                        if (ticket == (int)gridDim.x - 1) {
                            __threadfence_system();
                            for (int r = 0; r < a.xc.nranks; ++r)
                                st_release_sys(a.xc.flags[r] + a.xc.rank, a.xc.epoch);
                            atomicExch(a.counters, 0);
                        }
                    }
                }
            }
            return;
        }
        if (warp != kComputeWarps) return;   // the rest of the producer warpgroup idles out
        int slot = 0;
        uint32_t par = 0;
        for (int64_t pos = r0; pos < r1;) {
            const int64_t b = pos / a.seq_pos;
            const int64_t seg_end = min(r1, (b + 1) * a.seq_pos);
            const int64_t tb0 = max(pos - b * a.seq_pos - a.lead, (int64_t)0);
            const int64_t tb1 = max(seg_end - b * a.seq_pos - a.lead, (int64_t)0);
            const int64_t* ptb = a.pt + b * a.pt_stride_b;
            int64_t win = tb0;   // first tile of the page-id window held in registers
            int64_t pid = (win + lane < tb1) ? __ldg(ptb + win + lane) : 0;
            int rid = map_row(a, pid, b);   // the sequence's row in that page
            // Two arrangements of the same stage loop: one tile per lane (the 8-head instances)
            // or every lane holding all of the stage's tiles (the others).  Each measured the
            // faster of the two for its instances.
            if constexpr (GP == 8) {
                for (int64_t t0 = tb0; t0 < tb1; t0 += wph) {
                    const int ntile = (int)(tb1 - t0 < wph ? tb1 - t0 : wph);
                    if (t0 + ntile > win + 32) {   // slide the window (uniform across lanes)
                        win = t0;
                        pid = (win + lane < tb1) ? __ldg(ptb + win + lane) : 0;
                        rid = map_row(a, pid, b);
                    }
                    // lane s < ntile holds tile t0 + s: its slot and the sequence's row in it
                    const int src = (int)(t0 - win) + (lane < ntile ? lane : 0);
                    int64_t v = __shfl_sync(0xffffffffu, pid, src);
                    int r = __shfl_sync(0xffffffffu, rid, src);
                    if (app_new_page && lane < ntile && t0 + lane == new_tile) {
                        // the appended token opens a page: take the free stack's top; every
                        // sequence's rows of it are its own
                        v = __ldg(a.free_stack + a.free_top - 1);
                        r = (int)b;
                        a.pt_w[b * a.pt_stride_b + new_tile] = v;
                        if (a.row_map && v >= 0 && v < a.num_slots) a.row_map[v * a.B + b] = (int32_t)b;
                    }
                    const int ph = (v < 0 || v >= a.num_slots) ? -1 : (int)v;
                    const bool ok = mbar_wait(&sm.empty[slot], par ^ 1u, a.err, &sm.abort);
                    // lane 0 records every tile's slot before the arrive that releases them
    #pragma unroll 1
                    for (int s = 0; s < ntile; ++s) {
                        const int ph_s = __shfl_sync(0xffffffffu, ph, s);
                        if (lane == 0 && ok) {
                            if (ph_s < 0 && a.err) atomicExch(a.err, 2);
                            sm.phys[slot][s] = ph_s;
                        }
                    }
                    uint8_t* st = smem + slot * a.stage_bytes;
                    if (lane == 0 && ok) {
                        uint32_t bytes = (uint32_t)(ntile * a.tile_bytes);
                        if (a.score && a.sal_bulk) bytes += (uint32_t)(ntile * kTileTokens * 4);
                        mbar_arrive_expect_tx(&sm.full[slot], bytes);
                    }
    #pragma unroll 1
                    for (int s = 0; s < ntile; ++s) {
                        const int phys = max(__shfl_sync(0xffffffffu, ph, s), 0);
                        const int row = __shfl_sync(0xffffffffu, r, s);
                        if (lane == 0 && ok) {
                            int cc[3];
    #pragma unroll
                            for (int k = 0; k < 3; ++k)
                                cc[k] = a.role[k] == 0 ? 0 : a.role[k] == 1 ? row : phys;
                            uint8_t* tile = st + s * a.tile_bytes;
    #pragma unroll
                            for (int hf = 0; hf < HALVES; ++hf) {
                                tma_load_5d(tile + hf * a.half_bytes, &tmk, &sm.full[slot], hf * 64, 0,
                                            cc[0], cc[1], cc[2]);
                                if (a.attend)
                                    tma_load_5d(tile + a.kv_tile_bytes + hf * a.half_bytes, &tmv,
                                                &sm.full[slot], hf * 64, 0, cc[0], cc[1], cc[2]);
                            }
                            if (a.score && a.sal_bulk)
                                bulk_load(&sm.sal_old[slot][s][0],
                                          a.sal + (int64_t)phys * a.sal_stride_p + b * a.sal_stride_b,
                                          kTileTokens * 4, &sm.full[slot]);
                        }
                    }
                    __syncwarp();
                    if (++slot == NS) { slot = 0; par ^= 1u; }
                }
            } else {
                for (int64_t t0 = tb0; t0 < tb1; t0 += wph) {
                    const int ntile = (int)(tb1 - t0 < wph ? tb1 - t0 : wph);
                    int32_t ph[kComputeWarps], rw[kComputeWarps];
    #pragma unroll
                    for (int s = 0; s < kComputeWarps; ++s) {
                        if (s < ntile) {
                            const int64_t t = t0 + s;
                            if (t >= win + 32) {   // slide the window (uniform across lanes)
                                win = t;
                                pid = (win + lane < tb1) ? __ldg(ptb + win + lane) : 0;
                                rid = map_row(a, pid, b);
                            }
                            int64_t v = __shfl_sync(0xffffffffu, pid, (int)(t - win));
                            int r = __shfl_sync(0xffffffffu, rid, (int)(t - win));
                            if (app_new_page && t == new_tile) {
                                // the appended token opens a page: take the free stack's top;
                                // every sequence's rows of it are its own
                                v = __ldg(a.free_stack + a.free_top - 1);
                                r = (int)b;
                                if (lane == 0) {
                                    a.pt_w[b * a.pt_stride_b + t] = v;
                                    if (a.row_map && v >= 0 && v < a.num_slots)
                                        a.row_map[v * a.B + b] = (int32_t)b;
                                }
                            }
                            ph[s] = (v < 0 || v >= a.num_slots) ? -1 : (int32_t)v;
                            rw[s] = r;
                        }
                    }
                    const bool ok = mbar_wait(&sm.empty[slot], par ^ 1u, a.err, &sm.abort);
                    if (lane == 0 && ok) {
                        uint8_t* st = smem + slot * a.stage_bytes;
                        uint32_t bytes = (uint32_t)(ntile * a.tile_bytes);
                        for (int s = 0; s < ntile; ++s) {
                            if (ph[s] < 0 && a.err) atomicExch(a.err, 2);
                            sm.phys[slot][s] = ph[s];
                        }
                        if (a.score && a.sal_bulk) bytes += (uint32_t)(ntile * kTileTokens * 4);
                        mbar_arrive_expect_tx(&sm.full[slot], bytes);
                        for (int s = 0; s < ntile; ++s) {
                            const int phys = max(ph[s], 0);
                            int cc[3];
    #pragma unroll
                            for (int k = 0; k < 3; ++k)
                                cc[k] = a.role[k] == 0 ? 0 : a.role[k] == 1 ? rw[s] : phys;
                            uint8_t* tile = st + s * a.tile_bytes;
    #pragma unroll
                            for (int hf = 0; hf < HALVES; ++hf) {
                                tma_load_5d(tile + hf * a.half_bytes, &tmk, &sm.full[slot], hf * 64, 0,
                                            cc[0], cc[1], cc[2]);
                                if (a.attend)
                                    tma_load_5d(tile + a.kv_tile_bytes + hf * a.half_bytes, &tmv,
                                                &sm.full[slot], hf * 64, 0, cc[0], cc[1], cc[2]);
                            }
                            if (a.score && a.sal_bulk)
                                bulk_load(&sm.sal_old[slot][s][0],
                                          a.sal + (int64_t)phys * a.sal_stride_p + b * a.sal_stride_b,
                                          kTileTokens * 4, &sm.full[slot]);
                        }
                    }
                    __syncwarp();
                    if (++slot == NS) { slot = 0; par ^= 1u; }
                }
            }
            pos = seg_end;
        }
        return;
    }

    // ------------------------------------------------------------------- compute warps
    set_max_regs_inc<kComputeRegs>();
    const int h = warp % Hkv;       // kv head
    const int s = warp / Hkv;       // tile slot inside a stage
    const int g = lane >> 3, j = lane & 7;
    const int hl = head_of_lane<GP>(j);   // query head (within the group) this lane reduces to
    const int G = a.G;
    const bool head_writer = (j & ((8 / GP) - 1)) == 0;   // one lane per head in each group
    const uint32_t ps_base = smem_u32(&sm.ps[warp][0][0]);
    const bool qvec = !(reinterpret_cast<uintptr_t>(a.q) & 15) && !((a.q_stride_h * 2) & 15) &&
                      !((a.q_stride_b * 2) & 15);

    // MODE 0 / 2 without the screen: fl(q * scale) as (even, odd) element pairs
    uint64_t qreg[SCREEN ? 1 : GP][EPL / 2];
    uint32_t qf[D / 16][2];       // MODE 1 / 2 and screened MODE 0: q2^T as mma B fragments
    // screened MODE 2: the score query's fragments; screened modes: their magnitudes
    uint32_t qsf[(SCREEN && M == 2) ? D / 16 : 1][2];
    uint32_t qa[SCREEN ? D / 16 : 1][2];
    float acc[MT][4];
    int slot = 0;
    uint32_t par = 0;
    for (int64_t pos = r0; pos < r1;) {
        const int64_t b = pos / a.seq_pos;
        const int64_t seg_end = min(r1, (b + 1) * a.seq_pos);
        const int64_t tb0 = max(pos - b * a.seq_pos - a.lead, (int64_t)0);
        const int64_t tb1 = max(seg_end - b * a.seq_pos - a.lead, (int64_t)0);

        if constexpr (M != 0) {
            // B = q2^T (dims x heads): lane holds head lane/4, dims 16kk + 2(lane%4) + {0,1}
            // (b0) and the same + 8 (b1); heads past G are zero.  Issued first: in the
            // screened instances these loads overlap the staging of the scoring rows below.
            const int n = lane >> 2;
            const T* qr = static_cast<const T*>(a.q2) + b * a.q2_stride_b + (int64_t)(h * G + n) * a.q2_stride_h;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const int d0 = kk * 16 + 2 * (lane & 3);
                qf[kk][0] = n < G ? pack_elems<T>(qr[d0], qr[d0 + 1]) : 0u;
                qf[kk][1] = n < G ? pack_elems<T>(qr[d0 + 8], qr[d0 + 9]) : 0u;
            }
        }
        if constexpr (SCREEN) {
            // this warp's copy of the G scoring-query rows (q) for the canonical recompute
            // (16-byte rows; the host requires 16-byte aligned query rows for these
            // instances), then every fragment of q from the copy: one round trip to global
            // memory per segment instead of one per fragment set
            __syncwarp();   // the previous segment's reads of the copy are done
            const T* qg = static_cast<const T*>(a.q) + b * a.q_stride_b + (int64_t)(h * G) * a.q_stride_h;
            for (int idx = lane; idx < G * (D / 8); idx += 32) {
                const int i = idx / (D / 8), c8 = idx % (D / 8);
                const uint4 w = *reinterpret_cast<const uint4*>(qg + (int64_t)i * a.q_stride_h + c8 * 8);
                sts128(smem_u32(&qrows.q[warp][i][c8 * 8]), w);
            }
            __syncwarp();
            // B fragments of q (the attention query too in MODE 0, the score query in MODE 2)
            // and of its magnitudes; heads past G are zero
            const int n = lane >> 2;
            const uint32_t qrow = smem_u32(&qrows.q[warp][n < G ? n : 0][0]);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const int d0 = kk * 16 + 2 * (lane & 3);
                const uint32_t f0 = n < G ? lds32(qrow + d0 * 2) : 0u;
                const uint32_t f1 = n < G ? lds32(qrow + (d0 + 8) * 2) : 0u;
                if constexpr (M == 2) {
                    qsf[kk][0] = f0; qsf[kk][1] = f1;
                } else {
                    qf[kk][0] = f0; qf[kk][1] = f1;
                }
                qa[kk][0] = f0 & kAbsMask2;
                qa[kk][1] = f1 & kAbsMask2;
            }
        }
        if constexpr (M != 1 && !SCREEN) {
            // fl(q * scale) for this lane's K elements: chunk j of every 64-element half
            // (one 16-byte load per chunk when the query rows are 16-byte aligned)
            const T* qb = static_cast<const T*>(a.q) + b * a.q_stride_b;
            if (qvec) {
#pragma unroll
                for (int i = 0; i < GP; ++i) {
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) {
                        float f[8];
                        const uint4 w = i < G ? *reinterpret_cast<const uint4*>(
                                                    qb + (int64_t)(h * G + i) * a.q_stride_h + hf * 64 + 8 * j)
                                              : make_uint4(0u, 0u, 0u, 0u);
                        unpack8<T>(w, f);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            qreg[i][hf * 4 + e] = pack2(__fmul_rn(f[2 * e], a.scale_r),
                                                        __fmul_rn(f[2 * e + 1], a.scale_r));
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < GP; ++i) {
#pragma unroll
                    for (int e = 0; e < EPL; e += 2) {
                        const int dim = (e / 8) * 64 + 8 * j + (e % 8);
                        const T* qr = qb + (int64_t)(h * G + i) * a.q_stride_h + dim;
                        const float lo = i < G ? __fmul_rn(to_f<T>(qr[0]), a.scale_r) : 0.0f;
                        const float hi = i < G ? __fmul_rn(to_f<T>(qr[1]), a.scale_r) : 0.0f;
                        qreg[i][e / 2] = pack2(lo, hi);
                    }
                }
            }
        }
        float m_run = -INFINITY, l_run = 0.0f;   // MODE 0: running max / sum of head hl
        // MODE 1 / 2: the same for heads nA = 2(lane % 4) and nB = nA + 1 (the accumulator's
        // columns of this lane)
        float mrA = -INFINITY, mrB = -INFINITY, lrA = 0.0f, lrB = 0.0f;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;

        for (int t0 = (int)tb0; t0 < (int)tb1; t0 += wph) {
            const bool landed = mbar_wait(&sm.full[slot], par, a.err, &sm.abort);
            const int tile = t0 + s;
            if (landed && tile < tb1) {
                const int nv = (int)(a.N - tile * kTileTokens < kTileTokens ? a.N - tile * kTileTokens : kTileTokens);
                uint8_t* tbase = smem + slot * a.stage_bytes + s * a.tile_bytes;
                const uint32_t kb = smem_u32(tbase) + h * kTileTokens * 128;
                const uint32_t vb = kb + a.kv_tile_bytes;

                // ---- 0. fused append of the token at N - 1 --------------------------------
                // Copy this kv head's new K and V rows into the staged page (the page in HBM
                // still holds an older row there) and into the pool page for later steps, and
                // take ||k|| in the canonical order for the token's initial salience.
                const bool has_new = append && tile == new_tile;
                if (has_new) {
                    const int phys = sm.phys[slot][s];
                    constexpr int NCH = D / 8;   // 16-byte chunks per row
                    for (int i = lane; i < 2 * NCH; i += 32) {
                        const bool isv = i >= NCH;
                        const int cidx = isv ? i - NCH : i;
                        const T* src = static_cast<const T*>(isv ? a.v_new : a.k_new) +
                                       b * a.new_stride_b + (int64_t)h * a.new_stride_h + cidx * 8;
                        const uint4 w = *reinterpret_cast<const uint4*>(src);
                        const int hf = cidx >> 3, c8 = cidx & 7;
                        if (!isv || a.attend)   // without attention no V is staged
                            sts128((isv ? vb : kb) + hf * a.half_bytes + new_row * 128 +
                                       ((c8 ^ (new_row & 7)) << 4),
                                   w);
                        if (phys >= 0) {
                            T* dst = static_cast<T*>(isv ? a.vpool : a.kpool) + b * a.stride_b +
                                     (int64_t)h * a.stride_h + (int64_t)phys * a.stride_p +
                                     (int64_t)new_row * a.stride_t + cidx * 8;
                            *reinterpret_cast<uint4*>(dst) = w;
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    uint64_t x = 0ull;
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) {
                        uint64_t kq[4];
                        unpack8_pairs<T>(lds128(kb + hf * a.half_bytes + new_row * 128 +
                                                ((j ^ (new_row & 7)) << 4)),
                                         kq);
#pragma unroll
                        for (int e = 0; e < 4; ++e) ffma2(x, kq[e], kq[e]);
                    }
                    const float nrm = __fsqrt_rn(group8_sum(sum_pair(x)));
                    if (lane == 0) sm.new_norm[slot][s][h] = nrm;
                }

                // attention logits in the mma accumulator layout (MODE 1 / 2 and screened
                // MODE 0): tokens lane/4 and lane/4 + 8, heads 2(lane%4) and 2(lane%4) + 1
                float c4[4] = {0.0f, 0.0f, 0.0f, 0.0f};

                // ---- 1s. screened resonance (5-8 query heads per kv head) -----------------
                if constexpr (SCREEN) {
                    float cs[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // score query . k
                    float ca[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // |score query| . |k|
                    {
                        const int mi = lane >> 3;
                        const int tk = (lane & 7) + 8 * (mi & 1);
#pragma unroll
                        for (int kk = 0; kk < D / 16; ++kk) {
                            const int c8 = (kk & 3) * 2 + (mi >> 1);
                            uint32_t a0, a1, a2, a3;
                            ldsm_x4(kb + (kk >> 2) * a.half_bytes + tk * 128 + ((c8 ^ (tk & 7)) << 4),
                                    a0, a1, a2, a3);
                            if constexpr (M == 2) {
                                mma_16816<kBf16>(cs, a0, a1, a2, a3, qsf[kk][0], qsf[kk][1]);
                                if (a.attend) mma_16816<kBf16>(c4, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
                            } else {
                                mma_16816<kBf16>(cs, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
                            }
                            mma_16816<kBf16>(ca, a0 & kAbsMask2, a1 & kAbsMask2, a2 & kAbsMask2,
                                             a3 & kAbsMask2, qa[kk][0], qa[kk][1]);
                        }
                    }
                    if constexpr (M == 0) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) c4[e] = cs[e];
                    }
                    if (a.score) {
                        const int tA = lane >> 2, tB = tA + 8;
                        const int nA = 2 * (lane & 3), nB = nA + 1;
                        const int64_t gt = (int64_t)tile * kTileTokens;
                        const bool vA = tA < nv && gt + tA < a.score_n;
                        const bool vB = tB < nv && gt + tB < a.score_n;
                        const bool ok[4] = {vA && nA < G, vA && nB < G, vB && nA < G, vB && nB < G};
                        const float tol = a.scale_r * kScreenTol;
                        float ap[4], eb[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            ap[e] = cs[e] * a.scale_r;
                            eb[e] = ca[e] * tol;
                        }
                        // lower bound of each token's canonical max over its heads (the 8 heads
                        // of a token sit in 4 consecutive lanes, 2 per lane)
                        float lbA = fmaxf(ok[0] ? ap[0] - eb[0] : -INFINITY, ok[1] ? ap[1] - eb[1] : -INFINITY);
                        float lbB = fmaxf(ok[2] ? ap[2] - eb[2] : -INFINITY, ok[3] ? ap[3] - eb[3] : -INFINITY);
                        lbA = fmaxf(lbA, __shfl_xor_sync(0xffffffffu, lbA, 1));
                        lbB = fmaxf(lbB, __shfl_xor_sync(0xffffffffu, lbB, 1));
                        lbA = fmaxf(lbA, __shfl_xor_sync(0xffffffffu, lbA, 2));
                        lbB = fmaxf(lbB, __shfl_xor_sync(0xffffffffu, lbB, 2));
                        // candidate heads: upper bound not below the lower bound (NaN stays in)
                        uint32_t mA = ((ok[0] && !(ap[0] + eb[0] < lbA)) ? 1u << nA : 0u) |
                                      ((ok[1] && !(ap[1] + eb[1] < lbA)) ? 1u << nB : 0u);
                        uint32_t mB = ((ok[2] && !(ap[2] + eb[2] < lbB)) ? 1u << nA : 0u) |
                                      ((ok[3] && !(ap[3] + eb[3] < lbB)) ? 1u << nB : 0u);
                        mA |= __shfl_xor_sync(0xffffffffu, mA, 1);
                        mB |= __shfl_xor_sync(0xffffffffu, mB, 1);
                        mA |= __shfl_xor_sync(0xffffffffu, mA, 2);
                        mB |= __shfl_xor_sync(0xffffffffu, mB, 2);
                        // canonical dots of the candidates: round r, group g takes token 4r + g
                        // and its lowest candidate head (the four rounds run together); further
                        // candidates (rare) follow, four at a time
                        const uint32_t qb = smem_u32(&qrows.q[warp][0][0]);
                        uint32_t keyr[4], rem[4];
                        int tr[4], hr[4];
                        float vr[4];
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            tr[r] = 4 * r + g;
                            rem[r] = __shfl_sync(0xffffffffu, r < 2 ? mA : mB, (tr[r] & 7) * 4);
                            keyr[r] = 0u;
                        }
                        // one copy of the round body (instruction fetch is a limiter here):
                        // the first pass takes every token's lowest candidate, later passes the
                        // rest (rare)
                        do {
#pragma unroll
                            for (int r = 0; r < 4; ++r) hr[r] = rem[r] ? __ffs(rem[r]) - 1 : 0;
                            canon_dots4<T, D>(kb, a.half_bytes, tr, qb, hr, j, a.scale_r, vr);
#pragma unroll
                            for (int r = 0; r < 4; ++r) {
                                if (rem[r]) keyr[r] = max(keyr[r], ordered_key(vr[r]));
                                rem[r] &= rem[r] - 1u;
                            }
                        } while (__any_sync(0xffffffffu, (rem[0] | rem[1] | rem[2] | rem[3]) != 0u));
                        if (j == 0) {
#pragma unroll
                            for (int r = 0; r < 4; ++r) sm.red[slot][warp][4 * r + g] = keyr[r];
                        }
                        __syncwarp();   // orders the lanes' key stores before lane 0's release
                        if (lane == 0) mbar_arrive(&sm.scored[slot]);
                    }
                }

                // ---- 1. scores, canonical order (MODE 0: also the logits) ----------------
                float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if constexpr (M != 1 && !SCREEN) {
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int t = 4 * r + g;
                    uint64_t kp[EPL / 2];   // element pairs (even position, odd position)
#pragma unroll
                    for (int hf = 0; hf < HALVES; ++hf) {
                        const uint4 w = lds128(kb + hf * a.half_bytes + t * 128 + ((j ^ (t & 7)) << 4));
                        unpack8_pairs<T>(w, kp + hf * 4);
                    }
                    float part[GP];
#pragma unroll
                    for (int i = 0; i < GP; ++i) {
                        uint64_t x = 0ull;   // (+0.0f, +0.0f)
#pragma unroll
                        for (int e = 0; e < EPL / 2; ++e) ffma2(x, qreg[i][e], kp[e]);
                        part[i] = sum_pair(x);
                    }
                    sc[r] = group_transpose_reduce<GP>(part, j);
                }
                }

                // ---- 2. resonance: max over this warp's heads --------------------------
                // The fold over kv heads, the EWMA and the store are the salience
                // finisher's; this warp stores one key per token and arrives on scored.
                if (M != 1 && !SCREEN && a.score) {
                    // transpose-max over the 8 lanes of the group: afterwards lane j holds
                    // the max over heads of round rj = 2*bit2(j) + bit1(j), i.e. token 4*rj + g
                    uint32_t key[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        key[r] = (4 * r + g < nv && hl < G) ? ordered_key(sc[r]) : 0u;
                    {
                        const bool up = (j & 4) != 0;
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const uint32_t send = up ? key[i] : key[i + 2];
                            const uint32_t keep = up ? key[i + 2] : key[i];
                            key[i] = max(keep, __shfl_xor_sync(0xffffffffu, send, 4));
                        }
                    }
                    {
                        const bool up = (j & 2) != 0;
                        const uint32_t send = up ? key[0] : key[1];
                        const uint32_t keep = up ? key[1] : key[0];
                        key[0] = max(keep, __shfl_xor_sync(0xffffffffu, send, 2));
                    }
                    key[0] = max(key[0], __shfl_xor_sync(0xffffffffu, key[0], 1));
                    {
                        const int t = 4 * (((j >> 2) & 1) * 2 + ((j >> 1) & 1)) + g;
                        if ((j & 1) == 0) sm.red[slot][warp][t] = key[0];
                    }
                    __syncwarp();   // orders the lanes' key stores before lane 0's release
                    if (lane == 0) mbar_arrive(&sm.scored[slot]);
                }

                // ---- 3. online softmax + P.V on tensor cores ------------------------------
                if (a.attend) {
                    bool any_raise = false;
                    uint32_t pb0 = 0u, pb1 = 0u;   // P.V B fragments (tensor-core logits path)
                    if constexpr (M == 0 && !SCREEN) {
                        float z[4];
                        float mx = -INFINITY;
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const int t = 4 * r + g;
                            z[r] = (t < nv && hl < G) ? sc[r] * a.logit_log2 : -INFINITY;
                            mx = fmaxf(mx, z[r]);
                        }
                        // Lazy rescaling: the running reference max only moves when the tile
                        // max exceeds it by more than 2^8, so P stays <= 256 (exact range for
                        // bf16/fp16 and fp32 sums) and the accumulator is rescaled only on
                        // those rare tiles.  A head's tile max exceeds the bound exactly when
                        // one of its lanes' values does, so the max over the lanes is taken
                        // only on those tiles.
                        any_raise = __any_sync(0xffffffffu, mx > m_run + kRescaleLog2);   // includes m_run == -inf
                        if (any_raise) {
                            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                            const bool raise = mx > m_run + kRescaleLog2;
                            const float m_new = raise ? mx : m_run;
                            const float alpha = raise ? ex2(m_run - m_new) : 1.0f;   // ex2(-inf) = 0
                            l_run *= alpha;
                            m_run = m_new;
                            if (head_writer && g == 0) sm.alpha[warp][hl] = alpha;
                        }
                        const bool live = m_run != -INFINITY;
                        float psum = 0.0f;
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const float p = live ? ex2(z[r] - m_run) : 0.0f;
                            psum += p;
                            if (head_writer) sm.ps[warp][hl][4 * r + g] = to_bits<T>(p);
                        }
                        l_run += psum;
                    } else {
                        // logits S[16 tokens x 8 heads] = K tile . q2^T on tensor cores; A
                        // fragments straight from the swizzled K stage by ldmatrix.  Lane
                        // holds tokens tA = lane/4 and tA + 8 of heads nA = 2(lane%4), nA + 1
                        // -- the accumulator's own columns, so rescaling stays in the lane.
                        // (Screened instances computed them with the screen's mma above.)
                        if constexpr (!SCREEN) {
                            const int mi = lane >> 3;
                            const int tk = (lane & 7) + 8 * (mi & 1);
#pragma unroll
                            for (int kk = 0; kk < D / 16; ++kk) {
                                const int c8 = (kk & 3) * 2 + (mi >> 1);
                                uint32_t a0, a1, a2, a3;
                                ldsm_x4(kb + (kk >> 2) * a.half_bytes + tk * 128 +
                                            ((c8 ^ (tk & 7)) << 4),
                                        a0, a1, a2, a3);
                                mma_16816<kBf16>(c4, a0, a1, a2, a3, qf[kk][0], qf[kk][1]);
                            }
                        }
                        const int tA = lane >> 2, tB = tA + 8;
                        const int nA = 2 * (lane & 3), nB = nA + 1;
                        const float zA0 = (tA < nv && nA < G) ? c4[0] * a.attn_log2 : -INFINITY;
                        const float zB0 = (tA < nv && nB < G) ? c4[1] * a.attn_log2 : -INFINITY;
                        const float zA1 = (tB < nv && nA < G) ? c4[2] * a.attn_log2 : -INFINITY;
                        const float zB1 = (tB < nv && nB < G) ? c4[3] * a.attn_log2 : -INFINITY;
                        float mxA = fmaxf(zA0, zA1), mxB = fmaxf(zB0, zB1);
                        // as above: the max over a head's lanes only on tiles that raise it
                        if (__any_sync(0xffffffffu, mxA > mrA + kRescaleLog2 || mxB > mrB + kRescaleLog2)) {
#pragma unroll
                            for (int o = 4; o < 32; o <<= 1) {
                                mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, o));
                                mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, o));
                            }
                            const bool raiseA = mxA > mrA + kRescaleLog2;   // includes mr == -inf
                            const bool raiseB = mxB > mrB + kRescaleLog2;
                            const float alA = raiseA ? ex2(mrA - mxA) : 1.0f;   // ex2(-inf) = 0
                            const float alB = raiseB ? ex2(mrB - mxB) : 1.0f;
                            if (raiseA) { lrA *= alA; mrA = mxA; }
                            if (raiseB) { lrB *= alB; mrB = mxB; }
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                acc[mt][0] *= alA; acc[mt][1] *= alB;
                                acc[mt][2] *= alA; acc[mt][3] *= alB;
                            }
                        }
                        const bool liveA = mrA != -INFINITY, liveB = mrB != -INFINITY;
                        const float pA0 = liveA ? ex2(zA0 - mrA) : 0.0f;
                        const float pB0 = liveB ? ex2(zB0 - mrB) : 0.0f;
                        const float pA1 = liveA ? ex2(zA1 - mrA) : 0.0f;
                        const float pB1 = liveB ? ex2(zB1 - mrB) : 0.0f;
                        lrA += pA0 + pA1;
                        lrB += pB0 + pB1;
                        // P as the P.V mma's B fragments without a trip through shared
                        // memory: the lane's (token, head pair) in the accumulator layout is
                        // one element pair of an 8x8 row-major fragment (tokens 0-7 and 8-15),
                        // and the transposed fragment is exactly B's layout (tokens
                        // 2(lane%4) + {0,1} (+8), head lane/4)
                        pb0 = movmatrix_trans(pack_bits<T>(pA0, pB0));
                        pb1 = movmatrix_trans(pack_bits<T>(pA1, pB1));
                    }
                    if (nv < kTileTokens) {
                        // zero V rows past the last valid token (their P is 0; keep them finite)
                        for (int i = lane; i < (kTileTokens - nv) * 8 * HALVES; i += 32) {
                            const int row = nv + i / (8 * HALVES);
                            const int rem = i % (8 * HALVES);
                            const int hf = rem / 8, ch = rem % 8;
                            sts128(vb + hf * a.half_bytes + row * 128 + (ch << 4), make_uint4(0, 0, 0, 0));
                        }
                        fence_proxy_async_smem();
                    }
                    __syncwarp();
                    const int n0 = 2 * (lane & 3);
                    if (M == 0 && !SCREEN && any_raise) {
                        const float al0 = sm.alpha[warp][n0], al1 = sm.alpha[warp][n0 + 1];
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            acc[mt][0] *= al0; acc[mt][1] *= al1;
                            acc[mt][2] *= al0; acc[mt][3] *= al1;
                        }
                    }
                    uint32_t b0 = pb0, b1 = pb1;
                    if constexpr (M == 0 && !SCREEN) {
                        b0 = lds32(ps_base + ((lane >> 2) * kTileTokens + n0) * 2);
                        b1 = lds32(ps_base + ((lane >> 2) * kTileTokens + n0 + 8) * 2);
                    }
                    const int mi = lane >> 3;
                    const int tk = (mi >> 1) * 8 + (lane & 7);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const int cc = 2 * mt + (mi & 1);          // 8-dim chunk 0..D/8-1
                        const int hf = cc >> 3, c8 = cc & 7;
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4_trans(vb + hf * a.half_bytes + tk * 128 + ((c8 ^ (tk & 7)) << 4), a0, a1, a2, a3);
                        mma_16816<kBf16>(acc[mt], a0, a1, a2, a3, b0, b1);
                    }
                    __syncwarp();
                }
            } else if (a.score) {
                if (lane == 0) mbar_arrive(&sm.scored[slot]);   // no tile in this slot: keep the count whole
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[slot]);
            if (++slot == NS) { slot = 0; par ^= 1u; }
        }

        // ---- segment end: write this warp's partial --------------------------------------
        // partial row per query head: acc[0, D) | m (log2 units) at D | l at D+1 | pad;
        // merge_kernel combines the partials of a sequence once the whole grid is done
        bool writer = true;
        if constexpr (SCREEN || M != 0) {
            if (a.attend && a.pw == 1 && wph > 1) {
                // One-sequence launch: fold the tile slots' partials of each kv head here (the
                // merge then reads one partial per CTA).  Once every compute warp is past its
                // last tile the stage ring is idle (the CTA's only segment is done and every
                // copy has landed); warps of slot s >= 1 publish their state there, slot 0
                // folds it in the accumulator layout, which is the same for every warp of a
                // kv head.
                constexpr int SW = MT * 4 + 4;   // floats a lane publishes
                float* pub = reinterpret_cast<float*>(smem);
                compute_barrier(kComputeThreads);   // every warp is done reading the stages
                if (s > 0) {
                    float* my = pub + ((warp - Hkv) * 32 + lane) * SW;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) my[mt * 4 + e] = acc[mt][e];
                    my[MT * 4 + 0] = mrA; my[MT * 4 + 1] = mrB;
                    my[MT * 4 + 2] = lrA; my[MT * 4 + 3] = lrB;
                }
                compute_barrier(kComputeThreads);
                if (s == 0) {
                    for (int so = 1; so < wph; ++so) {
                        const float* ot = pub + ((so * Hkv + h - Hkv) * 32 + lane) * SW;
                        const float moA = ot[MT * 4 + 0], moB = ot[MT * 4 + 1];
                        const float mnA = fmaxf(mrA, moA), mnB = fmaxf(mrB, moB);
                        // weights 2^(m - max); a side that saw no token weighs 0
                        const float wsA = mrA == -INFINITY ? 0.f : ex2(mrA - mnA);
                        const float woA = moA == -INFINITY ? 0.f : ex2(moA - mnA);
                        const float wsB = mrB == -INFINITY ? 0.f : ex2(mrB - mnB);
                        const float woB = moB == -INFINITY ? 0.f : ex2(moB - mnB);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            acc[mt][0] = acc[mt][0] * wsA + ot[mt * 4 + 0] * woA;
                            acc[mt][1] = acc[mt][1] * wsB + ot[mt * 4 + 1] * woB;
                            acc[mt][2] = acc[mt][2] * wsA + ot[mt * 4 + 2] * woA;
                            acc[mt][3] = acc[mt][3] * wsB + ot[mt * 4 + 3] * woB;
                        }
                        lrA = lrA * wsA + ot[MT * 4 + 2] * woA;
                        lrB = lrB * wsB + ot[MT * 4 + 3] * woB;
                        mrA = mnA;
                        mrB = mnB;
                    }
                }
                writer = s == 0;
            }
        }
        if (a.attend && writer) {
            constexpr int RS = D + 4;
            const int64_t cfirst = (b * a.seq_pos) / a.W;
            const int64_t pidx = (c - cfirst) * a.pw + s;
            float* part = a.partials + ((b * a.maxc * wph + pidx) * a.Hq) * (int64_t)RS;
            if constexpr (M == 0 && !SCREEN) {
                float l_tot = l_run + __shfl_xor_sync(0xffffffffu, l_run, 8);
                l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 16);
                if (head_writer && g == 0 && hl < G) {
                    float* ph = part + (int64_t)(h * G + hl) * RS;
                    ph[D] = m_run;
                    ph[D + 1] = l_tot;
                }
            } else {
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    lrA += __shfl_xor_sync(0xffffffffu, lrA, o);
                    lrB += __shfl_xor_sync(0xffffffffu, lrB, o);
                }
                const int nA = 2 * lane;   // lanes 0..3 write heads 2 lane and 2 lane + 1
                if (lane < 4 && nA < G) {
                    float* ph = part + (int64_t)(h * G + nA) * RS;
                    ph[D] = mrA;
                    ph[D + 1] = lrA;
                }
                if (lane < 4 && nA + 1 < G) {
                    float* ph = part + (int64_t)(h * G + nA + 1) * RS;
                    ph[D] = mrB;
                    ph[D + 1] = lrB;
                }
            }
            const int n0 = 2 * (lane & 3);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int d0 = mt * 16 + (lane >> 2);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = n0 + (e & 1);
                    const int d = d0 + (e >> 1) * 8;
                    if (n < G) part[(int64_t)(h * G + n) * RS + d] = acc[mt][e];
                }
            }
        }
        pos = seg_end;
    }
}

// Log-sum-exp merge of the per-warp partials of each (sequence b, query head hq) row.
// merge_kernel: one CTA per row of kMergeGroups x D threads.  Group g folds its share of the
// partials with one lane per output dimension (every partial's (m, l, acc[d]) of a 32-partial
// chunk is loaded at once; the weights 2^(m_p - M) go through shuffles); the groups then
// combine in shared memory.
// merge_cluster_kernel, for rows with more than kMergePartialsPerCta partials (batch 1: a row
// has 150-300): a cluster of S <= kMergeMaxCluster CTAs serves one row, CTA r folding the
// contiguous share [np r / S, np (r + 1) / S) as above, then storing its fold into slot r of
// cluster rank 0's shared memory (distributed shared memory); after one cluster barrier rank
// 0 folds the S results in rank order and writes the row.  With one CTA per row a batch-1
// launch merged its 28-32 rows on 28-32 SMs.
constexpr int kMergeGroups = 4;
constexpr int kMergeMaxCluster = 8;
constexpr int kMergePartialsPerCta = 40;   // cluster size: ceil(partials / 40), at most 8

struct MergeArgs {
    const float* partials; void* out; int64_t o_stride_b, o_stride_h;
    int Hq, wph; int64_t seq_pos, W, maxc;   // stream-K positions per sequence (DevArgs)
    int pw;        // partials per CTA and row (DevArgs)
    int cluster;   // CTAs per row (the launch's cluster size)
};

template <typename T, int D>
__global__ void __launch_bounds__(kMergeGroups * D)
merge_kernel(const MergeArgs a) {
    // the next decode kernel may start its prologue now; it waits for this grid to finish
    // before it touches anything this grid reads
    grid_launch_dependents();
    grid_dependency_wait();   // the partials come from the decode kernel just before
    constexpr int RS = D + 4;
    __shared__ float s_o[kMergeGroups][D];
    __shared__ float s_m[kMergeGroups], s_l[kMergeGroups];
    const int lane = threadIdx.x & 31;
    const int grp = threadIdx.x / D;
    const int d = threadIdx.x % D;
    const int64_t b = blockIdx.x / a.Hq;
    const int hq = blockIdx.x % a.Hq;
    const int64_t cfirst = (b * a.seq_pos) / a.W;
    const int64_t clast = ((b + 1) * a.seq_pos - 1) / a.W;
    const int np = (int)(clast - cfirst + 1) * a.pw;
    // group g takes whole 32-partial chunks g, g + G, g + 2G, ...
    const float* pb = a.partials + ((b * a.maxc * a.wph) * a.Hq + hq) * (int64_t)RS;
    const int64_t pstride = (int64_t)a.Hq * RS;
    float M = -INFINITY, O = 0.f, L = 0.f;
    for (int p0 = grp * 32; p0 < np; p0 += kMergeGroups * 32) {
        const int n = min(32, np - p0);
        // lane p holds the stats of partial p0 + p
        const float mp = lane < n ? __ldcg(pb + (p0 + lane) * pstride + D) : -INFINITY;
        const float lp = lane < n ? __ldcg(pb + (p0 + lane) * pstride + D + 1) : 0.f;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = i < n ? __ldcg(pb + (p0 + i) * pstride + d) : 0.f;
        float Mc = mp;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, o));
        const float Mn = fmaxf(M, Mc);
        if (Mn == -INFINITY) continue;
        const float r = M == -INFINITY ? 0.f : ex2(M - Mn);
        const float wl = mp == -INFINITY ? 0.f : ex2(mp - Mn);
        float Lc = lp * wl;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Lc += __shfl_xor_sync(0xffffffffu, Lc, o);
        float Oc = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) Oc += acc[i] * __shfl_sync(0xffffffffu, wl, i);
        O = O * r + Oc;
        L = L * r + Lc;
        M = Mn;
    }
    s_o[grp][d] = O;
    if (d == 0) { s_m[grp] = M; s_l[grp] = L; }
    __syncthreads();
    if (grp != 0) return;
    float Mt = -INFINITY;
#pragma unroll
    for (int g = 0; g < kMergeGroups; ++g) Mt = fmaxf(Mt, s_m[g]);
    float Ot = 0.f, Lt = 0.f;
    if (Mt != -INFINITY) {
#pragma unroll
        for (int g = 0; g < kMergeGroups; ++g) {
            const float w = s_m[g] == -INFINITY ? 0.f : ex2(s_m[g] - Mt);
            Ot += s_o[g][d] * w;
            Lt += s_l[g] * w;
        }
    }
    T* ob = static_cast<T*>(a.out) + b * a.o_stride_b + (int64_t)hq * a.o_stride_h;
    ob[d] = from_f<T>(Lt > 0.f ? Ot / Lt : 0.f);
}

template <typename T, int D>
__global__ void __launch_bounds__(kMergeGroups * D)
merge_cluster_kernel(const MergeArgs a) {
    // the next decode kernel may start its prologue now; it waits for this grid to finish
    // before it touches anything this grid reads
    grid_launch_dependents();
    grid_dependency_wait();   // the partials come from the decode kernel just before
    constexpr int RS = D + 4;
    __shared__ float s_o[kMergeGroups][D];
    __shared__ float s_m[kMergeGroups], s_l[kMergeGroups];
    // rank 0 of a cluster: the folds of the cluster's CTAs, slot r from rank r
    __shared__ float c_o[kMergeMaxCluster][D];
    __shared__ float c_m[kMergeMaxCluster], c_l[kMergeMaxCluster];
    const int lane = threadIdx.x & 31;
    const int grp = threadIdx.x / D;
    const int d = threadIdx.x % D;
    const int S = a.cluster;
    const int rank = (int)(blockIdx.x % (unsigned)S);   // == the block's rank in its cluster
    const int row = (int)(blockIdx.x / (unsigned)S);
    const int64_t b = row / a.Hq;
    const int hq = row % a.Hq;
    const int64_t cfirst = (b * a.seq_pos) / a.W;
    const int64_t clast = ((b + 1) * a.seq_pos - 1) / a.W;
    const int np = (int)(clast - cfirst + 1) * a.pw;
    // this CTA's share of the row; group g takes its 32-partial chunks g, g + G, ...
    const int lo = np * rank / S, hi = np * (rank + 1) / S;
    const float* pb = a.partials + ((b * a.maxc * a.wph) * a.Hq + hq) * (int64_t)RS;
    const int64_t pstride = (int64_t)a.Hq * RS;
    float M = -INFINITY, O = 0.f, L = 0.f;
    for (int p0 = lo + grp * 32; p0 < hi; p0 += kMergeGroups * 32) {
        const int n = min(32, hi - p0);
        // lane p holds the stats of partial p0 + p
        const float mp = lane < n ? __ldcg(pb + (p0 + lane) * pstride + D) : -INFINITY;
        const float lp = lane < n ? __ldcg(pb + (p0 + lane) * pstride + D + 1) : 0.f;
        float acc[32];
        const float* pp = pb + p0 * pstride + d;   // walks the chunk's partials
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            acc[i] = i < n ? __ldcg(pp) : 0.f;
            pp += pstride;
        }
        float Mc = mp;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Mc = fmaxf(Mc, __shfl_xor_sync(0xffffffffu, Mc, o));
        const float Mn = fmaxf(M, Mc);
        if (Mn == -INFINITY) continue;
        const float r = M == -INFINITY ? 0.f : ex2(M - Mn);
        const float wl = mp == -INFINITY ? 0.f : ex2(mp - Mn);
        float Lc = lp * wl;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) Lc += __shfl_xor_sync(0xffffffffu, Lc, o);
        float Oc = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) Oc += acc[i] * __shfl_sync(0xffffffffu, wl, i);
        O = O * r + Oc;
        L = L * r + Lc;
        M = Mn;
    }
    s_o[grp][d] = O;
    if (d == 0) { s_m[grp] = M; s_l[grp] = L; }
    __syncthreads();
    if (grp == 0) {
        float Mt = -INFINITY;
#pragma unroll
        for (int g = 0; g < kMergeGroups; ++g) Mt = fmaxf(Mt, s_m[g]);
        float Ot = 0.f, Lt = 0.f;
        if (Mt != -INFINITY) {
#pragma unroll
            for (int g = 0; g < kMergeGroups; ++g) {
                const float w = s_m[g] == -INFINITY ? 0.f : ex2(s_m[g] - Mt);
                Ot += s_o[g][d] * w;
                Lt += s_l[g] * w;
            }
        }
        // push this CTA's fold into cluster rank 0's slot `rank` (distributed shared memory
        // stores; the cluster barrier below releases them)
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        *cluster.map_shared_rank(&c_o[rank][d], 0) = Ot;
        if (d == 0) {
            *cluster.map_shared_rank(&c_m[rank], 0) = Mt;
            *cluster.map_shared_rank(&c_l[rank], 0) = Lt;
        }
    }
    {
        // every thread of every CTA of the cluster reaches the barrier (no early return);
        // after it only rank 0 reads, and only its own shared memory
        namespace cg = cooperative_groups;
        cg::this_cluster().sync();
        if (rank == 0 && grp == 0) {
            float Mt = -INFINITY;
#pragma unroll
            for (int r = 0; r < kMergeMaxCluster; ++r)
                if (r < S) Mt = fmaxf(Mt, c_m[r]);
            float Ot = 0.f, Lt = 0.f;
            if (Mt != -INFINITY) {
#pragma unroll
                for (int r = 0; r < kMergeMaxCluster; ++r) {
                    if (r < S) {
                        const float w = c_m[r] == -INFINITY ? 0.f : ex2(c_m[r] - Mt);
                        Ot += c_o[r][d] * w;
                        Lt += c_l[r] * w;
                    }
                }
            }
            T* ob = static_cast<T*>(a.out) + b * a.o_stride_b + (int64_t)hq * a.o_stride_h;
            ob[d] = from_f<T>(Lt > 0.f ? Ot / Lt : 0.f);
        }
    }
}

// ------------------------------------------------------------------------------ host side
static int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

// Self-test of the bounded waits: every thread of one CTA waits on a barrier that nothing
// arrives on.  The first to reach the limit sets the CTA abort flag and the error flag; the
// others then return at once.  result[1]: some wait reported success (expected 0);
// result[2]: a second wait after the abort returned within half the limit (expected 1).
__global__ void __launch_bounds__(64) wait_timeout_kernel(int* result, long long limit) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    const bool first = mbar_wait(&bar, 0, result, &abort, limit);
    const long long t0 = clock64();
    const bool second = mbar_wait(&bar, 0, result, &abort, limit);
    const bool quick = clock64() - t0 < limit / 2;
    if (first || second) atomicExch(result + 1, 1);
    __syncthreads();
    if (threadIdx.x == 0) result[2] = quick ? 1 : 0;
}

struct Plan {
    int64_t n_tiles, seq_pos, lead, total, W, grid, maxc;
    int wph, stages, stage_bytes, tile_bytes, kv_tile_bytes, half_bytes, smem_bytes;
};

static Plan make_plan(int64_t B, int64_t N, int Hkv, int D, bool attend) {
    Plan p{};
    p.n_tiles = (N + kTileTokens - 1) / kTileTokens;
    p.wph = kComputeWarps / Hkv;
    // A CTA whose range crosses from one sequence to the next pays ~3-4.5 us more than the
    // others (the appended token at the first sequence's end, its partials out, the next
    // query in): a per-CTA timeline put those CTAs last in every launch.  Three stages of
    // empty positions before every sequence give them that much less real work, so they
    // finish with the rest (with one sequence no range crosses a boundary).
    p.lead = B > 1 ? 3 * p.wph : 0;
    p.seq_pos = p.n_tiles + p.lead;
    p.total = B * p.seq_pos;
    const int64_t sms = num_sms();
    const int64_t grid0 = p.total < sms ? p.total : sms;
    p.W = grid0 > 0 ? (p.total + grid0 - 1) / grid0 : 1;
    p.grid = p.W > 0 ? (p.total + p.W - 1) / p.W : 0;
    p.maxc = p.seq_pos / p.W + 2;
    p.half_bytes = Hkv * kTileTokens * 128;
    p.kv_tile_bytes = (D / 64) * p.half_bytes;
    p.tile_bytes = (attend ? 2 : 1) * p.kv_tile_bytes;
    p.stage_bytes = p.wph * p.tile_bytes;
    p.stages = kSmemBudget / p.stage_bytes;
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    p.smem_bytes = p.stages * p.stage_bytes + (int)sizeof(SmemTail) + 1024;
    return p;
}

// The driver's tensor-map encoder, looked up through the runtime so the library does not
// link libcuda (it loads on hosts without a driver; the lookup happens at the first launch).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// 5-D map over one K or V storage: dims (D, 16 tokens, then kv head / sequence / page slot
// in ascending stride order); the box covers 64 elements x 16 tokens x all kv heads, so it
// lands in shared memory as [Hkv][16][64] whatever the storage order.  role[] reports which
// of the three outer dims is which.
static bool encode_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int D, int Hkv,
                       int64_t B, int64_t slots, int64_t st_t, int64_t st_h, int64_t st_b,
                       int64_t st_p, int role[3]) {
    struct Dim { int64_t n, stride; int box, role; };
    Dim outer[3] = {{Hkv, st_h, Hkv, 0}, {B, st_b, 1, 1}, {slots, st_p, 1, 2}};
    for (int i = 0; i < 3; ++i)
        for (int k = i + 1; k < 3; ++k)
            if (outer[k].stride < outer[i].stride) { Dim t = outer[i]; outer[i] = outer[k]; outer[k] = t; }
    const cuuint64_t dims[5] = {(cuuint64_t)D, (cuuint64_t)kTileTokens, (cuuint64_t)outer[0].n,
                                (cuuint64_t)outer[1].n, (cuuint64_t)outer[2].n};
    const cuuint64_t strides[4] = {(cuuint64_t)st_t * 2, (cuuint64_t)outer[0].stride * 2,
                                   (cuuint64_t)outer[1].stride * 2, (cuuint64_t)outer[2].stride * 2};
    const cuuint32_t box[5] = {64, (cuuint32_t)kTileTokens, (cuuint32_t)outer[0].box,
                               (cuuint32_t)outer[1].box, (cuuint32_t)outer[2].box};
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    for (int i = 0; i < 3; ++i) role[i] = outer[i].role;
    const EncodeTiledFn encode = encode_tiled_fn();
    if (!encode) return false;
    CUresult r = encode(map, dt, 5, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <typename T, int D, int GP, int MODE>
static cudaError_t launch_t(const FusedParams& f, const Plan& pl, CUtensorMapDataType dt,
                            cudaStream_t stream) {
    CUtensorMap mk, mv;
    int role[3];
    if (!encode_map(&mk, f.k, dt, D, f.Hkv, f.B, f.num_slots, f.stride_t, f.stride_h, f.stride_b,
                    f.stride_p, role))
        return cudaErrorInvalidValue;
    if (f.attend) {
        if (!encode_map(&mv, f.v, dt, D, f.Hkv, f.B, f.num_slots, f.stride_t, f.stride_h,
                        f.stride_b, f.stride_p, role))
            return cudaErrorInvalidValue;
    } else {
        mv = mk;
    }
    auto kern = decode_kernel<T, D, GP, MODE>;
    {
        // function attributes are per device: set once on each device this process uses
        static std::mutex mu;
        static bool done[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 0 || dev >= 64 || !done[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(
                kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                kSmemBudget + (int)sizeof(SmemTail) + (int)sizeof(QRows) + 1024);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) done[dev] = true;
        }
    }
    DevArgs a{};
    a.q = f.q; a.q_stride_b = f.q_stride_b; a.q_stride_h = f.q_stride_h;
    a.Hq = f.Hq; a.Hkv = f.Hkv; a.G = f.Hq / f.Hkv; a.wph = pl.wph;
    a.B = f.B; a.N = f.N; a.n_tiles = pl.n_tiles; a.total = pl.total; a.W = pl.W; a.maxc = pl.maxc;
    a.seq_pos = pl.seq_pos; a.lead = pl.lead;
    // one-sequence launches of the instances with tensor-core logits fold their tile slots'
    // partials inside the CTA (one partial per CTA and row for the merge)
    constexpr bool kMmaLayout = GP == 8 || MODE == 1 || MODE == 2;
    a.pw = (kMmaLayout && f.B == 1 && pl.wph > 1 && f.attend) ? 1 : pl.wph;
    a.pt = f.page_table; a.pt_stride_b = f.pt_stride_b; a.num_slots = f.num_slots;
    a.row_map = f.row_map;
    a.sal = f.sal; a.sal_stride_b = f.sal_stride_b; a.sal_stride_p = f.sal_stride_p;
    a.scale_r = f.scale_r; a.logit_log2 = f.logit_mul * 1.4426950408889634f;
    a.decay = f.decay; a.omd = f.one_minus_decay;
    a.attend = f.attend; a.score = f.sal != nullptr || f.xc.x != nullptr;
    a.sal_bulk = f.sal && !f.xc.x && !(reinterpret_cast<uintptr_t>(f.sal) & 15) &&
                 !((f.sal_stride_b * 4) & 15) && !((f.sal_stride_p * 4) & 15);
    a.out = f.out; a.o_stride_b = f.o_stride_b; a.o_stride_h = f.o_stride_h;
    a.partials = f.partials; a.counters = f.counters; a.err = f.err;
    a.stages = pl.stages; a.stage_bytes = pl.stage_bytes; a.tile_bytes = pl.tile_bytes;
    a.kv_tile_bytes = pl.kv_tile_bytes; a.half_bytes = pl.half_bytes;
    for (int i = 0; i < 3; ++i) a.role[i] = role[i];
    a.k_new = (f.k_new && (f.sal || f.xc.x) && (f.attend || f.pool)) ? f.k_new : nullptr;
    a.v_new = f.v_new; a.new_stride_b = f.new_stride_b; a.new_stride_h = f.new_stride_h;
    a.pt_w = f.pt_w; a.free_stack = f.free_stack; a.free_top = f.free_top;
    a.sal_init_norm = f.sal_init_norm;
    a.kpool = const_cast<void*>(f.k); a.vpool = const_cast<void*>(f.v);
    a.stride_b = f.stride_b; a.stride_h = f.stride_h; a.stride_p = f.stride_p;
    a.stride_t = f.stride_t;
    const bool two_q = f.q2 != nullptr;
    a.q2 = two_q ? f.q2 : f.q;
    a.q2_stride_b = two_q ? f.q2_stride_b : f.q_stride_b;
    a.q2_stride_h = two_q ? f.q2_stride_h : f.q_stride_h;
    a.attn_log2 = f.scale_r * f.logit_mul * 1.4426950408889634f;
    a.score_n = f.has_score_n ? f.score_n : f.N;
    a.xc = f.xc;
    a.pool = f.pool; a.pool_first = f.pool_first; a.pool_num = f.pool_num;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    constexpr bool kScreen = GP == 8 && MODE != 1;   // as SCREEN in decode_kernel
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)pl.smem_bytes + (kScreen ? sizeof(QRows) : 0);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = counted(cudaLaunchKernelEx(&cfg, kern, mk, mv, a), 1);
    if (e != cudaSuccess || !f.attend) return e;
    // CTAs per row: enough that each folds ~kMergePartialsPerCta partials (rows of a batch-1
    // launch have hundreds); maxc * wph bounds the partials of every row
    const int64_t np_max = pl.maxc * a.pw;
    int S = (int)((np_max + kMergePartialsPerCta - 1) / kMergePartialsPerCta);
    S = S < 1 ? 1 : S > kMergeMaxCluster ? kMergeMaxCluster : S;
    MergeArgs m{f.partials, f.out, f.o_stride_b, f.o_stride_h, f.Hq, pl.wph, pl.seq_pos, pl.W,
                pl.maxc, a.pw, S};
    cudaLaunchAttribute mattr[2];
    mattr[0] = attr[0];
    mattr[1].id = cudaLaunchAttributeClusterDimension;
    mattr[1].val.clusterDim.x = (unsigned)S;
    mattr[1].val.clusterDim.y = 1;
    mattr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t mcfg{};
    mcfg.gridDim = dim3((unsigned)(f.B * f.Hq * S));
    mcfg.blockDim = dim3(kMergeGroups * D);
    mcfg.stream = stream;
    mcfg.attrs = mattr;
    mcfg.numAttrs = S > 1 ? 2 : 1;
    if (S > 1) return counted(cudaLaunchKernelEx(&mcfg, merge_cluster_kernel<T, D>, m), 1);
    return counted(cudaLaunchKernelEx(&mcfg, merge_kernel<T, D>, m), 1);
}

}  // namespace sm100

// ------------------------------------------------------------------------------ dispatch
bool fused_supported(int dtype, int D, int Hkv, int Hq, int64_t page_size, int64_t stride_t,
                     int64_t stride_h, int64_t stride_b, int64_t stride_p, const void* k,
                     const void* v) {
    if (dtype != RKV_BF16 && dtype != RKV_F16) return false;
    if (D != 64 && D != 128) return false;
    if (Hkv != 1 && Hkv != 2 && Hkv != 4 && Hkv != 8) return false;
    if (Hq % Hkv != 0 || Hq / Hkv > 8) return false;
    if (page_size != sm100::kTileTokens || stride_t != D) return false;
    const int64_t strides[3] = {stride_h, stride_b, stride_p};
    for (int64_t st : strides)
        if (st <= 0 || (st * 2) % 16 != 0 || st * 2 >= (int64_t(1) << 40)) return false;
    if ((reinterpret_cast<uintptr_t>(k) & 15) || (reinterpret_cast<uintptr_t>(v) & 15)) return false;
    return true;
}

size_t fused_workspace_bytes(int64_t B, int Hq, int Hkv, int D, int64_t N) {
    if (B <= 0 || Hkv <= 0) return 0;
    sm100::Plan pl = sm100::make_plan(B, N, Hkv, D, true);
    return (size_t)B * pl.maxc * pl.wph * Hq * (D + 4) * sizeof(float);
}

cudaError_t launch_wait_selftest(int* result, long long limit, cudaStream_t st) {
    sm100::wait_timeout_kernel<<<1, 64, 0, st>>>(result, limit);
    return counted(cudaGetLastError(), 1);
}

cudaError_t launch_fused(const FusedParams& p, cudaStream_t st) {
    using namespace sm100;
    if (p.B > (RKV_WORKSPACE_HEADER_BYTES - 256) / 4) return cudaErrorNotSupported;
    if (p.attend && (!p.partials || !p.counters || !p.out)) return cudaErrorInvalidValue;
    const int G = p.Hq / p.Hkv;
    const Plan pl = make_plan(p.B, p.N, p.Hkv, p.D, p.attend != 0);
    if (pl.grid == 0) return cudaSuccess;
    // attention only: tensor-core logits; two queries: canonical scores of q + tensor-core
    // logits of q2; otherwise one query serves both (canonical scores)
    const bool scoring = p.sal != nullptr || p.xc.x != nullptr;
    const int mode = !scoring ? 1 : (p.q2 && p.attend) ? 2 : p.xc.x ? 3 : p.pool ? 4 : 0;
    if (mode == 1 && !p.attend) return cudaErrorInvalidValue;
    if (p.q2 && p.xc.x) return cudaErrorNotSupported;   // partial scoring of the two-query step
    if (p.pool && (p.attend || p.xc.x || p.q2 || p.has_score_n || !p.sal))
        return cudaErrorInvalidValue;                     // pooling is the score-only pass
    const bool bf = p.dtype == RKV_BF16;
    const auto dt = bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int gp = G <= 2 ? 2 : G <= 4 ? 4 : 8;
    // MODE 1 has no canonical dots: its group width does not matter, one instance per shape
#define RKV_LAUNCH(T_, D_)                                                                     \
    (mode == 1   ? launch_t<T_, D_, 2, 1>(p, pl, dt, st)                                      \
     : mode == 2 ? (gp == 2 ? launch_t<T_, D_, 2, 2>(p, pl, dt, st)                           \
                    : gp == 4 ? launch_t<T_, D_, 4, 2>(p, pl, dt, st)                         \
                              : launch_t<T_, D_, 8, 2>(p, pl, dt, st))                        \
     : mode == 3 ? (gp == 2 ? launch_t<T_, D_, 2, 3>(p, pl, dt, st)                           \
                    : gp == 4 ? launch_t<T_, D_, 4, 3>(p, pl, dt, st)                         \
                              : launch_t<T_, D_, 8, 3>(p, pl, dt, st))                        \
     : mode == 4 ? (gp == 2 ? launch_t<T_, D_, 2, 4>(p, pl, dt, st)                           \
                    : gp == 4 ? launch_t<T_, D_, 4, 4>(p, pl, dt, st)                         \
                              : launch_t<T_, D_, 8, 4>(p, pl, dt, st))                        \
                 : (gp == 2 ? launch_t<T_, D_, 2, 0>(p, pl, dt, st)                           \
                    : gp == 4 ? launch_t<T_, D_, 4, 0>(p, pl, dt, st)                         \
                              : launch_t<T_, D_, 8, 0>(p, pl, dt, st)))
    cudaError_t e;
    if (bf) e = p.D == 128 ? RKV_LAUNCH(__nv_bfloat16, 128) : RKV_LAUNCH(__nv_bfloat16, 64);
    else e = p.D == 128 ? RKV_LAUNCH(__half, 128) : RKV_LAUNCH(__half, 64);
#undef RKV_LAUNCH
    return e;
}

}  // namespace rkv
