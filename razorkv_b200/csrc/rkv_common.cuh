// Shared device helpers of the RazorKV decode path (sm_100a).
//
// Canonical dot product.  The salience score of a token is
//     R = max over query rows of  sum_d fl(q_d * scale) * k_d        (razorkv/cache.py:274-280)
// computed in fp32.  Page selection is decided by these values, so every kernel that
// produces them uses one fixed evaluation order that a CPU restatement can repeat exactly:
// eight lanes cooperate on a row; lane j owns the 16-byte chunks c = j, j+8, j+16, ... of
// the K row (CH = 16 / sizeof(K element) elements per chunk).  Listing the lane's elements
// in ascending order, those at even positions accumulate into one chain and those at odd
// positions into a second, each by fused multiply-add from +0.0f (the two halves of one
// packed f32x2 FMA in the sm_100a kernel); the lane partial is even + odd.  The eight
// partials are then combined by an xor-4, xor-2, xor-1 butterfly, i.e.
//     ((p0 + p4) + (p2 + p6)) + ((p1 + p5) + (p3 + p7)).
// fp32 addition is commutative, so every lane of the group ends with the same value.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/razorkv_b200.h"

namespace rkv {

constexpr int kMaxHeadDim = 256;

__host__ __device__ inline int elt_bytes(int dtype) { return dtype == RKV_F32 ? 4 : 2; }

__device__ __forceinline__ float load_elt(const void* base, int64_t idx, int dtype) {
    if (dtype == RKV_F32) return static_cast<const float*>(base)[idx];
    if (dtype == RKV_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
    return __half2float(static_cast<const __half*>(base)[idx]);
}

__device__ __forceinline__ void store_elt(void* base, int64_t idx, int dtype, float v) {
    if (dtype == RKV_F32) static_cast<float*>(base)[idx] = v;
    else if (dtype == RKV_BF16) static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
    else static_cast<__half*>(base)[idx] = __float2half_rn(v);
}

// Sum of the eight lane partials of an 8-lane group (lanes 8g .. 8g+7 of a warp), in the
// canonical order.  All eight lanes return the same value.
__device__ __forceinline__ float group8_sum(float p) {
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 4));
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 2));
    p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 1));
    return p;
}

// Monotone mapping of fp32 to uint32 (every NaN maps to the top).
__device__ __forceinline__ uint32_t ordered_key(float f) {
    uint32_t u = __float_as_uint(f);
    if (f != f) return 0xffffffffu;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
    if (k == 0xffffffffu) return __uint_as_float(0x7fc00000u);
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Location of logical token t of one (sequence, kv-head) plane.
//   page_table == nullptr : contiguous rows, element offset t * stride_t
//   otherwise             : page page_table[t / P] (times stride_p) plus (t % P) * stride_t
//   num_slots > 0         : a page id outside [0, num_slots) reads physical page 0 instead
//                           (a caller's table is never trusted to stay inside the storage)
struct TokenMap {
    const int64_t* page_table;   // [.., n_pages] int64; row for this sequence already applied
    int64_t page_size;
    int64_t stride_p;            // elements between physical pages
    int64_t stride_t;            // elements between tokens inside a page
    int64_t num_slots = 0;       // physical pages in the storage (0: ids not checked)
    // optional row map of a cache pool ([slots][batch] int32): sequence `seq` of the page in
    // slot s lives in row row_map[s * batch + seq]; offset() then adds (row - seq) * stride_b
    // to a base that already holds seq * stride_b.  Entries outside [0, batch) read row seq.
    const int32_t* row_map = nullptr;
    int64_t batch = 0, seq = 0, stride_b = 0;
    __device__ __forceinline__ int64_t offset(int64_t t) const {
        if (page_table == nullptr) return t * stride_t;
        int64_t pg = page_table[t / page_size];
        if (num_slots > 0 && (pg < 0 || pg >= num_slots)) pg = 0;
        int64_t off = pg * stride_p + (t % page_size) * stride_t;
        if (row_map != nullptr) {
            const int64_t r = row_map[pg * batch + seq];
            if (r >= 0 && r < batch) off += (r - seq) * stride_b;
        }
        return off;
    }
};

}  // namespace rkv
