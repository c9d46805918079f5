// C-ABI entry points of librazorkv_b200.so: argument validation, path choice, launch.
// Every function returns an rkv_status and never allocates, frees or synchronises.
#include <cuda.h>
#include <math.h>
#include <string.h>

#include <atomic>

#include "../../include/razorkv_b200.h"
#include "rkv_common.cuh"
#include "rkv_kernels.h"

using namespace rkv;

namespace rkv {
static std::atomic<unsigned long long> g_launches{0};
void count_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }
}  // namespace rkv

namespace {

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

inline int status_of(cudaError_t e) {
    if (e == cudaSuccess) return RKV_OK;
    if (e == cudaErrorNotSupported) return RKV_ERR_UNSUPPORTED;
    return RKV_ERR_CUDA;
}

inline bool dtype_ok(int d) { return d == RKV_F32 || d == RKV_F16 || d == RKV_BF16; }

// Workspace layout: [0, 4) error flag, [256, header) cross-CTA counters (int32; every launch
// leaves them at zero), [header, ...) scratch of the call.
inline int* ws_err(void* ws) { return static_cast<int*>(ws); }
inline int* ws_counters(void* ws) { return reinterpret_cast<int*>(static_cast<char*>(ws) + 256); }
inline float* ws_body(void* ws) {
    return reinterpret_cast<float*>(static_cast<char*>(ws) + RKV_WORKSPACE_HEADER_BYTES);
}

int check_kv(const rkv_kv_layout* kv, bool need_v) {
    if (!kv || !kv->k || (need_v && !kv->v)) return RKV_ERR_INVALID_ARGUMENT;
    if (!dtype_ok(kv->dtype)) return RKV_ERR_UNSUPPORTED;
    if (kv->head_dim < 1 || kv->head_dim > kMaxHeadDim) return RKV_ERR_UNSUPPORTED;
    if (kv->batch < 0 || kv->num_kv_heads < 1 || kv->num_tokens < 0) return RKV_ERR_INVALID_ARGUMENT;
    if (kv->page_table && kv->page_size < 1) return RKV_ERR_INVALID_ARGUMENT;
    // a row map describes a cache pool: one page table shared by every sequence (without a
    // page table it is not read)
    if (kv->row_map && kv->page_table && kv->pt_stride_b != 0) return RKV_ERR_INVALID_ARGUMENT;
    return RKV_OK;
}

int check_q(const rkv_query* q, const rkv_kv_layout* kv) {
    if (!q || !q->q) return RKV_ERR_INVALID_ARGUMENT;
    if (!dtype_ok(q->dtype)) return RKV_ERR_UNSUPPORTED;
    if (q->num_heads < 1 || q->num_heads % kv->num_kv_heads != 0) return RKV_ERR_INVALID_ARGUMENT;
    if (q->q_len < 1) return RKV_ERR_INVALID_ARGUMENT;
    return RKV_OK;
}

float resonance_scale(int D) { return (float)(1.0 / sqrt((double)D)); }

AttnParams attn_params(const rkv_query* q, const rkv_kv_layout* kv, float scale, int causal,
                       const rkv_output* out) {
    AttnParams p{};
    p.q = q->q; p.q_dtype = q->dtype;
    p.q_stride_b = q->stride_b; p.q_stride_h = q->stride_h; p.q_stride_t = q->stride_t;
    p.Hq = q->num_heads; p.QL = (int)q->q_len;
    p.k = kv->k; p.v = kv->v; p.kv_dtype = kv->dtype; p.D = kv->head_dim;
    p.Hkv = (int)kv->num_kv_heads; p.B = kv->batch; p.N = kv->num_tokens;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.page_size = kv->page_size;
    p.page_table = kv->page_table; p.pt_stride_b = kv->pt_stride_b;
    p.num_slots = kv->page_table ? kv->num_slots : 0;
    p.row_map = kv->row_map;
    p.scale = scale > 0.0f ? scale : (float)(1.0 / sqrt((double)kv->head_dim));
    p.causal = causal;
    p.out = out->out; p.out_dtype = out->dtype;
    p.o_stride_b = out->stride_b; p.o_stride_h = out->stride_h; p.o_stride_t = out->stride_t;
    return p;
}

// The screened instances (5-8 query heads per kv head) read query rows of the scoring query
// with 16-byte loads: its base and head / sequence strides must keep rows 16-byte aligned.
bool q_rows_aligned(const rkv_query* q) {
    const int64_t eb = q->dtype == RKV_F32 ? 4 : 2;
    return !(reinterpret_cast<uintptr_t>(q->q) & 15) && (q->stride_b * eb) % 16 == 0 &&
           (q->stride_h * eb) % 16 == 0;
}

bool fast_ok(const rkv_query* q, const rkv_kv_layout* kv, bool need_v) {
    if (q->q_len != 1) return false;
    if (!kv->page_table) return false;
    if (q->num_heads / kv->num_kv_heads > 4 && !q_rows_aligned(q)) return false;
    return fused_supported(kv->dtype, kv->head_dim, (int)kv->num_kv_heads, q->num_heads,
                           kv->page_size, kv->stride_t, kv->stride_h, kv->stride_b,
                           kv->stride_p, kv->k, need_v ? kv->v : kv->k) &&
           q->dtype == kv->dtype;
}

FusedParams fused_params(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
                         float decay, float omd, float scale, const rkv_output* out) {
    FusedParams p{};
    p.q = q->q; p.q_stride_b = q->stride_b; p.q_stride_h = q->stride_h;
    p.Hq = q->num_heads; p.Hkv = (int)kv->num_kv_heads; p.D = kv->head_dim;
    p.dtype = kv->dtype; p.B = kv->batch; p.N = kv->num_tokens;
    p.k = kv->k; p.v = kv->v;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.num_slots = kv->num_slots;
    p.page_table = kv->page_table; p.pt_stride_b = kv->pt_stride_b;
    p.row_map = kv->row_map;
    p.sal = sal ? sal->s : nullptr;
    p.sal_stride_b = sal ? sal->stride_b : 0; p.sal_stride_p = sal ? sal->stride_p : 0;
    p.scale_r = resonance_scale(kv->head_dim);
    const float sc = scale > 0.0f ? scale : p.scale_r;
    p.logit_mul = sc / p.scale_r;
    p.decay = decay; p.one_minus_decay = omd;
    p.attend = out ? 1 : 0;
    if (out) { p.out = out->out; p.o_stride_b = out->stride_b; p.o_stride_h = out->stride_h; }
    return p;
}

}  // namespace

namespace rkv {
// The argument checks rkv_decode_attention makes before it touches the workspace (shared with
// the no-allocation entry point, which must reject a call before it queues any work).
int attention_args_status(const rkv_query* q, const rkv_kv_layout* kv, const rkv_output* out) {
    int st = check_kv(kv, true);
    if (st) return st;
    if ((st = check_q(q, kv))) return st;
    if (!out || !out->out || !dtype_ok(out->dtype)) return RKV_ERR_INVALID_ARGUMENT;
    return RKV_OK;
}
}  // namespace rkv

extern "C" {

const char* rkv_status_string(int s) {
    switch (s) {
        case RKV_OK: return "ok";
        case RKV_ERR_INVALID_ARGUMENT: return "invalid argument";
        case RKV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
        case RKV_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
        case RKV_ERR_FREE_LIST_EXHAUSTED: return "free page list exhausted";
        case RKV_ERR_ALIGNMENT: return "misaligned pointer or stride";
        case RKV_ERR_CUDA: return "CUDA launch or runtime error";
        case RKV_ERR_PAGE_OUT_OF_RANGE: return "page index out of range";
        default: return "unknown status";
    }
}

int rkv_abi_version(void) { return 1; }

unsigned long long rkv_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int rkv_selftest_wait_timeout(int* result, long long limit_cycles, void* stream) {
    if (!result || limit_cycles < 1 || limit_cycles > 10000000000LL) return RKV_ERR_INVALID_ARGUMENT;
    return status_of(launch_wait_selftest(result, limit_cycles, S(stream)));
}

size_t rkv_decode_attention_workspace_size(const rkv_query* q, const rkv_kv_layout* kv) {
    // sizes of a call rkv_decode_attention would reject: no workspace can make it valid
    if (!q || !kv || kv->num_kv_heads < 1 || kv->batch < 0 || kv->num_tokens < 0 ||
        q->num_heads < 1 || q->q_len < 1 || kv->head_dim < 1 || kv->head_dim > kMaxHeadDim)
        return 0;
    const int64_t G = q->num_heads / kv->num_kv_heads;
    int splits = attn_num_splits(kv->num_tokens, kv->batch, kv->num_kv_heads, G * q->q_len);
    size_t generic = attn_workspace_floats(kv->batch, q->num_heads, q->q_len, kv->head_dim, splits) *
                     sizeof(float);
    size_t fast = fused_workspace_bytes(kv->batch, q->num_heads, (int)kv->num_kv_heads, kv->head_dim, kv->num_tokens);
    return RKV_WORKSPACE_HEADER_BYTES + (generic > fast ? generic : fast);
}

int rkv_decode_attention(const rkv_query* q, const rkv_kv_layout* kv, float scale, int causal,
                         const rkv_output* out, void* workspace, size_t workspace_bytes,
                         void* stream) {
    int st = attention_args_status(q, kv, out);
    if (st) return st;
    if (kv->batch == 0) return RKV_OK;
    if (workspace_bytes < rkv_decode_attention_workspace_size(q, kv) || !workspace)
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    if (!causal && kv->num_tokens > 0 && fast_ok(q, kv, true)) {
        FusedParams p = fused_params(q, kv, nullptr, 0.f, 0.f, scale, out);
        p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
        return status_of(launch_fused(p, S(stream)));
    }
    AttnParams p = attn_params(q, kv, scale, causal, out);
    const int64_t G = q->num_heads / kv->num_kv_heads;
    p.num_splits = attn_num_splits(kv->num_tokens, kv->batch, kv->num_kv_heads, G * q->q_len);
    p.workspace = ws_body(workspace);
    return status_of(launch_attention(p, S(stream)));
}

int rkv_page_salience_pool(const float* sal, int64_t batch, int64_t seq_len, int64_t stride_b,
                           int64_t page_size, int pool_type, float* out, void* stream) {
    if (!sal || !out || batch < 0 || seq_len < 1 || page_size < 1) return RKV_ERR_INVALID_ARGUMENT;
    if (pool_type != RKV_POOL_MAX && pool_type != RKV_POOL_MEAN) return RKV_ERR_INVALID_ARGUMENT;
    if (seq_len < page_size) pool_type = RKV_POOL_MAX;   // the reference returns the row max
    return status_of(launch_pool(sal, batch, seq_len, stride_b, page_size,
                                 pool_type == RKV_POOL_MEAN, out, S(stream)));
}

// rkv_append and rkv_append_partial: sal may be null only with an exchange block (xc.x).
static int append_impl(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
                       const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                       int64_t new_stride_t, int64_t n_new, int64_t pos, int64_t* page_table,
                       const int64_t* free_stack, int64_t free_top, int salience_init,
                       const Exchange& xc, void* stream) {
    int st = check_kv(kv, true);
    if (st) return st;
    if ((!xc.x && (!sal || !sal->s)) || !k_new || !v_new || !page_table || !free_stack)
        return RKV_ERR_INVALID_ARGUMENT;
    if (n_new < 0 || pos < 0 || free_top < 0 || kv->page_size < 1) return RKV_ERR_INVALID_ARGUMENT;
    const int64_t P = kv->page_size;
    const int64_t first_new = (pos + P - 1) / P;
    const int64_t last_page = (pos + n_new + P - 1) / P;   // exclusive
    const int64_t need = last_page > first_new ? last_page - first_new : 0;
    if (need > free_top) return RKV_ERR_FREE_LIST_EXHAUSTED;
    AppendParams p{};
    p.k = const_cast<void*>(kv->k); p.v = const_cast<void*>(kv->v); p.dtype = kv->dtype;
    p.D = kv->head_dim; p.Hkv = (int)kv->num_kv_heads; p.B = kv->batch;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.page_size = P;
    p.sal = sal ? sal->s : nullptr; p.sal_stride_b = sal ? sal->stride_b : 0;
    p.sal_stride_p = sal ? sal->stride_p : 0;
    p.k_new = k_new; p.v_new = v_new;
    p.new_stride_b = new_stride_b; p.new_stride_h = new_stride_h; p.new_stride_t = new_stride_t;
    p.n_new = n_new; p.pos = pos;
    p.page_table = page_table; p.free_stack = free_stack; p.free_top = free_top;
    p.salience_init = salience_init;
    p.xc = xc;
    p.row_map = kv->row_map;
    {
        const int64_t eb = kv->dtype == RKV_F32 ? 4 : 2;
        const int64_t strides[7] = {new_stride_b, new_stride_h, new_stride_t, kv->stride_b,
                                    kv->stride_h, kv->stride_p, kv->stride_t};
        bool ok = (kv->head_dim * eb) % 16 == 0;
        for (int64_t s : strides) ok = ok && (s * eb) % 16 == 0;
        for (const void* ptr : {k_new, v_new, kv->k, kv->v})
            ok = ok && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0;
        p.vec_ok = ok ? 1 : 0;
    }
    return status_of(launch_append(p, S(stream)));
}

int rkv_append(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
               const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
               int64_t new_stride_t, int64_t n_new, int64_t pos, int64_t* page_table,
               const int64_t* free_stack, int64_t free_top, int salience_init, void* stream) {
    if (!sal || !sal->s) return RKV_ERR_INVALID_ARGUMENT;
    return append_impl(kv, sal, k_new, v_new, new_stride_b, new_stride_h, new_stride_t, n_new,
                       pos, page_table, free_stack, free_top, salience_init, Exchange{}, stream);
}

// rkv_score and rkv_score_partial: sal may be null only with an exchange block (xc.x).
static int score_impl(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
                      float decay, float one_minus_decay, int ewma, const Exchange& xc,
                      void* stream) {
    int st = check_kv(kv, false);
    if (st) return st;
    if ((st = check_q(q, kv))) return st;
    if (!xc.x && (!sal || !sal->s)) return RKV_ERR_INVALID_ARGUMENT;
    if (kv->batch == 0 || kv->num_tokens == 0) return RKV_OK;
    if ((ewma || xc.x) && fast_ok(q, kv, false)) {
        FusedParams p = fused_params(q, kv, xc.x ? nullptr : sal, decay, one_minus_decay, 0.f, nullptr);
        p.xc = xc;
        return status_of(launch_fused(p, S(stream)));
    }
    ScoreParams p{};
    p.q = q->q; p.q_dtype = q->dtype;
    p.q_stride_b = q->stride_b; p.q_stride_h = q->stride_h; p.q_stride_t = q->stride_t;
    p.Hq = q->num_heads; p.QL = (int)q->q_len;
    p.k = kv->k; p.kv_dtype = kv->dtype; p.D = kv->head_dim; p.Hkv = (int)kv->num_kv_heads;
    p.B = kv->batch; p.N = kv->num_tokens;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.page_size = kv->page_size;
    p.page_table = kv->page_table; p.pt_stride_b = kv->pt_stride_b;
    p.sal = sal ? sal->s : nullptr; p.sal_stride_b = sal ? sal->stride_b : 0;
    p.sal_stride_p = sal ? sal->stride_p : 0;
    p.scale_r = resonance_scale(kv->head_dim);
    p.decay = decay; p.one_minus_decay = one_minus_decay; p.ewma = ewma;
    p.xc = xc;
    p.row_map = kv->row_map;
    return status_of(launch_score(p, S(stream)));
}

int rkv_score(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
              float decay, float one_minus_decay, int ewma, void* stream) {
    if (!sal || !sal->s) return RKV_ERR_INVALID_ARGUMENT;
    return score_impl(q, kv, sal, decay, one_minus_decay, ewma, Exchange{}, stream);
}

size_t rkv_decode_fused_workspace_size(const rkv_query* q, const rkv_kv_layout* kv) {
    return rkv_decode_attention_workspace_size(q, kv);
}

int rkv_decode_fused(const rkv_query* q, const rkv_kv_layout* kv, const rkv_salience* sal,
                     float decay, float one_minus_decay, float scale, const rkv_output* out,
                     void* workspace, size_t workspace_bytes, void* stream) {
    int st = check_kv(kv, true);
    if (st) return st;
    if ((st = check_q(q, kv))) return st;
    if (!sal || !sal->s || !out || !out->out) return RKV_ERR_INVALID_ARGUMENT;
    if (q->q_len != 1) return RKV_ERR_UNSUPPORTED;
    if (kv->batch == 0) return RKV_OK;
    if (workspace_bytes < rkv_decode_fused_workspace_size(q, kv) || !workspace)
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    if (kv->num_tokens > 0 && fast_ok(q, kv, true)) {
        FusedParams p = fused_params(q, kv, sal, decay, one_minus_decay, scale, out);
        p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
        return status_of(launch_fused(p, S(stream)));
    }
    // shapes outside the fused kernel: the two shape-general kernels back to back
    if ((st = rkv_score(q, kv, sal, decay, one_minus_decay, 1, stream))) return st;
    return rkv_decode_attention(q, kv, scale, 0, out, workspace, workspace_bytes, stream);
}

size_t rkv_decode_scored_workspace_size(const rkv_query* q_attn, const rkv_kv_layout* kv) {
    return rkv_decode_attention_workspace_size(q_attn, kv);
}

int rkv_decode_scored(const rkv_query* q_score, const rkv_query* q_attn, const rkv_kv_layout* kv,
                      const rkv_salience* sal, int64_t score_tokens, float decay,
                      float one_minus_decay, float scale, const rkv_output* out,
                      void* workspace, size_t workspace_bytes, void* stream) {
    int st = check_kv(kv, true);
    if (st) return st;
    if ((st = check_q(q_score, kv)) || (st = check_q(q_attn, kv))) return st;
    if (!sal || !sal->s || !out || !out->out) return RKV_ERR_INVALID_ARGUMENT;
    if (q_score->q_len != 1 || q_attn->q_len != 1) return RKV_ERR_UNSUPPORTED;
    if (q_score->num_heads != q_attn->num_heads) return RKV_ERR_INVALID_ARGUMENT;
    if (score_tokens < 0 || score_tokens > kv->num_tokens) return RKV_ERR_INVALID_ARGUMENT;
    if (kv->batch == 0) return RKV_OK;
    if (workspace_bytes < rkv_decode_scored_workspace_size(q_attn, kv) || !workspace)
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    if (kv->num_tokens > 0 && fast_ok(q_attn, kv, true) && q_score->dtype == q_attn->dtype &&
        (q_score->num_heads / kv->num_kv_heads <= 4 || q_rows_aligned(q_score))) {
        FusedParams p = fused_params(q_score, kv, sal, decay, one_minus_decay, scale, out);
        p.q2 = q_attn->q; p.q2_stride_b = q_attn->stride_b; p.q2_stride_h = q_attn->stride_h;
        p.has_score_n = 1; p.score_n = score_tokens;
        p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
        return status_of(launch_fused(p, S(stream)));
    }
    // shapes outside the fused kernel: score the first score_tokens tokens, then attend
    if (score_tokens > 0) {
        rkv_kv_layout scored = *kv;
        scored.num_tokens = score_tokens;
        if ((st = rkv_score(q_score, &scored, sal, decay, one_minus_decay, 1, stream))) return st;
    }
    return rkv_decode_attention(q_attn, kv, scale, 0, out, workspace, workspace_bytes, stream);
}

int rkv_append_decode(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
                      const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                      int64_t* page_table, const int64_t* free_stack, int64_t free_top,
                      int salience_init, const rkv_query* q, float decay, float one_minus_decay,
                      float scale, const rkv_output* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (!kv) return RKV_ERR_INVALID_ARGUMENT;
    rkv_kv_layout grown = *kv;
    grown.num_tokens = kv->num_tokens + 1;
    // One kernel does the append, the scoring and the attention when the fused kernel covers
    // the shape and the new rows are 16-byte vectors; otherwise append, then score + attend.
    int st = check_kv(&grown, true);
    if (st) return st;
    if ((st = check_q(q, &grown))) return st;
    const bool rows_aligned = k_new && v_new && !(reinterpret_cast<uintptr_t>(k_new) & 15) &&
                              !(reinterpret_cast<uintptr_t>(v_new) & 15) &&
                              !((new_stride_b * 2) & 15) && !((new_stride_h * 2) & 15);
    if (sal && sal->s && out && out->out && page_table && free_stack && grown.batch > 0 &&
        grown.page_table == page_table && grown.pt_stride_b == 0 && rows_aligned &&
        fast_ok(q, &grown, true) && (kv->num_tokens % kv->page_size != 0 || free_top >= 1)) {
        if (workspace_bytes < rkv_decode_fused_workspace_size(q, &grown) || !workspace)
            return RKV_ERR_WORKSPACE_TOO_SMALL;
        FusedParams p = fused_params(q, &grown, sal, decay, one_minus_decay, scale, out);
        p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
        p.k_new = k_new; p.v_new = v_new; p.new_stride_b = new_stride_b;
        p.new_stride_h = new_stride_h; p.pt_w = page_table; p.free_stack = free_stack;
        p.free_top = free_top; p.sal_init_norm = salience_init == RKV_SAL_NORM;
        return status_of(launch_fused(p, S(stream)));
    }
    st = rkv_append(kv, sal, k_new, v_new, new_stride_b, new_stride_h, 0, 1, kv->num_tokens,
                    page_table, free_stack, free_top, salience_init, stream);
    if (st) return st;
    return rkv_decode_fused(q, &grown, sal, decay, one_minus_decay, scale, out, workspace,
                            workspace_bytes, stream);
}

// ---- KV-head sharding -----------------------------------------------------------------------
static int exchange_status(const rkv_exchange* xc, const rkv_kv_layout* kv, int64_t need_cols) {
    if (!xc || !xc->x || xc->stride_b < need_cols || xc->norm_off < 0) return RKV_ERR_INVALID_ARGUMENT;
    if (xc->head0 < 0 || xc->num_kv_heads_total < 1 ||
        xc->head0 + kv->num_kv_heads > xc->num_kv_heads_total)
        return RKV_ERR_INVALID_ARGUMENT;
    return RKV_OK;
}

static Exchange exchange_of(const rkv_exchange* xc) {
    Exchange e{};
    e.x = xc->x; e.stride_b = xc->stride_b; e.norm_off = xc->norm_off;
    e.h0 = xc->head0; e.htot = xc->num_kv_heads_total;
    return e;
}

int rkv_append_partial(const rkv_kv_layout* kv, const void* k_new, const void* v_new,
                       int64_t new_stride_b, int64_t new_stride_h, int64_t new_stride_t,
                       int64_t n_new, int64_t pos, int64_t* page_table, const int64_t* free_stack,
                       int64_t free_top, int salience_init, const rkv_exchange* xc, void* stream) {
    int st = check_kv(kv, true);
    if (st) return st;
    if (n_new < 0) return RKV_ERR_INVALID_ARGUMENT;
    if ((st = exchange_status(xc, kv, xc ? xc->norm_off + n_new * xc->num_kv_heads_total : 0)))
        return st;
    return append_impl(kv, nullptr, k_new, v_new, new_stride_b, new_stride_h, new_stride_t,
                       n_new, pos, page_table, free_stack, free_top, salience_init,
                       exchange_of(xc), stream);
}

int rkv_score_partial(const rkv_query* q, const rkv_kv_layout* kv, const rkv_exchange* xc,
                      void* stream) {
    int st = check_kv(kv, false);
    if (st) return st;
    if ((st = check_q(q, kv))) return st;
    if ((st = exchange_status(xc, kv, kv->num_tokens))) return st;
    return score_impl(q, kv, nullptr, 0.f, 0.f, 1, exchange_of(xc), stream);
}

int rkv_append_decode_partial(const rkv_kv_layout* kv,
                              const void* k_new, const void* v_new, int64_t new_stride_b,
                              int64_t new_stride_h, int64_t* page_table,
                              const int64_t* free_stack, int64_t free_top, int salience_init,
                              const rkv_query* q, float scale, const rkv_output* out,
                              const rkv_exchange* xc, void* workspace, size_t workspace_bytes,
                              void* stream) {
    if (!kv) return RKV_ERR_INVALID_ARGUMENT;
    rkv_kv_layout grown = *kv;
    grown.num_tokens = kv->num_tokens + 1;
    int st = check_kv(&grown, true);
    if (st) return st;
    if ((st = check_q(q, &grown))) return st;
    if ((st = exchange_status(xc, kv, grown.num_tokens))) return st;
    if (xc->stride_b < xc->norm_off + xc->num_kv_heads_total) return RKV_ERR_INVALID_ARGUMENT;
    if (!out || !out->out) return RKV_ERR_INVALID_ARGUMENT;
    const bool rows_aligned = k_new && v_new && !(reinterpret_cast<uintptr_t>(k_new) & 15) &&
                              !(reinterpret_cast<uintptr_t>(v_new) & 15) &&
                              !((new_stride_b * 2) & 15) && !((new_stride_h * 2) & 15);
    if (page_table && free_stack && grown.batch > 0 && grown.page_table == page_table &&
        grown.pt_stride_b == 0 && rows_aligned && fast_ok(q, &grown, true) &&
        (kv->num_tokens % kv->page_size != 0 || free_top >= 1)) {
        if (workspace_bytes < rkv_decode_fused_workspace_size(q, &grown) || !workspace)
            return RKV_ERR_WORKSPACE_TOO_SMALL;
        FusedParams p = fused_params(q, &grown, nullptr, 0.f, 0.f, scale, out);
        p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
        p.k_new = k_new; p.v_new = v_new; p.new_stride_b = new_stride_b;
        p.new_stride_h = new_stride_h; p.pt_w = page_table; p.free_stack = free_stack;
        p.free_top = free_top; p.sal_init_norm = salience_init == RKV_SAL_NORM;
        p.xc = exchange_of(xc);
        return status_of(launch_fused(p, S(stream)));
    }
    // shapes outside the fused kernel: append, score, attend
    if ((st = rkv_append_partial(kv, k_new, v_new, new_stride_b, new_stride_h, 0, 1,
                                 kv->num_tokens, page_table, free_stack, free_top, salience_init,
                                 xc, stream)))
        return st;
    if ((st = rkv_score_partial(q, &grown, xc, stream))) return st;
    return rkv_decode_attention(q, &grown, scale, 0, out, workspace, workspace_bytes, stream);
}

// ---- CUDA IPC of an exchange region -----------------------------------------------------------
using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

static GetAddressRangeFn address_range_fn() {
    static GetAddressRangeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<GetAddressRangeFn>(nullptr);
        return reinterpret_cast<GetAddressRangeFn>(p);
    }();
    return fn;
}

int rkv_ipc_export(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) return RKV_ERR_INVALID_ARGUMENT;
    GetAddressRangeFn range = address_range_fn();
    if (!range) return RKV_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return RKV_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return RKV_ERR_CUDA;
    static_assert(sizeof(h) == RKV_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return RKV_OK;
}

int rkv_ipc_import(const void* handle, int64_t offset, void** ptr) {
    if (!handle || !ptr || offset < 0) return RKV_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    // mapped into the current device's context, with peer access enabled as needed
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        return RKV_ERR_CUDA;
    *ptr = static_cast<char*>(base) + offset;
    return RKV_OK;
}

int rkv_ipc_release(void* ptr, int64_t offset) {
    if (!ptr || offset < 0) return RKV_ERR_INVALID_ARGUMENT;
    return cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) == cudaSuccess ? RKV_OK : RKV_ERR_CUDA;
}

static int peer_status(const rkv_peer_exchange* px) {
    if (!px || !px->regions || !px->flags || !px->my_region || !px->my_flags) return RKV_ERR_INVALID_ARGUMENT;
    if (px->nranks < 1 || px->rank < 0 || px->rank >= px->nranks || px->sub < 1 || px->buf_off < 0)
        return RKV_ERR_INVALID_ARGUMENT;
    return RKV_OK;
}

int rkv_append_decode_peer(const rkv_kv_layout* kv, const void* k_new, const void* v_new,
                           int64_t new_stride_b, int64_t new_stride_h, int64_t* page_table,
                           const int64_t* free_stack, int64_t free_top, int salience_init,
                           const rkv_query* q, float scale, const rkv_output* out,
                           const rkv_exchange* xc, const rkv_peer_exchange* px, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (!kv || !xc) return RKV_ERR_INVALID_ARGUMENT;
    rkv_kv_layout grown = *kv;
    grown.num_tokens = kv->num_tokens + 1;
    int st = check_kv(&grown, true);
    if (st) return st;
    if ((st = check_q(q, &grown))) return st;
    if ((st = peer_status(px))) return st;
    if (xc->stride_b < grown.num_tokens || xc->norm_off < grown.num_tokens ||
        xc->norm_off + xc->num_kv_heads_total > xc->stride_b || xc->head0 < 0 ||
        xc->head0 + kv->num_kv_heads > xc->num_kv_heads_total ||
        px->sub < grown.batch * xc->stride_b)
        return RKV_ERR_INVALID_ARGUMENT;
    if (!out || !out->out) return RKV_ERR_INVALID_ARGUMENT;
    const bool rows_aligned = k_new && v_new && !(reinterpret_cast<uintptr_t>(k_new) & 15) &&
                              !(reinterpret_cast<uintptr_t>(v_new) & 15) &&
                              !((new_stride_b * 2) & 15) && !((new_stride_h * 2) & 15);
    if (!(page_table && free_stack && grown.batch > 0 && grown.page_table == page_table &&
          grown.pt_stride_b == 0 && rows_aligned && fast_ok(q, &grown, true) &&
          (kv->num_tokens % kv->page_size != 0 || free_top >= 1)))
        return RKV_ERR_UNSUPPORTED;
    if (workspace_bytes < rkv_decode_fused_workspace_size(q, &grown) || !workspace)
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    FusedParams p = fused_params(q, &grown, nullptr, 0.f, 0.f, scale, out);
    p.partials = ws_body(workspace); p.counters = ws_counters(workspace); p.err = ws_err(workspace);
    p.k_new = k_new; p.v_new = v_new; p.new_stride_b = new_stride_b;
    p.new_stride_h = new_stride_h; p.pt_w = page_table; p.free_stack = free_stack;
    p.free_top = free_top; p.sal_init_norm = salience_init == RKV_SAL_NORM;
    p.xc = exchange_of(xc);
    p.xc.x = const_cast<int32_t*>(px->my_region);   // marks the partial mode
    p.xc.regions = px->regions; p.xc.flags = px->flags;
    p.xc.rank = px->rank; p.xc.nranks = px->nranks; p.xc.sub = px->sub;
    p.xc.buf_off = px->buf_off; p.xc.epoch = px->epoch;
    return status_of(launch_fused(p, S(stream)));
}

int rkv_salience_apply_peer(const rkv_kv_layout* kv, const rkv_salience* sal,
                            const rkv_exchange* xc, const rkv_peer_exchange* px,
                            int64_t score_tokens, int64_t new_first, int64_t n_new,
                            int salience_init, float decay, float one_minus_decay,
                            void* workspace, size_t workspace_bytes, void* stream) {
    if (!kv || !sal || !sal->s || !xc) return RKV_ERR_INVALID_ARGUMENT;
    int st = peer_status(px);
    if (st) return st;
    if (kv->batch < 0 || (kv->page_table && kv->page_size < 1)) return RKV_ERR_INVALID_ARGUMENT;
    if (score_tokens < 0 || new_first < 0 || n_new < 0) return RKV_ERR_INVALID_ARGUMENT;
    const int64_t end = score_tokens > new_first + n_new ? score_tokens : new_first + n_new;
    if (end > kv->num_tokens || xc->stride_b < score_tokens || xc->num_kv_heads_total < 1 ||
        px->sub < kv->batch * xc->stride_b ||
        (salience_init == RKV_SAL_NORM && n_new > 0 &&
         xc->stride_b < xc->norm_off + n_new * xc->num_kv_heads_total))
        return RKV_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < RKV_WORKSPACE_HEADER_BYTES) return RKV_ERR_WORKSPACE_TOO_SMALL;
    PeerApplyParams p{};
    p.sal = sal->s; p.sal_stride_b = sal->stride_b; p.sal_stride_p = sal->stride_p;
    p.page_table = kv->page_table; p.page_size = kv->page_size; p.B = kv->batch;
    p.region = px->my_region; p.flags = px->my_flags; p.nranks = px->nranks; p.sub = px->sub;
    p.buf_off = px->buf_off; p.epoch = px->epoch; p.stride_b = xc->stride_b;
    p.norm_off = xc->norm_off; p.htot = xc->num_kv_heads_total;
    p.score_tokens = score_tokens; p.new_first = new_first; p.n_new = n_new;
    p.norm_init = salience_init == RKV_SAL_NORM; p.decay = decay; p.one_minus_decay = one_minus_decay;
    p.err = ws_err(workspace);
    p.wait_limit = 2000000000LL;   // ~1 s at B200 clocks
    return status_of(launch_apply_peer(p, S(stream)));
}

int rkv_salience_apply(const rkv_kv_layout* kv, const rkv_salience* sal, const rkv_exchange* xc,
                       int64_t score_tokens, int64_t new_first, int64_t n_new,
                       int salience_init, float decay, float one_minus_decay, void* stream) {
    if (!kv || !sal || !sal->s) return RKV_ERR_INVALID_ARGUMENT;
    if (kv->batch < 0 || (kv->page_table && kv->page_size < 1)) return RKV_ERR_INVALID_ARGUMENT;
    if (score_tokens < 0 || new_first < 0 || n_new < 0) return RKV_ERR_INVALID_ARGUMENT;
    const int64_t end = score_tokens > new_first + n_new ? score_tokens : new_first + n_new;
    if (end > kv->num_tokens) return RKV_ERR_INVALID_ARGUMENT;
    if (!xc || !xc->x || xc->stride_b < score_tokens || xc->num_kv_heads_total < 1 ||
        (salience_init == RKV_SAL_NORM && n_new > 0 &&
         xc->stride_b < xc->norm_off + n_new * xc->num_kv_heads_total))
        return RKV_ERR_INVALID_ARGUMENT;
    ApplyParams p{};
    p.sal = sal->s; p.sal_stride_b = sal->stride_b; p.sal_stride_p = sal->stride_p;
    p.page_table = kv->page_table; p.page_size = kv->page_size; p.B = kv->batch;
    p.xc = exchange_of(xc);
    p.score_tokens = score_tokens; p.new_first = new_first; p.n_new = n_new;
    p.norm_init = salience_init == RKV_SAL_NORM; p.decay = decay; p.one_minus_decay = one_minus_decay;
    return status_of(launch_apply(p, S(stream)));
}

int rkv_append_score_pool(const rkv_kv_layout* kv, const rkv_salience* sal, const void* k_new,
                          const void* v_new, int64_t new_stride_b, int64_t new_stride_h,
                          int64_t* page_table, const int64_t* free_stack, int64_t free_top,
                          int salience_init, const rkv_query* q, float decay,
                          float one_minus_decay, int64_t first_token, int64_t num_pages,
                          float* scores, void* stream) {
    if (!kv || !sal || !sal->s || !scores) return RKV_ERR_INVALID_ARGUMENT;
    rkv_kv_layout grown = *kv;
    grown.num_tokens = kv->num_tokens + 1;
    int st = check_kv(&grown, true);
    if (st) return st;
    if ((st = check_q(q, &grown))) return st;
    if (first_token < 0 || num_pages < 0 || grown.page_size < 1 ||
        first_token + num_pages * grown.page_size > grown.num_tokens)
        return RKV_ERR_INVALID_ARGUMENT;
    const bool rows_aligned = k_new && v_new && !(reinterpret_cast<uintptr_t>(k_new) & 15) &&
                              !(reinterpret_cast<uintptr_t>(v_new) & 15) &&
                              !((new_stride_b * 2) & 15) && !((new_stride_h * 2) & 15);
    if (page_table && free_stack && grown.batch > 0 && grown.page_table == page_table &&
        grown.pt_stride_b == 0 && rows_aligned && fast_ok(q, &grown, true) &&
        first_token % grown.page_size == 0 &&
        (kv->num_tokens % kv->page_size != 0 || free_top >= 1)) {
        FusedParams p = fused_params(q, &grown, sal, decay, one_minus_decay, 0.f, nullptr);
        p.k_new = k_new; p.v_new = v_new; p.new_stride_b = new_stride_b;
        p.new_stride_h = new_stride_h; p.pt_w = page_table; p.free_stack = free_stack;
        p.free_top = free_top; p.sal_init_norm = salience_init == RKV_SAL_NORM;
        p.pool = scores; p.pool_first = first_token / grown.page_size; p.pool_num = num_pages;
        return status_of(launch_fused(p, S(stream)));
    }
    // shapes outside the fused kernel: append, score, pool
    if ((st = rkv_append(kv, sal, k_new, v_new, new_stride_b, new_stride_h, 0, 1, kv->num_tokens,
                         page_table, free_stack, free_top, salience_init, stream)))
        return st;
    if ((st = rkv_score(q, &grown, sal, decay, one_minus_decay, 1, stream))) return st;
    return num_pages ? rkv_page_scores(&grown, sal, first_token, num_pages, grown.page_size,
                                       scores, stream)
                     : RKV_OK;
}

int rkv_select_compact_pages(const float* scores, int64_t batch, int64_t num_pages, int64_t k,
                             int64_t* page_table, int64_t sink_pages, int64_t tail_first_page,
                             int64_t n_pages_total, int64_t* free_stack, int64_t free_top,
                             int64_t* kept, float* margin, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (!scores || !kept || !page_table || !free_stack || batch < 1 || num_pages < 1 || k < 1 ||
        k > num_pages || sink_pages < 0 || free_top < 0)
        return RKV_ERR_INVALID_ARGUMENT;
    if (tail_first_page != sink_pages + num_pages || n_pages_total < tail_first_page)
        return RKV_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < rkv_select_pages_workspace_size(num_pages))
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    return status_of(launch_select_compact(scores, batch, num_pages, k, kept, margin,
                                           reinterpret_cast<uint32_t*>(ws_body(workspace)),
                                           page_table, sink_pages, tail_first_page,
                                           n_pages_total, free_stack, free_top, S(stream)));
}

int rkv_page_scores(const rkv_kv_layout* kv, const rkv_salience* sal, int64_t first_token,
                    int64_t num_pages, int64_t sel_page_size, float* scores, void* stream) {
    if (!kv || !sal || !sal->s || !scores) return RKV_ERR_INVALID_ARGUMENT;
    if (first_token < 0 || num_pages < 0 || sel_page_size < 1) return RKV_ERR_INVALID_ARGUMENT;
    if (first_token + num_pages * sel_page_size > kv->num_tokens) return RKV_ERR_INVALID_ARGUMENT;
    PageScoreParams p{};
    p.sal = sal->s; p.sal_stride_b = sal->stride_b; p.sal_stride_p = sal->stride_p;
    p.page_table = kv->page_table; p.page_size = kv->page_size;
    p.B = kv->batch; p.first_token = first_token; p.num_pages = num_pages;
    p.sel_page_size = sel_page_size; p.scores = scores;
    return status_of(launch_page_scores(p, S(stream)));
}

size_t rkv_select_pages_workspace_size(int64_t num_pages) {
    return RKV_WORKSPACE_HEADER_BYTES + (size_t)(num_pages > 0 ? num_pages : 1) * sizeof(uint32_t);
}

size_t rkv_workspace_error_flag_offset(void) { return 0; }

int rkv_select_pages(const float* scores, int64_t batch, int64_t num_pages, int64_t k,
                     int64_t* kept, float* margin, void* workspace, size_t workspace_bytes,
                     void* stream) {
    if (!scores || !kept || batch < 1 || num_pages < 1 || k < 1 || k > num_pages)
        return RKV_ERR_INVALID_ARGUMENT;
    if (!workspace || workspace_bytes < rkv_select_pages_workspace_size(num_pages))
        return RKV_ERR_WORKSPACE_TOO_SMALL;
    return status_of(launch_select(scores, batch, num_pages, k, kept, margin,
                                   reinterpret_cast<uint32_t*>(ws_body(workspace)), S(stream)));
}

int rkv_compact_pages(int64_t* page_table, int64_t sink_pages, int64_t num_pages,
                      const int64_t* kept, int64_t k, int64_t tail_first_page,
                      int64_t n_pages_total, int64_t* free_stack, int64_t free_top,
                      void* stream) {
    if (!page_table || !kept || !free_stack) return RKV_ERR_INVALID_ARGUMENT;
    if (sink_pages < 0 || num_pages < 1 || k < 1 || k > num_pages || free_top < 0)
        return RKV_ERR_INVALID_ARGUMENT;
    if (tail_first_page != sink_pages + num_pages || n_pages_total < tail_first_page)
        return RKV_ERR_INVALID_ARGUMENT;
    return status_of(launch_compact_pages(page_table, sink_pages, num_pages, kept, k,
                                          tail_first_page, n_pages_total, free_stack, free_top,
                                          S(stream)));
}

int rkv_compact_tokens(const rkv_kv_layout* kv, const rkv_salience* sal,
                       int64_t* new_page_table, const int64_t* free_stack, int64_t free_top,
                       int64_t new_len, int64_t sink, const int64_t* kept, int64_t k,
                       int64_t sel_page_size, int64_t hay_start, int64_t tail_src_start,
                       void* stream) {
    int st = check_kv(kv, true);
    if (st) return st;
    if (!kv->page_table || !sal || !sal->s || !new_page_table || !free_stack)
        return RKV_ERR_INVALID_ARGUMENT;
    if (k > 0 && !kept) return RKV_ERR_INVALID_ARGUMENT;
    if (new_len < 0 || sink < 0 || k < 0 || sel_page_size < 1) return RKV_ERR_INVALID_ARGUMENT;
    if (sink + k * sel_page_size > new_len) return RKV_ERR_INVALID_ARGUMENT;
    if (tail_src_start + (new_len - sink - k * sel_page_size) > kv->num_tokens)
        return RKV_ERR_INVALID_ARGUMENT;
    const int64_t pages = (new_len + kv->page_size - 1) / kv->page_size;
    if (pages > free_top) return RKV_ERR_FREE_LIST_EXHAUSTED;
    CompactTokensParams p{};
    p.k = const_cast<void*>(kv->k); p.v = const_cast<void*>(kv->v); p.dtype = kv->dtype;
    p.D = kv->head_dim; p.Hkv = kv->num_kv_heads; p.B = kv->batch;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.page_size = kv->page_size;
    p.sal = sal->s; p.sal_stride_b = sal->stride_b; p.sal_stride_p = sal->stride_p;
    p.old_pt = kv->page_table; p.new_pt = new_page_table; p.free_stack = free_stack;
    p.free_top = free_top; p.new_len = new_len; p.sink = sink; p.n_kept = k; p.kept = kept;
    p.sel_page_size = sel_page_size; p.hay_start = hay_start; p.tail_src_start = tail_src_start;
    p.row_map = kv->row_map;
    return status_of(launch_compact_tokens(p, S(stream)));
}

int rkv_release_pages(const int64_t* pages, int64_t n, int64_t* free_stack, int64_t free_top,
                      void* stream) {
    if ((n > 0 && !pages) || !free_stack || n < 0 || free_top < 0) return RKV_ERR_INVALID_ARGUMENT;
    return status_of(launch_release(pages, n, free_stack, free_top, S(stream)));
}

int rkv_gather_tokens(const rkv_kv_layout* kv, int which, void* dst, const rkv_salience* sal,
                      float* sal_dst, void* stream) {
    int st = check_kv(kv, which == 1);
    if (st) return st;
    if (!dst || (sal_dst && (!sal || !sal->s))) return RKV_ERR_INVALID_ARGUMENT;
    GatherParams p{};
    p.src = which == 1 ? kv->v : kv->k; p.dst = dst; p.dtype = kv->dtype;
    p.B = kv->batch; p.Hkv = kv->num_kv_heads; p.N = kv->num_tokens; p.D = kv->head_dim;
    p.stride_b = kv->stride_b; p.stride_h = kv->stride_h; p.stride_p = kv->stride_p;
    p.stride_t = kv->stride_t; p.page_size = kv->page_size;
    p.page_table = kv->page_table; p.pt_stride_b = kv->pt_stride_b;
    p.sal = sal ? sal->s : nullptr; p.sal_stride_b = sal ? sal->stride_b : 0;
    p.sal_stride_p = sal ? sal->stride_p : 0; p.sal_dst = sal_dst;
    p.row_map = kv->row_map;
    return status_of(launch_gather(p, S(stream)));
}

int rkv_reindex_batch(const rkv_kv_layout* src, const rkv_salience* src_sal,
                      const rkv_kv_layout* dst, const rkv_salience* dst_sal,
                      const int64_t* index, const int64_t* slots, int64_t num_listed,
                      int64_t num_moved, int* err, void* stream) {
    int st = check_kv(src, false);
    if (st || (st = check_kv(dst, false))) return st;
    if (num_listed < 0 || (num_listed > 0 && !slots) || (dst->batch > 0 && !index))
        return RKV_ERR_INVALID_ARGUMENT;
    if (src->dtype != dst->dtype || src->head_dim != dst->head_dim ||
        src->num_kv_heads != dst->num_kv_heads || src->page_size != dst->page_size ||
        src->page_size < 1 || src->num_slots < 0 || dst->num_slots < 0)
        return RKV_ERR_INVALID_ARGUMENT;
    if (!src->v != !dst->v || !src_sal != !dst_sal || (src_sal && (!src_sal->s || !dst_sal->s)))
        return RKV_ERR_INVALID_ARGUMENT;
    const int64_t D = src->head_dim, P = src->page_size;
    // every (slot, sequence) plane of K and V must be one contiguous run of Hkv*P*D elements
    for (const rkv_kv_layout* l : {src, dst})
        if (l->stride_t != D || l->stride_h != P * D) return RKV_ERR_UNSUPPORTED;
    const bool in_place = src->k == dst->k;
    if (in_place != (src->v == dst->v) ||
        (src_sal && in_place != (src_sal->s == dst_sal->s)))
        return RKV_ERR_INVALID_ARGUMENT;
    if (in_place && (src->batch != dst->batch || src->stride_b != dst->stride_b ||
                     src->stride_p != dst->stride_p ||
                     (src_sal && (src_sal->stride_b != dst_sal->stride_b ||
                                  src_sal->stride_p != dst_sal->stride_p))))
        return RKV_ERR_INVALID_ARGUMENT;
    // in place the row map is src's own; out of place dst gets sequence b in row b
    if ((in_place && dst->row_map != src->row_map) || (!in_place && dst->row_map))
        return RKV_ERR_INVALID_ARGUMENT;
    if (num_moved < 0 || num_moved > num_listed) return RKV_ERR_INVALID_ARGUMENT;
    const bool compose = in_place && src->row_map != nullptr;
    const int64_t eb = elt_bytes(src->dtype);
    ReindexParams p{};
    p.src[0] = static_cast<const char*>(src->k); p.dst[0] = static_cast<char*>(const_cast<void*>(dst->k));
    p.src[1] = static_cast<const char*>(src->v); p.dst[1] = static_cast<char*>(const_cast<void*>(dst->v));
    p.src[2] = src_sal ? reinterpret_cast<const char*>(src_sal->s) : nullptr;
    p.dst[2] = dst_sal ? reinterpret_cast<char*>(dst_sal->s) : nullptr;
    const int64_t kv_row = src->num_kv_heads * P * D * eb;
    for (int w = 0; w < 2; ++w) {
        p.row_bytes[w] = p.src[w] ? kv_row : 0;
        p.src_slot_stride[w] = src->stride_p * eb; p.src_b_stride[w] = src->stride_b * eb;
        p.dst_slot_stride[w] = dst->stride_p * eb; p.dst_b_stride[w] = dst->stride_b * eb;
    }
    p.row_bytes[2] = src_sal ? P * 4 : 0;
    if (src_sal) {
        p.src_slot_stride[2] = src_sal->stride_p * 4; p.src_b_stride[2] = src_sal->stride_b * 4;
        p.dst_slot_stride[2] = dst_sal->stride_p * 4; p.dst_b_stride[2] = dst_sal->stride_b * 4;
    }
    // widest access every base, stride and row length allows
    int vec = 16;
    for (int w = 0; w < 3; ++w) {
        if (!p.src[w]) continue;
        const int64_t vals[] = {(int64_t)(uintptr_t)p.src[w], (int64_t)(uintptr_t)p.dst[w],
                                p.src_slot_stride[w], p.src_b_stride[w], p.dst_slot_stride[w],
                                p.dst_b_stride[w], p.row_bytes[w]};
        for (int64_t x : vals) {
            while (vec > 2 && x % vec != 0) vec = vec == 16 ? 4 : 2;
        }
    }
    p.vec = vec;
    p.chunk = reindex_chunk_bytes(dst->batch, kv_row > P * 4 ? kv_row : P * 4, vec);
    if (dst->batch > 0 && p.chunk == 0) return RKV_ERR_UNSUPPORTED;
    for (int w = 0; w < 3; ++w)
        p.chunks[w] = p.chunk ? (p.row_bytes[w] + p.chunk - 1) / p.chunk : 0;
    p.src_B = src->batch; p.dst_B = dst->batch;
    p.num_slots = src->num_slots < dst->num_slots ? src->num_slots : dst->num_slots;
    p.index = index; p.slots = slots; p.n_listed = num_listed; p.err = err;
    p.in_place = in_place ? 1 : 0;
    p.row_map = src->row_map;
    p.n_moved = compose ? num_moved : num_listed;
    const cudaError_t e = launch_reindex(p, S(stream));
    if (e != cudaSuccess || !compose) return status_of(e);
    return status_of(launch_row_map_compose(src->row_map, src->batch, index, slots, num_listed,
                                            num_moved, p.num_slots, S(stream)));
}

}  // extern "C"
