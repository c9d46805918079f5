/*
 * CPU oracle for the RazorKV decode path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's decode step so that
 * the CUDA path can be checked against it bit for bit.  It is linked only by the test
 * suite, by the package's smoke check and by the CPU-baseline leg of the benchmark; the
 * product library never calls it.
 *
 * Reference functions restated (paths inside the reference project):
 *   orc_norm_salience  razorkv/cache.py:239-247   mean over kv heads of ||k||_2 (fp32)
 *   orc_resonance      razorkv/cache.py:263-280   max over (q head, q row) of (fp32(q)*scale).k
 *   orc_ewma           razorkv/cache.py:282-287   S = decay*S + (1-decay)*R
 *   orc_attention      razorkv/kernels/torch_sparse.py:15-61 and
 *                      razorkv/kernels/triton_paged_sparse.py:105-174
 *                      softmax(q.k*scale).v with GQA head grouping, evaluated in fp64
 *
 * Canonical summation order.  torch's fp32 reductions (MKL sgemm for the scores,
 * vector_norm, mean) have ISA-dependent orders that no restatement can reproduce, so the
 * oracle and the CUDA kernels share ONE fixed order and agree bit for bit; the reference
 * differs from both by a few ulps.  A dot product over D elements of a K row whose
 * element size is E bytes is cut into 16-byte chunks of CH = 16/E elements.  Lane j
 * (j = 0..7) owns the chunks c = j, j+8, j+16, ...; listing its elements in ascending
 * order (chunk by chunk), the elements at even positions of that list accumulate into one
 * chain and those at odd positions into another, each with fused multiply-add starting
 * from +0.0f (the two halves of one packed f32x2 FMA on the GPU); partial p_j = even + odd.
 * The eight partials are combined as ((p0+p4)+(p2+p6)) + ((p1+p5)+(p3+p7)), which is the
 * xor-4 / xor-2 / xor-1 butterfly the GPU performs across eight lanes.
 *
 * Build: cc -O2 -ffp-contract=off -shared -fPIC -pthread (see oracle/Makefile).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- a minimal static-partition parallel-for over [0, n) on POSIX threads ---------------
 * Every output element is computed by exactly one thread in a fixed order, so results do
 * not depend on the thread count.  ORACLE_THREADS overrides the online-CPU count. */
typedef void (*range_fn)(int64_t lo, int64_t hi, void *ctx);
typedef struct { range_fn fn; void *ctx; int64_t lo, hi; } range_job;

static void *range_trampoline(void *p) {
    range_job *j = (range_job *)p;
    j->fn(j->lo, j->hi, j->ctx);
    return NULL;
}

static int oracle_threads(void) {
    const char *e = getenv("ORACLE_THREADS");
    long n = e ? atol(e) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 256) n = 256;
    return (int)n;
}

int orc_num_threads(void) { return oracle_threads(); }

static void parallel_for(int64_t n, range_fn fn, void *ctx) {
    int nt = oracle_threads();
    if (nt > n) nt = (int)(n > 0 ? n : 1);
    if (nt <= 1) { fn(0, n, ctx); return; }
    pthread_t th[256];
    range_job jobs[256];
    for (int i = 0; i < nt; ++i) {
        jobs[i].fn = fn; jobs[i].ctx = ctx;
        jobs[i].lo = n * i / nt; jobs[i].hi = n * (i + 1) / nt;
        pthread_create(&th[i], NULL, range_trampoline, &jobs[i]);
    }
    for (int i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

static float canon_dot(const float *a, const float *b, int64_t D, int64_t ch) {
    float p[8];
    for (int j = 0; j < 8; ++j) {
        float even = 0.0f, odd = 0.0f;
        int64_t pos = 0;
        for (int64_t c = j; c * ch < D; c += 8) {
            int64_t e0 = c * ch, e1 = e0 + ch < D ? e0 + ch : D;
            for (int64_t e = e0; e < e1; ++e, ++pos) {
                if (pos & 1) odd = fmaf(a[e], b[e], odd);
                else even = fmaf(a[e], b[e], even);
            }
        }
        p[j] = even + odd;
    }
    float s04 = p[0] + p[4], s26 = p[2] + p[6], s15 = p[1] + p[5], s37 = p[3] + p[7];
    return (s04 + s26) + (s15 + s37);
}

/* Canonical dot of two rows; exported so tests can check single values. */
float orc_canon_dot(const float *a, const float *b, int64_t D, int64_t ch) {
    return canon_dot(a, b, D, ch);
}

/* out[b, t] = (sum_h sqrt(canon_dot(k, k))) / H  with h summed in ascending order.
 * k is [B, H, T, D] contiguous fp32 (values already widened from the cache dtype). */
typedef struct { const float *k; int64_t B, H, T, D, ch; float *out; } norm_ctx;

static void norm_range(int64_t lo, int64_t hi, void *p) {
    norm_ctx *c = (norm_ctx *)p;
    for (int64_t i = lo; i < hi; ++i) {
        int64_t b = i / c->T, t = i % c->T;
        float acc = 0.0f;
        for (int64_t h = 0; h < c->H; ++h) {
            const float *row = c->k + ((b * c->H + h) * c->T + t) * c->D;
            acc = acc + sqrtf(canon_dot(row, row, c->D, c->ch));
        }
        c->out[i] = acc / (float)c->H;
    }
}

void orc_norm_salience(const float *k, int64_t B, int64_t H, int64_t T, int64_t D,
                       int64_t ch, float *out) {
    norm_ctx c = {k, B, H, T, D, ch, out};
    parallel_for(B * T, norm_range, &c);
}

/* R[b, n] = max over q rows r = (h, t) of canon_dot(fl(q[b,h,t,:] * scale), k[b, h/G, n, :]).
 * q is [B, Hq, QL, D] and k is [B, Hkv, N, D], both contiguous fp32.  NaN propagates like
 * torch.amax. */
typedef struct { const float *qs, *k; int64_t B, Hq, Hkv, QL, N, D, ch; float *R; } res_ctx;

static void res_range(int64_t lo, int64_t hi, void *p) {
    res_ctx *c = (res_ctx *)p;
    int64_t G = c->Hq / c->Hkv;
    for (int64_t i = lo; i < hi; ++i) {
        int64_t b = i / c->N, n = i % c->N;
        float m = -INFINITY;
        int nan = 0;
        for (int64_t h = 0; h < c->Hq; ++h) {
            const float *krow = c->k + ((b * c->Hkv + h / G) * c->N + n) * c->D;
            for (int64_t t = 0; t < c->QL; ++t) {
                float s = canon_dot(c->qs + ((b * c->Hq + h) * c->QL + t) * c->D, krow, c->D, c->ch);
                if (s != s) nan = 1;
                else if (s > m) m = s;
            }
        }
        c->R[i] = nan ? NAN : m;
    }
}

void orc_resonance(const float *q, const float *k, int64_t B, int64_t Hq, int64_t Hkv,
                   int64_t QL, int64_t N, int64_t D, int64_t ch, float scale, float *R) {
    float *qs = (float *)malloc(sizeof(float) * (size_t)(B * Hq * QL * D));
    for (int64_t i = 0; i < B * Hq * QL * D; ++i) qs[i] = q[i] * scale;
    res_ctx c = {qs, k, B, Hq, Hkv, QL, N, D, ch, R};
    parallel_for(B * N, res_range, &c);
    free(qs);
}

/* S = fl(fl(decay * S) + fl(one_minus_decay * R)), no contraction (matches torch's two
 * scalar multiplies and one add in fp32). */
void orc_ewma(float *S, const float *R, int64_t n, float decay, float one_minus_decay) {
    for (int64_t i = 0; i < n; ++i) {
        float a = decay * S[i];
        float c = one_minus_decay * R[i];
        S[i] = a + c;
    }
}

/* out[b, h, t, :] = softmax_j(q.k_j * scale) . v_j over the N keys of kv head h/G, in fp64.
 * causal != 0 masks key j > t (upper-left aligned, as torch SDPA with is_causal=True);
 * q [B,Hq,QL,D], k/v [B,Hkv,N,D], out [B,Hq,QL,D] fp64. */
typedef struct {
    const float *q, *k, *v; int64_t B, Hq, Hkv, QL, N, D; double scale; int causal; double *out;
} att_ctx;

static void att_range(int64_t lo, int64_t hi, void *p) {
    att_ctx *c = (att_ctx *)p;
    int64_t G = c->Hq / c->Hkv, N = c->N, D = c->D;
    double *w = (double *)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
    for (int64_t i = lo; i < hi; ++i) {
        int64_t b = i / c->Hq, h = i % c->Hq;
        const float *kb = c->k + (b * c->Hkv + h / G) * N * D;
        const float *vb = c->v + (b * c->Hkv + h / G) * N * D;
        for (int64_t t = 0; t < c->QL; ++t) {
            const float *qr = c->q + ((b * c->Hq + h) * c->QL + t) * D;
            double *o = c->out + ((b * c->Hq + h) * c->QL + t) * D;
            int64_t lim = c->causal ? t + 1 : N;
            if (lim > N) lim = N;
            double m = -INFINITY;
            for (int64_t j = 0; j < lim; ++j) {
                double s = 0.0;
                for (int64_t d = 0; d < D; ++d) s += (double)qr[d] * (double)kb[j * D + d];
                w[j] = s * c->scale;
                if (w[j] > m) m = w[j];
            }
            double l = 0.0;
            for (int64_t j = 0; j < lim; ++j) { w[j] = exp(w[j] - m); l += w[j]; }
            for (int64_t d = 0; d < D; ++d) o[d] = 0.0;
            for (int64_t j = 0; j < lim; ++j) {
                double pj = w[j] / l;
                for (int64_t d = 0; d < D; ++d) o[d] += pj * (double)vb[j * D + d];
            }
        }
    }
    free(w);
}

void orc_attention(const float *q, const float *k, const float *v, int64_t B, int64_t Hq,
                   int64_t Hkv, int64_t QL, int64_t N, int64_t D, double scale, int causal,
                   double *out) {
    att_ctx c = {q, k, v, B, Hq, Hkv, QL, N, D, scale, causal, out};
    parallel_for(B * Hq, att_range, &c);
}
