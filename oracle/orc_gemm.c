/*
 * ORACLE — test infrastructure only (see orc_rng.c for the usage rule).
 *
 * Host restatement of the reference's GEMM check, include/reference_matmul.cuh:17-32:
 *     C[m, n] = sum_k A[m, k] * B[n, k]
 * with A row-major [M, K] (the gathered activation, rank r's shard at rows
 * [r*M/P, (r+1)*M/P), vmm/main.cpp:302-309) and B row-major [N, K] (the
 * rank's own weight shard, read "transposed", reference_matmul.cuh:17-20).
 * The reference computes this with cublasGemmEx (bf16 inputs, fp32 compute,
 * reference_matmul.cuh:59-77); it has no CPU matmul of its own.
 *
 *   orc_gemm_f32    fp32 accumulate, multithreaded, register-blocked — the
 *                   "CPU fp32 matmul" that bench.py times as cpu_baseline;
 *   orc_gemm_f64    double accumulate, the exact-as-possible ground truth for
 *                   small parity cases;
 *   orc_check_close the reference's check_close (reference_matmul.cuh:99-145):
 *                   |a - e| <= atol + rtol * |e|, counted over rows x cols;
 *   orc_error_stats max |a - e|, max |e| and the normwise relative error
 *                   max|a - e| / max|e| used by the parity tests.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef float v8f __attribute__((vector_size(32)));

typedef struct gemm_job {
    const float* A;
    const float* B;
    float* C;
    long M, N, K, lda, ldb, ldc;
    long row_begin, row_end;
} gemm_job;

static inline float hsum8(v8f v) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += v[i];
    return s;
}

static inline v8f load8(const float* p) {
    v8f v;
    memcpy(&v, p, sizeof(v));
    return v;
}

/* 4 rows of A against 2 rows of B: 8 dot products sharing every load. */
static void block_4x2(const float* a0, const float* a1, const float* a2, const float* a3,
                      const float* b0, const float* b1, long K, float out[8]) {
    v8f c00 = {0}, c01 = {0}, c10 = {0}, c11 = {0};
    v8f c20 = {0}, c21 = {0}, c30 = {0}, c31 = {0};
    long k = 0;
    for (; k + 8 <= K; k += 8) {
        const v8f x0 = load8(a0 + k), x1 = load8(a1 + k), x2 = load8(a2 + k), x3 = load8(a3 + k);
        const v8f y0 = load8(b0 + k), y1 = load8(b1 + k);
        c00 += x0 * y0; c01 += x0 * y1;
        c10 += x1 * y0; c11 += x1 * y1;
        c20 += x2 * y0; c21 += x2 * y1;
        c30 += x3 * y0; c31 += x3 * y1;
    }
    float s[8] = {hsum8(c00), hsum8(c01), hsum8(c10), hsum8(c11),
                  hsum8(c20), hsum8(c21), hsum8(c30), hsum8(c31)};
    for (; k < K; ++k) {
        s[0] += a0[k] * b0[k]; s[1] += a0[k] * b1[k];
        s[2] += a1[k] * b0[k]; s[3] += a1[k] * b1[k];
        s[4] += a2[k] * b0[k]; s[5] += a2[k] * b1[k];
        s[6] += a3[k] * b0[k]; s[7] += a3[k] * b1[k];
    }
    memcpy(out, s, sizeof(s));
}

static float dot_f32(const float* a, const float* b, long K) {
    v8f c = {0};
    long k = 0;
    for (; k + 8 <= K; k += 8) c += load8(a + k) * load8(b + k);
    float s = hsum8(c);
    for (; k < K; ++k) s += a[k] * b[k];
    return s;
}

static void* gemm_worker(void* arg) {
    const gemm_job* j = (const gemm_job*)arg;
    const long NB = 64; /* columns of C per pass: keeps 64 rows of B hot in L2 */
    for (long n0 = 0; n0 < j->N; n0 += NB) {
        const long n1 = n0 + NB < j->N ? n0 + NB : j->N;
        long m = j->row_begin;
        for (; m + 4 <= j->row_end; m += 4) {
            const float* a0 = j->A + m * j->lda;
            const float* a1 = a0 + j->lda;
            const float* a2 = a1 + j->lda;
            const float* a3 = a2 + j->lda;
            long n = n0;
            for (; n + 2 <= n1; n += 2) {
                float o[8];
                block_4x2(a0, a1, a2, a3, j->B + n * j->ldb, j->B + (n + 1) * j->ldb, j->K, o);
                for (int r = 0; r < 4; ++r) {
                    j->C[(m + r) * j->ldc + n] = o[2 * r];
                    j->C[(m + r) * j->ldc + n + 1] = o[2 * r + 1];
                }
            }
            for (; n < n1; ++n)
                for (int r = 0; r < 4; ++r)
                    j->C[(m + r) * j->ldc + n] = dot_f32(j->A + (m + r) * j->lda, j->B + n * j->ldb, j->K);
        }
        for (; m < j->row_end; ++m)
            for (long n = n0; n < n1; ++n)
                j->C[m * j->ldc + n] = dot_f32(j->A + m * j->lda, j->B + n * j->ldb, j->K);
    }
    return NULL;
}

/* C[M, N] (ldc) = A[M, K] (lda) . B[N, K]^T (ldb), fp32 accumulate, nthreads threads. */
int orc_gemm_f32(const float* A, const float* B, float* C, long M, long N, long K,
                 long lda, long ldb, long ldc, int nthreads) {
    if (M <= 0 || N <= 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 512) nthreads = 512;
    if ((long)nthreads > M) nthreads = (int)M;
    pthread_t th[512];
    gemm_job jobs[512];
    /* split rows in multiples of 4 so every thread runs the blocked path */
    const long per = ((M + nthreads - 1) / nthreads + 3) / 4 * 4;
    int launched = 0;
    for (int t = 0; t < nthreads; ++t) {
        const long b = (long)t * per;
        if (b >= M) break;
        const long e = b + per < M ? b + per : M;
        jobs[t] = (gemm_job){A, B, C, M, N, K, lda, ldb, ldc, b, e};
        if (pthread_create(&th[t], NULL, gemm_worker, &jobs[t]) != 0) {
            gemm_worker(&jobs[t]);
            jobs[t].row_begin = jobs[t].row_end; /* already done inline */
            th[t] = 0;
        }
        launched = t + 1;
    }
    for (int t = 0; t < launched; ++t)
        if (th[t]) pthread_join(th[t], NULL);
    return 0;
}

/* Double-accumulate ground truth (single thread; small parity cases only). */
int orc_gemm_f64(const float* A, const float* B, double* C, long M, long N, long K,
                 long lda, long ldb, long ldc) {
    for (long m = 0; m < M; ++m)
        for (long n = 0; n < N; ++n) {
            double s = 0.0;
            const float* a = A + m * lda;
            const float* b = B + n * ldb;
            for (long k = 0; k < K; ++k) s += (double)a[k] * (double)b[k];
            C[m * ldc + n] = s;
        }
    return 0;
}

/*
 * check_close (reference_matmul.cuh:99-145): returns the number of elements
 * with |a - e| > atol + rtol*|e| (0 = pass) and records up to `max_report`
 * failing flat indices in `report`.
 */
long orc_check_close(const float* actual, const float* expected, long rows, long cols,
                     float atol, float rtol, long* report, int max_report) {
    long bad = 0;
    for (long r = 0; r < rows; ++r)
        for (long c = 0; c < cols; ++c) {
            const long i = r * cols + c;
            const float a = actual[i];
            const float e = expected[i];
            const float tol = atol + rtol * fabsf(e);
            if (fabsf(a - e) > tol || isnan(a) != isnan(e)) {
                if (report && bad < max_report) report[bad] = i;
                ++bad;
            }
        }
    return bad;
}

/* out[0] = max|a-e|, out[1] = max|e|, out[2] = max|a-e| / max|e|, out[3] = #NaN in a */
void orc_error_stats(const float* actual, const float* expected, long n, double out[4]) {
    double max_err = 0.0, max_ref = 0.0, nans = 0.0;
    for (long i = 0; i < n; ++i) {
        const double a = actual[i], e = expected[i];
        if (isnan(a)) { nans += 1.0; continue; }
        const double d = fabs(a - e);
        if (d > max_err) max_err = d;
        if (fabs(e) > max_ref) max_ref = fabs(e);
    }
    out[0] = max_err;
    out[1] = max_ref;
    out[2] = max_ref > 0.0 ? max_err / max_ref : max_err;
    out[3] = nans;
}

/* Widen bf16 payloads to float (the read_back_as_float conversion, random_fill.cuh:69-89). */
void orc_bf16_to_f32_array(const uint16_t* in, float* out, long n) {
    for (long i = 0; i < n; ++i) {
        uint32_t u = (uint32_t)in[i] << 16;
        memcpy(&out[i], &u, 4);
    }
}
