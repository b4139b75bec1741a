/*
 * fp4attn_oracle.c -- CPU restatement of the reference's FP4 attention path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker; see fp4attn_oracle.h).  Each function
 * cites the reference file:line it restates.  Parity of this file with the
 * reference is pinned by tests/test_oracle.py against oracle/_ref (the
 * reference's own sources compiled by oracle/Makefile) and against the
 * committed vectors in tests/golden/.
 */
#include "fp4attn_oracle.h"

#include <limits.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* common.h:21-36.  Thresholds are compared with >= so a tie rounds up; the
 * sign is taken from (v < 0), so -0.0 and NaN get sign 0 and a NaN magnitude
 * fails every comparison (code 0). */
uint8_t oracle_encode_e2m1(float v)
{
    uint8_t sign = (v < 0.f) ? 1 : 0;
    float a = fabsf(v);
    uint8_t n;
    if (a >= 5.0f)       n = 7;
    else if (a >= 3.5f)  n = 6;
    else if (a >= 2.5f)  n = 5;
    else if (a >= 1.75f) n = 4;
    else if (a >= 1.25f) n = 3;
    else if (a >= 0.75f) n = 2;
    else if (a >= 0.25f) n = 1;
    else                 n = 0;
    return (uint8_t)(n | (sign << 3));
}

/* (int)ceilf(x) as x86-64 executes it (cvttss2si): a NaN or a value outside
 * the int range gives INT_MIN.  The reference relies on this for an all-zero
 * block, where log2f(0) = -inf and the scale byte becomes 0x7F. */
static int x86_ceil_to_int(float x)
{
    float c = ceilf(x);
    if (!(c >= -2147483648.0f && c < 2147483648.0f)) return INT_MIN;
    return (int)c;
}

/* common.h:39-48: max |x| over 32 elements (NaN never wins the > test),
 * exponent = (int)ceilf(log2f(max)), byte = (uint8_t)(exponent + 127). */
uint8_t oracle_scale_ue8m0(const float* block, int scale_mode)
{
    float max_abs = 0.0f;
    for (int i = 0; i < 32; i++) {
        float a = fabsf(block[i]);
        if (a > max_abs) max_abs = a;
    }
    if (scale_mode == ORACLE_SCALE_OCP) max_abs = max_abs / 6.0f;
    volatile float m = max_abs; /* keep log2f a library call, never folded */
    int e = x86_ceil_to_int(log2f(m));
    return (uint8_t)((unsigned)(e + 127) & 0xFFu);
}

float oracle_e2m1_value(uint8_t code)
{
    static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    float v = mag[code & 7];
    return (code & 8) ? -v : v;
}

/* common.h:115-123 (Q) and :160-168 (K): per 32-element block, scale byte s,
 * scale_f = exp2f(s - 127), code = encode(x / scale_f). */
void oracle_quantize(const float* x, int64_t rows, int d, uint8_t* codes,
                     uint8_t* scales, int scale_mode)
{
    int nb = d / 32;
    for (int64_t r = 0; r < rows; r++) {
        for (int b = 0; b < nb; b++) {
            const float* blk = x + r * d + b * 32;
            uint8_t s = oracle_scale_ue8m0(blk, scale_mode);
            scales[r * nb + b] = s;
            volatile float ex = (float)((int)s - 127);
            float scale_f = exp2f(ex);
            for (int j = 0; j < 32; j++)
                codes[r * d + b * 32 + j] = oracle_encode_e2m1(blk[j] / scale_f);
        }
    }
}

void oracle_dequantize(const uint8_t* codes, const uint8_t* scales, int64_t rows,
                       int d, float* out)
{
    int nb = d / 32;
    for (int64_t r = 0; r < rows; r++)
        for (int j = 0; j < d; j++) {
            uint8_t c = codes[r * d + j];
            float v = oracle_e2m1_value(c);
            out[r * d + j] = (v == 0.f) ? 0.f : ldexpf(v, (int)scales[r * nb + j / 32] - 127);
        }
}

/* tests/test_attention.cu:33-54 with cpu_matmul (:9-19) and
 * cpu_softmax_rows (:21-31).  Loops are reordered for speed but every output
 * element is accumulated in FP32 over k in ascending order, as in :15-16. */
void oracle_attention(const float* Q, const float* K, const float* V, float* Out,
                      int sq, int sk, int d, float scale)
{
    float* Kt = (float*)malloc(sizeof(float) * (size_t)sk * d);
    float* row = (float*)malloc(sizeof(float) * (size_t)sk);
    float* acc = (float*)malloc(sizeof(float) * (size_t)d);
    for (int i = 0; i < sk; i++)
        for (int j = 0; j < d; j++) Kt[(size_t)j * sk + i] = K[(size_t)i * d + j];
    if (!(scale > 0.f)) scale = 1.0f / sqrtf((float)d);
    for (int i = 0; i < sq; i++) {
        for (int j = 0; j < sk; j++) row[j] = 0.f;
        for (int k = 0; k < d; k++) {
            float q = Q[(size_t)i * d + k];
            const float* kt = Kt + (size_t)k * sk;
            for (int j = 0; j < sk; j++) row[j] += q * kt[j];
        }
        for (int j = 0; j < sk; j++) row[j] *= scale;
        float m = row[0];
        for (int j = 1; j < sk; j++) m = fmaxf(m, row[j]);
        float sum = 0.f;
        for (int j = 0; j < sk; j++) { row[j] = expf(row[j] - m); sum += row[j]; }
        for (int j = 0; j < sk; j++) row[j] /= sum;
        for (int j = 0; j < d; j++) acc[j] = 0.f;
        for (int k = 0; k < sk; k++) {
            float p = row[k];
            const float* v = V + (size_t)k * d;
            for (int j = 0; j < d; j++) acc[j] += p * v[j];
        }
        for (int j = 0; j < d; j++) Out[(size_t)i * d + j] = acc[j];
    }
    free(Kt); free(row); free(acc);
}

/* The causal extension (our own; the reference has no mask): the row loop of
 * oracle_attention restricted to the visible keys [0, lim). */
void oracle_attention_causal(const float* Q, const float* K, const float* V, float* Out,
                             int sq, int sk, int d, float scale, int first_row, int sq_total)
{
    float* row = (float*)malloc(sizeof(float) * (size_t)(sk > 0 ? sk : 1));
    float* acc = (float*)malloc(sizeof(float) * (size_t)d);
    if (!(scale > 0.f)) scale = 1.0f / sqrtf((float)d);
    for (int i = 0; i < sq; i++) {
        long lim = (long)first_row + i + sk - sq_total + 1;
        if (lim > sk) lim = sk;
        for (int j = 0; j < d; j++) acc[j] = 0.f;
        if (lim > 0) {
            for (long j = 0; j < lim; j++) {
                float a = 0.f;
                for (int k = 0; k < d; k++) a += Q[(size_t)i * d + k] * K[(size_t)j * d + k];
                row[j] = a * scale;
            }
            float m = row[0];
            for (long j = 1; j < lim; j++) m = fmaxf(m, row[j]);
            float sum = 0.f;
            for (long j = 0; j < lim; j++) { row[j] = expf(row[j] - m); sum += row[j]; }
            for (long j = 0; j < lim; j++) row[j] /= sum;
            for (long k = 0; k < lim; k++) {
                float p = row[k];
                const float* v = V + (size_t)k * d;
                for (int j = 0; j < d; j++) acc[j] += p * v[j];
            }
        }
        for (int j = 0; j < d; j++) Out[(size_t)i * d + j] = acc[j];
    }
    free(row); free(acc);
}

static void quant_dequant(const float* x, int64_t rows, int d, int mode, float* out)
{
    uint8_t* codes = (uint8_t*)malloc((size_t)rows * d);
    uint8_t* sc = (uint8_t*)malloc((size_t)rows * (d / 32));
    oracle_quantize(x, rows, d, codes, sc, mode);
    oracle_dequantize(codes, sc, rows, d, out);
    free(codes); free(sc);
}

typedef struct {
    const float *Q, *K, *V; float* Out;
    int s0, s1, sq, sk, d, mode; float scale;
    int causal;
} slice_job;

static void* run_slices(void* arg)
{
    slice_job* j = (slice_job*)arg;
    size_t qn = (size_t)j->sq * j->d, kn = (size_t)j->sk * j->d;
    float* qd = (float*)malloc(sizeof(float) * qn);
    float* kd = (float*)malloc(sizeof(float) * kn);
    for (int s = j->s0; s < j->s1; s++) {
        quant_dequant(j->Q + s * qn, j->sq, j->d, j->mode, qd);
        quant_dequant(j->K + s * kn, j->sk, j->d, j->mode, kd);
        if (j->causal)
            oracle_attention_causal(qd, kd, j->V + s * kn, j->Out + s * qn, j->sq, j->sk, j->d, j->scale, 0, j->sq);
        else
            oracle_attention(qd, kd, j->V + s * kn, j->Out + s * qn, j->sq, j->sk, j->d, j->scale);
    }
    free(qd); free(kd);
    return NULL;
}

static void fp4_attention_slices(const float* Q, const float* K, const float* V, float* Out,
                                 int slices, int sq, int sk, int d, float scale, int mode,
                                 int threads, int causal)
{
    if (threads < 1) threads = 1;
    if (threads > slices) threads = slices;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    slice_job* jobs = (slice_job*)malloc(sizeof(slice_job) * threads);
    for (int t = 0; t < threads; t++) {
        slice_job jb = {Q, K, V, Out, slices * t / threads, slices * (t + 1) / threads,
                        sq, sk, d, mode, scale, causal};
        jobs[t] = jb;
        pthread_create(&tid[t], NULL, run_slices, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    free(tid); free(jobs);
}

void oracle_fp4_attention(const float* Q, const float* K, const float* V, float* Out,
                          int slices, int sq, int sk, int d, float scale, int mode,
                          int threads)
{
    fp4_attention_slices(Q, K, V, Out, slices, sq, sk, d, scale, mode, threads, 0);
}

void oracle_fp4_attention_causal(const float* Q, const float* K, const float* V, float* Out,
                                 int slices, int sq, int sk, int d, float scale, int mode,
                                 int threads)
{
    fp4_attention_slices(Q, K, V, Out, slices, sq, sk, d, scale, mode, threads, 1);
}

void oracle_fp4_attention_rows(const float* Q, const float* K, const float* V,
                               float* Out, int n, const int* slice_of, const int* rows,
                               int sq, int sk, int d, float scale, int mode)
{
    size_t qn = (size_t)sq * d, kn = (size_t)sk * d;
    float* qd = (float*)malloc(sizeof(float) * d);
    float* kd = (float*)malloc(sizeof(float) * kn);
    int cached = -1;
    for (int i = 0; i < n; i++) {
        int s = slice_of[i];
        if (s != cached) { quant_dequant(K + s * kn, sk, d, mode, kd); cached = s; }
        quant_dequant(Q + s * qn + (size_t)rows[i] * d, 1, d, mode, qd);
        oracle_attention(qd, kd, V + s * kn, Out + (size_t)i * d, 1, sk, d, scale);
    }
    free(qd); free(kd);
}

typedef struct {
    const float *qd, *kd, *V; float* Out;
    int r0, r1, sk, d; float scale;
} row_job;

static void* run_rows(void* arg)
{
    row_job* j = (row_job*)arg;
    if (j->r1 > j->r0)
        oracle_attention(j->qd + (size_t)j->r0 * j->d, j->kd, j->V, j->Out + (size_t)j->r0 * j->d,
                         j->r1 - j->r0, j->sk, j->d, j->scale);
    return NULL;
}

/* Rows of one slice over threads: Q and K are quantised and dequantised once
 * (as run_slices does per slice), then each thread runs oracle_attention
 * (tests/test_attention.cu:33-54) on its block of query rows. */
void oracle_fp4_attention_slice(const float* Q, const float* K, const float* V, float* Out,
                                int sq, int sk, int d, float scale, int mode, int threads)
{
    float* qd = (float*)malloc(sizeof(float) * (size_t)sq * d);
    float* kd = (float*)malloc(sizeof(float) * (size_t)sk * d);
    quant_dequant(Q, sq, d, mode, qd);
    quant_dequant(K, sk, d, mode, kd);
    if (threads < 1) threads = 1;
    if (threads > sq) threads = sq;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    row_job* jobs = (row_job*)malloc(sizeof(row_job) * threads);
    for (int t = 0; t < threads; t++) {
        row_job jb = {qd, kd, V, Out, (int)((int64_t)sq * t / threads), (int)((int64_t)sq * (t + 1) / threads),
                      sk, d, scale};
        jobs[t] = jb;
        pthread_create(&tid[t], NULL, run_rows, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    free(tid); free(jobs); free(qd); free(kd);
}

/* common.h:331-398 computes one 64x64 block of Q K^T on FP4 codes; this is the
 * same product with the reference's block scales applied (common.h:208-213). */
void oracle_fp4_scores(const float* Q, const float* K, float* S, int sq, int sk, int d,
                       int mode)
{
    float* qd = (float*)malloc(sizeof(float) * (size_t)sq * d);
    float* kd = (float*)malloc(sizeof(float) * (size_t)sk * d);
    quant_dequant(Q, sq, d, mode, qd);
    quant_dequant(K, sk, d, mode, kd);
    for (int i = 0; i < sq; i++)
        for (int j = 0; j < sk; j++) {
            float acc = 0.f;
            for (int k = 0; k < d; k++) acc += qd[(size_t)i * d + k] * kd[(size_t)j * d + k];
            S[(size_t)i * sk + j] = acc;
        }
    free(qd); free(kd);
}

/* tests/test_attention.cu:56-65, accumulated in double. */
double oracle_cosine(const float* a, const float* b, int64_t n)
{
    double dot = 0, na = 0, nb = 0;
    for (int64_t i = 0; i < n; i++) {
        dot += (double)a[i] * b[i];
        na += (double)a[i] * a[i];
        nb += (double)b[i] * b[i];
    }
    return dot / (sqrt(na) * sqrt(nb) + 1e-30);
}

/* ------------------------------------------------------------------ backward
 * Not part of the reference, which is forward only (common.h:68-328 has no
 * gradient path).  The gradient of the FP4 path above with the quantiser as a
 * straight-through estimator: with Qq, Kq the dequantised Q, K (quant_dequant,
 * i.e. common.h:21-48 and :115-123 / :160-168 followed by dequantisation),
 * z = scale * Qq Kq^T over the visible keys, P = softmax(z) row-wise:
 *   dV = P^T dO,  dP = dO V^T,  Dd_i = sum_j P_ij dP_ij,
 *   dZ = P o (dP - Dd),  dQ = scale * dZ Kq,  dK = scale * dZ^T Qq.
 * Everything is accumulated in double.  Dd_i = sum_j P_ij dP_ij equals
 * sum_c dO_ic O_ic for the exact O = P V. */

typedef struct {
    const float *qd, *kd, *V, *dO;
    float* dQ;
    double *dK, *dV;     /* this job's private accumulators [sk][d] */
    int r0, r1, sq, sk, d, causal;
    double scale;
} bwd_job;

static void* run_bwd_rows(void* arg)
{
    bwd_job* j = (bwd_job*)arg;
    const int sk = j->sk, d = j->d;
    double* p = (double*)malloc(sizeof(double) * (size_t)(sk > 0 ? sk : 1));
    double* dp = (double*)malloc(sizeof(double) * (size_t)(sk > 0 ? sk : 1));
    double* dq = (double*)malloc(sizeof(double) * (size_t)d);
    for (int i = j->r0; i < j->r1; i++) {
        long lim = sk;
        if (j->causal) {
            lim = (long)i + sk - j->sq + 1;
            if (lim > sk) lim = sk;
        }
        const float* q = j->qd + (size_t)i * d;
        const float* go = j->dO + (size_t)i * d;
        for (int c = 0; c < d; c++) dq[c] = 0.0;
        if (lim > 0) {
            double m = -INFINITY;
            for (long k = 0; k < lim; k++) {
                const float* kr = j->kd + (size_t)k * d;
                double a = 0.0;
                for (int c = 0; c < d; c++) a += (double)q[c] * kr[c];
                p[k] = a * j->scale;
                if (p[k] > m) m = p[k];
            }
            double sum = 0.0;
            for (long k = 0; k < lim; k++) { p[k] = exp(p[k] - m); sum += p[k]; }
            double dd = 0.0;
            for (long k = 0; k < lim; k++) {
                p[k] /= sum;
                const float* vr = j->V + (size_t)k * d;
                double a = 0.0;
                for (int c = 0; c < d; c++) a += (double)go[c] * vr[c];
                dp[k] = a;
                dd += p[k] * a;
            }
            for (long k = 0; k < lim; k++) {
                const double dz = p[k] * (dp[k] - dd);
                const float* kr = j->kd + (size_t)k * d;
                double* dkr = j->dK + (size_t)k * d;
                double* dvr = j->dV + (size_t)k * d;
                for (int c = 0; c < d; c++) {
                    dq[c] += dz * kr[c];
                    dkr[c] += dz * q[c];
                    dvr[c] += p[k] * go[c];
                }
            }
        }
        for (int c = 0; c < d; c++) j->dQ[(size_t)i * d + c] = (float)(dq[c] * j->scale);
    }
    free(p); free(dp); free(dq);
    return NULL;
}

void oracle_fp4_attention_backward(const float* Q, const float* K, const float* V, const float* dO,
                                   float* dQ, float* dK, float* dV, int slices, int sq, int sk, int d,
                                   float scale, int mode, int causal, int threads)
{
    const double sc = scale > 0.f ? (double)scale : 1.0 / sqrt((double)d);
    const size_t qn = (size_t)sq * d, kn = (size_t)sk * d;
    if (threads < 1) threads = 1;
    if (threads > sq) threads = sq;
    float* qd = (float*)malloc(sizeof(float) * qn);
    float* kd = (float*)malloc(sizeof(float) * kn);
    double* acc = (double*)malloc(sizeof(double) * kn * 2 * (size_t)threads);
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    bwd_job* jobs = (bwd_job*)malloc(sizeof(bwd_job) * threads);
    for (int s = 0; s < slices; s++) {
        quant_dequant(Q + s * qn, sq, d, mode, qd);
        quant_dequant(K + s * kn, sk, d, mode, kd);
        memset(acc, 0, sizeof(double) * kn * 2 * (size_t)threads);
        for (int t = 0; t < threads; t++) {
            bwd_job jb = {qd, kd, V + s * kn, dO + s * qn, dQ + s * qn, acc + kn * 2 * t, acc + kn * (2 * t + 1),
                          (int)((int64_t)sq * t / threads), (int)((int64_t)sq * (t + 1) / threads), sq, sk, d,
                          causal, sc};
            jobs[t] = jb;
            pthread_create(&tid[t], NULL, run_bwd_rows, &jobs[t]);
        }
        for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
        for (size_t e = 0; e < kn; e++) {
            double gk = 0.0, gv = 0.0;
            for (int t = 0; t < threads; t++) {
                gk += acc[kn * 2 * t + e];
                gv += acc[kn * (2 * t + 1) + e];
            }
            dK[s * kn + e] = (float)(gk * sc);
            dV[s * kn + e] = (float)gv;
        }
    }
    free(qd); free(kd); free(acc); free(tid); free(jobs);
}

/* Per query row, ln(sum_j exp(scale * Qq_i . Kq_j)) over the visible keys (in
 * double; +inf for a row that sees no key): the statistic the forward returns
 * for the backward pass. */
void oracle_fp4_attention_lse(const float* Q, const float* K, float* lse, int slices, int sq, int sk, int d,
                              float scale, int mode, int causal)
{
    const double sc = scale > 0.f ? (double)scale : 1.0 / sqrt((double)d);
    const size_t qn = (size_t)sq * d, kn = (size_t)sk * d;
    float* qd = (float*)malloc(sizeof(float) * qn);
    float* kd = (float*)malloc(sizeof(float) * kn);
    double* z = (double*)malloc(sizeof(double) * (size_t)(sk > 0 ? sk : 1));
    for (int s = 0; s < slices; s++) {
        quant_dequant(Q + s * qn, sq, d, mode, qd);
        quant_dequant(K + s * kn, sk, d, mode, kd);
        for (int i = 0; i < sq; i++) {
            long lim = sk;
            if (causal) {
                lim = (long)i + sk - sq + 1;
                if (lim > sk) lim = sk;
            }
            if (lim <= 0) {
                lse[(size_t)s * sq + i] = INFINITY;
                continue;
            }
            double m = -INFINITY;
            for (long k = 0; k < lim; k++) {
                double a = 0.0;
                for (int c = 0; c < d; c++) a += (double)qd[(size_t)i * d + c] * kd[(size_t)k * d + c];
                z[k] = a * sc;
                if (z[k] > m) m = z[k];
            }
            double sum = 0.0;
            for (long k = 0; k < lim; k++) sum += exp(z[k] - m);
            lse[(size_t)s * sq + i] = (float)(m + log(sum));
        }
    }
    free(qd); free(kd); free(z);
}
