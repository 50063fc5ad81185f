/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the MoE layer; never part
 * of the product path.  See moe_oracle.h for what each function restates and
 * the reference file:line it follows.
 *
 * Built with -ffp-contract=off so that the only fused multiply-adds are the
 * explicit fmaf() calls, which are exactly the contractions GCC performs on
 * the reference's `sum += a * b` and `y += w * out` loops.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

/* C[m][n] = sum_p A[m][p] * B[n][p], k-ascending fmaf chain from 0.0f.
 * src/tensor.cu:136-148 (matmul_transposed).  Eight independent output
 * chains are interleaved for throughput; each one is still strictly serial
 * in p, so the bits are those of the reference loop. */
static void matmul_nt(const float* A, const float* B, float* C, int m, int k, int n) {
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)m; ++i) {
        const float* a = A + (size_t)i * k;
        float* c = C + (size_t)i * n;
        int j = 0;
        for (; j + 8 <= n; j += 8) {
            const float* b0 = B + (size_t)(j + 0) * k;
            const float* b1 = B + (size_t)(j + 1) * k;
            const float* b2 = B + (size_t)(j + 2) * k;
            const float* b3 = B + (size_t)(j + 3) * k;
            const float* b4 = B + (size_t)(j + 4) * k;
            const float* b5 = B + (size_t)(j + 5) * k;
            const float* b6 = B + (size_t)(j + 6) * k;
            const float* b7 = B + (size_t)(j + 7) * k;
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f, s4 = 0.f, s5 = 0.f, s6 = 0.f, s7 = 0.f;
            for (int p = 0; p < k; ++p) {
                const float av = a[p];
                s0 = fmaf(av, b0[p], s0);
                s1 = fmaf(av, b1[p], s1);
                s2 = fmaf(av, b2[p], s2);
                s3 = fmaf(av, b3[p], s3);
                s4 = fmaf(av, b4[p], s4);
                s5 = fmaf(av, b5[p], s5);
                s6 = fmaf(av, b6[p], s6);
                s7 = fmaf(av, b7[p], s7);
            }
            c[j + 0] = s0; c[j + 1] = s1; c[j + 2] = s2; c[j + 3] = s3;
            c[j + 4] = s4; c[j + 5] = s5; c[j + 6] = s6; c[j + 7] = s7;
        }
        for (; j < n; ++j) {
            const float* b = B + (size_t)j * k;
            float s = 0.f;
            for (int p = 0; p < k; ++p) s = fmaf(a[p], b[p], s);
            c[j] = s;
        }
    }
}

/* src/tensor.cu:132-134 accurate_exp and :169-172 silu. */
static inline float silu_ref(float x) {
    const float e = (float)exp((double)(-x));
    return x / (1.0f + e);
}

void oracle_router_logits(const float* x, const float* wg, const float* bias,
                          int T, int d, int E, float* logits, int nthreads) {
    set_threads(nthreads);
    matmul_nt(x, wg, logits, T, d, E);
    if (bias) {
        for (long long i = 0; i < (long long)T * E; ++i) logits[i] = logits[i] + bias[i % E];
    }
}

/* src/layer.cu:47-70.  Every operation is a single IEEE fp32 operation in the
 * reference too (no multiply feeds an add, so nothing is contracted). */
void oracle_route_phi(const float* logits, int E, float quantum, float tie_eps,
                      int* idx, float* w) {
    float scores[1024];
    for (int e = 0; e < E; ++e) {
        const float score = logits[e];
        const float rounded = floorf(fabsf(score) / quantum + 0.5f) * quantum;
        scores[e] = score < 0.0f ? -rounded : rounded;
    }
    int sel[2];
    for (int s = 0; s < 2; ++s) {
        const int excluded = s == 0 ? -1 : sel[0];
        int best = -1;
        float best_value = -INFINITY;
        for (int e = 0; e < E; ++e) {
            if (e == excluded) continue;
            if (best < 0 || scores[e] > best_value + tie_eps) {
                best = e;
                best_value = scores[e];
            }
        }
        sel[s] = best;
    }
    idx[0] = sel[0]; idx[1] = sel[1];
    w[0] = 0.5f; w[1] = 0.5f;
}

/* Ordering key: NaN sorts below every number. */
static inline float route_key(float v) { return v != v ? -INFINITY : v; }

void oracle_route_softmax(const float* logits, int E, int k, int* idx, float* w) {
    unsigned char taken[1024];
    memset(taken, 0, (size_t)E);
    for (int s = 0; s < k; ++s) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
            if (taken[e]) continue;
            if (best < 0 || route_key(logits[e]) > route_key(logits[best])) best = e;
        }
        taken[best] = 1;
        idx[s] = best;
    }
    const double m = (double)logits[idx[0]];
    double p[1024], sum = 0.0;
    for (int s = 0; s < k; ++s) { p[s] = exp((double)logits[idx[s]] - m); sum += p[s]; }
    for (int s = 0; s < k; ++s) w[s] = (float)(p[s] / sum);
}

void oracle_route(const float* logits, int T, int E, int k, int policy,
                  float quantum, float tie_eps, int* idx, float* w) {
    for (int t = 0; t < T; ++t) {
        if (policy == ORACLE_POLICY_PHI)
            oracle_route_phi(logits + (size_t)t * E, E, quantum, tie_eps, idx + (size_t)t * k, w + (size_t)t * k);
        else
            oracle_route_softmax(logits + (size_t)t * E, E, k, idx + (size_t)t * k, w + (size_t)t * k);
    }
}

/* src/tensor.cu:174-189 tensor_ops::layer_norm. */
void oracle_layer_norm(const float* x, const float* w, const float* b, float eps, int T, int d,
                       float* y) {
#pragma omp parallel for schedule(static)
    for (long long r = 0; r < (long long)T; ++r) {
        const float* xr = x + (size_t)r * d;
        float* yr = y + (size_t)r * d;
        float mean = 0.0f;
        for (int j = 0; j < d; ++j) mean += xr[j];
        mean /= (float)d;
        float var = 0.0f;
        for (int j = 0; j < d; ++j) {
            const float dv = xr[j] - mean;
            var += dv * dv;   /* not contracted in the reference build: rounded product */
        }
        const float inv = 1.0f / sqrtf(var / (float)d + eps);
        for (int j = 0; j < d; ++j) yr[j] = fmaf((xr[j] - mean) * inv, w[j], b[j]);
    }
}

/* src/layer.cu:32-45 PhiMLP::forward. */
void oracle_expert_ffn(const float* X, int rows, int d, int ff,
                       const float* w1, const float* w3, const float* w2,
                       float* out, int nthreads) {
    set_threads(nthreads);
    float* gate = (float*)malloc(sizeof(float) * (size_t)rows * ff);
    float* up = (float*)malloc(sizeof(float) * (size_t)rows * ff);
    matmul_nt(X, w1, gate, rows, d, ff);
    matmul_nt(X, w3, up, rows, d, ff);
    for (long long i = 0; i < (long long)rows * ff; ++i) {
        const float a = silu_ref(gate[i]);
        gate[i] = a * up[i];
    }
    matmul_nt(gate, w2, out, rows, ff, d);
    free(gate);
    free(up);
}

/* src/layer.cu:80-103 PhiMoE::forward. */
int oracle_moe_forward(const float* x, int T, int d, int ff, int E, int k,
                       int policy, float quantum, float tie_eps,
                       const float* wg, const float* bias,
                       const float* const* w1, const float* const* w3,
                       const float* const* w2,
                       const int* sample, int n_sample,
                       float* y, int* idx, float* w, float* logits,
                       int nthreads) {
    if (T < 0 || d <= 0 || ff <= 0 || E <= 0 || k <= 0 || k > E || E > 1024) return -1;
    if (policy == ORACLE_POLICY_PHI && k != 2) return -1;
    float* lg = (float*)malloc(sizeof(float) * ((size_t)T * E + 1));
    int* id = (int*)malloc(sizeof(int) * ((size_t)T * k + 1));
    float* wt = (float*)malloc(sizeof(float) * ((size_t)T * k + 1));
    oracle_router_logits(x, wg, bias, T, d, E, lg, nthreads);
    oracle_route(lg, T, E, k, policy, quantum, tie_eps, id, wt);

    /* Which tokens need their output row. */
    unsigned char* want = (unsigned char*)calloc((size_t)T + 1, 1);
    if (sample) {
        for (int i = 0; i < n_sample; ++i)
            if (sample[i] >= 0 && sample[i] < T) want[sample[i]] = 1;
    } else {
        memset(want, 1, (size_t)T);
    }
    for (int t = 0; t < T; ++t)
        if (want[t]) memset(y + (size_t)t * d, 0, sizeof(float) * (size_t)d);

    int* rows_tok = (int*)malloc(sizeof(int) * ((size_t)T + 1));
    float* rows_w = (float*)malloc(sizeof(float) * ((size_t)T + 1));
    for (int e = 0; e < E; ++e) {
        /* assignments[e], ascending token order (src/layer.cu:86-91). */
        int n = 0;
        for (int t = 0; t < T; ++t) {
            if (!want[t]) continue;
            for (int s = 0; s < k; ++s)
                if (id[(size_t)t * k + s] == e) { rows_tok[n] = t; rows_w[n] = wt[(size_t)t * k + s]; ++n; }
        }
        if (n == 0) continue;
        float* X = (float*)malloc(sizeof(float) * (size_t)n * d);
        float* out = (float*)malloc(sizeof(float) * (size_t)n * d);
        for (int i = 0; i < n; ++i) memcpy(X + (size_t)i * d, x + (size_t)rows_tok[i] * d, sizeof(float) * (size_t)d);
        oracle_expert_ffn(X, n, d, ff, w1[e], w3[e], w2[e], out, nthreads);
        for (int i = 0; i < n; ++i) {
            float* yr = y + (size_t)rows_tok[i] * d;
            const float* o = out + (size_t)i * d;
            const float wv = rows_w[i];
            for (int j = 0; j < d; ++j) yr[j] = fmaf(wv, o[j], yr[j]);
        }
        free(X);
        free(out);
    }
    if (idx) memcpy(idx, id, sizeof(int) * (size_t)T * k);
    if (w) memcpy(w, wt, sizeof(float) * (size_t)T * k);
    if (logits) memcpy(logits, lg, sizeof(float) * (size_t)T * E);
    free(rows_tok); free(rows_w); free(want); free(lg); free(id); free(wt);
    return 0;
}
