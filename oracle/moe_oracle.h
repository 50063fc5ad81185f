/*
 * TEST INFRASTRUCTURE ONLY -- never linked into the product library.
 *
 * CPU restatement of the reference MoE FFN layer (songsnim/accelerating-MoE-inference):
 *   router     matmul_transposed(x, gate, logits)   src/layer.cu:84, src/tensor.cu:136-148
 *   PHI route  quantise 1e-3, tie-eps 2e-2 top-2     src/layer.cu:47-70
 *   dispatch   assignments[e] in ascending token     src/layer.cu:86-91
 *   expert     PhiMLP::forward (w1, silu, w3, mul, w2) src/layer.cu:32-45
 *   combine    y[t] += w * out, ascending expert     src/layer.cu:92-102
 * plus the softmax / top-k / renormalise policy that the reference declares
 * (include/tensor.h:67, softmax_last_dim) but never defines.
 *
 * Arithmetic follows the reference as its own Makefile builds it (g++ -O3
 * -march=native on an FMA-capable host): every `sum += a * b` is contracted
 * by GCC into a fused multiply-add, so each dot product is a k-ascending
 * fmaf() chain from 0.0f.  silu is x / (1 + (float)exp((double)-x))
 * (src/tensor.cu:132-134, 169-172).  The combine `y += w * out` is likewise a
 * fused multiply-add into y.
 *
 * Parity is pinned by comparing this file's output bit for bit against the
 * reference's own PhiMoE::forward compiled from its sources (oracle/_ref,
 * built by oracle/Makefile); see tests/test_oracle.py.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_POLICY_PHI = 0, ORACLE_POLICY_SOFTMAX = 1 };

/* logits[t][e] = bias[e] + sum_k x[t][k] * wg[e][k]  (k-ascending fma chain;
 * the bias, if non-NULL, is one fp32 add after the chain). */
void oracle_router_logits(const float* x, const float* wg, const float* bias,
                          int T, int d, int E, float* logits, int nthreads);

/* Reference top-2 policy on one token's E logits (src/layer.cu:47-70).
 * idx[0..1] = (first, second) in selection order, w[0..1] = 0.5f. */
void oracle_route_phi(const float* logits, int E, float quantum, float tie_eps,
                      int* idx, float* w);

/* Softmax -> top-k -> renormalise on one token's logits.  Selection order is
 * descending logit (NaN ranks below every number); exact ties go to the
 * lower expert index.  Weights are
 * exp(l - l_max) in double over the selected k, renormalised, rounded to
 * float once. */
void oracle_route_softmax(const float* logits, int E, int k, int* idx, float* w);

/* Route every token: idx/w are [T][k]. */
void oracle_route(const float* logits, int T, int E, int k, int policy,
                  float quantum, float tie_eps, int* idx, float* w);

/* One expert's SwiGLU FFN on `rows` gathered rows (PhiMLP::forward):
 * out[rows][d] = (silu(X w1^T) * (X w3^T)) w2^T. */
void oracle_expert_ffn(const float* X, int rows, int d, int ff,
                       const float* w1, const float* w3, const float* w2,
                       float* out, int nthreads);

/* tensor_ops::layer_norm (src/tensor.cu:174-189) per row of x [T][d]:
 * mean = serial sum / d; var = serial sum of rounded (x - mean)^2, / d;
 * inv = 1 / sqrt(var + eps); y = fma((x - mean) * inv, w, b).  GCC contracts
 * the output expression but leaves the variance accumulation unfused; both
 * were established bit-exactly against the reference's compiled function. */
void oracle_layer_norm(const float* x, const float* w, const float* b, float eps, int T, int d,
                       float* y);

/* Full layer.  w1[e], w3[e]: [ff][d]; w2[e]: [d][ff].  y is [T][d] and is
 * overwritten.  idx/w/logits outputs may be NULL.  If `sample` is non-NULL
 * only the n_sample listed tokens get their y rows computed (routing is still
 * done for all T tokens); other rows of y are left untouched. */
int oracle_moe_forward(const float* x, int T, int d, int ff, int E, int k,
                       int policy, float quantum, float tie_eps,
                       const float* wg, const float* bias,
                       const float* const* w1, const float* const* w3,
                       const float* const* w2,
                       const int* sample, int n_sample,
                       float* y, int* idx, float* w, float* logits,
                       int nthreads);

#ifdef __cplusplus
}
#endif
#endif
