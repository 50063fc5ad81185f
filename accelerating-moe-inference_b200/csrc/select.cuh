// Expert selection of one token from its router logits, shared by the
// router kernels (route.cu) and the fused batch-1 decode step
// (decode_step.cu), so both choose experts with the same code.
#pragma once

#include <climits>
#include <cmath>

#include "moe_internal.h"

namespace moe {

// Softmax ordering key: NaN sorts below every number (as -inf).
__device__ __forceinline__ float route_key(float v) { return v != v ? -INFINITY : v; }

// Expert selection for one token's logits l[0..E): warp-collective (every
// lane calls it); the k selected experts and combine weights are valid on
// lane 0.
//   PHI_QUANTISED (src/layer.cu:47-70): quantise, then two hysteresis scans;
//     the scan is order-dependent, so one lane runs it serially.
//   SOFTMAX_TOPK: k rounds of a warp-wide argmax over (key, index), larger
//     key first, exact ties to the lower index; weights are the softmax of
//     the chosen logits in double, renormalised over the k.
__device__ __forceinline__ void select_experts(const float* l, int E, int k, int policy,
                                               float quantum, float tie_eps, int lane,
                                               int (&sel)[kMaxTopK], float (&wsel)[kMaxTopK]) {
    if (policy == MOE_ROUTER_PHI_QUANTISED) {
        if (lane == 0) {
            for (int s = 0; s < 2; ++s) {
                const int excluded = s == 0 ? -1 : sel[0];
                int best = -1;
                float best_value = -INFINITY;
                for (int e = 0; e < E; ++e) {
                    if (e == excluded) continue;
                    const float score = l[e];
                    const float rounded =
                        floorf(__fadd_rn(__fdiv_rn(fabsf(score), quantum), 0.5f)) * quantum;
                    const float v = score < 0.0f ? -rounded : rounded;
                    if (best < 0 || v > __fadd_rn(best_value, tie_eps)) {
                        best = e;
                        best_value = v;
                    }
                }
                sel[s] = best;
                wsel[s] = 0.5f;
            }
        }
        return;
    }
    unsigned taken = 0;  // bit i: expert lane + 32 i already chosen
    for (int s = 0; s < k; ++s) {
        float bk = -INFINITY;
        int bi = INT_MAX;
        for (int i = 0, e = lane; e < E; ++i, e += 32) {
            if (taken & (1u << i)) continue;
            const float kv = route_key(l[e]);
            if (bi == INT_MAX || kv > bk) { bk = kv; bi = e; }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ok = __shfl_xor_sync(0xffffffffu, bk, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (ok > bk || (ok == bk && oi < bi)) { bk = ok; bi = oi; }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        sel[s] = bi;
    }
    // Lane s < k computes p_s = e^(l_s - l_0) and its weight p_s / sum at
    // the same time (one exp and one divide of latency instead of k); every
    // lane adds the p_s in ascending s, the order a serial loop would use.
    float ls = 0.0f;
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
        if (s < k && lane == s) ls = l[sel[s]];
    const double m = (double)l[sel[0]];
    const double p = lane < k ? exp((double)ls - m) : 0.0;
    double sum = 0.0;
    for (int s = 0; s < k; ++s) sum += __shfl_sync(0xffffffffu, p, s);
    const float w = (float)(p / sum);
#pragma unroll
    for (int s = 0; s < kMaxTopK; ++s)
        if (s < k) wsel[s] = __shfl_sync(0xffffffffu, w, s);
}

}  // namespace moe
