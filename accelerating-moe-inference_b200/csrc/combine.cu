// The ordered combine: y[t] = sum over token t's k routed experts, in
// ascending expert order, of  acc = fmaf(w, v, acc)  from acc = 0, where v is
// that expert's output row for t and w its routing weight -- exactly the
// reference's combine, `y.at(t, j) += w * output.at(i, j)` run expert by
// expert over a zeroed y (src/layer.cu:85,98-101) with the multiply-add
// contracted into one fma as GCC builds it.  The result does not depend on
// how the expert GEMMs were scheduled, so a forward is bit-reproducible for
// every top-k and for split-K.
//
// The down GEMM (or the decode down kernel) stores each routed row's output
// unweighted at part[split][slot] (slot = t * k + s, the s-th selection of
// token t); split-K partials of one slot add in ascending split order before
// the fma.  An optional residual r is added last: y = combine + r (the
// decoder layer's `moe_out + x`, src/layer.cu:160-161).
#include <climits>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

constexpr int kCombineThreads = 256;
constexpr int kCombineWarps = kCombineThreads / 32;

// kU float4 columns per lane per unit (more for large batches); the k * nsplit
// partial rows a column needs are loaded kB at a time, all in flight, then
// consumed in the fixed order: slot by ascending expert, split by split.
template <int KMAX, int kU, int kB>
__global__ void __launch_bounds__(kCombineThreads)
combine_kernel(const float* __restrict__ part, int nsplit, size_t split_stride,
               const int* __restrict__ idx, const float* __restrict__ wts, int T, int k, int d,
               int units_per_token, const float* resid, float* y) {
    wait_predecessor_grid();
    launch_dependents();
    const int lane = threadIdx.x & 31;
    const long long unit = (long long)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);
    if (unit >= (long long)T * units_per_token) return;
    const int t = (int)(unit / units_per_token);
    const int chunk = (int)(unit % units_per_token);
    int ord[KMAX];
    float ow[KMAX];
    slot_order<KMAX>(idx + (size_t)t * k, wts + (size_t)t * k, k, lane, ord, ow);
    // Lane r holds the r-th slot (ascending expert): its row offset and weight.
    const int nv = d / 4;
    size_t my_off = 0;
    float my_w = 0.0f;
#pragma unroll
    for (int r = 0; r < KMAX; ++r)
        if (lane == r) {
            my_off = ((size_t)t * k + ord[r]) * nv;
            my_w = ow[r];
        }
    const float4* base = reinterpret_cast<const float4*>(part);
    const size_t sstride = split_stride / 4;
    const int v0 = chunk * 32 * kU + lane;
    const int total = k * nsplit;
    float4 acc[kU], v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
        acc[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        v[u] = acc[u];
    }
    for (int b0 = 0; b0 < total; b0 += kB) {
        float4 q[kB][kU];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = b0 + j;
            const int r = i / nsplit, sp = i - r * nsplit;
            const size_t off = __shfl_sync(0xffffffffu, my_off, r < 32 ? r : 0);
            if (i < total) {
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    const int c = v0 + 32 * u;
                    if (c < nv) q[j][u] = __ldcs(base + off + sp * sstride + c);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int i = b0 + j;
            const int r = i / nsplit, sp = i - r * nsplit;
            const float w = __shfl_sync(0xffffffffu, my_w, r < 32 ? r : 0);
            if (i < total) {
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    if (sp == 0) {
                        v[u] = q[j][u];
                    } else {
                        v[u].x = __fadd_rn(v[u].x, q[j][u].x);
                        v[u].y = __fadd_rn(v[u].y, q[j][u].y);
                        v[u].z = __fadd_rn(v[u].z, q[j][u].z);
                        v[u].w = __fadd_rn(v[u].w, q[j][u].w);
                    }
                    if (sp == nsplit - 1) {
                        acc[u].x = __fmaf_rn(w, v[u].x, acc[u].x);
                        acc[u].y = __fmaf_rn(w, v[u].y, acc[u].y);
                        acc[u].z = __fmaf_rn(w, v[u].z, acc[u].z);
                        acc[u].w = __fmaf_rn(w, v[u].w, acc[u].w);
                    }
                }
            }
        }
    }
    float4* yr = reinterpret_cast<float4*>(y) + (size_t)t * nv;
    const float4* rr = resid ? reinterpret_cast<const float4*>(resid) + (size_t)t * nv : nullptr;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
        const int c = v0 + 32 * u;
        if (c >= nv) continue;
        float4 o = acc[u];
        if (rr) {
            const float4 q = rr[c];
            o.x = __fadd_rn(o.x, q.x);
            o.y = __fadd_rn(o.y, q.y);
            o.z = __fadd_rn(o.z, q.z);
            o.w = __fadd_rn(o.w, q.w);
        }
        yr[c] = o;
    }
}

template <int KMAX, int kU, int kB>
cudaError_t launch_t(const Layer& L, int T, int nsplit, size_t split_stride, const float* resid,
                     float* y, cudaStream_t s) {
    const int units = (L.d / 4 + 32 * kU - 1) / (32 * kU);
    const long long warps = (long long)T * units;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((warps + kCombineWarps - 1) / kCombineWarps));
    cfg.blockDim = dim3(kCombineThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.profile ? 0 : 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, combine_kernel<KMAX, kU, kB>, (const float*)L.ws.part, nsplit,
                              split_stride, (const int*)L.ws.idx, (const float*)L.ws.wts, T, L.k,
                              L.d, units, resid, y);
}

}  // namespace

cudaError_t launch_combine(const Layer& L, int T, int nsplit, const float* resid, float* y,
                           cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const size_t stride = (size_t)T * L.k * L.d;
    // Decode-sized batches: one float4 per lane per unit, so a token's row is
    // spread over d / 128 warps.
    // Large batches (one split): 4 columns per lane, all k slots' loads in
    // flight (k <= 2) or 2 columns and 8 slots (k <= 8).
    const bool small = (long long)T * (L.d / 512) < 8LL * L.sm_count;
    if (small) {
        if (L.k <= 2) return launch_t<2, 1, 16>(L, T, nsplit, stride, resid, y, s);
        return launch_t<kMaxTopK, 1, 16>(L, T, nsplit, stride, resid, y, s);
    }
    if (L.k <= 2) return launch_t<2, 4, 2>(L, T, nsplit, stride, resid, y, s);
    return launch_t<kMaxTopK, 2, 8>(L, T, nsplit, stride, resid, y, s);
}

}  // namespace moe
