// Weight-streaming decode path (small T): the layer is bound by reading the
// routed experts' weights once from HBM, so these kernels stream exactly
// those weights with coalesced 128-bit loads, several loads in flight per
// lane, and do the math on CUDA cores in fp32.  The reference has no
// decode-specialised kernel; its decode re-runs the prefill path per token
// (src/model.cu:2061-2104).
//
// Inputs come from the dispatch: the packed activation rows A (expert e's
// tokens at rows eoff[e] .. eoff[e] + counts[e], ascending token order; fp32
// in FP32 precision, bf16 in BF16 precision), row_token / row_weight.
//
// decode_gateup: the (active expert, intermediate column) pairs are split
//   into equal contiguous ranges, one per warp.  A warp takes two columns at
//   a time -- their gate and up rows of w13, 4 weight rows -- and each lane
//   streams 16 bytes of each row per step; the expert's token rows are read
//   through L1 (they are tiny and shared by every warp).  Warp reductions
//   give the dots; SwiGLU is applied and H (fp32, one row per routed token,
//   unpadded) is written.
// decode_down: work items are (active expert, 4 output columns, 2048-wide K
//   chunk of the padded d_ff), again in equal contiguous ranges per warp.
//   Each partial dot is stored, unweighted, at part[chunk][slot of the row];
//   the ordered combine (combine.cu) adds the chunks in order and the
//   experts in ascending order, so the result is bit-reproducible.
// No shared-memory staging and no block-wide synchronisation: warps are
// independent, and the ranges balance the bytes each warp streams to within
// one step.
#include <cuda_bf16.h>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

constexpr int kDecThreads = 512;            // 16 warps per CTA
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kMaxDecodeTokens = 64;

// Weights are read exactly once: bypass L1 so the stream does not evict the
// token rows every warp re-reads from it.
__device__ __forceinline__ uint4 stream_load(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 16 bytes of a row -> V fp32 values.
template <typename T>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int N = 4;
    using Raw = float4;
    __device__ static Raw load(const float* p) {
        const uint4 u = stream_load(p);
        return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z),
                           __uint_as_float(u.w));
    }
    __device__ static void unpack(const Raw& r, float (&v)[4]) {
        v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
    }
};
template <>
struct Vec<__nv_bfloat16> {
    static constexpr int N = 8;
    using Raw = uint4;
    __device__ static Raw load(const __nv_bfloat16* p) { return stream_load(p); }
    __device__ static void unpack(const Raw& r, float (&v)[8]) {
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Active experts and the unpadded offset of each one's H rows, per CTA.
struct Active {
    int n;
    int act[kMaxExperts];
    int coff[kMaxExperts];
};

// Warp 0 builds it: each lane loads a run of consecutive experts' counts at
// once (no chain of dependent global loads before the first weight load),
// and two warp scans give the row offsets and the active list's positions,
// so the list stays in ascending expert order.
__device__ void build_active(Active& a, const int* __restrict__ counts, int E) {
    if (threadIdx.x < 32) {
        constexpr int kPer = kMaxExperts / 32;
        const int lane = threadIdx.x;
        const int per = (E + 31) / 32;
        const int e0 = lane * per;
        int c[kPer];
        int sum = 0, nact = 0;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            c[i] = (i < per && e0 + i < E) ? counts[e0 + i] : 0;
            sum += c[i];
            nact += c[i] > 0 ? 1 : 0;
        }
        int s = sum, n = nact;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ts = __shfl_up_sync(0xffffffffu, s, o);
            const int tn = __shfl_up_sync(0xffffffffu, n, o);
            if (lane >= o) {
                s += ts;
                n += tn;
            }
        }
        int off = s - sum, pos = n - nact;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            if (i < per && e0 + i < E) {
                a.coff[e0 + i] = off;
                off += c[i];
                if (c[i] > 0) a.act[pos++] = e0 + i;
            }
        }
        if (lane == 31) a.n = n;
    }
    __syncthreads();
}

// acc[r][m] += dot(w rows r, activation rows m) over K positions
// [k_begin, k_end), lane-strided by 16-byte vectors.  W rows are of type WT,
// activation rows of type AT; each row pointer points at K position 0.
template <typename WT, typename AT, int R, int TM>
__device__ __forceinline__ void stream_dots(const WT* const (&w)[R], const AT* const (&a)[TM],
                                            int gm, int k_begin, int k_end, int lane,
                                            float (&acc)[R][TM]) {
    constexpr int V = Vec<WT>::N;
    // 16-byte loads per weight row in flight per lane: more when fewer token
    // rows share the registers.
    constexpr int kInFlight = V * TM >= 32 ? 1 : (V * TM >= 16 ? 2 : 4);
    for (int k0 = k_begin + lane * V; k0 < k_end; k0 += 32 * V * kInFlight) {
        typename Vec<WT>::Raw raw[kInFlight][R];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int kk = k0 + u * 32 * V;
            if (kk < k_end) {
#pragma unroll
                for (int r = 0; r < R; ++r) raw[u][r] = Vec<WT>::load(w[r] + kk);
            }
        }
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int kk = k0 + u * 32 * V;
            if (kk >= k_end) break;
            float wv[R][V];
#pragma unroll
            for (int r = 0; r < R; ++r) Vec<WT>::unpack(raw[u][r], wv[r]);
#pragma unroll
            for (int m = 0; m < TM; ++m) {
                if (m >= gm) break;
                float av[V];
                if constexpr (sizeof(AT) == 4) {
#pragma unroll
                    for (int q = 0; q < V; q += 4) {
                        const float4 f = __ldg(reinterpret_cast<const float4*>(
                            reinterpret_cast<const float*>(a[m]) + kk + q));
                        av[q] = f.x; av[q + 1] = f.y; av[q + 2] = f.z; av[q + 3] = f.w;
                    }
                } else {
                    static_assert(V == 8, "bf16 activations pair with bf16 weights");
                    Vec<__nv_bfloat16>::unpack(
                        __ldg(reinterpret_cast<const uint4*>(
                            reinterpret_cast<const __nv_bfloat16*>(a[m]) + kk)),
                        reinterpret_cast<float(&)[8]>(av));
                }
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int q = 0; q < V; ++q) acc[r][m] = fmaf(wv[r][q], av[q], acc[r][m]);
            }
        }
    }
}

template <typename WT, typename AT, int TM>
__global__ void __launch_bounds__(kDecThreads, 1)
decode_gateup_kernel(const AT* __restrict__ a_rows, const WT* __restrict__ w13, int d, int ffp,
                     int E, const int* __restrict__ counts, const int* __restrict__ eoff,
                     float* __restrict__ h) {
    __shared__ Active A;
    wait_predecessor_grid();
    launch_dependents();
    build_active(A, counts, E);
    const int lane = threadIdx.x & 31;
    const long long W = (long long)gridDim.x * kDecWarps;
    const long long gw = (long long)blockIdx.x * kDecWarps + (threadIdx.x >> 5);
    const long long total = (long long)A.n * ffp;          // (expert, column) pairs
    long long j = total * gw / W;
    const long long j_end = total * (gw + 1) / W;
    while (j < j_end) {
        const int ai = (int)(j / ffp);
        const int e = A.act[ai];
        const int c = (int)(j % ffp);
        // Two columns when both are in range and in the same expert.
        const int nc = (j + 1 < j_end && c + 1 < ffp) ? 2 : 1;
        const size_t base = (size_t)e * 2 * ffp;
        const size_t rg0 = (size_t)(c / kFfBlock) * (2 * kFfBlock) + (c % kFfBlock);
        const size_t rg1 = (size_t)((c + nc - 1) / kFfBlock) * (2 * kFfBlock) + ((c + nc - 1) % kFfBlock);
        const WT* const w[4] = {w13 + (base + rg0) * d, w13 + (base + rg0 + kFfBlock) * d,
                                w13 + (base + rg1) * d, w13 + (base + rg1 + kFfBlock) * d};
        const int n_e = counts[e];
        const int r0 = eoff[e];
        for (int g0 = 0; g0 < n_e; g0 += TM) {
            const int gm = min(TM, n_e - g0);
            const AT* a[TM];
#pragma unroll
            for (int m = 0; m < TM; ++m) a[m] = a_rows + (size_t)(r0 + g0 + min(m, gm - 1)) * d;
            float acc[4][TM];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int m = 0; m < TM; ++m) acc[r][m] = 0.0f;
            stream_dots<WT, AT, 4, TM>(w, a, gm, 0, d, lane, acc);
#pragma unroll
            for (int m = 0; m < TM; ++m) {
                if (m >= gm) break;
                const float g0v = warp_sum(acc[0][m]), u0v = warp_sum(acc[1][m]);
                const float g1v = warp_sum(acc[2][m]), u1v = warp_sum(acc[3][m]);
                if (lane == 0) {
                    float* hr = h + (size_t)(A.coff[e] + g0 + m) * ffp + c;
                    hr[0] = g0v / (1.0f + __expf(-g0v)) * u0v;
                    if (nc == 2) hr[1] = g1v / (1.0f + __expf(-g1v)) * u1v;
                }
            }
        }
        j += nc;
    }
}

template <typename WT, int TM>
__global__ void __launch_bounds__(kDecThreads, 1)
decode_down_kernel(const float* __restrict__ h, const WT* __restrict__ w2, int d, int ffp,
                   int E, const int* __restrict__ counts, const int* __restrict__ eoff,
                   const int* __restrict__ row_slot, float* __restrict__ part,
                   size_t split_stride) {
    __shared__ Active A;
    // The routing (counts) comes from the kernel before decode_gateup, and a
    // dependent launch of this kernel happens only once every decode_gateup
    // CTA has passed its own wait (launch_dependents follows it), so counts
    // are final here already: the active list is built, and each warp's first
    // work item's weight rows are prefetched into L2, while decode_gateup is
    // still streaming.  h (decode_gateup's output) is read after the wait.
    build_active(A, counts, E);
    const int lane = threadIdx.x & 31;
    const int nq = (d + 3) / 4;                    // column quads per expert
    const int nk = (ffp + kDownChunk - 1) / kDownChunk;
    const long long W = (long long)gridDim.x * kDecWarps;
    const long long gw = (long long)blockIdx.x * kDecWarps + (threadIdx.x >> 5);
    const long long total = (long long)A.n * nq * nk;
    {
        const long long it = total * gw / W;
        if (lane < 4 && it < total * (gw + 1) / W) {
            const int e = A.act[(int)(it / ((long long)nq * nk))];
            const int rem = (int)(it % ((long long)nq * nk));
            const int n = min((rem / nk) * 4 + lane, d - 1);
            const int k0 = (rem % nk) * kDownChunk;
            const int k1 = min(ffp, k0 + kDownChunk);
            prefetch_l2_bulk(w2 + ((size_t)e * d + n) * ffp + k0, (uint32_t)((k1 - k0) * sizeof(WT)));
        }
    }
    wait_predecessor_grid();
    launch_dependents();
    for (long long it = total * gw / W; it < total * (gw + 1) / W; ++it) {
        const int ai = (int)(it / ((long long)nq * nk));
        const int rem = (int)(it % ((long long)nq * nk));
        const int e = A.act[ai];
        const int n0 = (rem / nk) * 4;
        const int k0 = (rem % nk) * kDownChunk;
        const int k1 = min(ffp, k0 + kDownChunk);
        const WT* const w[4] = {w2 + ((size_t)e * d + min(n0, d - 1)) * ffp,
                                w2 + ((size_t)e * d + min(n0 + 1, d - 1)) * ffp,
                                w2 + ((size_t)e * d + min(n0 + 2, d - 1)) * ffp,
                                w2 + ((size_t)e * d + min(n0 + 3, d - 1)) * ffp};
        const int n_e = counts[e];
        const int r0 = eoff[e];
        for (int g0 = 0; g0 < n_e; g0 += TM) {
            const int gm = min(TM, n_e - g0);
            const float* a[TM];
#pragma unroll
            for (int m = 0; m < TM; ++m)
                a[m] = h + (size_t)(A.coff[e] + g0 + min(m, gm - 1)) * ffp;
            float acc[4][TM];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int m = 0; m < TM; ++m) acc[r][m] = 0.0f;
            stream_dots<WT, float, 4, TM>(w, a, gm, k0, k1, lane, acc);
#pragma unroll
            for (int m = 0; m < TM; ++m) {
                if (m >= gm) break;
                const int prow = r0 + g0 + m;
                float* dst = part + (size_t)(k0 / kDownChunk) * split_stride +
                             (size_t)row_slot[prow] * d + n0;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float v = warp_sum(acc[r][m]);
                    if (lane == r && n0 + r < d) dst[r] = v;
                }
            }
        }
    }
}

// One CTA per SM, launched with programmatic stream serialisation (the
// kernel waits for its predecessor itself).  Profiling disables it so the
// stage events stay between the kernels.
template <typename Kern, typename... Args>
cudaError_t launch_dependent(const Layer& L, Kern kern, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.sm_count);
    cfg.blockDim = dim3(kDecThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.profile ? 0 : 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename WT, typename AT, int TM>
cudaError_t launch_t(Layer& L, size_t stride, cudaStream_t s, const WT* w13, const WT* w2) {
    const Workspace& W = L.ws;
    cudaError_t err = launch_dependent(L, decode_gateup_kernel<WT, AT, TM>, s,
                                       static_cast<const AT*>(W.a_hi), w13, L.d, L.ffp, L.E,
                                       (const int*)W.counts, (const int*)W.eoff, W.h_dec);
    if (err != cudaSuccess) return err;
    prof_mark(L, 4, s);
    return launch_dependent(L, decode_down_kernel<WT, TM>, s, (const float*)W.h_dec, w2, L.d,
                            L.ffp, L.E, (const int*)W.counts, (const int*)W.eoff,
                            (const int*)W.row_slot, W.part, stride);
}

template <typename WT, typename AT>
cudaError_t launch_w(Layer& L, int T, cudaStream_t s, const WT* w13, const WT* w2) {
    // Token rows per pass over the weights: up to 4 (the weights of a pass
    // are re-read from L1/L2 for further passes).
    const int tm = T >= 4 ? 4 : (T >= 2 ? 2 : 1);
    const size_t stride = (size_t)T * L.k * L.d;
    switch (tm) {
        case 4: return launch_t<WT, AT, 4>(L, stride, s, w13, w2);
        case 2: return launch_t<WT, AT, 2>(L, stride, s, w13, w2);
        default: return launch_t<WT, AT, 1>(L, stride, s, w13, w2);
    }
}

}  // namespace

int decode_max_supported_tokens() { return kMaxDecodeTokens; }

int decode_chunks(const Layer& L) { return (L.ffp + kDownChunk - 1) / kDownChunk; }

cudaError_t launch_decode(Layer& L, const float* x, int T, int* nsplit, cudaStream_t s,
                          const NormRef& nr, bool packed) {
    if (T > kMaxDecodeTokens || !L.ws.h_dec) return cudaErrorInvalidValue;
    *nsplit = decode_chunks(L);
    // Pack the routed token rows (fp32 as is in FP32 precision, bf16 in BF16),
    // normalised on the way when nr is active -- unless the small-batch
    // router already did.
    if (!packed) {
        cudaError_t err = launch_dispatch_permute_raw(L, x, T, s, nr);
        if (err != cudaSuccess) return err;
    }
    prof_mark(L, 3, s);
    if (L.cfg.precision == MOE_PREC_BF16)
        return launch_w<__nv_bfloat16, __nv_bfloat16>(
            L, T, s, static_cast<const __nv_bfloat16*>(L.w13_hi),
            static_cast<const __nv_bfloat16*>(L.w2_hi));
    return launch_w<float, float>(L, T, s, L.w13_f32, L.w2_f32);
}

}  // namespace moe
