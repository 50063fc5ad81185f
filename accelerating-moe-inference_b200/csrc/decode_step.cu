// Fused batch-1 decode step of the toy MoE decoder: the
// counterpart of one iteration of the reference's generate_decode loop
// (src/model.cu:2061-2104) for a single sequence, in ONE launch.
//
// At one token per step every projection is a weight-streaming GEMV and the
// step is bound by reading the weights once (about 1.6 GB at config 4).  As a
// chain of ordinary kernels the step is about ten launches per layer, and
// each boundary costs a drain, a completion flush and a ramp-up of several
// microseconds -- more than the bytes of most of the phases.  Here one
// cooperative grid of one 512-thread CTA per SM runs the phases back to back,
// separated by a grid-wide barrier (one arrival counter in global memory
// that only grows), and each warp prefetches its slice of the next phase's weights
// into L2 before it arrives at the barrier.
//
// Per layer (x: the residual row, every CTA keeps a copy in shared memory):
//   A  x += ordered MoE combine of the previous layer (the embedding row for
//      layer 0); RMSNorm -> bf16 row; q/k/v GEMV (3d weight rows split over
//      all warps)
//   B  split-K decode attention: one 128-thread group per (head, 64-key
//      chunk), RoPE of q (and of the new key, written with its value into
//      the cache by the chunk that holds the position), the chunk's partial
//      softmax
//   C  every CTA merges the chunks of all heads (the attention output), then
//      the o-projection GEMV rows: xm = x + o . Wo^T
//   D  every CTA: x = xm, RMSNorm (post-attention) -> bf16 row; CTA e < E
//      runs expert e's router chain (the reference's serial fp32 FMA chain)
//   E  every CTA: top-k selection from the E logits; gate/up GEMV of the k
//      routed experts' columns with SwiGLU -> h
//   F  down GEMV in (expert, columns, 2048-wide K chunk) items -> part
// then the final RMSNorm and the output-head GEMV into the logits; greedy
// selection and the step counters stay separate small kernels.
//
// Arithmetic: every phase evaluates the same expressions in the same order
// as the kernel it replaces (rms_pack_row_kernel, dense_gemv_kernel,
// attn_decode_partial/combine_kernel, router_small_kernel with its in-kernel
// RMS statistics, decode_gateup/down_kernel, combine_kernel), so the fused
// step's logits are bit-identical to the unfused chain's.
//
// Every barrier wait is bounded (kWaitBudgetNs of %globaltimer): a CTA whose
// wait runs out sets the error flag and the abort word, and every CTA leaves
// at its next barrier; the host reads MOE_ERR_TIMEOUT and resets the words.
#include <cuda_bf16.h>

#include <cfloat>
#include <climits>
#include <cmath>

#include "decode_step.h"
#include "moe_internal.h"
#include "ptx.cuh"
#include "select.cuh"

namespace moe {
namespace {

constexpr int kWarps = kStepThreads / 32;
constexpr int kGroupThreads = 128;                 // attention group
constexpr int kGroups = kStepThreads / kGroupThreads;
constexpr int kChunk = 64;                         // keys per attention item
constexpr int kNormThreads = 256;                  // rms_pack_row's block
constexpr int kNormVec = 8;                        // float4 per thread: d <= 8192
constexpr int kGemvVecs = 4;                       // 16-byte loads per row per lane per pass
constexpr uint32_t kPrefetchCap = 8192;            // bytes of one L2 prefetch instruction
constexpr int kDownCols = 2;                       // down GEMV columns per item
constexpr int kDevErrTimeoutStep = 1 << 14;        // a fused-step barrier wait ran out
constexpr int kStepBarriersPerLayer = 6;           // grid barriers per layer (phases A-F)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Weights are read once per step: past L1.
__device__ __forceinline__ uint4 stream_load(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void bf16x8(const uint4& r, float (&v)[8]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

__device__ __forceinline__ void group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kGroupThreads) : "memory");
}

// Contiguous share [r0, r1) of n items for warp gw of nw.
__device__ __forceinline__ void warp_range(long long n, long long gw, long long nw, long long& r0,
                                           long long& r1) {
    r0 = n * gw / nw;
    r1 = n * (gw + 1) / nw;
}

// Grid-wide barrier on a 64-bit arrival counter (sync[0..1]) that only
// grows.  A launch makes exactly nb barriers, so every launch starts with the
// counter at a multiple of nb * G; thread 0 of each CTA reads it at the start
// and rounds down (at most G - 1 arrivals at the first barrier can precede
// the read, since that barrier waits for this CTA), which gives the launch's
// base.  Barrier i: after the CTA's work, one release reduction adds 1 (no
// returned value, so the arrival is a single one-way message), then thread 0
// polls with acquire loads until the counter reaches base + (i + 1) * G.
// sync[2] is the abort word: a wait that runs out sets it and the error flag,
// and every CTA leaves at its next barrier; the host then zeroes the words.
// Returns false when the CTA must leave.
struct GridBarrier {
    unsigned long long* count;
    unsigned* abort;
    int* err;
    unsigned long long target;   // thread 0's copy: the next barrier's count
};

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ bool grid_barrier(GridBarrier& b, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        red_release_gpu_add(b.count, 1ull);
        b.target += gridDim.x;
        const unsigned long long t0 = global_timer_ns();
        while (ld_acquire_gpu_u64(b.count) < b.target) {
            if (*reinterpret_cast<volatile unsigned*>(b.abort)) {
                ok = 0;
                break;
            }
            if (global_timer_ns() - t0 > kWaitBudgetNs) {
                atomicOr(b.err, kDevErrTimeoutStep);
                atomicExch(b.abort, 1u);
                ok = 0;
                break;
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Rotate-half RoPE of one head vector, kPer values per lane (lane l holds
// dims l * kPer ..); the partner of dim j < hd/2 is j + hd/2, in lane l ^ 16.
template <int HD>
__device__ __forceinline__ void rope_lane(float (&v)[HD / 32], int lane,
                                          const float2* __restrict__ cs_row) {
    constexpr int kPer = HD / 32;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], 16);
        const int j = (lane & 15) * kPer + i;
        const float2 cs = __ldg(cs_row + j);
        v[i] = lane < 16 ? v[i] * cs.x - other * cs.y : v[i] * cs.x + other * cs.y;
    }
}

// Shared memory of one CTA (dynamic part): the residual row, the normalised
// fp32 row (router chains), the router row of this CTA's expert, the bf16
// GEMV operand row, the staged attention chunk statistics and the attention
// groups' scratch.
struct Smem {
    float* res;              // [d]
    float* xn;               // [d]
    float* wrow;             // [d]
    __nv_bfloat16* a;        // [d]
    float* ml;               // [2][H * nch]
    float* att;              // [kGroups][kChunk + 4 * kGroupThreads]
};

__device__ __forceinline__ Smem carve(float* base, int d, int H, int nch) {
    Smem s;
    s.res = base;
    s.xn = s.res + d;
    s.wrow = s.xn + d;
    s.a = reinterpret_cast<__nv_bfloat16*>(s.wrow + d);
    s.ml = s.wrow + d + d / 2;
    s.att = s.ml + 2 * H * nch;
    return s;
}

}  // namespace

size_t step_fused_smem(int d, int H, int nch) {
    return sizeof(float) * ((size_t)3 * d + d / 2 + (size_t)2 * H * nch +
                            (size_t)kGroups * (kChunk + 4 * kGroupThreads));
}

namespace {

// RMSNorm of the residual row into the bf16 GEMV operand, with
// rms_pack_row_kernel's arithmetic: threads t < 256 sum the squares of
// float4 t, t + 256, ... in order, warp trees, then the 8 warp sums in warp
// order; out = bf16((x * inv) * w).
__device__ __noinline__ void norm_to_a(const Smem& s, const float* __restrict__ w, int d, float eps,
                          float* s_part) {
    __builtin_assume(__isShared(s.res) && __isShared(s.a) && __isShared(s_part));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nv = d / 4;
    const float4* x4 = reinterpret_cast<const float4*>(s.res);
    float ss = 0.0f;
    if (tid < kNormThreads) {
#pragma unroll
        for (int i = 0; i < kNormVec; ++i) {
            const int v = tid + i * kNormThreads;
            if (v < nv) {
                const float4 a = x4[v];
                ss = __fmaf_rn(a.x, a.x, ss);
                ss = __fmaf_rn(a.y, a.y, ss);
                ss = __fmaf_rn(a.z, a.z, ss);
                ss = __fmaf_rn(a.w, a.w, ss);
            }
        }
    }
    ss = warp_sum(ss);
    if (lane == 0 && warp < kNormThreads / 32) s_part[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += s_part[i];
    const float inv = 1.0f / sqrtf(tot / (float)d + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    __nv_bfloat162* a2 = reinterpret_cast<__nv_bfloat162*>(s.a);
    for (int v = tid; v < nv; v += blockDim.x) {
        const float4 a = x4[v], g = __ldg(w4 + v);
        a2[2 * v] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(a.x, inv), g.x),
                                          __fmul_rn(__fmul_rn(a.y, inv), g.y));
        a2[2 * v + 1] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(a.z, inv), g.z),
                                              __fmul_rn(__fmul_rn(a.w, inv), g.w));
    }
    __syncthreads();
}

// y[r] = (base ? base[r] : 0) + W[r] . a for this warp's rows [r0, r1) of W
// [N][K] bf16 (dense_gemv_kernel's per-row arithmetic: lane-strided 8-wide
// groups, fmaf in order, warp tree), two rows per pass, 16 loads in flight.
__device__ __noinline__ void gemv_rows(const __nv_bfloat16* __restrict__ W, int K, long long r0, long long r1,
                          const __nv_bfloat16* s_a, const float* base, float* __restrict__ y) {
    __builtin_assume(__isShared(s_a));
    const int lane = threadIdx.x & 31;
    const uint4* a8 = reinterpret_cast<const uint4*>(s_a);
    for (long long r = r0; r < r1; r += 2) {
        const bool two = r + 1 < r1;
        const __nv_bfloat16* w0 = W + (size_t)r * K;
        const __nv_bfloat16* w1 = two ? w0 + K : w0;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int k0 = lane * 8; k0 < K; k0 += 32 * 8 * kGemvVecs) {
            uint4 raw[kGemvVecs][2];
#pragma unroll
            for (int u = 0; u < kGemvVecs; ++u) {
                const int kk = k0 + u * 256;
                if (kk < K) {
                    raw[u][0] = stream_load(w0 + kk);
                    raw[u][1] = stream_load(w1 + kk);
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvVecs; ++u) {
                const int kk = k0 + u * 256;
                if (kk >= K) break;
                float wv0[8], wv1[8], av[8];
                bf16x8(raw[u][0], wv0);
                bf16x8(raw[u][1], wv1);
                bf16x8(a8[kk / 8], av);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    acc0 = fmaf(wv0[q], av[q], acc0);
                    acc1 = fmaf(wv1[q], av[q], acc1);
                }
            }
        }
        const float v0 = warp_sum(acc0);
        const float v1 = warp_sum(acc1);
        if (lane == 0) {
            y[r] = (base ? base[r] : 0.0f) + v0;
            if (two) y[r + 1] = (base ? base[r + 1] : 0.0f) + v1;
        }
    }
}

// Prefetch rows [r0, r1) of a [N][K] bf16 matrix into L2: the warp's whole
// contiguous slice, in pieces of kPrefetchCap bytes spread over the lanes.
__device__ __forceinline__ void prefetch_rows(const __nv_bfloat16* W, int K, long long r0,
                                              long long r1) {
    if (r1 <= r0) return;
    const int lane = threadIdx.x & 31;
    const size_t bytes = (size_t)(r1 - r0) * K * sizeof(__nv_bfloat16);
    const char* base = reinterpret_cast<const char*>(W + (size_t)r0 * K);
    for (size_t off = (size_t)lane * kPrefetchCap; off < bytes; off += 32 * (size_t)kPrefetchCap) {
        const size_t n = bytes - off < kPrefetchCap ? bytes - off : kPrefetchCap;
        prefetch_l2_bulk(base + off, (uint32_t)n);
    }
}

// One (head, chunk) item of the split-K decode attention on one 128-thread
// group g: attn_decode_partial_kernel's arithmetic, with the group's named
// barrier in place of the block barrier.
template <int HD>
__device__ __noinline__ void attn_item(const StepArgs& a, const StepLayer& L, int h, int c, int pos, int g,
                          float* sp, float* sacc) {
    __builtin_assume(__isShared(sp) && __isShared(sacc));
    constexpr int kPer = HD / 32;
    constexpr int kParts = kGroupThreads / HD;
    constexpr int kGWarps = kGroupThreads / 32;
    constexpr int kKeysPerWarp = kChunk / kGWarps;
    const int tid = threadIdx.x - g * kGroupThreads, warp = tid >> 5, lane = tid & 31;
    const int n = pos + 1;
    const int k0 = c * kChunk;
    const int nk = min(kChunk, n - k0);
    const int d = a.d;
    const float* q = a.qkv + h * HD;
    const float* kb = L.kc + ((size_t)h * a.max_seq + k0) * HD;
    const float* vb = L.vc + ((size_t)h * a.max_seq + k0) * HD;
    const float2* cs_row = a.rope + (size_t)pos * (HD / 2);
    float qv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) qv[i] = __ldcg(q + lane * kPer + i);
    rope_lane<HD>(qv, lane, cs_row);
#pragma unroll
    for (int i = 0; i < kPer; ++i) qv[i] *= a.scale;
    if (pos < k0 + kChunk) {
        // This chunk holds the new position: its key and value enter the cache.
        if (warp == 0) {
            float kv[kPer];
#pragma unroll
            for (int i = 0; i < kPer; ++i) kv[i] = __ldcg(q + d + lane * kPer + i);
            rope_lane<HD>(kv, lane, cs_row);
            float* kd = L.kc + ((size_t)h * a.max_seq + pos) * HD;
#pragma unroll
            for (int i = 0; i < kPer; ++i) kd[lane * kPer + i] = kv[i];
        } else if (warp == 1) {
            float* vd = L.vc + ((size_t)h * a.max_seq + pos) * HD;
#pragma unroll
            for (int i = 0; i < kPer; ++i) vd[lane * kPer + i] = __ldcg(q + 2 * d + lane * kPer + i);
        }
        group_sync(g);
    }
    float dots[kKeysPerWarp];
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i) {
        const int j = warp + kGWarps * i;
        float acc = 0.0f;
        if (j < nk) {
            const float* kr = kb + (size_t)j * HD + lane * kPer;
            float kv[kPer];
            if constexpr (kPer == 4) {
                const float4 f = *reinterpret_cast<const float4*>(kr);
                kv[0] = f.x; kv[1] = f.y; kv[2] = f.z; kv[3] = f.w;
            } else {
#pragma unroll
                for (int e = 0; e < kPer; e += 2) {
                    const float2 f = *reinterpret_cast<const float2*>(kr + e);
                    kv[e] = f.x; kv[e + 1] = f.y;
                }
            }
#pragma unroll
            for (int e = 0; e < kPer; ++e) acc = fmaf(qv[e], kv[e], acc);
        }
        dots[i] = acc;
    }
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i) {
        const float v = warp_sum(dots[i]);
        const int j = warp + kGWarps * i;
        if (lane == 0 && j < nk) sp[j] = v;
    }
    group_sync(g);
    float* out = a.attn_part + ((size_t)h * a.nch + c) * (HD + 2);
    if (warp == 0) {
        const float s0 = lane < nk ? sp[lane] : -INFINITY;
        const float s1 = lane + 32 < nk ? sp[lane + 32] : -INFINITY;
        const float mx = warp_max(fmaxf(s0, s1));
        const float p0 = lane < nk ? expf(s0 - mx) : 0.0f;
        const float p1 = lane + 32 < nk ? expf(s1 - mx) : 0.0f;
        if (lane < nk) sp[lane] = p0;
        if (lane + 32 < nk) sp[lane + 32] = p1;
        const float l = warp_sum(p0 + p1);
        if (lane == 0) {
            out[HD] = mx;
            out[HD + 1] = l;
        }
    }
    group_sync(g);
    // Values.  attn_decode_partial_kernel's thread (class, column) sums keys
    // cls, cls + kParts, ... into four accumulators by key position mod 4,
    // i.e. by key mod kClasses = 4 * kParts.  Here thread (m, c4) owns one
    // such accumulator -- keys j = m (mod kClasses), ascending -- for four
    // adjacent columns, with 16-byte loads all in flight; the accumulators
    // then combine per column exactly as there:
    //   ((A[cls] + A[cls + kParts]) + (A[cls + 2 kParts] + A[cls + 3 kParts]))
    // summed over cls in order.
    constexpr int kClasses = 4 * kParts;
    constexpr int kTpc = kGroupThreads / kClasses;       // threads per class (HD / 4)
    constexpr int kKeysPerThread = kChunk / kClasses;
    const int m = tid / kTpc, c4 = tid % kTpc;
    float4 vv[kKeysPerThread];
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
        const int j = m + i * kClasses;
        vv[i] = j < nk ? *reinterpret_cast<const float4*>(vb + (size_t)j * HD + 4 * c4)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
        const int j = m + i * kClasses;
        if (j < nk) {
            const float p = sp[j];
            acc.x = fmaf(p, vv[i].x, acc.x);
            acc.y = fmaf(p, vv[i].y, acc.y);
            acc.z = fmaf(p, vv[i].z, acc.z);
            acc.w = fmaf(p, vv[i].w, acc.w);
        }
    }
    reinterpret_cast<float4*>(sacc + m * HD)[c4] = acc;
    group_sync(g);
    if (tid < HD) {
        float v = 0.0f;
#pragma unroll
        for (int cls = 0; cls < kParts; ++cls) {
            const float* A = sacc + cls * HD + tid;
            const float sc = (A[0] + A[kParts * HD]) + (A[2 * kParts * HD] + A[3 * kParts * HD]);
            v = cls == 0 ? sc : v + sc;
        }
        out[tid] = v;
    }
    group_sync(g);   // sp / sacc are reused by the group's next item
}

// The attention output (all heads) into the bf16 operand row:
// attn_decode_combine_kernel's per-dimension arithmetic, chunk statistics
// staged in shared memory first.
template <int HD>
__device__ __noinline__ void attn_merge(const StepArgs& a, const Smem& s, int pos) {
    __builtin_assume(__isShared(s.ml) && __isShared(s.a));
    const int used = (pos + kChunk) / kChunk;
    const int H = a.H;
    float* sm = s.ml;               // [H][used] maxima
    float* sl = s.ml + H * a.nch;   // [H][used] sums
    for (int i = threadIdx.x; i < H * used; i += blockDim.x) {
        const int h = i / used, c = i % used;
        const float* base = a.attn_part + ((size_t)h * a.nch + c) * (HD + 2);
        sm[i] = __ldcg(base + HD);
        sl[i] = __ldcg(base + HD + 1);
    }
    __syncthreads();
    for (int dim = threadIdx.x; dim < a.d; dim += blockDim.x) {
        const int h = dim / HD, t = dim % HD;
        const float* base = a.attn_part + (size_t)h * a.nch * (HD + 2);
        float M = -INFINITY;
        for (int c = 0; c < used; ++c) M = fmaxf(M, sm[h * used + c]);
        float Ls = 0.0f, o = 0.0f;
        constexpr int kU = 16;
        for (int c0 = 0; c0 < used; c0 += kU) {
            float pv[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u)
                pv[u] = c0 + u < used ? __ldcg(base + (size_t)(c0 + u) * (HD + 2) + t) : 0.0f;
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int c = c0 + u;
                if (c < used) {
                    const float w = expf(sm[h * used + c] - M);
                    Ls = fmaf(w, sl[h * used + c], Ls);
                    o = fmaf(w, pv[u], o);
                }
            }
        }
        s.a[dim] = __float2bfloat16_rn(o / Ls);
    }
    __syncthreads();
}

__device__ __forceinline__ float4 lds4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

// One chunk of kKC columns, fully unrolled (router_small_kernel's loop).
template <int kKC>
__device__ __forceinline__ float router_chain_chunk(uint32_t xs, uint32_t ws, float acc) {
    float4 xa[4], wa[4], xb[4], wb[4];
    auto load = [&](float4 (&xv)[4], float4 (&wv)[4], int k) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            xv[q] = lds4(xs + 4u * (uint32_t)(k + 4 * q));
            wv[q] = lds4(ws + 4u * (uint32_t)(k + 4 * q));
        }
    };
    auto chain = [&](const float4 (&xv)[4], const float4 (&wv)[4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            acc = __fmaf_rn(xv[q].x, wv[q].x, acc);
            acc = __fmaf_rn(xv[q].y, wv[q].y, acc);
            acc = __fmaf_rn(xv[q].z, wv[q].z, acc);
            acc = __fmaf_rn(xv[q].w, wv[q].w, acc);
        }
    };
    load(xa, wa, 0);
#pragma unroll
    for (int kk = 0; kk < kKC; kk += 32) {
        load(xb, wb, kk + 16);
        chain(xa, wa);
        if (kk + 32 < kKC) load(xa, wa, kk + 32);
        chain(xb, wb);
    }
    return acc;
}

// One router logit: fp32 FMA chain over k ascending from 0 (the reference's
// matmul_transposed order, src/tensor.cu:136-148), on one thread, in chunks
// of 128 columns (d is a multiple of 128).  Explicit shared-memory loads:
// through a generic pointer each would take the longer generic path, and
// on a dependent chain every cycle of load latency not covered shows.
__device__ __noinline__ float router_chain(const float* xn, const float* w, int d) {
    const uint32_t xs = smem_u32(xn), ws = smem_u32(w);
    float acc = 0.0f;
    for (int k0 = 0; k0 < d; k0 += 128)
        acc = router_chain_chunk<128>(xs + 4u * (uint32_t)k0, ws + 4u * (uint32_t)k0, acc);
    return acc;
}

// Phase D: x = xm; the post-attention RMSNorm with router_small_kernel's
// in-kernel statistics (warp 0 sums the squares of float4 lane, lane + 32,
// ... in order, then the xor tree); xn = fma((x - 0) * inv, w, b) in fp32
// and its bf16 copy (the routed row of the expert GEMVs).  CTA e < E then
// runs expert e's logit: one fp32 FMA chain over k ascending, the
// reference's matmul_transposed order (src/tensor.cu:136-148).
__device__ __noinline__ void router_phase(const StepArgs& a, const StepLayer& L, const Smem& s, float* s_inv) {
    __builtin_assume(__isShared(s.res) && __isShared(s.xn) && __isShared(s.a) && __isShared(s.wrow));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int d = a.d, nv = d / 4;
    const int e = blockIdx.x;
    float4* r4 = reinterpret_cast<float4*>(s.res);
    for (int v = tid; v < nv; v += blockDim.x) r4[v] = __ldcg(reinterpret_cast<const float4*>(a.xm) + v);
    __syncthreads();   // s.wrow: loaded in phase C (load_router_row)
    if (warp == 0) {
        float ss = 0.0f;
        for (int v = lane; v < nv; v += 32) {
            const float4 x = r4[v];
            ss = __fmaf_rn(x.x, x.x, ss);
            ss = __fmaf_rn(x.y, x.y, ss);
            ss = __fmaf_rn(x.z, x.z, ss);
            ss = __fmaf_rn(x.w, x.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) *s_inv = 1.0f / sqrtf(ss / (float)d + L.ffn_eps);
    }
    __syncthreads();
    const float inv = *s_inv;
    const float4* w4 = reinterpret_cast<const float4*>(L.ffn_norm);
    const float4* b4 = reinterpret_cast<const float4*>(L.ffn_norm_b);
    __nv_bfloat162* a2 = reinterpret_cast<__nv_bfloat162*>(s.a);
    for (int v = tid; v < nv; v += blockDim.x) {
        const float4 f = layer_norm_out4(r4[v], 0.0f, inv, __ldg(w4 + v), __ldg(b4 + v));
        reinterpret_cast<float4*>(s.xn)[v] = f;
        a2[2 * v] = __floats2bfloat162_rn(f.x, f.y);
        a2[2 * v + 1] = __floats2bfloat162_rn(f.z, f.w);
    }
    __syncthreads();
    if (e < a.E && tid == 0) {
        const float acc = router_chain(s.xn, s.wrow, d);
        float v = acc;
        if (L.bias) v = __fadd_rn(v, L.bias[e]);
        a.logits_e[e] = v;
    }
}

// CTA e < E: expert e's router row into shared memory, ahead of phase D (it
// depends on nothing the step computes).
__device__ __forceinline__ void load_router_row(const StepArgs& a, const StepLayer& L,
                                                const Smem& s) {
    const int e = blockIdx.x;
    if (e >= a.E) return;
    const float4* src = reinterpret_cast<const float4*>(L.wg + (size_t)e * a.d);
    for (int v = threadIdx.x; v < a.d / 4; v += blockDim.x)
        reinterpret_cast<float4*>(s.wrow)[v] = __ldg(src + v);
}

// Phase E's selection: warp 0 selects the k experts from the E logits with
// the router kernels' code; s_act lists them in ascending expert order,
// s_slot[r] is the selection index of s_act[r], s_wsel[s] the weight of
// selection s.
__device__ __noinline__ void select_phase(const StepArgs& a, float* s_lg, int* s_act, int* s_slot,
                             float* s_wsel) {
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        for (int e = lane; e < a.E; e += 32) s_lg[e] = __ldcg(a.logits_e + e);
        __syncwarp();
        int sel[kMaxTopK];
        float wsel[kMaxTopK];
        select_experts(s_lg, a.E, a.k, a.policy, a.quantum, a.tie_eps, lane, sel, wsel);
        if (lane == 0) {
            for (int s = 0; s < a.k; ++s) {
                int r = 0;
                for (int s2 = 0; s2 < a.k; ++s2) r += sel[s2] < sel[s] || (sel[s2] == sel[s] && s2 < s);
                s_act[r] = sel[s];
                s_slot[r] = s;
                s_wsel[s] = wsel[s];
            }
        }
    }
    __syncthreads();
}

// Two dots of one routed row against bf16 weight rows w0, w1 over K
// positions [k_begin, k_end): lane-strided 8-wide groups, fmaf in order
// (decode_gateup_kernel's and decode_down_kernel's per-lane arithmetic).
template <typename AT, int kInFlight>
__device__ __forceinline__ void dot2(const __nv_bfloat16* w0, const __nv_bfloat16* w1,
                                     const AT* act, int k_begin, int k_end, int lane,
                                     float& acc0, float& acc1) {
    for (int k0 = k_begin + lane * 8; k0 < k_end; k0 += 32 * 8 * kInFlight) {
        uint4 raw[kInFlight][2];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int kk = k0 + u * 256;
            if (kk < k_end) {
                raw[u][0] = stream_load(w0 + kk);
                raw[u][1] = stream_load(w1 + kk);
            }
        }
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const int kk = k0 + u * 256;
            if (kk >= k_end) break;
            float wv0[8], wv1[8], av[8];
            bf16x8(raw[u][0], wv0);
            bf16x8(raw[u][1], wv1);
            if constexpr (sizeof(AT) == 4) {
                const float4 f0 = __ldcg(reinterpret_cast<const float4*>(act + kk));
                const float4 f1 = __ldcg(reinterpret_cast<const float4*>(act + kk + 4));
                av[0] = f0.x; av[1] = f0.y; av[2] = f0.z; av[3] = f0.w;
                av[4] = f1.x; av[5] = f1.y; av[6] = f1.z; av[7] = f1.w;
            } else {
                bf16x8(*reinterpret_cast<const uint4*>(act + kk), av);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                acc0 = fmaf(wv0[q], av[q], acc0);
                acc1 = fmaf(wv1[q], av[q], acc1);
            }
        }
    }
}

// Rows gate and up of intermediate column c of expert e in w13.
__device__ __forceinline__ size_t gate_row(int e, int c, int ffp) {
    return (size_t)e * 2 * ffp + (size_t)(c / kFfBlock) * (2 * kFfBlock) + (c % kFfBlock);
}

// Phase E's GEMV: items (rank r, column c) of k * ffp, contiguous per warp.
__device__ __noinline__ void gateup_phase(const StepArgs& a, const StepLayer& L, const Smem& s,
                             const int* s_act, long long gw, long long nw) {
    __builtin_assume(__isShared(s.a));
    const int lane = threadIdx.x & 31, d = a.d, ffp = a.ffp;
    long long j0, j1;
    warp_range((long long)a.k * ffp, gw, nw, j0, j1);
    // The experts are known only now: the warp's whole slice (a gate and an
    // up row per column) into L2 at once, so the loads below find their
    // lines in flight or landed instead of each paying the DRAM latency.
    for (long long j = j0 + lane / 2; j < j1; j += 16) {
        const size_t g = gate_row(s_act[(int)(j / ffp)], (int)(j % ffp), ffp) + (lane & 1) * kFfBlock;
        prefetch_l2_bulk(L.w13 + g * d, (uint32_t)(d * sizeof(__nv_bfloat16)));
    }
    for (long long j = j0; j < j1; ++j) {
        const int r = (int)(j / ffp), c = (int)(j % ffp);
        const size_t g = gate_row(s_act[r], c, ffp);
        float acc0 = 0.0f, acc1 = 0.0f;
        dot2<__nv_bfloat16, 4>(L.w13 + g * d, L.w13 + (g + kFfBlock) * d, s.a, 0, d, lane, acc0, acc1);
        const float gv = warp_sum(acc0), uv = warp_sum(acc1);
        if (lane == 0) a.h[(size_t)r * ffp + c] = gv / (1.0f + __expf(-gv)) * uv;
    }
}

// Down items of one warp: (rank r, kDownCols output columns, K chunk).
__device__ __forceinline__ void down_item(long long it, int nq, int nk, int& r, int& n0,
                                          int& ch) {
    r = (int)(it / ((long long)nq * nk));
    const int rem = (int)(it % ((long long)nq * nk));
    n0 = (rem / nk) * kDownCols;
    ch = rem % nk;
}

// Phase F: part[chunk][slot][n] = the chunk's partial dot of column n.
__device__ __noinline__ void down_phase(const StepArgs& a, const StepLayer& L, const int* s_act,
                           const int* s_slot, long long gw, long long nw) {
    static_assert(kDownCols == 2, "dot2 computes two columns");
    const int lane = threadIdx.x & 31, d = a.d, ffp = a.ffp;
    const int nq = (d + kDownCols - 1) / kDownCols;
    const int nk = (ffp + kDownChunk - 1) / kDownChunk;
    long long i0, i1;
    warp_range((long long)a.k * nq * nk, gw, nw, i0, i1);
    for (long long it = i0; it < i1; ++it) {
        int r, n0, ch;
        down_item(it, nq, nk, r, n0, ch);
        const int e = s_act[r];
        const int k0 = ch * kDownChunk, k1 = min(ffp, k0 + kDownChunk);
        const __nv_bfloat16* w0 = L.w2 + ((size_t)e * d + min(n0, d - 1)) * ffp;
        const __nv_bfloat16* w1 = L.w2 + ((size_t)e * d + min(n0 + 1, d - 1)) * ffp;
        float acc0 = 0.0f, acc1 = 0.0f;
        dot2<float, 4>(w0, w1, a.h + (size_t)r * ffp, k0, k1, lane, acc0, acc1);
        const float v0 = warp_sum(acc0), v1 = warp_sum(acc1);
        float* dst = a.part + (size_t)ch * a.k * d + (size_t)s_slot[r] * d + n0;
        if (lane == 0) dst[0] = v0;
        if (lane == 1 && n0 + 1 < d) dst[1] = v1;
    }
}

// This warp's down items' weight rows into L2 (lane j: row j % 2 of item
// i0 + j / 2, then the next 16 items).
__device__ __noinline__ void prefetch_down(const StepArgs& a, const StepLayer& L, const int* s_act,
                                           long long gw, long long nw) {
    const int lane = threadIdx.x & 31, d = a.d, ffp = a.ffp;
    const int nq = (d + kDownCols - 1) / kDownCols;
    const int nk = (ffp + kDownChunk - 1) / kDownChunk;
    long long i0, i1;
    warp_range((long long)a.k * nq * nk, gw, nw, i0, i1);
    for (long long it = i0 + lane / 2; it < i1; it += 16) {
        int r, n0, ch;
        down_item(it, nq, nk, r, n0, ch);
        const int k0 = ch * kDownChunk, k1 = min(ffp, k0 + kDownChunk);
        const int n = min(n0 + (lane & 1), d - 1);
        prefetch_l2_bulk(L.w2 + ((size_t)s_act[r] * d + n) * ffp + k0,
                         (uint32_t)((k1 - k0) * sizeof(__nv_bfloat16)));
    }
}

// x += the ordered combine of the last MoE block (combine_kernel's
// arithmetic): per column, each selection's K chunks added in chunk order,
// then fma(w, v, acc) over the selections in ascending expert order.  The
// k * nk partials of a column are loaded kB at a time, all in flight.
__device__ __noinline__ void combine_into_res(const StepArgs& a, const Smem& s, const int* s_slot,
                                              const float* s_wsel) {
    __builtin_assume(__isShared(s.res));
    constexpr int kB = 8;
    const int d = a.d, nv = d / 4;
    const int nk = (a.ffp + kDownChunk - 1) / kDownChunk;
    const int total = a.k * nk;
    const float4* p4 = reinterpret_cast<const float4*>(a.part);
    const size_t sstride = (size_t)a.k * nv;
    float4* r4 = reinterpret_cast<float4*>(s.res);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f), val = acc;
        for (int b0 = 0; b0 < total; b0 += kB) {
            float4 q[kB];
#pragma unroll
            for (int j = 0; j < kB; ++j) {
                const int i = b0 + j;
                if (i < total)
                    q[j] = __ldcg(p4 + (i % nk) * sstride + (size_t)s_slot[i / nk] * nv + v);
            }
#pragma unroll
            for (int j = 0; j < kB; ++j) {
                const int i = b0 + j;
                if (i >= total) break;
                const int r = i / nk, sp = i % nk;
                if (sp == 0) {
                    val = q[j];
                } else {
                    val.x = __fadd_rn(val.x, q[j].x);
                    val.y = __fadd_rn(val.y, q[j].y);
                    val.z = __fadd_rn(val.z, q[j].z);
                    val.w = __fadd_rn(val.w, q[j].w);
                }
                if (sp == nk - 1) {
                    const float w = s_wsel[s_slot[r]];
                    acc.x = __fmaf_rn(w, val.x, acc.x);
                    acc.y = __fmaf_rn(w, val.y, acc.y);
                    acc.z = __fmaf_rn(w, val.z, acc.z);
                    acc.w = __fmaf_rn(w, val.w, acc.w);
                }
            }
        }
        const float4 x = r4[v];
        r4[v] = make_float4(__fadd_rn(acc.x, x.x), __fadd_rn(acc.y, x.y), __fadd_rn(acc.z, x.z),
                            __fadd_rn(acc.w, x.w));
    }
    __syncthreads();
}

template <int HD>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepArgs a) {
    extern __shared__ __align__(16) float smem_raw[];
    __shared__ float s_part[kWarps];
    __shared__ float s_inv;
    __shared__ int s_ok;
    __shared__ float s_lg[kMaxExperts];
    __shared__ int s_act[kMaxTopK], s_slot[kMaxTopK];
    __shared__ float s_wsel[kMaxTopK];
    const Smem s = carve(smem_raw, a.d, a.H, a.nch);
    const int tid = threadIdx.x, warp = tid >> 5;
    GridBarrier bar{reinterpret_cast<unsigned long long*>(a.sync), a.sync + 2, a.err, 0ull};
    if (tid == 0) {
        // The launch's base count (see GridBarrier); an abort left by an
        // earlier launch (not yet cleared by the host) ends this one at once.
        const unsigned long long per = (unsigned long long)kStepBarriersPerLayer * a.nl * gridDim.x;
        const unsigned long long c = ld_acquire_gpu_u64(bar.count);
        bar.target = c - c % per;
        s_ok = *reinterpret_cast<volatile unsigned*>(bar.abort) == 0u;
    }
    __syncthreads();
    if (!s_ok) return;
    const int G = gridDim.x;
    const long long nw = (long long)G * kWarps;
    const long long gw = (long long)blockIdx.x * kWarps + warp;
    const int d = a.d, nv = d / 4;
    const int pos = *a.pos_dev;
    const int used = (pos + kChunk) / kChunk;
    const int items = a.H * used;
    long long r0, r1;
    warp_range(3LL * d, gw, nw, r0, r1);
    prefetch_rows(a.layers[0].wqkv, d, r0, r1);
    {
        // x = embed[tok] (a zero row and the token error for an id outside
        // [0, vocab), as embed_gather_kernel does).
        const int t = *a.tok;
        const bool ok = t >= 0 && t < a.V;
        if (!ok && blockIdx.x == 0 && tid == 0) atomicOr(a.err, kDecErrToken);
        const float4* src = reinterpret_cast<const float4*>(a.embed + (size_t)(ok ? t : 0) * d);
        for (int v = tid; v < nv; v += blockDim.x)
            reinterpret_cast<float4*>(s.res)[v] = ok ? __ldg(src + v) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        __syncthreads();
    }
    for (int l = 0; l < a.nl; ++l) {
        const StepLayer& L = a.layers[l];
        // ---- A: residual, input norm, q/k/v
        if (l > 0) combine_into_res(a, s, s_slot, s_wsel);
        norm_to_a(s, L.attn_norm, d, a.eps, s_part);
        warp_range(3LL * d, gw, nw, r0, r1);
        gemv_rows(L.wqkv, d, r0, r1, s.a, nullptr, a.qkv);
        // This CTA's attention items' cached keys and values, and this
        // warp's o-projection rows, into L2.
        for (int i = blockIdx.x + G * (tid >> 1); i < items; i += G * (kStepThreads >> 1)) {
            const int kk0 = (i % used) * kChunk;
            if (kk0 < pos) {
                const int rows = min(kChunk, pos - kk0);
                const float* src = ((tid & 1) ? L.vc : L.kc) + ((size_t)(i / used) * a.max_seq + kk0) * HD;
                prefetch_l2_bulk(src, (uint32_t)(rows * HD * sizeof(float)));
            }
        }
        warp_range(d, gw, nw, r0, r1);
        prefetch_rows(L.wo, d, r0, r1);
        if (!grid_barrier(bar, &s_ok)) return;
        // ---- B: attention partials
        {
            const int g = tid / kGroupThreads;
            float* sp = s.att + g * (kChunk + 4 * kGroupThreads);
            for (int i = blockIdx.x + G * g; i < items; i += G * kGroups)
                attn_item<HD>(a, L, i / used, i % used, pos, g, sp, sp + kChunk);
        }
        if (!grid_barrier(bar, &s_ok)) return;
        // ---- C: merge, o projection
        attn_merge<HD>(a, s, pos);
        warp_range(d, gw, nw, r0, r1);
        gemv_rows(L.wo, d, r0, r1, s.a, s.res, a.xm);
        load_router_row(a, L, s);
        if (!grid_barrier(bar, &s_ok)) return;
        // ---- D: post-attention norm, router chains
        router_phase(a, L, s, &s_inv);
        if (!grid_barrier(bar, &s_ok)) return;
        // ---- E: selection, gate/up
        select_phase(a, s_lg, s_act, s_slot, s_wsel);
        gateup_phase(a, L, s, s_act, gw, nw);
        prefetch_down(a, L, s_act, gw, nw);
        if (!grid_barrier(bar, &s_ok)) return;
        // ---- F: down
        down_phase(a, L, s_act, s_slot, gw, nw);
        if (l + 1 < a.nl) {
            warp_range(3LL * d, gw, nw, r0, r1);
            prefetch_rows(a.layers[l + 1].wqkv, d, r0, r1);
        } else {
            warp_range(a.V, gw, nw, r0, r1);
            prefetch_rows(a.head, d, r0, r1);
        }
        if (!grid_barrier(bar, &s_ok)) return;
    }
    // ---- the last block's residual, final norm, output head
    combine_into_res(a, s, s_slot, s_wsel);
    norm_to_a(s, a.final_norm, d, a.eps, s_part);
    warp_range(a.V, gw, nw, r0, r1);
    gemv_rows(a.head, d, r0, r1, s.a, nullptr, a.logits);
}

template <int HD>
cudaError_t launch_hd(const StepArgs& a, int grid, size_t smem, cudaStream_t s) {
    auto kern = decode_step_kernel<HD>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

int step_fused_occupancy(int head_dim, size_t smem) {
    int n = 0;
    cudaError_t e;
    if (head_dim == 128) {
        e = cudaFuncSetAttribute(decode_step_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_step_kernel<128>, kStepThreads, smem);
    } else {
        e = cudaFuncSetAttribute(decode_step_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_step_kernel<64>, kStepThreads, smem);
    }
    return e == cudaSuccess ? n : 0;
}

cudaError_t launch_step_fused(const StepArgs& a, int head_dim, int grid, size_t smem,
                              cudaStream_t s) {
    if (head_dim == 128) return launch_hd<128>(a, grid, smem, s);
    if (head_dim == 64) return launch_hd<64>(a, grid, smem, s);
    return cudaErrorInvalidValue;
}

}  // namespace moe
