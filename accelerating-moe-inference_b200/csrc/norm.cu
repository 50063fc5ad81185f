// The decoder layer's post-attention LayerNorm and residual around the MoE
// (PhiDecoderLayer::forward, src/layer.cu:157-161):
//
//   post = layer_norm(attn);  ff = moe(post);  y = ff + attn
//
// tensor_ops::layer_norm (src/tensor.cu:174-189), as GCC builds it, computes
// per row
//   mean = ((x0 + x1) + x2 ...) / d              j-ascending rounded adds
//   var  = (((x0-mean)^2 + ...) / d              rounded squares, rounded adds
//   inv  = 1 / sqrt(var + eps)
//   y_j  = fma((x_j - mean) * inv, w_j, b_j)     only this expression is
//                                                contracted to an FMA
// The two sums are sequential by definition, so a bit-exact result keeps one
// chain per row: row_stats_kernel gives each lane one row and streams the
// rows through shared memory with TMA so that the chains, not the loads, set
// the pace.  The output expression needs only the two per-row scalars, so it
// is applied where the normalised values are consumed -- by the router on the
// x chunks it stages and by the dispatch permute on the rows it converts --
// and the normalised activations are never written to HBM.  The standalone
// form (moe_layer_norm_device) lets the same kernel finish each row itself.
#include "moe_internal.h"
#include "ptx.cuh"

#include <string>

namespace moe {
namespace {

constexpr int kStatRows = 32;                         // rows per CTA: one lane each
constexpr int kBoxCols = 32;                          // one 128-byte swizzled box row
constexpr int kBoxBytes = kStatRows * kBoxCols * 4;   // 4 KB

// Ring geometry for KB boxes (32 * KB columns) per stage: 8 boxes (32 KB) x 6
// stages when d % 256 == 0, else 4 boxes (16 KB) x 8 stages; either way about
// 160 / 112 KB of loads in flight.
template <int KB>
struct StatRing {
    static constexpr int kStages = KB == 8 ? 6 : 8;
    static constexpr int kStageBytes = KB * kBoxBytes;
    static constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024;   // + alignment slack
};

// float4 j (columns 4j .. 4j+3) of row r inside a [32][32] fp32 box stored
// with the 128-byte swizzle: the 16-byte chunks of row r are permuted by
// r % 8, so 8 lanes reading the same chunk index of 8 consecutive rows hit
// 8 different bank groups.
__device__ __forceinline__ float4 box_ld(const unsigned char* box, int r, int j) {
    return *reinterpret_cast<const float4*>(box + r * 128 + ((j ^ (r & 7)) << 4));
}

__device__ __forceinline__ float comp(const float4 (&v)[8], int i) {
    const float4 q = v[i >> 2];
    return (i & 3) == 0 ? q.x : (i & 3) == 1 ? q.y : (i & 3) == 2 ? q.z : q.w;
}

// Pass 0 over one stage: acc += x, column by column, the next box's loads
// issued before the current box's adds (measured on B200: 4.2 cycles per
// element, the latency of the dependent add).
template <int KB>
__device__ __forceinline__ void stage_sum(const unsigned char* sbase, int lane, float& acc) {
    float4 v[8], vn[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = box_ld(sbase, lane, j);
#pragma unroll
    for (int bx = 0; bx < KB; ++bx) {
        if (bx + 1 < KB) {
#pragma unroll
            for (int j = 0; j < 8; ++j) vn[j] = box_ld(sbase + (bx + 1) * kBoxBytes, lane, j);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc = __fadd_rn(acc, comp(v, i));
        if (bx + 1 < KB) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = vn[j];
        }
    }
}

// Pass 1 over one stage: acc += (x - mean)^2 (rounded square, rounded add).
// The deviations and squares are formed two columns per instruction (packed
// f32x2: x + (-mean) is exactly x - mean) a box ahead of the chain, and are
// interleaved with its adds so that they fill the adds' latency (measured:
// 5.7 cycles per element).
template <int KB>
__device__ __forceinline__ void stage_sumsq(const unsigned char* sbase, int lane, float mean,
                                            float& acc) {
    const float2 nm = make_float2(-mean, -mean);
    float4 v[8];
    float2 q[16], qn[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = box_ld(sbase, lane, j);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float2 a = __fadd2_rn(make_float2(v[j].x, v[j].y), nm);
        const float2 c = __fadd2_rn(make_float2(v[j].z, v[j].w), nm);
        q[2 * j] = __fmul2_rn(a, a);
        q[2 * j + 1] = __fmul2_rn(c, c);
    }
#pragma unroll
    for (int bx = 0; bx < KB; ++bx) {
        if (bx + 1 < KB) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = box_ld(sbase + (bx + 1) * kBoxBytes, lane, j);
        }
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            acc = __fadd_rn(acc, q[p].x);
            acc = __fadd_rn(acc, q[p].y);
            if (bx + 1 < KB && (p & 1) == 0) {
                const int j = p >> 1;
                const float2 a = __fadd2_rn(make_float2(v[j].x, v[j].y), nm);
                const float2 c = __fadd2_rn(make_float2(v[j].z, v[j].w), nm);
                qn[p] = __fmul2_rn(a, a);
                qn[p + 1] = __fmul2_rn(c, c);
            }
        }
        if (bx + 1 < KB) {
#pragma unroll
            for (int p = 0; p < 16; ++p) q[p] = qn[p];
        }
    }
}

// Up to 32 rows per CTA, a lane of warp 0 per row.  The rows stream through a
// ring of [32 rows][32 * KB cols] stages, each filled by KB 2-D TMA loads of
// [box_rows][32] boxes completing on the stage's `full` mbarrier (box_rows =
// min(T, 32); rows past T arrive zero-filled, rows past box_rows are never
// written and their lanes' results are discarded).  The stages in order are
// pass 0 (sum), pass 1 (sum of squared deviations) and, for kApply, pass 2
// (normalise into y, the warp on one row at a time so the stores are
// coalesced); the next pass's loads are in flight while a pass finishes.
//
// Warp 1 (one lane) issues the loads, refilling a stage once warp 0 has
// released it on `empty`, so warp 0's instruction stream is the chains alone.
// Waits are bounded: on a timeout warp 0 flags err and `abort`, writes NaN
// for its rows, and warp 1 stops issuing and lets its loads land before the
// CTA's shared memory is released.  d % (32 * KB) == 0.
template <bool kApply, int KB>
__global__ void __launch_bounds__(64, 1)
row_stats_kernel(const __grid_constant__ CUtensorMap tm, int box_rows, int T, int d, float eps,
                 float* __restrict__ mean_out, float* __restrict__ inv_out,
                 const float* __restrict__ w, const float* __restrict__ b, float* __restrict__ y,
                 int* err) {
    using R = StatRing<KB>;
    constexpr int S = R::kStages;
    constexpr int kCols = 32 * KB;
    extern __shared__ unsigned char stat_smem[];
    __shared__ uint64_t full[S], empty[S];
    __shared__ volatile int abort_flag;
    unsigned char* ring = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(stat_smem) + 1023) & ~static_cast<uintptr_t>(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * kStatRows;
    const int nrows = min(kStatRows, T - r0);
    const int nchunks = d / kCols;
    const int total = (kApply ? 3 : 2) * nchunks;
    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm);
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 1) {
        if (lane != 0) return;
        const uint32_t bytes = (uint32_t)(KB * box_rows * kBoxCols * 4);
        int g = 0;
        for (int c = 0; g < total; ++g) {
            const int st = g % S;
            if (g >= S && !mbar_wait(&empty[st], ((g / S) - 1) & 1, err, kDevErrTimeoutNorm)) break;
            if (abort_flag) break;
            mbar_arrive_expect_tx(&full[st], bytes);
#pragma unroll
            for (int bx = 0; bx < KB; ++bx)
                tma_load_2d(ring + st * R::kStageBytes + bx * kBoxBytes, &tm, &full[st],
                            c * kCols + bx * kBoxCols, r0);
            if (++c == nchunks) c = 0;
        }
        // Every load issued has landed before the CTA exits (at once in the
        // normal case: warp 0 consumed them all).
        for (int h = g - 1; h >= 0 && h >= g - S; --h)
            mbar_wait(&full[h % S], (h / S) & 1, nullptr, 0);
        return;
    }

    float acc = 0.0f, mean = 0.0f, inv = 0.0f;
    bool ok = true;
    int st = 0;
    uint32_t phase = 0;
    for (int pass = 0; pass < (kApply ? 3 : 2) && ok; ++pass) {
        for (int c = 0; c < nchunks; ++c) {
            if (!mbar_wait(&full[st], phase, err, kDevErrTimeoutNorm)) {
                ok = false;
                abort_flag = 1;
                break;
            }
            const unsigned char* sbase = ring + st * R::kStageBytes;
            if (pass == 0) {
                stage_sum<KB>(sbase, lane, acc);
            } else if (pass == 1) {
                stage_sumsq<KB>(sbase, lane, mean, acc);
            } else {
                // Lane l holds columns 4l .. 4l+3 of each 128-column half:
                // box (l / 8) + 4h, chunk l % 8.
#pragma unroll
                for (int h = 0; h < KB / 4; ++h) {
                    const int col4 = c * (kCols / 4) + h * 32 + lane;
                    const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + col4);
                    const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + col4);
                    const unsigned char* box = sbase + ((lane >> 3) + 4 * h) * kBoxBytes;
                    for (int rr = 0; rr < nrows; ++rr) {   // nrows is warp-uniform
                        const float m = __shfl_sync(0xffffffffu, mean, rr);
                        const float iv = __shfl_sync(0xffffffffu, inv, rr);
                        reinterpret_cast<float4*>(y + (size_t)(r0 + rr) * d)[col4] =
                            layer_norm_out4(box_ld(box, rr, lane & 7), m, iv, wv, bv);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            if (++st == S) {
                st = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        if (pass == 0) {
            mean = __fdiv_rn(acc, (float)d);
            acc = 0.0f;
        } else if (pass == 1) {
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)d), eps)));
        }
    }
    if (!ok) mean = inv = __int_as_float(0x7fc00000);
    if constexpr (!kApply) {
        if (lane < nrows) {
            mean_out[r0 + lane] = mean;
            inv_out[r0 + lane] = inv;
        }
    } else if (!ok) {
        for (int rr = 0; rr < nrows; ++rr)
            for (int j = lane; j < d; j += 32) y[(size_t)(r0 + rr) * d + j] = mean;
    }
}

__global__ void residual_add_kernel(float4* __restrict__ y, const float4* __restrict__ r, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        float4 a = y[i];
        const float4 b = r[i];
        a.x = __fadd_rn(a.x, b.x);
        a.y = __fadd_rn(a.y, b.y);
        a.z = __fadd_rn(a.z, b.z);
        a.w = __fadd_rn(a.w, b.w);
        y[i] = a;
    }
}

int stream_grid(const Layer* L, size_t n4) {
    const int sms = L ? L->sm_count : 148;
    return (int)std::min<size_t>((n4 + 255) / 256, (size_t)sms * 8);
}

template <bool kApply, int KB>
cudaError_t launch_stats_t(const float* x, int T, int d, float eps, float* mean, float* inv,
                           const float* w, const float* b, float* y, int* err, cudaStream_t s) {
    // Boxes are as high as the batch (up to 32 rows): the TMA unit's time goes
    // by the box rows it fills, out-of-range ones included.
    const int box_rows = T < kStatRows ? T : kStatRows;
    CUtensorMap tm;
    std::string msg;
    if (!make_tmap_2d(&tm, x, /*bf16=*/false, d, T, kBoxCols, box_rows, &msg))
        return cudaErrorInvalidValue;
    auto kern = row_stats_kernel<kApply, KB>;
    const size_t smem = StatRing<KB>::kSmem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    kern<<<(T + kStatRows - 1) / kStatRows, 64, smem, s>>>(tm, box_rows, T, d, eps, mean, inv, w, b,
                                                           y, err);
    return cudaGetLastError();
}

template <bool kApply>
cudaError_t launch_stats(const float* x, int T, int d, float eps, float* mean, float* inv,
                         const float* w, const float* b, float* y, int* err, cudaStream_t s) {
    if (d % 256 == 0) return launch_stats_t<kApply, 8>(x, T, d, eps, mean, inv, w, b, y, err, s);
    return launch_stats_t<kApply, 4>(x, T, d, eps, mean, inv, w, b, y, err, s);
}

}  // namespace

bool norm_supported(int d) { return d > 0 && d % 128 == 0; }

cudaError_t launch_row_stats(const float* x, int T, int d, float eps, float* mean, float* inv,
                             int* err, cudaStream_t s) {
    if (!norm_supported(d)) return cudaErrorInvalidValue;
    return launch_stats<false>(x, T, d, eps, mean, inv, nullptr, nullptr, nullptr, err, s);
}

cudaError_t launch_layer_norm(const float* x, int T, int d, float eps, const float* w,
                              const float* b, float* y, cudaStream_t s) {
    if (!norm_supported(d)) return cudaErrorInvalidValue;
    return launch_stats<true>(x, T, d, eps, nullptr, nullptr, w, b, y, nullptr, s);
}

namespace {
// One warp per row: fp32 sum of squares (each lane walks its float4 columns,
// then a butterfly), mean 0, inv = 1 / sqrt(ss / d + eps).
__global__ void __launch_bounds__(256)
rms_stats_kernel(const float* __restrict__ x, int T, int d, float eps, float* __restrict__ mean,
                 float* __restrict__ inv) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= T) return;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * d);
    float ss = 0.0f;
    for (int v = lane; v < d / 4; v += 32) {
        const float4 a = __ldg(xr + v);
        ss = __fmaf_rn(a.x, a.x, ss);
        ss = __fmaf_rn(a.y, a.y, ss);
        ss = __fmaf_rn(a.z, a.z, ss);
        ss = __fmaf_rn(a.w, a.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) {
        mean[row] = 0.0f;
        inv[row] = 1.0f / sqrtf(ss / (float)d + eps);
    }
}
}  // namespace

cudaError_t launch_rms_stats(const float* x, int T, int d, float eps, float* mean, float* inv,
                             cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    rms_stats_kernel<<<(T + 7) / 8, 256, 0, s>>>(x, T, d, eps, mean, inv);
    return cudaGetLastError();
}

cudaError_t launch_residual_add(const Layer& L, float* y, const float* r, size_t n,
                                cudaStream_t s) {
    const size_t n4 = n / 4;
    residual_add_kernel<<<stream_grid(&L, n4), 256, 0, s>>>(reinterpret_cast<float4*>(y),
                                                           reinterpret_cast<const float4*>(r), n4);
    return cudaGetLastError();
}

}  // namespace moe
