// Weight ingestion: one expert's fp32 nn.Linear weights (already on the
// device) into the layouts the kernels read.  Runs once per layer at
// creation, outside any timed region -- the counterpart of DeviceMoE's
// upload and w1/w3 interleave (src/model.cu:1340-1365, 1491-1513).
//
//   w13 row r of expert e (r < 2*ffp): block b = r / 256, i = r % 256;
//       i <  128: w1 row 128b + i        (gate)
//       i >= 128: w3 row 128b + i - 128  (up)
//       rows past d_ff are zero.
//   w2  [d][ffp]: w2 columns past d_ff are zero.
// BF16 precision writes bf16 (RNE).  FP32 precision writes the tf32 hi
// plane, the lo plane (tf32 of the remainder) and the plain fp32 copy read
// by the decode kernels; FP32_BF16X3 the bf16 hi plane, the bf16 lo plane
// (bf16 of the remainder) and the fp32 copy.
#include <cuda_bf16.h>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

// One weight in the layout of GEMM scheme gp (GemmPrec) at element i.
__device__ __forceinline__ void store_weight(int gp, size_t i, float v, void* hi, void* lo,
                                             float* f32) {
    if (gp == kGemmBf16) {
        static_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v);
        return;
    }
    if (gp == kGemm3xTf32) {
        const float h = to_tf32(v);
        static_cast<float*>(hi)[i] = h;
        static_cast<float*>(lo)[i] = to_tf32(v - h);
    } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        static_cast<__nv_bfloat16*>(hi)[i] = h;
        static_cast<__nv_bfloat16*>(lo)[i] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
    }
    if (f32) f32[i] = v;   // a dense projection keeps no decode copy
}

__global__ void gateup_kernel(const float* __restrict__ w1, const float* __restrict__ w3, int ff,
                              int ffp, int d, int gp, void* __restrict__ hi,
                              void* __restrict__ lo, float* __restrict__ f32) {
    const size_t n = (size_t)2 * ffp * d;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / d);
        const int c = (int)(i % d);
        const int b = r / (2 * kFfBlock), w = r % (2 * kFfBlock);
        const int src_row = b * kFfBlock + (w < kFfBlock ? w : w - kFfBlock);
        const float* src = w < kFfBlock ? w1 : w3;
        const float v = src_row < ff ? src[(size_t)src_row * d + c] : 0.0f;
        store_weight(gp, i, v, hi, lo, f32);
    }
}

__global__ void down_kernel(const float* __restrict__ w2, int ff, int ffp, int d, int gp,
                            void* __restrict__ hi, void* __restrict__ lo,
                            float* __restrict__ f32) {
    const size_t n = (size_t)d * ffp;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / ffp);
        const int c = (int)(i % ffp);
        const float v = c < ff ? w2[(size_t)r * ff + c] : 0.0f;
        store_weight(gp, i, v, hi, lo, f32);
    }
}

// One thread waits, with the production bounded-wait routine, on an mbarrier
// that nothing arrives on; the wait runs out and records the timeout flag.
__global__ void selftest_wait_kernel(int* err, unsigned long long budget_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, err, kDevErrTimeoutSelftest, budget_ns);
    }
}

}  // namespace

cudaError_t launch_selftest_wait(int* err, unsigned long long budget_ns) {
    selftest_wait_kernel<<<1, 32>>>(err, budget_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return cudaDeviceSynchronize();
}

cudaError_t convert_gateup(const Layer& L, int e, const float* w1_dev, const float* w3_dev,
                           cudaStream_t s) {
    const size_t per = (size_t)2 * L.ffp * L.d;
    const size_t eb = plane_bytes(L);
    void* hi = static_cast<char*>(L.w13_hi) + per * e * eb;
    void* lo = L.w13_lo ? static_cast<char*>(L.w13_lo) + per * e * eb : nullptr;
    float* f32 = L.w13_f32 ? L.w13_f32 + per * e : nullptr;
    gateup_kernel<<<4 * L.sm_count, 256, 0, s>>>(w1_dev, w3_dev, L.ff, L.ffp, L.d, gemm_prec(L),
                                                 hi, lo, f32);
    return cudaGetLastError();
}

cudaError_t convert_down(const Layer& L, int e, const float* w2_dev, cudaStream_t s) {
    const size_t per = (size_t)L.d * L.ffp;
    const size_t eb = plane_bytes(L);
    void* hi = static_cast<char*>(L.w2_hi) + per * e * eb;
    void* lo = L.w2_lo ? static_cast<char*>(L.w2_lo) + per * e * eb : nullptr;
    float* f32 = L.w2_f32 ? L.w2_f32 + per * e : nullptr;
    down_kernel<<<4 * L.sm_count, 256, 0, s>>>(w2_dev, L.ff, L.ffp, L.d, gemm_prec(L), hi, lo,
                                               f32);
    return cudaGetLastError();
}

}  // namespace moe
