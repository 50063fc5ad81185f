// moe_dispatch_noalloc: token dispatch for callers that cannot allocate
// device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a
// CUDA stream capture that must not touch the allocator, under a serving
// framework that owns every byte of device memory through its own pool, or
// in a real-time path where an allocation's implicit synchronisation and
// unbounded latency are not acceptable.  Such callers already hold their
// inputs and outputs; what they cannot provide is the per-block histogram the
// dispatch needs between its passes.
//
// This file therefore keeps that scratch in a fixed, file-scope device array
// (kScratchBytes, 1 MiB on every GPU that loads the library, held until the
// process exits) and never allocates.  The passes are the same counting sort
// as the forward path's dispatch (histogram per 32-token block, exclusive
// scan per expert over the blocks, padded expert offsets, stable placement in
// ascending token order), written as separate kernels here so the forward
// path is untouched.
//
// Contract:
//   - the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture begins;
//   - every call on a device shares the one array, so calls whose GPU work
//     overlaps (different streams, or concurrent host threads) race -- order
//     them on one stream or synchronise between them;
//   - the array keeps the previous call's contents; each pass writes every
//     scratch word it later reads, so nothing needs clearing between calls.
#include <mutex>

#include "moe_internal.h"

namespace moe {
namespace {

constexpr size_t kScratchBytes = size_t(1) << 20;
constexpr int kScratchInts = int(kScratchBytes / sizeof(int));
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int g_dispatch_scratch[kScratchInts];

std::mutex g_scratch_mu;
int* g_scratch_ptr[kMaxDevices] = {};

// Per 32-token block: how many (token, slot) entries go to each expert.
// Entries whose expert index is out of range are not counted (and not placed).
__global__ void __launch_bounds__(256)
noalloc_count_kernel(const int* __restrict__ idx, int T, int E, int k, int* __restrict__ hist) {
    __shared__ int h[kMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
    __syncthreads();
    const int t0 = blockIdx.x * kRouteTokens;
    const int n = min(kRouteTokens, T - t0) * k;
    if ((int)threadIdx.x < n) {
        const int e = idx[(size_t)t0 * k + threadIdx.x];
        if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(size_t)blockIdx.x * E + e] = h[e];
}

constexpr int kScanThreads = 1024;

// One CTA per expert: exclusive scan of the expert's per-block counts over
// the blocks, in place, 1024 blocks per round (warp shuffles, then the warp
// totals); the expert's total goes to counts.
__global__ void __launch_bounds__(kScanThreads)
noalloc_scan_kernel(int* __restrict__ hist, int nblk, int E, int* __restrict__ counts) {
    __shared__ int s_warp[kScanThreads / 32];
    __shared__ int s_carry;
    const int e = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_carry = 0;
    __syncthreads();
    for (int b0 = 0; b0 < nblk; b0 += kScanThreads) {
        const int b = b0 + tid;
        const int c = b < nblk ? hist[(size_t)b * E + e] : 0;
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) s_warp[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            int w = s_warp[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += v;
            }
            s_warp[lane] = w;   // inclusive over warps
        }
        __syncthreads();
        const int carry = s_carry;
        const int before = (warp ? s_warp[warp - 1] : 0) + incl - c;
        if (b < nblk) hist[(size_t)b * E + e] = carry + before;
        __syncthreads();
        if (tid == 0) s_carry = carry + s_warp[kScanThreads / 32 - 1];
        __syncthreads();
    }
    if (tid == 0) counts[e] = s_carry;
}

// One CTA: expert offsets padded to 128 rows from the counts, and the
// padding rows' token -1 / weight 0.
__global__ void __launch_bounds__(256)
noalloc_offsets_kernel(const int* __restrict__ counts, int E, int* __restrict__ eoff,
                       int* __restrict__ row_token, float* __restrict__ row_weight) {
    __shared__ int s_off[kMaxExperts + 1];
    if (threadIdx.x == 0) {
        int off = 0;
        for (int x = 0; x < E; ++x) {
            s_off[x] = off;
            eoff[x] = off;
            off += (counts[x] + kTileM - 1) / kTileM * kTileM;
        }
        s_off[E] = off;
        eoff[E] = off;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = warp; e < E; e += blockDim.x >> 5)
        for (int r = s_off[e] + counts[e] + lane; r < s_off[e + 1]; r += 32) {
            row_token[r] = -1;
            row_weight[r] = 0.0f;
        }
}

// Stable placement: within an expert, entries in ascending (token, slot)
// order.  An entry's rank inside its block counts the block's earlier
// entries with the same expert, so an expert that a token lists twice gets
// two rows, in slot order.
__global__ void __launch_bounds__(256)
noalloc_place_kernel(const int* __restrict__ idx, const float* __restrict__ wts, int T, int E,
                     int k, const int* __restrict__ hist, const int* __restrict__ eoff,
                     int* __restrict__ row_token, float* __restrict__ row_weight) {
    __shared__ int s_e[kRouteTokens * kMaxTopK];
    const int t0 = blockIdx.x * kRouteTokens;
    const int n = min(kRouteTokens, T - t0) * k;
    const int i = threadIdx.x;
    int e = -1;
    if (i < n) {
        e = idx[(size_t)t0 * k + i];
        if (e < 0 || e >= E) e = -1;
        s_e[i] = e;
    }
    __syncthreads();
    if (e >= 0) {
        int rank = 0;
        for (int j = 0; j < i; ++j) rank += s_e[j] == e;
        const int pos = eoff[e] + hist[(size_t)blockIdx.x * E + e] + rank;
        row_token[pos] = t0 + i / k;
        row_weight[pos] = wts[(size_t)t0 * k + i];
    }
}

int set_error(int code, const char* msg) { return report_error(code, msg); }

}  // namespace
}  // namespace moe

extern "C" int moe_dispatch_noalloc(const int32_t* idx, const float* weights, int32_t T,
                         int32_t num_experts, int32_t top_k, int32_t* row_token,
                         float* row_weight, int32_t rows_cap, int32_t* expert_offsets,
                         int32_t* counts, void* stream) {
    using namespace moe;
    if (T < 0 || num_experts < 1 || num_experts > kMaxExperts || top_k < 1 ||
        top_k > kMaxTopK || top_k > num_experts)
        return set_error(MOE_ERR_INVALID,
                         "moe_dispatch_noalloc: need T >= 0, 1 <= num_experts <= 256, "
                         "1 <= top_k <= min(8, num_experts)");
    const long long nblk = (T + kRouteTokens - 1) / kRouteTokens;
    if (nblk * num_experts > kScratchInts)
        return set_error(MOE_ERR_INVALID,
                         "moe_dispatch_noalloc: ceil(T / 32) * num_experts exceeds the 262144-entry "
                         "(1 MiB) static scratch; split the tokens into smaller calls");
    const long long rows_needed =
        ((long long)T * top_k / kTileM + num_experts + 1) * (long long)kTileM;
    if (rows_cap < rows_needed)
        return set_error(MOE_ERR_INVALID,
                         "moe_dispatch_noalloc: rows_cap must be at least "
                         "(T * top_k / 128 + num_experts + 1) * 128");
    if (!row_token || !row_weight || !expert_offsets || !counts || (T > 0 && (!idx || !weights)))
        return set_error(MOE_ERR_INVALID, "moe_dispatch_noalloc: null pointer argument");

    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(MOE_ERR_CUDA, "moe_dispatch_noalloc: no usable current device");
    int* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_dispatch_scratch);
            if (e != cudaSuccess || !p)
                return set_error(MOE_ERR_CUDA,
                                 "moe_dispatch_noalloc: cudaGetSymbolAddress of the static "
                                 "scratch failed");
            g_scratch_ptr[dev] = static_cast<int*>(p);
        }
        scratch = g_scratch_ptr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int nb = (int)nblk;
    // T == 0 runs only the last two kernels, which write zero counts and
    // offsets.
    if (nb > 0) noalloc_count_kernel<<<nb, 256, 0, s>>>(idx, T, num_experts, top_k, scratch);
    noalloc_scan_kernel<<<num_experts, kScanThreads, 0, s>>>(scratch, nb, num_experts, counts);
    noalloc_offsets_kernel<<<1, 256, 0, s>>>(counts, num_experts, expert_offsets, row_token,
                                             row_weight);
    if (nb > 0)
        noalloc_place_kernel<<<nb, 256, 0, s>>>(idx, weights, T, num_experts, top_k, scratch,
                                                expert_offsets, row_token, row_weight);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(MOE_ERR_CUDA, cudaGetErrorString(e));
    return MOE_OK;
}
