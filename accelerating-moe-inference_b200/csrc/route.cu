// Router and dispatch kernels.
//
//   router_kernel     logits = x . wg^T (+ bias), one fp32 fused-multiply-add
//                     chain per (token, expert), k ascending -- the exact
//                     arithmetic of the reference's matmul_transposed as its
//                     Makefile builds it (src/tensor.cu:136-148, contracted to
//                     FMA under -O3 -march=native) and of its device gate GEMM
//                     (src/model.cu:505-616).  Then top-k selection per token
//                     (PHI policy src/layer.cu:47-70 / src/model.cu:878-904, or
//                     softmax top-k with a warp-shuffle argmax), the combine
//                     weights, and the block's per-expert histogram
//                     (src/model.cu:921-942).
//   dispatch_scan     per-expert exclusive scan over blocks, expert offsets
//                     padded to 128 rows, the GEMM m-tile list
//                     (src/model.cu:953-1003).
//   dispatch_permute  stable placement (ascending token order within each
//                     expert, as assignments[e] in src/layer.cu:86-91 and
//                     route_place src/model.cu:1009-1030) fused with the row
//                     gather and the conversion of x into the GEMM operand
//                     format (bf16, or tf32 hi + lo planes).
#include <cuda_bf16.h>

#include <algorithm>
#include <cfloat>
#include <type_traits>
#include <climits>
#include <cmath>

#include "moe_internal.h"
#include "ptx.cuh"
#include "select.cuh"

namespace moe {
namespace {

constexpr int kRouterThreads = 256;

// Outputs of the scan, handed to the permute kernel when it also does the
// scan (single-block dispatch); all null otherwise.
struct ScanOut {
    int* counts = nullptr;
    int* eoff = nullptr;
    MTile* mtiles = nullptr;
    int* num_mtiles = nullptr;
    MTile* ptiles = nullptr;
    int* num_ptiles = nullptr;
    // Selection slot maps (written whenever non-null, scan or not): packed
    // row -> slot t * k + s, and slot -> packed row.
    int* row_slot = nullptr;
    int* slot_row = nullptr;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const uint32_t s = smem_u32(smem);
    const int n = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Thread layout: el = tid % 8 is the expert lane, tt = tid / 8 the token
// (0..31).  Thread (tt, el) owns the chains of experts el, el + 8, ...,
// el + 8 (EJ - 1) for token tt.  Per 4-wide k step a warp reads 4 distinct x
// rows and 8 distinct weight rows out of shared memory.
// kBlk (E a multiple of 32): 2E threads, thread (tq = tid % 8, eq = tid / 8)
// owning the 16 chains of tokens tq + 8a and experts eq + (E/4) b (a, b < 4):
// 4 x and 4 weight float4 per 4-wide k step for 64 FMAs instead of 9 for 32,
// each load's rows consecutive (bank-conflict free).  Every chain is still
// one serial fused multiply-add per k, ascending.
template <int EJ, int KC, bool kBlk = false>
__global__ void __launch_bounds__(kBlk ? 512 : kRouterThreads)
router_kernel(const float* __restrict__ x, const float* __restrict__ wg,
              const float* __restrict__ bias, int T, int d, int E, int k, int policy,
              float quantum, float tie_eps, float* __restrict__ logits_out,
              int* __restrict__ idx_out, float* __restrict__ w_out,
              int* __restrict__ blockhist, NormRef nr, const int* __restrict__ eperm) {
    constexpr int kStages = 4;
    constexpr int kLd = KC + 4;              // padded row stride (floats)
    constexpr int kXs = kRouteTokens * kLd;  // x floats per stage
    const int kWs = (kBlk ? E : 8 * EJ) * kLd;   // wg floats per stage
    extern __shared__ __align__(16) float rsm[];
    float* xs = rsm;                       // [kStages][32][kLd]
    float* ws = rsm + kStages * kXs;       // [kStages][wg rows][kLd]
    float* nws = ws + kStages * kWs;       // [kStages][2][KC] norm weight, bias chunks
    float* nst = nws + kStages * 2 * KC;   // [2][32] norm mean, inverse std of the tokens
    float* lg = nst + 2 * kRouteTokens;    // [32][E + 1]
    int* hist = reinterpret_cast<int*>(lg + kRouteTokens * (E + 1));

    const int tid = threadIdx.x;
    const int el = tid & 7;
    const int tt = tid >> 3;
    const int t0 = blockIdx.x * kRouteTokens;
    const int n_tok = min(kRouteTokens, T - t0);
    const int nchunks = d / KC;
    if (nr.mean) {
        for (int t = tid; t < n_tok; t += blockDim.x) {
            nst[t] = nr.mean[t0 + t];
            nst[kRouteTokens + t] = nr.inv[t0 + t];
        }
    }

    // Stage loader: x chunk is 32 rows x KC floats, wg chunk E rows x KC.
    // Token rows this CTA stages (kBlk: all 32, the rows past T zero-filled).
    const int x_rows = kBlk ? kRouteTokens : (int)(blockDim.x / 8);
    auto load_chunk = [&](int chunk, int stage) {
        const int kbase = chunk * KC;
        const int kXv = x_rows * KC / 4;   // float4 per x chunk
        for (int v = tid; v < kXv; v += blockDim.x) {
            const int r = v / (KC / 4), c = (v % (KC / 4)) * 4;
            const bool ok = r < n_tok;
            const float* src = x + (size_t)(ok ? t0 + r : 0) * d + kbase + c;
            cp_async16(xs + stage * kXs + r * kLd + c, src, ok);
        }
        const int wv = E * KC / 4;
        for (int v = tid; v < wv; v += blockDim.x) {
            const int r = v / (KC / 4), c = (v % (KC / 4)) * 4;
            cp_async16(ws + stage * kWs + r * kLd + c, wg + (size_t)r * d + kbase + c, true);
        }
        if (nr.mean) {
            for (int v = tid; v < KC / 2; v += blockDim.x) {
                const int c = (v % (KC / 4)) * 4;
                const float* src = (v < KC / 4 ? nr.w : nr.b) + kbase + c;
                cp_async16(nws + stage * 2 * KC + (v < KC / 4 ? 0 : KC) + c, src, true);
            }
        }
    };

    constexpr int kAcc = kBlk ? 16 : EJ;
    float acc[kAcc];
#pragma unroll
    for (int j = 0; j < kAcc; ++j) acc[j] = 0.0f;

    for (int s = 0; s < kStages - 1; ++s) {
        if (s < nchunks) load_chunk(s, s);
        cp_async_commit();
    }
    for (int c = 0; c < nchunks; ++c) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        // Refill the stage consumed in the previous iteration.
        const int nxt = c + kStages - 1;
        if (nxt < nchunks) load_chunk(nxt, nxt % kStages);
        cp_async_commit();
        const int st = c % kStages;
        if (nr.mean) {
            // Post-attention LayerNorm: normalise the landed x chunk in place,
            // once per element, before the chains read it (the norm's weight
            // and bias chunk landed with it).
            const int kXv = x_rows * KC / 4;
            const float* nw = nws + st * 2 * KC;
            for (int v = tid; v < kXv; v += blockDim.x) {
                const int r = v / (KC / 4), cc = (v % (KC / 4)) * 4;
                if (r < n_tok) {
                    float4* p = reinterpret_cast<float4*>(xs + st * kXs + r * kLd + cc);
                    *p = layer_norm_out4(*p, nst[r], nst[kRouteTokens + r],
                                         *reinterpret_cast<const float4*>(nw + cc),
                                         *reinterpret_cast<const float4*>(nw + KC + cc));
                }
            }
            __syncthreads();
        }
        if constexpr (kBlk) {
            const int tq = tid & 7, eq = tid >> 3, es = E / 4;
            const float* xr = xs + st * kXs + tq * kLd;
            const float* wr = ws + st * kWs + eq * kLd;
            float4 xa[4], wa[4], xb[4], wb[4];
            auto load_q = [&](float4 (&xv)[4], float4 (&wv)[4], int kk) {
#pragma unroll
                for (int a = 0; a < 4; ++a) xv[a] = *reinterpret_cast<const float4*>(xr + 8 * a * kLd + kk);
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    wv[b] = *reinterpret_cast<const float4*>(wr + (size_t)es * b * kLd + kk);
            };
            auto chain_q = [&](const float4 (&xv)[4], const float4 (&wv)[4]) {
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        float& c = acc[a * 4 + b];
                        c = __fmaf_rn(xv[a].x, wv[b].x, c);
                        c = __fmaf_rn(xv[a].y, wv[b].y, c);
                        c = __fmaf_rn(xv[a].z, wv[b].z, c);
                        c = __fmaf_rn(xv[a].w, wv[b].w, c);
                    }
            };
            load_q(xa, wa, 0);
#pragma unroll
            for (int kk = 0; kk < KC; kk += 8) {
                load_q(xb, wb, kk + 4);
                chain_q(xa, wa);
                if (kk + 8 < KC) load_q(xa, wa, kk + 8);
                chain_q(xb, wb);
            }
        } else {
            const float* xr = xs + st * kXs + tt * kLd;
            const float* wr = ws + st * kWs + el * kLd;
            // Fully unrolled over the chunk, every shared-memory offset an
            // immediate.  Two register sets alternate (ping-pong, no copies): the
            // loads of the next 16-wide group are issued before the current
            // group's dependent FMAs, which the loads then overlap.  Lanes whose
            // expert index is past E run chains on unused rows that are never
            // stored.
            // Group width: 16 columns for 1-2 chains per thread, 8 for 4, 4 for
            // 8 or more, so that both register sets (4 kQ (1 + EJ) floats each)
            // stay in registers whatever the expert count.
            constexpr int kQ = EJ >= 8 ? 1 : (EJ >= 4 ? 2 : 4);   // float4 per row per group
            constexpr int kGw = 4 * kQ;                            // columns per group
            float4 xa[kQ], wa[EJ][kQ], xb[kQ], wb[EJ][kQ];
            auto load_group = [&](float4 (&xv)[kQ], float4 (&wv)[EJ][kQ], int kk) {
    #pragma unroll
                for (int q = 0; q < kQ; ++q) xv[q] = *reinterpret_cast<const float4*>(xr + kk + 4 * q);
    #pragma unroll
                for (int j = 0; j < EJ; ++j)
    #pragma unroll
                    for (int q = 0; q < kQ; ++q)
                        wv[j][q] = *reinterpret_cast<const float4*>(wr + 8 * j * kLd + kk + 4 * q);
            };
            auto chain_group = [&](const float4 (&xv)[kQ], const float4 (&wv)[EJ][kQ]) {
    #pragma unroll
                for (int q = 0; q < kQ; ++q)
    #pragma unroll
                    for (int j = 0; j < EJ; ++j) {
                        acc[j] = __fmaf_rn(xv[q].x, wv[j][q].x, acc[j]);
                        acc[j] = __fmaf_rn(xv[q].y, wv[j][q].y, acc[j]);
                        acc[j] = __fmaf_rn(xv[q].z, wv[j][q].z, acc[j]);
                        acc[j] = __fmaf_rn(xv[q].w, wv[j][q].w, acc[j]);
                    }
            };
            load_group(xa, wa, 0);
    #pragma unroll
            for (int kk = 0; kk < KC; kk += 2 * kGw) {
                load_group(xb, wb, kk + kGw);
                chain_group(xa, wa);
                if (kk + 2 * kGw < KC) load_group(xa, wa, kk + 2 * kGw);
                chain_group(xb, wb);
            }
        }
    }
    cp_async_wait<0>();

    for (int e = tid; e < E; e += blockDim.x) hist[e] = 0;
    if constexpr (kBlk) {
        const int tq = tid & 7, eq = tid >> 3;
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int t = tq + 8 * a, e = eq + (E / 4) * b;
                float v = acc[a * 4 + b];
                if (bias) v = __fadd_rn(v, bias[e]);
                lg[t * (E + 1) + e] = v;
                if (logits_out && t < n_tok) logits_out[(size_t)(t0 + t) * E + e] = v;
            }
    } else {
#pragma unroll
        for (int j = 0; j < EJ; ++j) {
            const int e = el + 8 * j;
            if (e < E) {
                float v = acc[j];
                if (bias) v = __fadd_rn(v, bias[e]);
                lg[tt * (E + 1) + e] = v;
                if (logits_out && tt < n_tok) logits_out[(size_t)(t0 + tt) * E + e] = v;
            }
        }
    }
    __syncthreads();

    // Selection: warp w handles tokens per * w .. per * w + per - 1 (4 per
    // warp with 8 warps; kBlk: 32 / warps).
    const int warp = tid >> 5, lane = tid & 31;
    const int per = kBlk ? kRouteTokens / (int)(blockDim.x >> 5) : 4;
    for (int q = 0; q < per; ++q) {
        const int tk = warp * per + q;
        if (tk >= n_tok) break;
        int sel[kMaxTopK];
        float wsel[kMaxTopK];
        select_experts(lg + tk * (E + 1), E, k, policy, quantum, tie_eps, lane, sel, wsel);
        if (lane == 0) {
            const int t = t0 + tk;
            for (int s = 0; s < k; ++s) {
                // Expert parallelism: the dispatch position of the expert
                // (placement), selection having used its own index.
                const int e = eperm ? eperm[sel[s]] : sel[s];
                idx_out[(size_t)t * k + s] = e;
                w_out[(size_t)t * k + s] = wsel[s];
                atomicAdd(&hist[e], 1);
            }
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) blockhist[(size_t)blockIdx.x * E + e] = hist[e];
}

// One block of 32 warps.  Warp w scans experts w, w + 32, ... over the
// blocks with warp shuffles, turning blockhist into each block's base row
// inside its expert's run; warp 0 then scans the experts' padded sizes into
// offsets; finally every warp writes its experts' m-tiles and marks their
// padding rows (token -1, weight 0).
constexpr int kScanThreads = 1024;

__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += n;
    }
    return v;
}

__global__ void __launch_bounds__(kScanThreads)
dispatch_scan_kernel(int* __restrict__ blockhist, int nblk, int E, int granule,
                     int* __restrict__ counts, int* __restrict__ eoff, MTile* __restrict__ mtiles,
                     int* __restrict__ num_mtiles, MTile* __restrict__ ptiles,
                     int* __restrict__ num_ptiles, int* __restrict__ row_token,
                     float* __restrict__ row_weight) {
    __shared__ int s_cnt[kMaxExperts];
    __shared__ int s_off[kMaxExperts + 1];
    __shared__ int s_mst[kMaxExperts + 1];
    __shared__ int s_pst[kMaxExperts + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kWarps = kScanThreads / 32;
    for (int e = warp; e < E; e += kWarps) {
        int carry = 0;
        for (int b0 = 0; b0 < nblk; b0 += 32) {
            const int b = b0 + lane;
            const int c = b < nblk ? blockhist[(size_t)b * E + e] : 0;
            const int incl = warp_inclusive_scan(c, lane);
            if (b < nblk) blockhist[(size_t)b * E + e] = carry + incl - c;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            s_cnt[e] = carry;
            counts[e] = carry;
        }
    }
    __syncthreads();
    if (warp == 0) {
        int run_off = 0, run_m = 0, run_p = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < E ? s_cnt[e] : 0;
            const int mc = (c + kTileM - 1) / kTileM;
            const int qc = (mc + 1) / 2;                  // 256-row pair tiles
            const int pc = (c + granule - 1) / granule * granule;
            const int ipc = warp_inclusive_scan(pc, lane);
            const int imc = warp_inclusive_scan(mc, lane);
            const int iqc = warp_inclusive_scan(qc, lane);
            if (e < E) {
                s_off[e] = run_off + ipc - pc;
                s_mst[e] = run_m + imc - mc;
                s_pst[e] = run_p + iqc - qc;
                eoff[e] = s_off[e];
            }
            run_off += __shfl_sync(0xffffffffu, ipc, 31);
            run_m += __shfl_sync(0xffffffffu, imc, 31);
            run_p += __shfl_sync(0xffffffffu, iqc, 31);
        }
        if (lane == 0) {
            s_off[E] = run_off;
            s_mst[E] = run_m;
            s_pst[E] = run_p;
            eoff[E] = run_off;
            if (num_mtiles) *num_mtiles = run_m;
            if (num_ptiles) *num_ptiles = run_p;
        }
    }
    __syncthreads();
    if (!mtiles) return;   // compact layout (granule 1): no GEMM tiles, no padding rows
    for (int e = warp; e < E; e += kWarps) {
        const int c = s_cnt[e];
        const int mst = s_mst[e];
        const int mc = s_mst[e + 1] - mst;
        for (int i = lane; i < mc; i += 32) {
            MTile mt;
            mt.expert = e;
            mt.row0 = s_off[e] + i * kTileM;
            mt.rows = min(kTileM, c - i * kTileM);
            mt.mstart = mst;
            mt.mcount = mc;
            mt.pad[0] = mt.pad[1] = mt.pad[2] = 0;
            mtiles[mst + i] = mt;
        }
        if (ptiles) {
            const int pst = s_pst[e];
            const int pc = s_pst[e + 1] - pst;
            for (int i = lane; i < pc; i += 32) {
                MTile pt;
                pt.expert = e;
                pt.row0 = s_off[e] + 2 * i * kTileM;
                pt.rows = min(kTileM, c - 2 * i * kTileM);
                pt.mstart = pst;
                pt.mcount = pc;
                pt.pad[0] = max(0, min(kTileM, c - (2 * i + 1) * kTileM));   // second half
                pt.pad[1] = pt.pad[2] = 0;
                ptiles[pst + i] = pt;
            }
        }
        for (int r = s_off[e] + c + lane; r < s_off[e + 1]; r += 32) {
            row_token[r] = -1;
            row_weight[r] = 0.0f;
        }
    }
}

// Tiles of one expert-block layout from per-expert counts held in shared
// memory (single-block dispatch: T fits one 32-token router block, so the
// block histogram is the whole count and the scan is a prefix over experts).
// Called by every thread of the CTA; writes the layout only if `write`.
// Warp 0 scans 32 experts at a time with shuffles (expert e's lane writes
// its own offsets and tiles); the padding rows are then spread over all
// warps.
__device__ __forceinline__ void store_tile(MTile* dst, int expert, int row0, int rows, int mstart,
                                           int mcount, int second) {
    int4* p = reinterpret_cast<int4*>(dst);
    p[0] = make_int4(expert, row0, rows, mstart);
    p[1] = make_int4(mcount, second, 0, 0);
}

__device__ void single_block_layout(const int* __restrict__ cnt, int E, int* s_off, bool write,
                                    int* __restrict__ counts, int* __restrict__ eoff,
                                    MTile* __restrict__ mtiles, int* __restrict__ num_mtiles,
                                    MTile* __restrict__ ptiles, int* __restrict__ num_ptiles,
                                    int* __restrict__ row_token, float* __restrict__ row_weight) {
    static_assert(sizeof(MTile) == 32, "MTile is stored as two int4");
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int off = 0, nm = 0, np = 0;   // running totals of the experts before this group
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < E ? cnt[e] : 0;
            const int mc = (c + kTileM - 1) / kTileM;
            const int qc = (mc + 1) / 2;
            int srow = mc * kTileM, smc = mc, sqc = qc;   // inclusive prefix sums
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, srow, o);
                const int b = __shfl_up_sync(0xffffffffu, smc, o);
                const int q = __shfl_up_sync(0xffffffffu, sqc, o);
                if (lane >= o) {
                    srow += a;
                    smc += b;
                    sqc += q;
                }
            }
            const int my_off = off + srow - mc * kTileM;
            const int my_m = nm + smc - mc, my_p = np + sqc - qc;
            if (e < E) {
                s_off[e] = my_off;
                if (write) {
                    counts[e] = c;
                    eoff[e] = my_off;
                    for (int i = 0; i < mc; ++i)
                        store_tile(mtiles + my_m + i, e, my_off + i * kTileM,
                                   min(kTileM, c - i * kTileM), my_m, mc, 0);
                    for (int i = 0; i < qc; ++i)
                        store_tile(ptiles + my_p + i, e, my_off + 2 * i * kTileM,
                                   min(kTileM, c - 2 * i * kTileM), my_p, qc,
                                   max(0, min(kTileM, c - (2 * i + 1) * kTileM)));
                }
            }
            off += __shfl_sync(0xffffffffu, srow, 31);
            nm += __shfl_sync(0xffffffffu, smc, 31);
            np += __shfl_sync(0xffffffffu, sqc, 31);
        }
        if (lane == 0) {
            s_off[E] = off;
            if (write) {
                eoff[E] = off;
                *num_mtiles = nm;
                *num_ptiles = np;
            }
        }
    }
    __syncthreads();
    if (write) {
        // Padding rows of every expert block (token -1, weight 0).
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
        for (int e = warp; e < E; e += nw)
            for (int r = s_off[e] + cnt[e] + lane; r < s_off[e + 1]; r += 32) {
                row_token[r] = -1;
                row_weight[r] = 0.0f;
            }
    }
}

// kMode: ActFormat -- bf16 plane, tf32 hi + lo planes, fp32 as is (decode),
// or bf16 hi + lo planes.
template <int kMode>
__global__ void __launch_bounds__(256)
dispatch_permute_kernel(const float* __restrict__ x, int T, int d, int E, int k,
                        const int* __restrict__ idx, const float* __restrict__ wts,
                        const int* __restrict__ blockbase, const int* __restrict__ eoff,
                        int* __restrict__ row_token, float* __restrict__ row_weight,
                        void* __restrict__ a_hi, void* __restrict__ a_lo, ScanOut so,
                        NormRef nr) {
    __shared__ unsigned s_mask[kMaxExperts];
    __shared__ int s_base[kMaxExperts + 1];
    __shared__ int s_dest[kRouteTokens * kMaxTopK];
    __shared__ float s_nmean[kRouteTokens], s_ninv[kRouteTokens];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kRouteTokens;
    const int n_tok = min(kRouteTokens, T - t0);
    if (nr.mean && tid < n_tok) {
        s_nmean[tid] = nr.mean[t0 + tid];
        s_ninv[tid] = nr.inv[t0 + tid];
    }
    if (so.counts) {
        // Single-block dispatch: this kernel also does the scan.  blockbase
        // holds the one block's histogram.
        single_block_layout(blockbase, E, s_base, blockIdx.y == 0, so.counts, so.eoff, so.mtiles,
                            so.num_mtiles, so.ptiles, so.num_ptiles, row_token, row_weight);
        for (int e = tid; e < E; e += blockDim.x) s_mask[e] = 0u;
    } else {
        for (int e = tid; e < E; e += blockDim.x) {
            s_mask[e] = 0u;
            s_base[e] = eoff[e] + blockbase[(size_t)blockIdx.x * E + e];
        }
    }
    __syncthreads();
    const int n_ent = n_tok * k;
    int my_e = -1, my_t = 0;
    if (tid < n_ent) {
        my_t = tid / k;
        my_e = idx[(size_t)(t0 + my_t) * k + (tid % k)];
        atomicOr(&s_mask[my_e], 1u << my_t);
    }
    __syncthreads();
    if (tid < n_ent) {
        const int rank = __popc(s_mask[my_e] & ((1u << my_t) - 1u));
        const int pos = s_base[my_e] + rank;
        s_dest[tid] = pos;
        if (blockIdx.y == 0) {
            const int slot = (t0 + my_t) * k + (tid % k);
            row_token[pos] = t0 + my_t;
            row_weight[pos] = wts[slot];
            if (so.row_slot) so.row_slot[pos] = slot;
            if (so.slot_row) so.slot_row[slot] = pos;
        }
    }
    __syncthreads();
    // This CTA copies columns [c0, c1) (in float4 units) of its block's rows.
    const int nv = d / 4;
    const int per = (nv + gridDim.y - 1) / gridDim.y;
    const int c0 = blockIdx.y * per, c1 = min(nv, c0 + per);
    const int width = max(0, c1 - c0);
    const int total = n_tok * width;
    constexpr int kUnroll = 8;
    const float4* nw4 = reinterpret_cast<const float4*>(nr.w);
    const float4* nb4 = reinterpret_cast<const float4*>(nr.b);
    for (int base = tid; base < total; base += kUnroll * 256) {
        float4 f[kUnroll];
        if (nr.mean) {
            // The post-attention LayerNorm's weight and bias columns are
            // loaded in the same batch as the rows.
            float4 wv[kUnroll], bv[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * 256;
                if (i < total) {
                    const int v = c0 + i % width;
                    f[u] = reinterpret_cast<const float4*>(x + (size_t)(t0 + i / width) * d)[v];
                    wv[u] = __ldg(nw4 + v);
                    bv[u] = __ldg(nb4 + v);
                }
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * 256;
                if (i < total) {
                    const int t = i / width;
                    f[u] = layer_norm_out4(f[u], s_nmean[t], s_ninv[t], wv[u], bv[u]);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int i = base + u * 256;
                if (i < total)
                    f[u] = reinterpret_cast<const float4*>(x + (size_t)(t0 + i / width) * d)[c0 + i % width];
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int i = base + u * 256;
            if (i >= total) break;
            const int t = i / width, v = c0 + i % width;
            if constexpr (kMode == 0) {
                __nv_bfloat162 lo2 = __floats2bfloat162_rn(f[u].x, f[u].y);
                __nv_bfloat162 hi2 = __floats2bfloat162_rn(f[u].z, f[u].w);
                uint2 packed;
                packed.x = *reinterpret_cast<uint32_t*>(&lo2);
                packed.y = *reinterpret_cast<uint32_t*>(&hi2);
                for (int s = 0; s < k; ++s) {
                    const size_t row = (size_t)s_dest[t * k + s];
                    reinterpret_cast<uint2*>(a_hi)[row * nv + v] = packed;
                }
            } else if constexpr (kMode == kActF32) {
                for (int s = 0; s < k; ++s) {
                    const size_t row = (size_t)s_dest[t * k + s];
                    reinterpret_cast<float4*>(a_hi)[row * nv + v] = f[u];
                }
            } else if constexpr (kMode == kActBf16x2) {
                uint2 hp, lp;
                split_bf16x2(f[u].x, f[u].y, hp.x, lp.x);
                split_bf16x2(f[u].z, f[u].w, hp.y, lp.y);
                for (int s = 0; s < k; ++s) {
                    const size_t row = (size_t)s_dest[t * k + s];
                    reinterpret_cast<uint2*>(a_hi)[row * nv + v] = hp;
                    reinterpret_cast<uint2*>(a_lo)[row * nv + v] = lp;
                }
            } else {
                float4 h, l;
                h.x = to_tf32(f[u].x); l.x = to_tf32(f[u].x - h.x);
                h.y = to_tf32(f[u].y); l.y = to_tf32(f[u].y - h.y);
                h.z = to_tf32(f[u].z); l.z = to_tf32(f[u].z - h.z);
                h.w = to_tf32(f[u].w); l.w = to_tf32(f[u].w - h.w);
                for (int s = 0; s < k; ++s) {
                    const size_t row = (size_t)s_dest[t * k + s];
                    reinterpret_cast<float4*>(a_hi)[row * nv + v] = h;
                    reinterpret_cast<float4*>(a_lo)[row * nv + v] = l;
                }
            }
        }
    }
}

// ------------------------------------------------------------ small batches
// A decode-sized batch (T <= 4) is routed and dispatched by one CTA in one
// launch.  Warp 0's lane 0 streams K chunks of the router weights and of the
// token rows (and the post-attention norm's weight and bias) into a ring of
// shared-memory stages with 1-D bulk copies, one per row, each stage
// completing on its `full` mbarrier.  Every (token, expert) pair has a thread
// in warps 1.. that runs its logit's fused-multiply-add chain out of the ring
// (with the norm applied in registers), so the chains -- 4.5 cycles per FMA,
// d of them -- and not the loads set the kernel's length.  Warp t then
// selects token t's experts, the whole CTA builds the single-block layout,
// and the routed rows are written in the format the next stage reads.
constexpr int kSmallMaxTokens = 4;
constexpr int kSmallChainThreads = 256;
constexpr int kSmallThreads = 32 + kSmallChainThreads;
constexpr int kSmallMaxStages = 8;

struct SmallGeom {
    int kc;       // K columns per stage
    int stages;
    int rows;     // E router rows, T token rows, then norm weight and bias rows
    int ld;       // padded row stride in floats: kc + 4 (LDS.128 of 8 rows conflict-free)
    // RMSNorm statistics computed here from the token rows in shared memory
    // (every K chunk resident) instead of by rms_stats_kernel beforehand:
    // the same sum order and expression, written to stat_mean / stat_inv.
    int rms_inline;
    float rms_eps;
    float* stat_mean;
    float* stat_inv;
};

// Columns 4v .. 4v+3 of packed row `row` in the format of kMode (ActFormat).
template <int kMode>
__device__ __forceinline__ void store_row4(void* a_hi, void* a_lo, size_t row, int nv, int v,
                                           float4 f) {
    if constexpr (kMode == kActBf16x2) {
        uint2 hp, lp;
        split_bf16x2(f.x, f.y, hp.x, lp.x);
        split_bf16x2(f.z, f.w, hp.y, lp.y);
        reinterpret_cast<uint2*>(a_hi)[row * nv + v] = hp;
        reinterpret_cast<uint2*>(a_lo)[row * nv + v] = lp;
    } else if constexpr (kMode == 0) {
        __nv_bfloat162 lo2 = __floats2bfloat162_rn(f.x, f.y);
        __nv_bfloat162 hi2 = __floats2bfloat162_rn(f.z, f.w);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&lo2);
        packed.y = *reinterpret_cast<uint32_t*>(&hi2);
        reinterpret_cast<uint2*>(a_hi)[row * nv + v] = packed;
    } else if constexpr (kMode == 2) {
        reinterpret_cast<float4*>(a_hi)[row * nv + v] = f;
    } else {
        float4 h, l;
        h.x = to_tf32(f.x); l.x = to_tf32(f.x - h.x);
        h.y = to_tf32(f.y); l.y = to_tf32(f.y - h.y);
        h.z = to_tf32(f.z); l.z = to_tf32(f.z - h.z);
        h.w = to_tf32(f.w); l.w = to_tf32(f.w - h.w);
        reinterpret_cast<float4*>(a_hi)[row * nv + v] = h;
        reinterpret_cast<float4*>(a_lo)[row * nv + v] = l;
    }
}

// kMode: ActFormat of the routed rows.  KC: K columns
// per stage (the chain loop is fully unrolled over it); kNorm: apply the
// post-attention LayerNorm.
template <int kMode, int KC, bool kNorm>
__global__ void __launch_bounds__(kSmallThreads, 1)
router_small_kernel(const float* __restrict__ x, const float* __restrict__ wg,
                    const float* __restrict__ bias, int T, int d, int E, int k, int policy,
                    float quantum, float tie_eps, NormRef nr, SmallGeom gm,
                    float* __restrict__ logits_out, int* __restrict__ idx_out,
                    float* __restrict__ w_out, ScanOut so, int* __restrict__ row_token,
                    float* __restrict__ row_weight, void* __restrict__ a_hi,
                    void* __restrict__ a_lo, int* err) {
    extern __shared__ __align__(16) float ring[];
    __shared__ uint64_t full[kSmallMaxStages], empty[kSmallMaxStages];
    __shared__ float lg[kSmallMaxTokens * (kMaxExperts + 1)];
    __shared__ int hist[kMaxExperts];
    __shared__ int s_base[kMaxExperts + 1];
    __shared__ int s_sel[kSmallMaxTokens * kMaxTopK];
    __shared__ float s_w[kSmallMaxTokens * kMaxTopK];
    __shared__ int s_dest[kSmallMaxTokens * kMaxTopK];
    __shared__ volatile int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nchunks = d / KC;
    const int chain_warps = (blockDim.x >> 5) - 1;
    // Dependent launch: nothing the previous kernel may write (x, the norm
    // statistics, the workspace) is read or written before it has completed;
    // the layer's constants (router rows, the norm's weight and bias) are
    // loaded before that wait, so their latency overlaps the previous kernel.
    constexpr bool norm = kNorm;
    const int rows_used = E + T + (norm ? 2 : 0);
    if (tid == 0) {
        for (int st = 0; st < gm.stages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], chain_warps);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    for (int e = tid; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();

    // When every K chunk has a stage of its own (nchunks <= stages), all
    // threads fill the ring with plain 16-byte loads, 16 in flight each, and
    // the chains run once the whole ring has landed: one SM's bulk copies
    // deliver only a few bytes per cycle, many threads' loads far more.
    const bool direct = nchunks <= gm.stages;
    if (direct) {
        constexpr int kV = KC / 4;     // float4 per row chunk
        constexpr int kInFlight = 16;
        const int nw = blockDim.x >> 5;
        // Pass 0: the constant rows (router, norm weight and bias); pass 1,
        // after the wait for the previous kernel: the token rows.
        for (int pass = 0; pass < 2; ++pass) {
            if (pass == 1) {
                wait_predecessor_grid();
                launch_dependents();
            }
            for (int r = warp; r < rows_used; r += nw) {
                const bool token_row = r >= E && r < E + T;
                if (token_row != (pass == 1)) continue;
                const float* src = r < E ? wg + (size_t)r * d
                                 : token_row ? x + (size_t)(r - E) * d
                                 : (r == E + T ? nr.w : nr.b);
                for (int v0 = lane; v0 < d / 4; v0 += 32 * kInFlight) {
                    float4 f[kInFlight];
#pragma unroll
                    for (int u = 0; u < kInFlight; ++u) {
                        const int v = v0 + 32 * u;
                        if (v < d / 4) f[u] = __ldg(reinterpret_cast<const float4*>(src) + v);
                    }
#pragma unroll
                    for (int u = 0; u < kInFlight; ++u) {
                        const int v = v0 + 32 * u;
                        if (v < d / 4)
                            *reinterpret_cast<float4*>(ring + (size_t)(v / kV) * gm.rows * gm.ld +
                                                       (size_t)r * gm.ld + 4 * (v % kV)) = f[u];
                    }
                }
            }
        }
        __syncthreads();
        if constexpr (kNorm) {
            __shared__ float s_mean[kSmallMaxTokens], s_inv[kSmallMaxTokens];
            if (gm.rms_inline) {
                // Warp t: token t's sum of squares in rms_stats_kernel's order
                // (lane-strided float4 fma chain, then the xor-shuffle tree).
                if (warp < T) {
                    float ss = 0.0f;
                    for (int v = lane; v < d / 4; v += 32) {
                        const float4 a = *reinterpret_cast<const float4*>(
                            ring + (size_t)(v / kV) * gm.rows * gm.ld + (size_t)(E + warp) * gm.ld +
                            4 * (v % kV));
                        ss = __fmaf_rn(a.x, a.x, ss);
                        ss = __fmaf_rn(a.y, a.y, ss);
                        ss = __fmaf_rn(a.z, a.z, ss);
                        ss = __fmaf_rn(a.w, a.w, ss);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                    if (lane == 0) {
                        s_mean[warp] = 0.0f;
                        s_inv[warp] = 1.0f / sqrtf(ss / (float)d + gm.rms_eps);
                        gm.stat_mean[warp] = 0.0f;
                        gm.stat_inv[warp] = s_inv[warp];
                    }
                }
            } else if (tid < T) {
                s_mean[tid] = nr.mean[tid];
                s_inv[tid] = nr.inv[tid];
            }
            __syncthreads();
            // Every expert's chain reads the same normalised token row:
            // normalise it once, in place, with the expression the chains
            // would apply (bit-identical), instead of in each chain.
            for (int i = tid; i < T * (d / 4); i += blockDim.x) {
                const int t = i / (d / 4), v = i % (d / 4);
                float* sb = ring + (size_t)(v / kV) * gm.rows * gm.ld + 4 * (v % kV);
                float4* xp = reinterpret_cast<float4*>(sb + (size_t)(E + t) * gm.ld);
                *xp = layer_norm_out4(*xp, s_mean[t], s_inv[t],
                                      *reinterpret_cast<const float4*>(sb + (size_t)(E + T) * gm.ld),
                                      *reinterpret_cast<const float4*>(sb + (size_t)(E + T + 1) * gm.ld));
            }
            __syncthreads();
        }
    }

    if (!direct) {
        wait_predecessor_grid();
        launch_dependents();
    }
    if (warp == 0) {
        if (lane == 0 && !direct) {
            // ------------------------------------------------ loads
            const uint32_t bytes = (uint32_t)rows_used * KC * 4;
            for (int g = 0; g < nchunks; ++g) {
                const int st = g % gm.stages;
                if (g >= gm.stages &&
                    !mbar_wait(&empty[st], ((g / gm.stages) - 1) & 1, err, kDevErrTimeoutProducer)) {
                    abort_flag = 1;
                    break;
                }
                if (abort_flag) break;
                mbar_arrive_expect_tx(&full[st], bytes);
                float* sb = ring + (size_t)st * gm.rows * gm.ld;
                const size_t c0 = (size_t)g * KC;
                for (int r = 0; r < rows_used; ++r) {
                    const float* src = r < E ? wg + (size_t)r * d + c0
                                     : r < E + T ? x + (size_t)(r - E) * d + c0
                                     : (r == E + T ? nr.w : nr.b) + c0;
                    bulk_load(sb + (size_t)r * gm.ld, src, KC * 4, &full[st]);
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------- chains
        const int ci = tid - 32;
        const bool active = ci < T * E;
        const int t = active ? ci / E : 0, e = active ? ci % E : 0;
        float m = 0.0f, iv = 0.0f;
        if (norm && active) {
            m = nr.mean[t];
            iv = nr.inv[t];
        }
        float acc = 0.0f;
        for (int g = 0; g < nchunks; ++g) {
            const int st = g % gm.stages;
            if (!direct && !mbar_wait(&full[st], (g / gm.stages) & 1, err, kDevErrTimeoutMma)) {
                abort_flag = 1;
                break;
            }
            const float* sb = ring + (size_t)st * gm.rows * gm.ld;
            const float* xr = sb + (size_t)(E + t) * gm.ld;
            const float* wr = sb + (size_t)e * gm.ld;
            const float* nw = sb + (size_t)(E + T) * gm.ld;
            const float* nb = nw + gm.ld;
            if (active) {
                // Two register groups alternate: the next 16 columns' loads
                // are issued before the current group's dependent FMAs.
                float4 xa[4], wa[4], xb[4], wb[4];
                // kApply: the norm is applied here (ring path); the direct
                // path normalised the token rows in shared memory already.
                auto run = [&](auto apply_tag) {
                    constexpr bool kApply = decltype(apply_tag)::value;
                    auto load = [&](float4 (&xv)[4], float4 (&wv)[4], int kk) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            float4 xq = *reinterpret_cast<const float4*>(xr + kk + 4 * q);
                            if constexpr (kApply)
                                xq = layer_norm_out4(xq, m, iv,
                                                     *reinterpret_cast<const float4*>(nw + kk + 4 * q),
                                                     *reinterpret_cast<const float4*>(nb + kk + 4 * q));
                            xv[q] = xq;
                            wv[q] = *reinterpret_cast<const float4*>(wr + kk + 4 * q);
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
                    for (int kk = 0; kk < KC; kk += 32) {
                        load(xb, wb, kk + 16);
                        chain(xa, wa);
                        if (kk + 32 < KC) load(xa, wa, kk + 32);
                        chain(xb, wb);
                    }
                };
                if (kNorm && !direct)
                    run(std::integral_constant<bool, kNorm>{});
                else
                    run(std::integral_constant<bool, false>{});
            }
            __syncwarp();
            if (lane == 0 && !direct) mbar_arrive(&empty[st]);
        }
        if (active) {
            float v = acc;
            if (bias) v = __fadd_rn(v, bias[e]);
            lg[t * (E + 1) + e] = v;
            if (logits_out) logits_out[(size_t)t * E + e] = v;
        }
    }
    __syncthreads();
    if (abort_flag) return;   // err is set; outputs are left as they were

    // ---------------------------------------------------- selection: warp t, token t
    if (warp < T) {
        const int t = warp;
        int sel[kMaxTopK];
        float wsel[kMaxTopK];
        select_experts(lg + t * (E + 1), E, k, policy, quantum, tie_eps, lane, sel, wsel);
        if (lane == 0) {
            for (int s2 = 0; s2 < k; ++s2) {
                idx_out[(size_t)t * k + s2] = sel[s2];
                w_out[(size_t)t * k + s2] = wsel[s2];
                s_sel[t * k + s2] = sel[s2];
                s_w[t * k + s2] = wsel[s2];
                atomicAdd(&hist[sel[s2]], 1);
            }
        }
    }
    __syncthreads();
    single_block_layout(hist, E, s_base, true, so.counts, so.eoff, so.mtiles, so.num_mtiles,
                        so.ptiles, so.num_ptiles, row_token, row_weight);
    // Stable placement: within an expert, tokens in ascending order.
    if (tid < T * k) {
        const int t = tid / k, e = s_sel[tid];
        int rank = 0;
        for (int t2 = 0; t2 < t; ++t2)
            for (int s2 = 0; s2 < k; ++s2) rank += s_sel[t2 * k + s2] == e;
        const int pos = s_base[e] + rank;
        s_dest[tid] = pos;
        row_token[pos] = t;
        row_weight[pos] = s_w[tid];
        so.row_slot[pos] = tid;
    }
    __syncthreads();
    // The routed rows, normalised if the norm is active, in the next stage's
    // format: each token row is read once (16 loads in flight per thread, so
    // a batch takes about one round trip) and written to its k packed rows.
    const int nv = d / 4;
    if (direct) {
        // The token rows are still in the ring: chunk v / (KC / 4) of row E + t.
        constexpr int kV = KC / 4;
        for (int i = tid; i < T * nv; i += blockDim.x) {
            const int t = i / nv, v = i % nv;
            const float* sb = ring + (size_t)(v / kV) * gm.rows * gm.ld + 4 * (v % kV);
            // Already normalised in place when the norm is active.
            const float4 f = *reinterpret_cast<const float4*>(sb + (size_t)(E + t) * gm.ld);
            for (int s2 = 0; s2 < k; ++s2)
                store_row4<kMode>(a_hi, a_lo, (size_t)s_dest[t * k + s2], nv, v, f);
        }
        return;
    }
    constexpr int kU = 16;
    for (int i0 = tid; i0 < T * nv; i0 += kU * blockDim.x) {
        float4 fv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int i = i0 + u * blockDim.x;
            if (i < T * nv) {
                fv[u] = reinterpret_cast<const float4*>(x + (size_t)(i / nv) * d)[i % nv];
                if (norm) fv[u] = nr.apply4(fv[u], i / nv, i % nv);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int i = i0 + u * blockDim.x;
            if (i >= T * nv) break;
            const int t = i / nv, v = i % nv;
            for (int s2 = 0; s2 < k; ++s2)
                store_row4<kMode>(a_hi, a_lo, (size_t)s_dest[t * k + s2], nv, v, fv[u]);
        }
    }
}

// T fits one router block: the permute kernel does the scan as well.
bool single_block(int T) { return T <= kRouteTokens; }


// Token blocks x column splits: enough CTAs (about 4 per SM) to keep tens of
// MB of row loads in flight.
dim3 permute_grid(const Layer& L, int T) {
    const int nblk = (T + kRouteTokens - 1) / kRouteTokens;
    int splits = (4 * L.sm_count + nblk - 1) / nblk;
    const int max_splits = max(1, L.d / 4 / 256);   // at least 256 float4 columns per CTA
    splits = max(1, min(splits, max_splits));
    return dim3(nblk, splits);
}

template <int EJ, int KC, bool kBlk = false>
cudaError_t launch_router_t(const Layer& L, const float* x, int T, float* logits, int* idx,
                            float* wts, int* blockhist, cudaStream_t s, const NormRef& nr,
                            const int* eperm) {
    const int E = L.E_route;
    const int wrows = kBlk ? E : 8 * EJ;
    const size_t smem = sizeof(float) * (4 * (kRouteTokens * (KC + 4) + wrows * (KC + 4) + 2 * KC) +
                                         2 * kRouteTokens + kRouteTokens * (E + 1)) +
                        sizeof(int) * E;
    auto kern = router_kernel<EJ, KC, kBlk>;
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
    if (err != cudaSuccess) return err;
    const int nblk = (T + kRouteTokens - 1) / kRouteTokens;
    // A single block of fewer than 32 tokens runs only the warps it needs
    // (8 threads per token, whole warps): at decode sizes the dependent FMA
    // chain is the critical path and idle warps would only take issue slots.
    const int tok = T < kRouteTokens ? (T + 3) / 4 * 4 : kRouteTokens;
    kern<<<nblk, kBlk ? 2 * E : 8 * tok, smem, s>>>(x, L.wg, L.bias, T, L.d, E, L.k,
                                            L.cfg.router_policy, L.cfg.router_quantum,
                                            L.cfg.router_tie_eps, logits, idx, wts, blockhist, nr,
                                            eperm);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router(const Layer& L, const float* x, int T, float* logits, int* idx,
                          float* wts, int* blockhist, cudaStream_t s, const NormRef& nr,
                          const int* eperm) {
    // K chunk per pipeline stage: as wide as shared memory allows, so each
    // SM keeps 100-200 KB of x / wg loads in flight (the dot-product chains
    // themselves are serial and cannot be split).
    const int ej = (L.E_route + 7) / 8;
    // Expert counts that are multiples of 32: the 4 x 4 register-blocked
    // chains (K chunk sized so two CTAs fit an SM up to 64 experts).
    if (L.E_route % 32 == 0) {
        if (L.E_route <= 128 && L.d % 64 == 0)
            return launch_router_t<1, 64, true>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
        if (L.E_route <= 256 && L.d % 32 == 0)
            return launch_router_t<1, 32, true>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    }
    if (L.d % 256 == 0) {
        if (ej <= 1) return launch_router_t<1, 256>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
        if (ej <= 2) return launch_router_t<2, 256>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    }
    if (L.d % 128 == 0) {
        if (ej <= 1) return launch_router_t<1, 128>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
        if (ej <= 2) return launch_router_t<2, 128>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
        if (ej <= 4) return launch_router_t<4, 128>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
        if (ej <= 8) return launch_router_t<8, 128>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    }
    if (ej <= 1) return launch_router_t<1, 64>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    if (ej <= 2) return launch_router_t<2, 64>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    if (ej <= 4) return launch_router_t<4, 64>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    if (ej <= 8) return launch_router_t<8, 64>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    if (ej <= 16) return launch_router_t<16, 32>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
    return launch_router_t<32, 32>(L, x, T, logits, idx, wts, blockhist, s, nr, eperm);
}

bool route_small_geometry(const Layer& L, int T, bool norm, int* kc_out, int* stages_out) {
    if (T < 1 || T > kSmallMaxTokens || T * L.E_route > kSmallChainThreads || L.E != L.E_route)
        return false;
    const int rows = L.E_route + T + (norm ? 2 : 0);
    for (int kc : {512, 256, 128, 64}) {
        if (L.d % kc) continue;
        // 218 KB of ring plus the kernel's ~7 KB of static shared memory stay
        // under the 227 KB a CTA may hold; that keeps every K chunk resident
        // (the direct-load path) up to T = 4 at d 4096 with 8 experts.
        const size_t stage = (size_t)rows * (kc + 4) * 4;
        const int stages = (int)std::min<size_t>(kSmallMaxStages, (218u << 10) / stage);
        if (stages >= 3) {
            *kc_out = kc;
            *stages_out = stages;
            return true;
        }
    }
    return false;
}

bool route_small_resident(const Layer& L, int kc, int stages) { return L.d / kc <= stages; }

cudaError_t launch_route_small(const Layer& L, const float* x, int T, const NormRef& nr,
                               bool decode, cudaStream_t s, bool rms_inline) {
    const Workspace& W = L.ws;
    const bool norm = nr.mean != nullptr;
    SmallGeom gm;
    if (!route_small_geometry(L, T, norm, &gm.kc, &gm.stages)) return cudaErrorInvalidValue;
    gm.rows = L.E_route + T + (norm ? 2 : 0);
    gm.ld = gm.kc + 4;
    gm.rms_inline = rms_inline && norm && route_small_resident(L, gm.kc, gm.stages);
    if (rms_inline && !gm.rms_inline) return cudaErrorInvalidValue;
    gm.rms_eps = L.norm_eps;
    gm.stat_mean = W.row_mean;
    gm.stat_inv = W.row_inv;
    const size_t smem = (size_t)gm.stages * gm.rows * gm.ld * 4;
    ScanOut so;
    so.counts = W.counts; so.eoff = W.eoff; so.mtiles = W.mtiles;
    so.num_mtiles = W.num_mtiles; so.ptiles = W.ptiles; so.num_ptiles = W.num_ptiles;
    so.row_slot = W.row_slot;
    // All chain warps are launched whatever T x E is: the tail (layout and
    // row copies) uses every thread.
    const int threads = kSmallThreads;
    // Row format: the decode kernels read fp32 (fp32-faithful) or bf16 (BF16)
    // rows, the grouped GEMMs their operand planes.
    const int mode = act_format(L, decode);
    auto launch = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = L.profile ? 0 : 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, x, L.wg, (const float*)L.bias, T, L.d, L.E_route,
                                  L.k, L.cfg.router_policy, L.cfg.router_quantum,
                                  L.cfg.router_tie_eps, nr, gm, W.logits, W.idx, W.wts, so,
                                  W.row_token, W.row_weight, W.a_hi, W.a_lo, W.dev_err);
    };
    auto by_kc = [&](auto mode_c, auto norm_c) {
        constexpr int M = decltype(mode_c)::value;
        constexpr bool N = decltype(norm_c)::value;
        if (gm.kc == 512) return launch(router_small_kernel<M, 512, N>);
        if (gm.kc == 256) return launch(router_small_kernel<M, 256, N>);
        if (gm.kc == 128) return launch(router_small_kernel<M, 128, N>);
        return launch(router_small_kernel<M, 64, N>);
    };
    using T0 = std::integral_constant<int, kActBf16>;
    using T1 = std::integral_constant<int, kActTf32x2>;
    using T2 = std::integral_constant<int, kActF32>;
    using T3 = std::integral_constant<int, kActBf16x2>;
    using NF = std::false_type;
    using NT = std::true_type;
    if (mode == kActBf16) return norm ? by_kc(T0{}, NT{}) : by_kc(T0{}, NF{});
    if (mode == kActTf32x2) return norm ? by_kc(T1{}, NT{}) : by_kc(T1{}, NF{});
    if (mode == kActBf16x2) return norm ? by_kc(T3{}, NT{}) : by_kc(T3{}, NF{});
    return norm ? by_kc(T2{}, NT{}) : by_kc(T2{}, NF{});
}

cudaError_t launch_dispatch_scan(const Layer& L, int T, cudaStream_t s) {
    const int nblk = (T + kRouteTokens - 1) / kRouteTokens;
    const Workspace& W = L.ws;
    dispatch_scan_kernel<<<1, kScanThreads, 0, s>>>(W.blockhist, nblk, L.E_route, kTileM, W.counts,
                                                  W.eoff, W.mtiles, W.num_mtiles, W.ptiles,
                                                  W.num_ptiles, W.row_token, W.row_weight);
    return cudaGetLastError();
}

cudaError_t launch_scan_generic(int* hist, int nblk, int E, int granule, int* counts, int* eoff,
                                MTile* mtiles, int* num_mtiles, MTile* ptiles, int* num_ptiles,
                                int* row_token, float* row_weight, cudaStream_t s) {
    dispatch_scan_kernel<<<1, kScanThreads, 0, s>>>(hist, nblk, E, granule, counts, eoff, mtiles,
                                                  num_mtiles, ptiles, num_ptiles, row_token,
                                                  row_weight);
    return cudaGetLastError();
}

cudaError_t launch_dispatch_permute_raw(const Layer& L, const float* x, int T, cudaStream_t s,
                                        const NormRef& nr) {
    const Workspace& W = L.ws;
    const dim3 grid = permute_grid(L, T);
    ScanOut so;
    if (single_block(T)) {
        so.counts = W.counts; so.eoff = W.eoff; so.mtiles = W.mtiles;
        so.num_mtiles = W.num_mtiles; so.ptiles = W.ptiles; so.num_ptiles = W.num_ptiles;
    }
    so.row_slot = W.row_slot;
    if (fp32_faithful(L))
        dispatch_permute_kernel<kActF32><<<grid, 256, 0, s>>>(x, T, L.d, L.E_route, L.k, W.idx,
                                                              W.wts, W.blockhist, W.eoff,
                                                              W.row_token, W.row_weight, W.a_hi,
                                                              nullptr, so, nr);
    else
        dispatch_permute_kernel<kActBf16><<<grid, 256, 0, s>>>(x, T, L.d, L.E_route, L.k, W.idx,
                                                               W.wts, W.blockhist, W.eoff,
                                                               W.row_token, W.row_weight, W.a_hi,
                                                               nullptr, so, nr);
    return cudaGetLastError();
}

cudaError_t launch_dispatch_permute_to(const Layer& L, const float* x, int T, int E,
                                       const int* eoff, int* row_token, float* row_weight,
                                       int* slot_row, void* rows, cudaStream_t s) {
    const Workspace& W = L.ws;
    const dim3 grid = permute_grid(L, T);
    ScanOut so;
    so.slot_row = slot_row;
    // Rows on the wire: fp32 in the fp32-faithful precisions, else bf16.
    if (fp32_faithful(L))
        dispatch_permute_kernel<kActF32><<<grid, 256, 0, s>>>(x, T, L.d, E, L.k, W.idx, W.wts,
                                                              W.blockhist, eoff, row_token,
                                                              row_weight, rows, nullptr, so,
                                                              NormRef{});
    else
        dispatch_permute_kernel<kActBf16><<<grid, 256, 0, s>>>(x, T, L.d, E, L.k, W.idx, W.wts,
                                                               W.blockhist, eoff, row_token,
                                                               row_weight, rows, nullptr, so,
                                                               NormRef{});
    return cudaGetLastError();
}

cudaError_t launch_dispatch_permute(const Layer& L, const float* x, int T, cudaStream_t s,
                                    const NormRef& nr) {
    const Workspace& W = L.ws;
    const dim3 grid = permute_grid(L, T);
    ScanOut so;
    if (single_block(T)) {
        so.counts = W.counts; so.eoff = W.eoff; so.mtiles = W.mtiles;
        so.num_mtiles = W.num_mtiles; so.ptiles = W.ptiles; so.num_ptiles = W.num_ptiles;
    }
    so.row_slot = W.row_slot;
    auto run = [&](auto kern) {
        kern<<<grid, 256, 0, s>>>(x, T, L.d, L.E_route, L.k, W.idx, W.wts, W.blockhist, W.eoff,
                                  W.row_token, W.row_weight, W.a_hi, W.a_lo, so, nr);
    };
    switch (act_format(L, false)) {
        case kActTf32x2: run(dispatch_permute_kernel<kActTf32x2>); break;
        case kActBf16x2: run(dispatch_permute_kernel<kActBf16x2>); break;
        default: run(dispatch_permute_kernel<kActBf16>); break;
    }
    return cudaGetLastError();
}

}  // namespace moe
