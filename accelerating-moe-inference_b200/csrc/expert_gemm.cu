// Grouped expert GEMMs on tcgen05 tensor cores.
//
// gate/up:  H[r, j] = silu(A[r] . w1[e, j]) * (A[r] . w3[e, j])
//           A = packed activations (rows grouped by expert), B = w13[e], the
//           row-interleaved gate/up weights: one 128 x 256 tile gives the gate
//           and up values of the same 128 intermediate columns, so SwiGLU is
//           applied in the epilogue straight out of TMEM.  Replaces
//           gemm_grouped<true,true> (src/model.cu:618-643) and
//           PhiMLP::forward's w1/w3/silu/mul (src/layer.cu:32-41).
// down:     out[r] = H[r] . w2[e], stored unweighted at the row's selection
//           slot (part[split][row_slot[r]]) for the ordered combine
//           (combine.cu), which adds a token's k rows in ascending expert
//           order with the reference's fma -- the combine of
//           gemm_grouped_combine<1,2> (src/model.cu:645-667, 417-449) and of
//           src/layer.cu:100-101, independent of the tile schedule.  Two
//           other epilogues serve the decoder's dense projections (add
//           weight * out into y[row_token[r]]) and the NCCL expert-parallel
//           transport (store out at y[row_token[r]]).
//
// One persistent CTA per SM, 6 warps:
//   warp 0      TMA producer (one thread): A and B K-blocks into a ring of
//               shared-memory stages, completion on a per-stage mbarrier.
//   warp 1      MMA issuer (one thread) and TMEM owner: tcgen05.mma
//               128 x 256 x (32 bytes of K) per instruction into one of two
//               256-column fp32 accumulators in TMEM; tcgen05.commit releases
//               smem stages and hands finished accumulators to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, one row per thread.
// Precision (GemmPrec): BF16 (kind::f16, 64 bf16 per 128-byte K-block, 4
// stages); FP32 as 3xTF32 (kind::tf32 on hi/lo planes: lo*hi + hi*lo + hi*hi,
// 32 fp32 per K-block, 2 stages); FP32_BF16X3 (kind::f16 on bf16 hi/lo
// planes, the same three products at the bf16 rate, 64 per K-block, 2
// stages).  All use 128-byte-swizzled K-major tiles.
#include <cuda_bf16.h>

#include <algorithm>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

enum Epi { kEpiGateUp = 0, kEpiDown = 1, kEpiDownStore = 2, kEpiDownSlot = 3 };

struct GemmParams {
    const MTile* mtiles;
    const int* num_mtiles;
    int n_tiles;       // N tiles per expert
    int k_blocks;      // K / (elements per 128-byte block)
    int k_splits;      // K splits per tile (down with the adding epilogue only; else 1)
    int kb_per;        // K blocks per split; k_splits = ceil(k_blocks / kb_per), none empty
    int b_rows_per_expert;
    // gate/up epilogue
    void* h_hi;
    void* h_lo;
    int ldh;           // padded d_ff
    // down epilogue
    const int* row_token;
    const float* row_weight;
    float* y;          // Down: [T][d] accumulated; DownStore: [rows][d], row row_token[prow]
    const int* row_slot;   // DownSlot: packed row -> selection slot
    float* part;           // DownSlot: [k_splits][slots][d]
    size_t split_stride;   // DownSlot: floats between the splits' planes
    int d;
    int* err;
};

constexpr int kThreads = 192;
constexpr int kABytes = kTileM * 128;   // one A plane per stage: 128 rows x 128 B
constexpr int kBBytes = kTileN * 128;   // one B plane per stage: 256 rows x 128 B
constexpr int kAccCols = kTileN;        // fp32 columns per accumulator
constexpr int kTmemCols = 2 * kAccCols;

// kP: GemmPrec.  Two-plane schemes issue three MMAs per K step.
template <int kP>
struct Cfg {
    static constexpr int kPlanes = kP == kGemmBf16 ? 1 : 2;
    static constexpr bool kTfKind = kP == kGemm3xTf32;
    static constexpr int kElems = kTfKind ? 32 : 64;   // K elements per 128-byte block
    static constexpr int kStageBytes = kPlanes * (kABytes + kBBytes);
    static constexpr int kStages = kPlanes == 2 ? 2 : 4;
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // barriers + alignment slack
    static constexpr uint32_t kIdesc = mma_idesc(kTfKind ? 2u : 1u, kTileM, kTileN);
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

// Tile order: expert by expert; inside an expert, n-tile major and m-tile
// minor.  The CTAs running at once then share one expert's activation rows
// (which stay in L2) and each weight tile is fetched from HBM once, by the
// m-tiles of its expert running side by side.
struct TileCoord {
    int mt;
    int nt;
};
__device__ __forceinline__ TileCoord decode_tile(const MTile* __restrict__ mtiles, int t,
                                                 int n_tiles) {
    const MTile& head = mtiles[t / n_tiles];
    const int local = t - head.mstart * n_tiles;
    TileCoord c;
    c.nt = local / head.mcount;
    c.mt = head.mstart + local % head.mcount;
    return c;
}

// One accumulator tile out of TMEM for the calling warp's 32 rows: lane i
// holds row (lane quarter base + i); `valid` rows are written.  tcgen05.ld is
// warp-collective, so every lane runs the loads.
template <int kP, int kEpi>
__device__ __forceinline__ void epilogue_rows(const GemmParams& p, uint32_t tbase, bool valid,
                                              size_t prow, int nt, int split) {
    if constexpr (kEpi == kEpiGateUp) {
#pragma unroll 1
        for (int c = 0; c < kTileN / 2; c += 32) {
            uint32_t g[32], u[32];
            tmem_ld32(tbase + c, g);
            tmem_ld32(tbase + kTileN / 2 + c, u);
            tmem_ld_wait();
            const int col = nt * (kTileN / 2) + c;
            if (valid) {
                if constexpr (kP == kGemm3xTf32) {
                    float4* dh = reinterpret_cast<float4*>(
                        static_cast<float*>(p.h_hi) + prow * p.ldh + col);
                    float4* dl = reinterpret_cast<float4*>(
                        static_cast<float*>(p.h_lo) + prow * p.ldh + col);
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 hv, lv;
                        float h0 = silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
                        float h1 = silu_f(__uint_as_float(g[j + 1])) * __uint_as_float(u[j + 1]);
                        float h2 = silu_f(__uint_as_float(g[j + 2])) * __uint_as_float(u[j + 2]);
                        float h3 = silu_f(__uint_as_float(g[j + 3])) * __uint_as_float(u[j + 3]);
                        hv.x = to_tf32(h0); lv.x = to_tf32(h0 - hv.x);
                        hv.y = to_tf32(h1); lv.y = to_tf32(h1 - hv.y);
                        hv.z = to_tf32(h2); lv.z = to_tf32(h2 - hv.z);
                        hv.w = to_tf32(h3); lv.w = to_tf32(h3 - hv.w);
                        dh[j / 4] = hv;
                        dl[j / 4] = lv;
                    }
                } else if constexpr (kP == kGemmBf16x3) {
                    const size_t off = prow * p.ldh + col;
                    uint4* dh = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.h_hi) + off);
                    uint4* dl = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.h_lo) + off);
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint32_t hw[4], lw[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float a = silu_f(__uint_as_float(g[j + 2 * i])) *
                                            __uint_as_float(u[j + 2 * i]);
                            const float b = silu_f(__uint_as_float(g[j + 2 * i + 1])) *
                                            __uint_as_float(u[j + 2 * i + 1]);
                            split_bf16x2(a, b, hw[i], lw[i]);
                        }
                        dh[j / 8] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                        dl[j / 8] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    }
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(
                        static_cast<__nv_bfloat16*>(p.h_hi) + prow * p.ldh + col);
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint32_t w4[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float a = silu_f(__uint_as_float(g[j + 2 * i])) *
                                            __uint_as_float(u[j + 2 * i]);
                            const float b = silu_f(__uint_as_float(g[j + 2 * i + 1])) *
                                            __uint_as_float(u[j + 2 * i + 1]);
                            __nv_bfloat162 v2 = __floats2bfloat162_rn(a, b);
                            w4[i] = *reinterpret_cast<uint32_t*>(&v2);
                        }
                        dst[j / 8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
            }
        }
    } else if constexpr (kEpi == kEpiDownSlot) {
        // The row's result, unweighted and in fp32, at its selection slot.
        const int slot = valid ? p.row_slot[prow] : 0;
        float* rowp = p.part + (size_t)split * p.split_stride + (size_t)slot * p.d;
#pragma unroll 1
        for (int c = 0; c < kTileN; c += 32) {
            uint32_t v[32];
            tmem_ld32(tbase + c, v);
            tmem_ld_wait();
            const int col = nt * kTileN + c;
            if (valid && col < p.d) {
                float4* out = reinterpret_cast<float4*>(rowp + col);
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    out[j / 4] = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                             __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
            }
        }
    } else if constexpr (kEpi == kEpiDownStore) {
        // Expert parallelism (NCCL transport): each row's result is stored
        // at the row it arrived in -- fp32 in FP32 precision, bf16 in BF16
        // precision (half the return bytes).
        const int dst = valid ? p.row_token[prow] : 0;
        constexpr bool kF32 = kP != kGemmBf16;   // fp32-faithful precisions return fp32
        constexpr size_t kEs = kF32 ? 4 : 2;
        char* rowp = reinterpret_cast<char*>(p.y) + static_cast<size_t>(dst) * p.d * kEs;
#pragma unroll 1
        for (int c = 0; c < kTileN; c += 32) {
            uint32_t v[32];
            tmem_ld32(tbase + c, v);
            tmem_ld_wait();
            const int col = nt * kTileN + c;
            if (valid && col < p.d) {
                if constexpr (kF32) {
                    float4* out = reinterpret_cast<float4*>(rowp) + col / 4;
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        out[j / 4] = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]),
                                                 __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]));
                } else {
                    uint4* out = reinterpret_cast<uint4*>(rowp) + col / 8;
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint32_t w4[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(v[j + 2 * i]),
                                                                      __uint_as_float(v[j + 2 * i + 1]));
                            w4[i] = *reinterpret_cast<uint32_t*>(&b2);
                        }
                        out[j / 8] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                    }
                }
            }
        }
    } else {
        int tok = 0;
        float wgt = 0.0f;
        if (valid) {
            tok = p.row_token[prow];
            wgt = p.row_weight[prow];
        }
#pragma unroll 1
        for (int c = 0; c < kTileN; c += 32) {
            uint32_t v[32];
            tmem_ld32(tbase + c, v);
            tmem_ld_wait();
            const int col = nt * kTileN + c;
            if (valid && col < p.d) {
                float* dst = p.y + static_cast<size_t>(tok) * p.d + col;
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    float4 o;
                    o.x = wgt * __uint_as_float(v[j]);
                    o.y = wgt * __uint_as_float(v[j + 1]);
                    o.z = wgt * __uint_as_float(v[j + 2]);
                    o.w = wgt * __uint_as_float(v[j + 3]);
                    atomicAdd(reinterpret_cast<float4*>(dst + j), o);
                }
            }
        }
    }
}

template <int kP, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
expert_gemm_kernel(const __grid_constant__ CUtensorMap tmA_hi,
                   const __grid_constant__ CUtensorMap tmA_lo,
                   const __grid_constant__ CUtensorMap tmB_hi,
                   const __grid_constant__ CUtensorMap tmB_lo, const GemmParams p) {
    using C = Cfg<kP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint64_t* empty = full + C::kStages;
    uint64_t* tfull = empty + C::kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 4);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA_hi);
        tma_prefetch_desc(&tmB_hi);
        if constexpr (C::kPlanes == 2) {
            tma_prefetch_desc(&tmA_lo);
            tma_prefetch_desc(&tmB_lo);
        }
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything below reads what the previous kernel on the stream wrote.
    wait_predecessor_grid();

    const int m_tiles = *p.num_mtiles;
    // Work items: tiles x K splits, the split fastest, so the splits of one
    // tile (which share its activation rows) run side by side.
    const int total = m_tiles * p.n_tiles * p.k_splits;
    const int kb_per = p.kb_per;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------ TMA producer
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            // Activation rows are re-read by every N tile of their expert over
            // the whole expert's run, while the weights stream past: keep the
            // activations in L2 (evict_last; 6% fewer DRAM reads for bf16x3
            // gate/up at config-2 shapes).  Weights keep the default policy --
            // evict_first doubled their reads, since the M tiles sharing a
            // weight tile do not read it at the same instant.
            const uint64_t pol_a = l2_policy_evict_last();
            const uint64_t pol_b = 0;
            for (int t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x) {
                const TileCoord tc = decode_tile(p.mtiles, t / p.k_splits, p.n_tiles);
                const int mt = tc.mt, nt = tc.nt;
                const MTile tile = p.mtiles[mt];
                const int brow = tile.expert * p.b_rows_per_expert + nt * kTileN;
                constexpr int kElems = C::kElems;
                const int kb0 = (t % p.k_splits) * kb_per;
                const int kb1 = min(p.k_blocks, kb0 + kb_per);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, kDevErrTimeoutProducer)) {
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* sbase = smem + stage * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
                    const int kx = kb * kElems;
                    auto ld = [&](uint8_t* dst, const CUtensorMap* tm, int y, uint64_t pol) {
                        if (pol) tma_load_2d_hint(dst, tm, &full[stage], kx, y, pol);
                        else tma_load_2d(dst, tm, &full[stage], kx, y);
                    };
                    ld(sbase, &tmA_hi, tile.row0, pol_a);
                    if constexpr (C::kPlanes == 2) {
                        ld(sbase + kABytes, &tmA_lo, tile.row0, pol_a);
                        ld(sbase + 2 * kABytes, &tmB_hi, brow, pol_b);
                        ld(sbase + 2 * kABytes + kBBytes, &tmB_lo, brow, pol_b);
                    } else {
                        ld(sbase + kABytes, &tmB_hi, brow, pol_b);
                    }
                    ++issued;
                    if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (*abort_flag) {
                // Let every load already issued land before the CTA leaves.
                const int pending = issued < C::kStages ? issued : C::kStages;
                int s = stage;
                uint32_t ph = phase;
                for (int i = 0; i < pending; ++i) {
                    if (--s < 0) { s = C::kStages - 1; ph ^= 1u; }
                    mbar_wait(&full[s], ph, p.err, kDevErrTimeoutDrain);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------ MMA issuer
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err, kDevErrTimeoutMma)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kAccCols;
                bool ok = true;
                const int kb0 = (t % p.k_splits) * kb_per;
                const int kb1 = min(p.k_blocks, kb0 + kb_per);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&full[stage], phase, p.err, kDevErrTimeoutMma)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(smem + stage * C::kStageBytes);
                    const uint64_t a_hi = smem_desc_sw128(sbase);
                    uint64_t a_lo = 0, b_hi, b_lo = 0;
                    if constexpr (C::kPlanes == 2) {
                        a_lo = smem_desc_sw128(sbase + kABytes);
                        b_hi = smem_desc_sw128(sbase + 2 * kABytes);
                        b_lo = smem_desc_sw128(sbase + 2 * kABytes + kBBytes);
                    } else {
                        b_hi = smem_desc_sw128(sbase + kABytes);
                    }
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        // 32 bytes of K per instruction: +2 in the >>4 address field.
                        const uint64_t off = static_cast<uint64_t>(ks * 2);
                        const uint32_t accum = (kb != kb0 || ks != 0) ? 1u : 0u;
                        if constexpr (C::kPlanes == 2) {
                            // Small products first: lo*hi, hi*lo, then hi*hi.
                            tc_mma<C::kTfKind>(d_tmem, a_lo + off, b_hi + off, C::kIdesc, accum);
                            tc_mma<C::kTfKind>(d_tmem, a_hi + off, b_lo + off, C::kIdesc, 1u);
                            tc_mma<C::kTfKind>(d_tmem, a_hi + off, b_hi + off, C::kIdesc, 1u);
                        } else {
                            tc_mma<false>(d_tmem, a_hi + off, b_hi + off, C::kIdesc, accum);
                        }
                    }
                    tc_commit(&empty[stage]);
                    if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            // Every MMA issued by this thread has completed once `done` fires.
            tc_commit(done);
            mbar_wait(done, 0, p.err, kDevErrTimeoutDrain);
        }
    } else {
        // ---------------------------------------------------- epilogue
        const int q = warp & 3;            // TMEM lane quarter this warp may read
        const int row_in_tile = q * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            // Exit decisions are warp-uniform: tcgen05.ld below is .sync.aligned.
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const TileCoord tc = decode_tile(p.mtiles, t / p.k_splits, p.n_tiles);
            const int mt = tc.mt, nt = tc.nt;
            const bool ready = mbar_wait(&tfull[acc], acc_phase, p.err, kDevErrTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, ready)) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const MTile tile = p.mtiles[mt];
            const bool valid = row_in_tile < tile.rows;
            const size_t prow = static_cast<size_t>(tile.row0 + row_in_tile);
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kAccCols);
            epilogue_rows<kP, kEpi>(p, tbase, valid, prow, nt, t % p.k_splits);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------ CTA-pair GEMM
// The same grouped GEMM on 256 x 256 tiles computed by a 2-CTA cluster with
// tcgen05.mma.cta_group::2: each CTA loads 128 rows of A and 128 rows (half
// the N tile) of B into its own shared memory, the leader CTA issues the MMAs
// (which read both CTAs' operands) and each CTA's TMEM holds its 128 rows x
// 256 columns of the accumulator.  Per SM this halves the B traffic from L2
// and shared memory.  Barrier protocol:
//   full[s]    leader only; its producer arms it with both CTAs' bytes, both
//              CTAs' TMA loads complete on it (cluster address of rank 0);
//   empty[s]   both CTAs; the leader's commit arrives on both;
//   tfull[a]   both CTAs; the leader's commit arrives on both;
//   tempty[a]  leader only; 4 epilogue warps x 2 CTAs arrive.
template <int kP>
struct PairCfg {
    static constexpr int kPlanes = kP == kGemmBf16 ? 1 : 2;
    static constexpr bool kTfKind = kP == kGemm3xTf32;
    static constexpr int kElems = kTfKind ? 32 : 64;
    static constexpr int kHalfA = kTileM * 128;          // 128 rows of A
    static constexpr int kHalfB = (kTileN / 2) * 128;    // 128 rows of B
    static constexpr int kStageBytes = kPlanes * (kHalfA + kHalfB);
    static constexpr int kStages = kPlanes == 2 ? 3 : 6;
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kSmemBytes = kBarOffset + 256 + 1024;
    static constexpr uint32_t kIdesc = mma_idesc(kTfKind ? 2u : 1u, 2 * kTileM, kTileN);
};

template <int kP, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
expert_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA_hi,
                        const __grid_constant__ CUtensorMap tmA_lo,
                        const __grid_constant__ CUtensorMap tmB_hi,
                        const __grid_constant__ CUtensorMap tmB_lo, const GemmParams p) {
    using C = PairCfg<kP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
    uint64_t* empty = full + C::kStages;
    uint64_t* tfull = empty + C::kStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();
    const bool leader = crank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], 8);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA_hi);
        tma_prefetch_desc(&tmB_hi);
        if constexpr (C::kPlanes == 2) {
            tma_prefetch_desc(&tmA_lo);
            tma_prefetch_desc(&tmB_lo);
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();                     // barriers of both CTAs initialised
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything below reads what the previous kernel on the stream wrote.
    wait_predecessor_grid();

    const int p_tiles = *p.num_mtiles;  // pair tiles (num_ptiles)
    const int total = p_tiles * p.n_tiles;
    const int cid = blockIdx.x >> 1;
    const int nclusters = gridDim.x >> 1;
    const uint32_t full0 = mapa_shared(&full[0], 0);     // leader's full[0]
    const uint32_t tempty0 = mapa_shared(&tempty[0], 0); // leader's tempty[0]

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            constexpr int kElems = C::kElems;
            // Activation rows are re-read by every N tile of their expert over
            // the whole expert's run, while the weights stream past: keep the
            // activations in L2 (evict_last; 6% fewer DRAM reads for bf16x3
            // gate/up at config-2 shapes).  Weights keep the default policy --
            // evict_first doubled their reads, since the M tiles sharing a
            // weight tile do not read it at the same instant.
            const uint64_t pol_a = l2_policy_evict_last();
            const uint64_t pol_b = 0;
            for (int t = cid; t < total && !*abort_flag; t += nclusters) {
                const TileCoord tc = decode_tile(p.mtiles, t, p.n_tiles);
                const MTile tile = p.mtiles[tc.mt];
                const int arow = tile.row0 + (int)crank * kTileM;
                const int brow = tile.expert * p.b_rows_per_expert + tc.nt * kTileN +
                                 (int)crank * (kTileN / 2);
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, kDevErrTimeoutProducer)) {
                        *abort_flag = 1;
                        break;
                    }
                    uint8_t* sbase = smem + stage * C::kStageBytes;
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::kStageBytes);
                    const uint32_t fb = full0 + stage * 8;
                    const int kx = kb * kElems;
                    auto ld = [&](uint8_t* dst, const CUtensorMap* tm, int y, uint64_t pol) {
                        if (pol) tma_load_2d_pair_hint(dst, tm, fb, kx, y, pol);
                        else tma_load_2d_pair(dst, tm, fb, kx, y);
                    };
                    ld(sbase, &tmA_hi, arow, pol_a);
                    if constexpr (C::kPlanes == 2) {
                        ld(sbase + C::kHalfA, &tmA_lo, arow, pol_a);
                        ld(sbase + 2 * C::kHalfA, &tmB_hi, brow, pol_b);
                        ld(sbase + 2 * C::kHalfA + C::kHalfB, &tmB_lo, brow, pol_b);
                    } else {
                        ld(sbase + C::kHalfA, &tmB_hi, brow, pol_b);
                    }
                    ++issued;
                    if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
                }
            }
            if (*abort_flag && leader) {
                const int pending = issued < C::kStages ? issued : C::kStages;
                int s = stage;
                uint32_t ph = phase;
                for (int i = 0; i < pending; ++i) {
                    if (--s < 0) { s = C::kStages - 1; ph ^= 1u; }
                    mbar_wait(&full[s], ph, p.err, kDevErrTimeoutDrain);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int t = cid; t < total && !*abort_flag; t += nclusters) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err, kDevErrTimeoutMma)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kAccCols;
                bool ok = true;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, p.err, kDevErrTimeoutMma)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sbase = smem_u32(smem + stage * C::kStageBytes);
                    const uint64_t a_hi = smem_desc_sw128(sbase);
                    uint64_t a_lo = 0, b_hi, b_lo = 0;
                    if constexpr (C::kPlanes == 2) {
                        a_lo = smem_desc_sw128(sbase + C::kHalfA);
                        b_hi = smem_desc_sw128(sbase + 2 * C::kHalfA);
                        b_lo = smem_desc_sw128(sbase + 2 * C::kHalfA + C::kHalfB);
                    } else {
                        b_hi = smem_desc_sw128(sbase + C::kHalfA);
                    }
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t off = static_cast<uint64_t>(ks * 2);
                        const uint32_t accum = (kb | ks) != 0 ? 1u : 0u;
                        if constexpr (C::kPlanes == 2) {
                            tc_mma_pair<C::kTfKind>(d_tmem, a_lo + off, b_hi + off, C::kIdesc, accum);
                            tc_mma_pair<C::kTfKind>(d_tmem, a_hi + off, b_lo + off, C::kIdesc, 1u);
                            tc_mma_pair<C::kTfKind>(d_tmem, a_hi + off, b_hi + off, C::kIdesc, 1u);
                        } else {
                            tc_mma_pair<false>(d_tmem, a_hi + off, b_hi + off, C::kIdesc, accum);
                        }
                    }
                    tc_commit_pair(&empty[stage], 0x3);
                    if (++stage == C::kStages) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                tc_commit_pair(&tfull[acc], 0x3);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            tc_commit_pair(done, 0x1);
            mbar_wait(done, 0, p.err, kDevErrTimeoutDrain);
        }
    } else {
        const int q = warp & 3;
        const int row_in_tile = q * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = cid; t < total; t += nclusters) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const TileCoord tc = decode_tile(p.mtiles, t, p.n_tiles);
            const bool ready = mbar_wait(&tfull[acc], acc_phase, p.err, kDevErrTimeoutEpilogue);
            if (!__all_sync(0xffffffffu, ready)) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const MTile tile = p.mtiles[tc.mt];
            const int half_rows = crank == 0 ? tile.rows : tile.pad[0];
            const bool valid = row_in_tile < half_rows;
            const size_t prow = static_cast<size_t>(tile.row0 + (int)crank * kTileM + row_in_tile);
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kAccCols);
            epilogue_rows<kP, kEpi>(p, tbase, valid, prow, tc.nt, 0);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + acc * 8);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();                     // the leader's MMAs (which read both CTAs) are done
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

template <int kP, int kEpi>
cudaError_t launch_pair(const CUtensorMap& a_hi, const CUtensorMap& a_lo, const CUtensorMap& b_hi,
                        const CUtensorMap& b_lo, const GemmParams& p, int clusters,
                        bool pdl, cudaStream_t s) {
    using C = PairCfg<kP>;
    auto kern = expert_gemm_pair_kernel<kP, kEpi>;
    cudaError_t err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a_hi, a_lo, b_hi, b_lo, p);
}

template <int kP, int kEpi>
cudaError_t launch_one(const Layer& L, const CUtensorMap& a_hi, const CUtensorMap& a_lo,
                       const CUtensorMap& b_hi, const CUtensorMap& b_lo, const GemmParams& p,
                       int grid, cudaStream_t s) {
    using C = Cfg<kP>;
    auto kern = expert_gemm_kernel<kP, kEpi>;
    cudaError_t err =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (err != cudaSuccess) return err;
    // Dependent launch: the kernel waits for its predecessor itself, after
    // its prologue (barriers, TMEM); the stage timers turn it off.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.profile ? 0 : 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a_hi, a_lo, b_hi, b_lo, p);
}

// One template instantiation per (precision, epilogue) for each tile shape.
template <int kP, int kEpi>
cudaError_t dispatch_shape(const Layer& L, bool pair, const GemmParams& g, int clusters,
                           int grid, cudaStream_t s) {
    const Workspace& W = L.ws;
    constexpr bool two = kP != kGemmBf16;
    const bool gu = kEpi == kEpiGateUp;
    const CUtensorMap& a_hi = gu ? W.tm_a_hi : W.tm_h_hi;
    const CUtensorMap& a_lo = two ? (gu ? W.tm_a_lo : W.tm_h_lo) : a_hi;
    if (pair) {
        const CUtensorMap& b_hi = gu ? L.tm_w13_hi2 : L.tm_w2_hi2;
        const CUtensorMap& b_lo = two ? (gu ? L.tm_w13_lo2 : L.tm_w2_lo2) : b_hi;
        return launch_pair<kP, kEpi>(a_hi, a_lo, b_hi, b_lo, g, clusters, !L.profile, s);
    }
    const CUtensorMap& b_hi = gu ? L.tm_w13_hi : L.tm_w2_hi;
    const CUtensorMap& b_lo = two ? (gu ? L.tm_w13_lo : L.tm_w2_lo) : b_hi;
    return launch_one<kP, kEpi>(L, a_hi, a_lo, b_hi, b_lo, g, grid, s);
}

template <int kP>
cudaError_t dispatch_mode(const Layer& L, int mode, bool pair, const GemmParams& g, int clusters,
                          int grid, cudaStream_t s) {
    switch (mode) {
        case 0: return dispatch_shape<kP, kEpiGateUp>(L, pair, g, clusters, grid, s);
        case 1: return dispatch_shape<kP, kEpiDown>(L, pair, g, clusters, grid, s);
        case 2: return dispatch_shape<kP, kEpiDownStore>(L, pair, g, clusters, grid, s);
        default: return dispatch_shape<kP, kEpiDownSlot>(L, pair, g, clusters, grid, s);
    }
}

cudaError_t dispatch_prec(const Layer& L, int mode, bool pair, const GemmParams& g,
                          int clusters, int grid, cudaStream_t s) {
    switch (gemm_prec(L)) {
        case kGemm3xTf32: return dispatch_mode<kGemm3xTf32>(L, mode, pair, g, clusters, grid, s);
        case kGemmBf16x3: return dispatch_mode<kGemmBf16x3>(L, mode, pair, g, clusters, grid, s);
        default: return dispatch_mode<kGemmBf16>(L, mode, pair, g, clusters, grid, s);
    }
}

}  // namespace

cudaError_t launch_expert_gemm_rows(const Layer& L, int routed_rows, float* y, cudaStream_t s,
                                    int mode, size_t split_stride, int* nsplit) {
    const bool down = mode != 0;
    const Workspace& W = L.ws;
    const int elems = kblock_elems(L);
    const int max_mtiles = (routed_rows + kTileM - 1) / kTileM + L.E;

    GemmParams g{};
    g.mtiles = W.mtiles;
    g.num_mtiles = W.num_mtiles;
    g.err = W.dev_err;
    g.row_token = W.row_token;
    g.row_weight = W.row_weight;
    g.y = y;
    g.row_slot = W.row_slot;
    g.part = W.part;
    g.split_stride = split_stride;
    g.d = L.d;
    g.h_hi = W.h_hi;
    g.h_lo = W.h_lo;
    g.ldh = L.ffp;
    g.k_splits = 1;
    if (!down) {
        // gate/up: N = 2 * ffp per expert, K = d.
        g.n_tiles = 2 * L.ffp / kTileN;
        g.k_blocks = L.d / elems;
        g.b_rows_per_expert = 2 * L.ffp;
    } else {
        // down: N = d per expert, K = ffp.
        g.n_tiles = (L.d + kTileN - 1) / kTileN;
        g.k_blocks = L.ffp / elems;
        g.b_rows_per_expert = L.d;
    }
    g.kb_per = g.k_blocks;
    if (nsplit) *nsplit = 1;
    // CTA-pair tiles pay off when experts have at least 256 routed rows on
    // average; below that (decode-sized T) most of a 256-row tile would be
    // padding and the 1-CTA tiles spread the weight stream over twice as many
    // SMs.
    const bool pair = L.gemm_variant == MOE_GEMM_CTA_PAIR ||
                      (L.gemm_variant == MOE_GEMM_AUTO && routed_rows >= 2 * kTileM * L.E);
    if (pair) {
        // CTA-pair tiles: 256 rows x 256 columns per 2-SM cluster.
        g.mtiles = W.ptiles;
        g.num_mtiles = W.num_ptiles;
        int clusters = ((routed_rows + 2 * kTileM - 1) / (2 * kTileM) + L.E) * g.n_tiles;
        if (clusters > L.sm_count / 2) clusters = L.sm_count / 2;
        return dispatch_prec(L, mode, true, g, clusters, 0, s);
    }
    // Decode-sized batches leave the down GEMM with few tiles (d / 256 per
    // routed expert), too few to keep every SM streaming weights: split K
    // until there are about two work items per SM.  Each split's partial
    // goes to its own plane (slot epilogue; the ordered combine adds the
    // planes in split order) or is added into y (dense projections).
    const bool can_split = mode == 1 || (mode == 3 && split_stride > 0);
    if (can_split && routed_rows <= kSplitMaxRows) {
        const int tiles = std::min(routed_rows, L.E) * g.n_tiles;
        int ks = (2 * L.sm_count) / std::max(tiles, 1);
        ks = std::max(1, std::min(ks, g.k_blocks / kSplitMinBlocks));
        g.kb_per = (g.k_blocks + ks - 1) / ks;
        g.k_splits = (g.k_blocks + g.kb_per - 1) / g.kb_per;
        if (nsplit) *nsplit = g.k_splits;
    }
    int grid = max_mtiles * g.n_tiles * g.k_splits;
    if (grid > L.sm_count) grid = L.sm_count;
    return dispatch_prec(L, mode, false, g, 0, grid, s);
}

}  // namespace moe
