// Internal declarations shared by the translation units of libmoe_b200.so.
//
// HBM layout of one layer (all row-major, 256-byte aligned allocations):
//   router    wg [E][d] fp32, bias [E] fp32
//   gate/up   w13 [E][2*ffp][d]: per 128-row block b of the padded d_ff
//             (ffp = d_ff rounded up to 128), rows [256b, 256b+128) are
//             w1 rows [128b, 128b+128) and rows [256b+128, 256b+256) are the
//             matching w3 rows, so one 256-wide MMA tile holds the gate and
//             up halves of the same 128 intermediate columns.  Padding rows
//             are zero.
//   down      w2 [E][d][ffp], padding columns zero.
//   BF16 precision stores these once in bf16.  FP32 precision stores a tf32
//   "hi" plane and a tf32 "lo" plane (the remainder) for the 3xTF32
//   tensor-core path, FP32_BF16X3 a bf16 "hi" plane and a bf16 "lo" plane;
//   both also keep the plain fp32 weights for the decode path.
// Workspace per forward (capacity grows, never shrinks):
//   logits [T][E], idx/wts [T][k], blockhist [nblk][E], counts [E],
//   eoff [E+1] (packed-row offset of each expert, multiples of 128),
//   mtiles [max_mtiles] (expert, first row, valid rows) and their number,
//   row_token/row_weight [rows] (packed row -> token, combine weight),
//   A [rows][d] and H [rows][ffp] activation planes (bf16, or tf32 hi + lo).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "moe_b200.h"

namespace moe {

constexpr int kRouteTokens = 32;   // tokens per router / dispatch block
constexpr int kTileM = 128;        // GEMM tile rows (= expert block alignment)
constexpr int kTileN = 256;        // GEMM tile columns
constexpr int kFfBlock = 128;      // d_ff padding granule (half of kTileN)
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;
constexpr int kProfileStages = 8;
constexpr int kProfileMarks = 24;  // stage boundaries one forward may record
constexpr int kProfEnd = -1;       // the mark closing the last stage
// Split-K of the down GEMM (single-CTA tiles): only for at most this many
// routed rows, with at least this many 128-byte K blocks per split.
constexpr int kSplitMaxRows = 64;
constexpr int kSplitMinBlocks = 8;
// K chunk of the decode down kernel (its split-K granule).
constexpr int kDownChunk = 2048;

// One 128-row slice of an expert's packed block.  m-tiles are listed expert
// by expert; mstart / mcount locate the expert's own run in that list.  The
// pair list (CTA-pair GEMM) uses the same struct for 256-row slices: rows is
// the first half's valid rows and pad[0] the second half's.
struct MTile {
    int expert;
    int row0;    // first packed row
    int rows;    // valid rows (<= kTileM)
    int mstart;  // index of the expert's first m-tile
    int mcount;  // m-tiles of this expert
    int pad[3];
};

struct Workspace {
    int cap_T = 0;
    int cap_rows = 0;
    int cap_mtiles = 0;
    float* logits = nullptr;
    int* idx = nullptr;
    float* wts = nullptr;
    int* blockhist = nullptr;
    int* counts = nullptr;
    int* eoff = nullptr;
    MTile* mtiles = nullptr;
    int* num_mtiles = nullptr;
    MTile* ptiles = nullptr;    // 256-row pair tiles (two m-tiles of one expert)
    int* num_ptiles = nullptr;
    int* row_token = nullptr;
    float* row_weight = nullptr;
    // Packed row -> selection slot t * k + s (the ordered combine's index).
    int* row_slot = nullptr;
    // Expert output rows, unweighted, one per selection slot and K split:
    // [splits][T * k][d] fp32, read by the ordered combine (combine.cu).
    float* part = nullptr;
    size_t part_rows = 0;
    void* a_hi = nullptr;
    void* a_lo = nullptr;
    void* h_hi = nullptr;
    void* h_lo = nullptr;
    float* x_stage = nullptr;   // host-API staging, [cap_T][d]
    float* y_stage = nullptr;
    int* dev_err = nullptr;     // device-side error flags (timeouts)
    float* row_mean = nullptr;  // post-attention LayerNorm statistics, [cap_T]
    float* row_inv = nullptr;
    float* h_dec = nullptr;     // decode-path H, fp32 [64 * k][ffp]
    int* dec_counter = nullptr; // decode-path work counters [2]
    CUtensorMap tm_a_hi, tm_a_lo, tm_h_hi, tm_h_lo;
    size_t bytes = 0;
};

#ifdef __CUDACC__
// A token's k selections ordered by ascending key (the expert index): ord[r]
// is the slot of rank r and ow[r] its weight.  Warp-collective (k and KMAX
// warp-uniform, k <= KMAX <= 32); lane s < k supplies slot s's key and
// weight, other lanes' values are ignored.  Equal keys keep slot order.
template <int KMAX>
__device__ __forceinline__ void slot_order_keys(int key, float wv, int k, int lane,
                                                int (&ord)[KMAX], float (&ow)[KMAX]) {
    if (lane >= k) key = 0x7fffffff;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
        if (j >= k) break;
        const int kj = __shfl_sync(0xffffffffu, key, j);
        rank += (kj < key) || (kj == key && j < lane);
    }
#pragma unroll
    for (int r = 0; r < KMAX; ++r) {
        const unsigned m = __ballot_sync(0xffffffffu, lane < k && rank == r);
        const int s = m ? __ffs(m) - 1 : 0;
        ord[r] = s;
        ow[r] = __shfl_sync(0xffffffffu, wv, s);
    }
}

// The same with the keys and weights read from idx[0..k) / w[0..k).
template <int KMAX>
__device__ __forceinline__ void slot_order(const int* idx, const float* w, int k, int lane,
                                           int (&ord)[KMAX], float (&ow)[KMAX]) {
    int key = 0;
    float wv = 0.0f;
    if (lane < k) {
        key = idx[lane];
        wv = w[lane];
    }
    slot_order_keys<KMAX>(key, wv, k, lane, ord, ow);
}

// Output expression of tensor_ops::layer_norm (src/tensor.cu:187) as GCC
// contracts it: fma((x - mean) * inv, w, b), four columns at a time.
__device__ __forceinline__ float4 layer_norm_out4(float4 x, float m, float iv, float4 w,
                                                  float4 b) {
    float4 o;
    o.x = __fmaf_rn(__fmul_rn(__fsub_rn(x.x, m), iv), w.x, b.x);
    o.y = __fmaf_rn(__fmul_rn(__fsub_rn(x.y, m), iv), w.y, b.y);
    o.z = __fmaf_rn(__fmul_rn(__fsub_rn(x.z, m), iv), w.z, b.z);
    o.w = __fmaf_rn(__fmul_rn(__fsub_rn(x.w, m), iv), w.w, b.w);
    return o;
}
#endif

// The LayerNorm applied on load (norm.cu): row t's mean and inverse standard
// deviation from row_stats_kernel, and the norm's weight and bias.  Inactive
// (mean == nullptr) for the plain MoE forward.
struct NormRef {
    const float* mean = nullptr;   // [T]
    const float* inv = nullptr;    // [T]
    const float* w = nullptr;      // [d]
    const float* b = nullptr;      // [d]
#ifdef __CUDACC__
    // Columns 4v .. 4v+3 of row t, normalised.
    __device__ __forceinline__ float4 apply4(float4 x, int t, int v) const {
        return layer_norm_out4(x, __ldg(mean + t), __ldg(inv + t),
                               __ldg(reinterpret_cast<const float4*>(w) + v),
                               __ldg(reinterpret_cast<const float4*>(b) + v));
    }
#endif
};

struct EpState;  // expert-parallel group (ep.cu)

struct Layer {
    MoeConfig cfg{};
    int d = 0, ff = 0, ffp = 0, E = 0, k = 0;
    // Experts the router scores.  Equal to E except under expert parallelism,
    // where E is the number of experts this rank holds and E_route the global
    // count; the rank's experts are [e_first, e_first + E).
    int E_route = 0;
    int e_first = 0;
    EpState* ep = nullptr;
    int sm_count = 148;
    float* wg = nullptr;
    float* bias = nullptr;
    void* w13_hi = nullptr;
    void* w13_lo = nullptr;
    void* w2_hi = nullptr;
    void* w2_lo = nullptr;
    float* w13_f32 = nullptr;
    float* w2_f32 = nullptr;
    CUtensorMap tm_w13_hi, tm_w13_lo, tm_w2_hi, tm_w2_lo;
    // The same weights in 128-row boxes: each CTA of a pair loads half of the
    // 256-wide N tile.
    CUtensorMap tm_w13_hi2, tm_w13_lo2, tm_w2_hi2, tm_w2_lo2;
    int gemm_variant = 0;       // MoeGemmVariant
    // Post-attention LayerNorm (moe_set_post_norm): weight and bias [d].
    float* norm_w = nullptr;
    float* norm_b = nullptr;
    float norm_eps = 0.0f;
    // RMSNorm instead (moe_set_post_rms_norm): the statistics kernel writes
    // mean 0 and norm_b holds zeros, so the LayerNorm apply expression
    // fma((x - 0) * inv, w, 0) is exactly (x * inv) * w.
    bool norm_rms = false;
    Workspace ws;
    size_t weight_bytes = 0;
    cudaStream_t last_stream = nullptr;
    int last_T = 0;
    // Stage timers (moe_profile_enable): the marks of the last forward, in
    // stream order; mark j's event starts stage prof_stage[j] (kProfEnd
    // closes the last), which lasts until mark j + 1.  A stage may recur; its
    // intervals add up.
    bool profile = false;
    cudaEvent_t prof_ev[kProfileMarks] = {};
    int prof_stage[kProfileMarks] = {};
    int prof_n = 0;
};

// Start stage `i` (kProfEnd: close the last one); no-op unless profiling.
inline void prof_mark(Layer& L, int i, cudaStream_t s) {
    if (!L.profile || L.prof_n >= kProfileMarks) return;
    cudaEventRecord(L.prof_ev[L.prof_n], s);
    L.prof_stage[L.prof_n++] = i;
}

// ------------------------------------------------------------ launchers
// route.cu
// nr active: x is normalised on load (the post-attention LayerNorm).  eperm
// (expert parallelism): idx and the histogram get eperm[expert], the
// expert's dispatch position, instead of the expert itself.
cudaError_t launch_router(const Layer& L, const float* x, int T, float* logits, int* idx,
                          float* wts, int* blockhist, cudaStream_t s, const NormRef& nr = {},
                          const int* eperm = nullptr);
cudaError_t launch_dispatch_scan(const Layer& L, int T, cudaStream_t s);
// Batches of at most 4 tokens: router, selection, layout and the routed rows
// in one single-CTA launch (rows in the decode kernels' format if `decode`,
// else the GEMMs').  route_small_geometry says whether it applies.
bool route_small_geometry(const Layer& L, int T, bool norm, int* kc, int* stages);
// Every K chunk of the geometry has a stage of its own (the direct-load path).
bool route_small_resident(const Layer& L, int kc, int stages);
// rms_inline: the RMSNorm statistics are computed in the kernel (needs the
// resident geometry) instead of read from the workspace.
cudaError_t launch_route_small(const Layer& L, const float* x, int T, const NormRef& nr,
                               bool decode, cudaStream_t s, bool rms_inline = false);
cudaError_t launch_dispatch_permute(const Layer& L, const float* x, int T, cudaStream_t s,
                                    const NormRef& nr = {});
// The same placement with the rows copied in the decode kernels' format:
// fp32 as is (FP32 precision) or bf16 (BF16 precision).
cudaError_t launch_dispatch_permute_raw(const Layer& L, const float* x, int T, cudaStream_t s,
                                        const NormRef& nr = {});
// Placement into explicit outputs, routing over E experts with offsets eoff;
// slot_row[t * k + s] receives the row of token t's s-th selection.
cudaError_t launch_dispatch_permute_to(const Layer& L, const float* x, int T, int E,
                                       const int* eoff, int* row_token, float* row_weight,
                                       int* slot_row, void* rows, cudaStream_t s);
// The scan on any [nblk][E] count matrix, expert blocks rounded to `granule`
// rows; mtiles == nullptr gives a compact layout with no tiles or padding.
cudaError_t launch_scan_generic(int* hist, int nblk, int E, int granule, int* counts, int* eoff,
                                MTile* mtiles, int* num_mtiles, MTile* ptiles, int* num_ptiles,
                                int* row_token, float* row_weight, cudaStream_t s);

// expert_gemm.cu
// Grouped GEMMs over `routed_rows` packed rows.  mode:
//   0 gate/up with the SwiGLU epilogue into H;
//   1 down, adding into y: y[row_token[row]] += row_weight[row] * result
//     (the dense projections of the decoder: one contribution per element
//     unless K is split);
//   2 down storing each row's result at y[row_token[row]] (bf16 in BF16
//     precision; the NCCL expert-parallel transport);
//   3 down storing each row's unweighted result at
//     part[split][row_slot[row]] for the ordered combine.
// split_stride (floats between the K splits' part planes; mode 3 only): 0
// keeps K whole.  *nsplit receives the number of K splits (may be null).
cudaError_t launch_expert_gemm_rows(const Layer& L, int routed_rows, float* y, cudaStream_t s,
                                    int mode, size_t split_stride = 0, int* nsplit = nullptr);

// combine.cu: y[t] = the ordered combine of token t's k expert rows in
// part ([nsplit][T * k][d]) with weights wts, plus resid[t] when non-null.
cudaError_t launch_combine(const Layer& L, int T, int nsplit, const float* resid, float* y,
                           cudaStream_t s);

// decode.cu: T <= decode_max_supported_tokens() (64)
// packed: the routed rows are already in the decode format (launch_route_small).
// The down kernel stores each slot's partial dots per K chunk into part;
// *nsplit receives the number of chunks for the ordered combine.
cudaError_t launch_decode(Layer& L, const float* x, int T, int* nsplit, cudaStream_t s,
                          const NormRef& nr = {}, bool packed = false);
int decode_chunks(const Layer& L);
int decode_max_supported_tokens();
// What MOE_DECODE_AUTO resolves to for a precision (capi.cu).
int auto_decode_max_tokens(int precision);

// norm.cu: per-row LayerNorm statistics, the whole LayerNorm into y (d a
// multiple of 128: norm_supported), and y += r over n floats (n a multiple
// of 4).  err collects timed-out waits (may be null).
bool norm_supported(int d);
cudaError_t launch_row_stats(const float* x, int T, int d, float eps, float* mean, float* inv,
                             int* err, cudaStream_t s);
cudaError_t launch_layer_norm(const float* x, int T, int d, float eps, const float* w,
                              const float* b, float* y, cudaStream_t s);
cudaError_t launch_residual_add(const Layer& L, float* y, const float* r, size_t n,
                                cudaStream_t s);
// RMSNorm statistics: mean[t] = 0, inv[t] = 1 / sqrt(sum_j x[t][j]^2 / d + eps)
// (fp32 sum of squares; d a multiple of 4).
cudaError_t launch_rms_stats(const float* x, int T, int d, float eps, float* mean, float* inv,
                             cudaStream_t s);

// weights.cu
// Runs one bounded mbarrier wait that nothing completes (timeout self-test).
cudaError_t launch_selftest_wait(int* err, unsigned long long budget_ns);
cudaError_t convert_gateup(const Layer& L, int e, const float* w1_dev, const float* w3_dev,
                           cudaStream_t s);
cudaError_t convert_down(const Layer& L, int e, const float* w2_dev, cudaStream_t s);

// Record `msg` as this thread's moe_last_error() and return `code` (capi.cu).
int report_error(int code, const std::string& msg);
// Grow the workspace to T tokens (capi.cu).
int ensure_workspace(Layer& L, int T);
// Supplies one expert tensor on the host during handle construction
// (which: 0 w1, 1 w3, 2 w2; n floats into dst); a non-zero return is an
// MoeStatus with moe_last_error set.  Lets a loader stream the experts from
// a file one tensor at a time instead of holding the layer in host memory.
struct ExpertReader {
    virtual ~ExpertReader() = default;
    virtual int read(int e, int which, float* dst, size_t n) = 0;
};
// Handle construction for experts [e_first, e_first + e_count) (capi.cu).
// With a reader (host weights only), w's expert pointers are not used.
int create_slice(const MoeConfig* cfg, const MoeWeightsHost* w, bool device_ptrs, int e_first,
                 int e_count, MoeHandle** out, ExpertReader* reader = nullptr);
// Expert-parallel teardown (ep.cu).
void ep_destroy(Layer& L);

// tensor maps (capi.cpp)
bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer, std::string* err);

}  // namespace moe

struct MoeHandle {
    moe::Layer L;
    cudaStream_t own_stream = nullptr;   // compute stream of the host-buffer API
    // Copy streams and chunk events of the pipelined host-buffer forward.
    cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
    static constexpr int kMaxChunks = 4;
    cudaEvent_t in_ev[kMaxChunks] = {}, out_ev[kMaxChunks] = {};
};

namespace moe {

// Tensor-core operand scheme of the grouped GEMMs: one bf16 plane; tf32 hi +
// lo planes (fp32 storage) with three tf32 MMAs; bf16 hi + lo planes with
// three bf16 MMAs.
enum GemmPrec : int { kGemmBf16 = 0, kGemm3xTf32 = 1, kGemmBf16x3 = 2 };
inline int gemm_prec(const Layer& L) {
    return L.cfg.precision == MOE_PREC_BF16 ? kGemmBf16
         : L.cfg.precision == MOE_PREC_FP32 ? kGemm3xTf32 : kGemmBf16x3;
}
// fp32-faithful precisions: decode streams fp32 weights, expert-parallel rows
// travel in fp32.
inline bool fp32_faithful(const Layer& L) { return L.cfg.precision != MOE_PREC_BF16; }
// GEMM operands in two planes (hi and lo).
inline bool split_planes(const Layer& L) { return gemm_prec(L) != kGemmBf16; }
// Bytes of one element of one operand plane, and whether the planes are bf16.
inline size_t plane_bytes(const Layer& L) { return gemm_prec(L) == kGemm3xTf32 ? 4 : 2; }
inline bool planes_bf16(const Layer& L) { return gemm_prec(L) != kGemm3xTf32; }
// Bytes per element of an expert-parallel row on the wire.
inline size_t wire_bytes(const Layer& L) { return fp32_faithful(L) ? 4 : 2; }
// Elements of one 128-byte K block of an operand plane.
inline int kblock_elems(const Layer& L) { return gemm_prec(L) == kGemm3xTf32 ? 32 : 64; }

// Format of the packed activation rows: the GEMM operand planes of each
// precision, or (decode kernels) the rows as the decode kernels read them.
enum ActFormat : int { kActBf16 = 0, kActTf32x2 = 1, kActF32 = 2, kActBf16x2 = 3 };
inline int act_format(const Layer& L, bool decode) {
    if (decode) return fp32_faithful(L) ? kActF32 : kActBf16;
    const int g = gemm_prec(L);
    return g == kGemmBf16 ? kActBf16 : g == kGemm3xTf32 ? kActTf32x2 : kActBf16x2;
}

}  // namespace moe
