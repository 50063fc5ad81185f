// Toy MoE decoder: whole-model greedy generation around
// the MoE layers -- the counterpart of the reference's PhiTinyMoEModel
// (include/model.h:8-30; generate src/model.cu:1575-2058, generate_decode
// src/model.cu:2061-2104).
//
// Per layer, on the decoder's stream:
//   rms_pack        x -> rms_norm(x) in the GEMM's A format (bf16, or tf32
//                   hi + lo), and the projection's output zeroed
//   qkv GEMM        the tcgen05 grouped GEMM with one group and an identity
//                   row map (combine epilogue, weight 1): qkv = A . Wqkv^T
//   rope_kv         rotate-half RoPE on q and k (tensor_ops::apply_rope,
//                   src/tensor.cu:191-210); k and v into the KV cache (a
//                   decode step does this inside its attention kernel)
//   attention       causal softmax(q k^T / sqrt(hd)) v per (sequence, head),
//                   output straight into the A format
//   o GEMM          x += A . Wo^T (the combine epilogue adds into the
//                   residual stream itself)
//   MoE block       x' = x + MoE(rms_norm(x)) (moe_block_forward_device with
//                   the RMSNorm attached; norm applied inside the router and
//                   the dispatch)
// then rms_pack of each sequence's last row, the output-head GEMM against the
// (tied) embedding matrix, and a greedy argmax.
//
// The reference's generate_decode re-runs the whole prefix for every new
// token; here a KV cache [layer][sequence][head][position][head_dim] (fp32)
// keeps keys and values, so a decode step processes one row per sequence.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "decode_step.h"
#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

// ------------------------------------------------------------ A-format stores
// Columns c .. c+3 of row `row` of a [rows][ld] A operand: bf16 (kTf = false)
// or the tf32 hi and lo planes of the 3xTF32 path.
template <bool kTf>
__device__ __forceinline__ void store_a4(void* a_hi, void* a_lo, size_t row, int ld, int c,
                                         float4 f) {
    if constexpr (kTf) {
        float4 h, l;
        h.x = to_tf32(f.x); l.x = to_tf32(f.x - h.x);
        h.y = to_tf32(f.y); l.y = to_tf32(f.y - h.y);
        h.z = to_tf32(f.z); l.z = to_tf32(f.z - h.z);
        h.w = to_tf32(f.w); l.w = to_tf32(f.w - h.w);
        *reinterpret_cast<float4*>(static_cast<float*>(a_hi) + row * ld + c) = h;
        *reinterpret_cast<float4*>(static_cast<float*>(a_lo) + row * ld + c) = l;
    } else {
        __nv_bfloat162 lo2 = __floats2bfloat162_rn(f.x, f.y);
        __nv_bfloat162 hi2 = __floats2bfloat162_rn(f.z, f.w);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&lo2);
        packed.y = *reinterpret_cast<uint32_t*>(&hi2);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a_hi) + row * ld + c) = packed;
    }
}

template <bool kTf>
__device__ __forceinline__ void store_a1(void* a_hi, void* a_lo, size_t row, int ld, int c,
                                         float f) {
    if constexpr (kTf) {
        const float h = to_tf32(f);
        static_cast<float*>(a_hi)[row * ld + c] = h;
        static_cast<float*>(a_lo)[row * ld + c] = to_tf32(f - h);
    } else {
        static_cast<__nv_bfloat16*>(a_hi)[row * ld + c] = __float2bfloat16_rn(f);
    }
}

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

// ------------------------------------------------------------ embedding
// x[r] = embed[tok[r]]: one block per row.  An id outside [0, vocab) gives a
// zero row and sets kDecErrToken.
__global__ void __launch_bounds__(256)
embed_gather_kernel(const int* __restrict__ tok, const float* __restrict__ embed, int vocab,
                    int d, float* __restrict__ x, int* __restrict__ err) {
    const int r = blockIdx.x;
    const int t = tok[r];
    const bool ok = t >= 0 && t < vocab;
    if (!ok && threadIdx.x == 0) atomicOr(err, kDecErrToken);
    const float4* src = reinterpret_cast<const float4*>(embed + (size_t)(ok ? t : 0) * d);
    float4* dst = reinterpret_cast<float4*>(x + (size_t)r * d);
    for (int v = threadIdx.x; v < d / 4; v += blockDim.x)
        dst[v] = ok ? __ldg(src + v) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// ------------------------------------------------------------ RMSNorm -> A
// One warp per packed row r < rows_pad.  Row r < T is row src0 + r * stride
// of x, written as (x * inv) * w with inv = 1 / sqrt(sum x^2 / d + eps) (the
// same arithmetic as the MoE block's norm); rows past T are zero.  The grid
// also zeroes the n4 float4 at `zero` -- the output the following GEMM adds
// into -- so that no separate memset sits between this kernel and the GEMM.
template <bool kTf>
__global__ void __launch_bounds__(256)
rms_pack_kernel(const float* __restrict__ x, int src0, int stride, int T, int rows_pad, int d,
                float eps, const float* __restrict__ w, void* __restrict__ a_hi,
                void* __restrict__ a_lo, float4* __restrict__ zero, size_t zero_n4) {
    // Dependent launch: x and the buffers below belong to earlier kernels.
    wait_predecessor_grid();
    launch_dependents();
    const size_t gtid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t gthreads = (size_t)gridDim.x * blockDim.x;
    for (size_t i = gtid; i < zero_n4; i += gthreads) zero[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows_pad) return;
    if (r >= T) {
        for (int c = lane * 4; c < d; c += 128)
            store_a4<kTf>(a_hi, a_lo, r, d, c, make_float4(0.0f, 0.0f, 0.0f, 0.0f));
        return;
    }
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(src0 + (size_t)r * stride) * d);
    float ss = 0.0f;
    for (int v = lane; v < d / 4; v += 32) {
        const float4 a = __ldg(xr + v);
        ss = __fmaf_rn(a.x, a.x, ss);
        ss = __fmaf_rn(a.y, a.y, ss);
        ss = __fmaf_rn(a.z, a.z, ss);
        ss = __fmaf_rn(a.w, a.w, ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    for (int v = lane; v < d / 4; v += 32) {
        const float4 a = __ldg(xr + v), g = __ldg(w4 + v);
        float4 o;
        o.x = __fmul_rn(__fmul_rn(a.x, inv), g.x);
        o.y = __fmul_rn(__fmul_rn(a.y, inv), g.y);
        o.z = __fmul_rn(__fmul_rn(a.z, inv), g.z);
        o.w = __fmul_rn(__fmul_rn(a.w, inv), g.w);
        store_a4<kTf>(a_hi, a_lo, r, d, 4 * v, o);
    }
}

// Decode-sized batches (the GEMV path): one CTA per row instead of one warp,
// so every x and w load of the row is issued at once (one memory round trip
// instead of a lane's serial walk), and a block reduction of the sum of
// squares; same expression (x * inv) * w.  Rows past T are not written (the
// GEMV reads only T rows).
constexpr int kPackThreads = 256;
constexpr int kPackMaxVec = 8;   // float4 per thread: d <= 8192

template <bool kTf>
__global__ void __launch_bounds__(kPackThreads)
rms_pack_row_kernel(const float* __restrict__ x, int src0, int stride, int d, float eps,
                    const float* __restrict__ w, void* __restrict__ a_hi,
                    void* __restrict__ a_lo, float4* __restrict__ zero, size_t zero_n4) {
    __shared__ float s_part[kPackThreads / 32];
    wait_predecessor_grid();   // dependent launch: x and the buffers below
    launch_dependents();
    const int r = blockIdx.x, tid = threadIdx.x;
    for (size_t i = (size_t)r * kPackThreads + tid; i < zero_n4; i += (size_t)gridDim.x * kPackThreads)
        zero[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(src0 + (size_t)r * stride) * d);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const int nv = d / 4;
    float4 a[kPackMaxVec], g[kPackMaxVec];
#pragma unroll
    for (int i = 0; i < kPackMaxVec; ++i) {
        const int v = tid + i * kPackThreads;
        if (v < nv) {
            a[i] = __ldcg(xr + v);   // written by the previous kernel: through L2
            g[i] = __ldg(w4 + v);
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kPackMaxVec; ++i) {
        if (tid + i * kPackThreads < nv) {
            ss = __fmaf_rn(a[i].x, a[i].x, ss);
            ss = __fmaf_rn(a[i].y, a[i].y, ss);
            ss = __fmaf_rn(a[i].z, a[i].z, ss);
            ss = __fmaf_rn(a[i].w, a[i].w, ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) s_part[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kPackThreads / 32; ++i) tot += s_part[i];
    const float inv = 1.0f / sqrtf(tot / (float)d + eps);
#pragma unroll
    for (int i = 0; i < kPackMaxVec; ++i) {
        const int v = tid + i * kPackThreads;
        if (v < nv) {
            float4 o;
            o.x = __fmul_rn(__fmul_rn(a[i].x, inv), g[i].x);
            o.y = __fmul_rn(__fmul_rn(a[i].y, inv), g[i].y);
            o.z = __fmul_rn(__fmul_rn(a[i].z, inv), g[i].z);
            o.w = __fmul_rn(__fmul_rn(a[i].w, inv), g[i].w);
            store_a4<kTf>(a_hi, a_lo, r, d, 4 * v, o);
        }
    }
}

// ------------------------------------------------------------ tile list
// The grouped GEMM's tile list for a dense projection over T rows: one group
// (expert 0), rows 0..T-1 in order, row r's output row r with weight 1;
// rows T..rows_pad-1 are padding (token -1, weight 0).  Same fields as the
// dispatch scan writes for an expert block.
__global__ void dense_tiles_kernel(int T, int rows_pad, MTile* __restrict__ mtiles,
                                   int* __restrict__ num_mtiles, MTile* __restrict__ ptiles,
                                   int* __restrict__ num_ptiles, int* __restrict__ row_token,
                                   float* __restrict__ row_weight) {
    const int mc = (T + kTileM - 1) / kTileM;
    const int qc = (mc + 1) / 2;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows_pad; r += gridDim.x * blockDim.x) {
        row_token[r] = r < T ? r : -1;
        row_weight[r] = r < T ? 1.0f : 0.0f;
    }
    if (blockIdx.x != 0) return;
    for (int i = threadIdx.x; i < mc; i += blockDim.x) {
        MTile mt;
        mt.expert = 0; mt.row0 = i * kTileM; mt.rows = min(kTileM, T - i * kTileM);
        mt.mstart = 0; mt.mcount = mc; mt.pad[0] = mt.pad[1] = mt.pad[2] = 0;
        mtiles[i] = mt;
    }
    for (int i = threadIdx.x; i < qc; i += blockDim.x) {
        MTile pt;
        pt.expert = 0; pt.row0 = 2 * i * kTileM; pt.rows = min(kTileM, T - 2 * i * kTileM);
        pt.mstart = 0; pt.mcount = qc;
        pt.pad[0] = max(0, min(kTileM, T - (2 * i + 1) * kTileM));
        pt.pad[1] = pt.pad[2] = 0;
        ptiles[i] = pt;
    }
    if (threadIdx.x == 0) {
        *num_mtiles = mc;
        *num_ptiles = qc;
    }
}

// ------------------------------------------------------------ RoPE + cache
// Row r of qkv [T][3d] is token r % rps of sequence r / rps, at position
// pos0 (+ *pos_dev, a decode step's position kept on the device) + r % rps.  q and k are rotated in the reference's rotate-half form
// (tensor_ops::apply_rope, src/tensor.cu:191-210): for j < hd/2,
//   x_j' = x_j cos - x_{j+hd/2} sin,  x_{j+hd/2}' = x_{j+hd/2} cos + x_j sin
// with (cos, sin) of position p and pair j from the table [max_seq][hd/2][2].
// q stays in qkv (rotated); k and v go to the cache at their position.
template <int HD>
__global__ void __launch_bounds__(256)
rope_kv_kernel(float* __restrict__ qkv, int rps, int pos0, const int* __restrict__ pos_dev, int H,
               const float2* __restrict__ rope, float* __restrict__ kc, float* __restrict__ vc,
               int max_seq) {
    constexpr int kHalf = HD / 2;
    const int r = blockIdx.x;
    const int b = r / rps, pos = pos0 + (pos_dev ? *pos_dev : 0) + r % rps;
    const int d = H * HD;
    float* q = qkv + (size_t)r * 3 * d;
    const float* k = q + d;
    const float* v = q + 2 * d;
    for (int i = threadIdx.x; i < H * kHalf; i += blockDim.x) {
        const int h = i / kHalf, j = i % kHalf;
        const float2 cs = __ldg(rope + (size_t)pos * kHalf + j);
        const float q0 = q[h * HD + j], q1 = q[h * HD + j + kHalf];
        q[h * HD + j] = q0 * cs.x - q1 * cs.y;
        q[h * HD + j + kHalf] = q1 * cs.x + q0 * cs.y;
        const float k0 = k[h * HD + j], k1 = k[h * HD + j + kHalf];
        float* kd = kc + (((size_t)b * H + h) * max_seq + pos) * HD;
        kd[j] = k0 * cs.x - k1 * cs.y;
        kd[j + kHalf] = k1 * cs.x + k0 * cs.y;
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const int h = i / HD, c = i % HD;
        vc[(((size_t)b * H + h) * max_seq + pos) * HD + c] = v[i];
    }
}

// ------------------------------------------------------------ attention
// Prefill: causal attention of the S queries of one sequence and head over
// keys 0..S-1, a 64-query block per CTA, keys in blocks of 64 with an online
// softmax.  256 threads: thread (ti, tj) = (tid / 16, tid % 16) scores
// queries ti + 16a against keys tj + 16b (a, b < 4) and accumulates the
// output of queries ti + 16a in dims 4 tj + 64 u .. +3.  Rows are padded to
// hd + 4 floats so the float4 shared loads of 16 different rows fall in
// different banks.  Output: row b*S + q of the A operand, cols h*hd..
constexpr int kAttBQ = 64;
constexpr int kAttBK = 64;

template <int HD>
struct AttnSmem {
    static constexpr int kLd = HD + 4;
    static constexpr int kLdP = kAttBK + 4;
    static constexpr size_t kBytes =
        sizeof(float) * ((size_t)kAttBQ * kLd + 2 * (size_t)kAttBK * kLd + (size_t)kAttBQ * kLdP);
};

template <int HD, bool kTf>
__global__ void __launch_bounds__(256)
attn_prefill_kernel(const float* __restrict__ qkv, int S, int H, const float* __restrict__ kc,
                    const float* __restrict__ vc, int max_seq, float scale,
                    void* __restrict__ a_hi, void* __restrict__ a_lo) {
    using Sm = AttnSmem<HD>;
    constexpr int kLd = Sm::kLd, kLdP = Sm::kLdP;
    constexpr int kU = HD / 64;   // 64-dim slices per thread row
    extern __shared__ __align__(16) float sm[];
    float* sQ = sm;
    float* sK = sQ + kAttBQ * kLd;
    float* sV = sK + kAttBK * kLd;
    float* sP = sV + kAttBK * kLd;
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
    const int q0 = qb * kAttBQ;
    const int d = H * HD;
    const float* kbase = kc + ((size_t)b * H + h) * max_seq * HD;
    const float* vbase = vc + ((size_t)b * H + h) * max_seq * HD;

    for (int i = tid; i < kAttBQ * HD / 4; i += 256) {
        const int r = i / (HD / 4), c4 = i % (HD / 4);
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (q0 + r < S) {
            v = *reinterpret_cast<const float4*>(qkv + ((size_t)b * S + q0 + r) * 3 * d + h * HD + 4 * c4);
            v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
        }
        *reinterpret_cast<float4*>(sQ + r * kLd + 4 * c4) = v;
    }
    float m[4], l[4], o[4][4 * kU];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.0f;
#pragma unroll
        for (int c = 0; c < 4 * kU; ++c) o[a][c] = 0.0f;
    }
    const int last_q = min(q0 + kAttBQ, S) - 1;
    for (int k0 = 0; k0 <= last_q; k0 += kAttBK) {
        __syncthreads();   // the previous block's sK / sV / sP reads are done
        for (int i = tid; i < kAttBK * HD / 4; i += 256) {
            const int r = i / (HD / 4), c4 = i % (HD / 4);
            float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vv = kv;
            if (k0 + r < S) {
                kv = *reinterpret_cast<const float4*>(kbase + (size_t)(k0 + r) * HD + 4 * c4);
                vv = *reinterpret_cast<const float4*>(vbase + (size_t)(k0 + r) * HD + 4 * c4);
            }
            *reinterpret_cast<float4*>(sK + r * kLd + 4 * c4) = kv;
            *reinterpret_cast<float4*>(sV + r * kLd + 4 * c4) = vv;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) s[a][bb] = 0.0f;
#pragma unroll 4
        for (int c = 0; c < HD; c += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a)
                qv[a] = *reinterpret_cast<const float4*>(sQ + (ti + 16 * a) * kLd + c);
#pragma unroll
            for (int bb = 0; bb < 4; ++bb)
                kv[bb] = *reinterpret_cast<const float4*>(sK + (tj + 16 * bb) * kLd + c);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int bb = 0; bb < 4; ++bb) {
                    s[a][bb] = fmaf(qv[a].x, kv[bb].x, s[a][bb]);
                    s[a][bb] = fmaf(qv[a].y, kv[bb].y, s[a][bb]);
                    s[a][bb] = fmaf(qv[a].z, kv[bb].z, s[a][bb]);
                    s[a][bb] = fmaf(qv[a].w, kv[bb].w, s[a][bb]);
                }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int qpos = q0 + ti + 16 * a;
            float mt = -INFINITY;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const int kpos = k0 + tj + 16 * bb;
                if (kpos > qpos || kpos >= S) s[a][bb] = -INFINITY;
                mt = fmaxf(mt, s[a][bb]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1)
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
            const float mn = fmaxf(m[a], mt);
            // Every visited block holds at least one key at or before each
            // valid query (key k0 <= q0); rows past S may be all -inf.
            const float corr = mn == -INFINITY ? 1.0f : expf(m[a] - mn);
            m[a] = mn;
            float ps = 0.0f;
#pragma unroll
            for (int bb = 0; bb < 4; ++bb) {
                const float p = s[a][bb] == -INFINITY ? 0.0f : expf(s[a][bb] - mn);
                sP[(ti + 16 * a) * kLdP + tj + 16 * bb] = p;
                ps += p;
            }
            l[a] = l[a] * corr + ps;
#pragma unroll
            for (int c = 0; c < 4 * kU; ++c) o[a][c] *= corr;
        }
        __syncthreads();
        const int nk = min(kAttBK, last_q + 1 - k0);
#pragma unroll 2
        for (int j = 0; j < nk; ++j) {
            float4 vv[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u)
                vv[u] = *reinterpret_cast<const float4*>(sV + j * kLd + 4 * tj + 64 * u);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float p = sP[(ti + 16 * a) * kLdP + j];
#pragma unroll
                for (int u = 0; u < kU; ++u) {
                    o[a][4 * u + 0] = fmaf(p, vv[u].x, o[a][4 * u + 0]);
                    o[a][4 * u + 1] = fmaf(p, vv[u].y, o[a][4 * u + 1]);
                    o[a][4 * u + 2] = fmaf(p, vv[u].z, o[a][4 * u + 2]);
                    o[a][4 * u + 3] = fmaf(p, vv[u].w, o[a][4 * u + 3]);
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        float lt = l[a];
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, off);
        const int q = q0 + ti + 16 * a;
        if (q >= S) continue;
        const float il = 1.0f / lt;
        const size_t row = (size_t)b * S + q;
#pragma unroll
        for (int u = 0; u < kU; ++u)
            store_a4<kTf>(a_hi, a_lo, row, d, h * HD + 4 * tj + 64 * u,
                          make_float4(o[a][4 * u] * il, o[a][4 * u + 1] * il,
                                      o[a][4 * u + 2] * il, o[a][4 * u + 3] * il));
    }
}

// Prefill on the tensor cores (BF16 precision): one CTA per (128-query
// block, head, sequence), 128 threads, thread r owning query row r (TMEM
// lane r).  Two passes over the key blocks up to the diagonal, so the output
// accumulator never needs rescaling:
//   pass 1   S = Q K^T (tcgen05, M 128, N 128 keys, K = hd) -> each thread
//            reads its row of S from TMEM and updates its running max m and
//            sum l of e^(s - m);
//   pass 2   S again; P = e^(s - m) / l written as bf16 into shared memory;
//            O += P V (tcgen05, M 128, N = hd, K = 128 keys), O in TMEM.
// Operands are staged by the threads themselves from the fp32 cache into the
// K-major, 128-byte-swizzled layout the GEMMs' descriptors read (16-byte
// chunk c of row r at chunk c ^ (r % 8)): Q and K as [rows][hd], V
// transposed as [hd][keys] so that both MMAs read K-major operands.  q is
// scaled by 1/sqrt(hd) before rounding to bf16, as the CUDA-core kernel
// scales it.  Every wait is bounded; a CTA whose wait runs out drains its
// MMAs, frees TMEM and leaves (error flag set).
constexpr int kTcBQ = 128;   // queries per CTA
constexpr int kTcBK = 128;   // keys per block

template <int HD>
struct TcAttn {
    static constexpr int kQBytes = kTcBQ * HD * 2;      // [128][hd] bf16
    static constexpr int kKBytes = kTcBK * HD * 2;
    static constexpr int kVBytes = HD * kTcBK * 2;      // [hd][128 keys] bf16
    static constexpr int kPBytes = kTcBQ * kTcBK * 2;
    static constexpr int kQ = 0, kK = kQ + kQBytes, kV = kK + kKBytes, kP = kV + kVBytes;
    static constexpr int kBar = kP + kPBytes;
    static constexpr size_t kSmem = (size_t)kBar + 64 + 1024;   // barriers + alignment slack
    static constexpr uint32_t kIdescS = mma_idesc(1u, kTcBQ, kTcBK);
    static constexpr uint32_t kIdescO = mma_idesc(1u, kTcBQ, HD);
};

// Byte offset of element (row, col) of a [rows][w] bf16 K-major operand made
// of w/64 column blocks of [rows][64], each 128-byte swizzled.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int rows) {
    const int blk = col >> 6, c = col & 63;
    return (uint32_t)(blk * rows * 128 + row * 128 + ((((c >> 3) ^ (row & 7))) << 4) + (c & 7) * 2);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

// One row of 64 fp32 (scaled) into 8 swizzled 16-byte chunks of a bf16 tile.
__device__ __forceinline__ void stage_row64(uint8_t* tile, int row, int col0, int rows,
                                            const float* __restrict__ src, float scale, bool zero) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (!zero) {
            const float4 a = *reinterpret_cast<const float4*>(src + ch * 8);
            const float4 b = *reinterpret_cast<const float4*>(src + ch * 8 + 4);
            u.x = pack_bf16x2(a.x * scale, a.y * scale);
            u.y = pack_bf16x2(a.z * scale, a.w * scale);
            u.z = pack_bf16x2(b.x * scale, b.y * scale);
            u.w = pack_bf16x2(b.z * scale, b.w * scale);
        }
        *reinterpret_cast<uint4*>(tile + sw128_off(row, col0 + ch * 8, rows)) = u;
    }
}

__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int HD>
__global__ void __launch_bounds__(128, 1)
attn_prefill_tc_kernel(const float* __restrict__ qkv, int S, int H, const float* __restrict__ kc,
                       const float* __restrict__ vc, int max_seq, float scale,
                       void* __restrict__ a_out, int* __restrict__ err) {
    using L = TcAttn<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
    uint8_t* sQ = sm + L::kQ;
    uint8_t* sK = sm + L::kK;
    uint8_t* sV = sm + L::kV;
    uint8_t* sP = sm + L::kP;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::kBar);   // [0] S done, [1] O done, [2] drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 3);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int q0 = qb * kTcBQ;
    const int d = H * HD;
    const float* kbase = kc + ((size_t)b * H + h) * max_seq * HD;
    const float* vbase = vc + ((size_t)b * H + h) * max_seq * HD;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 256);
        tmem_relinquish();
    }
    // Q tile: row tid = query q0 + tid.
    {
        const bool valid = q0 + tid < S;
        const float* src = qkv + ((size_t)b * S + q0 + tid) * 3 * d + h * HD;
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 64)
            stage_row64(sQ, tid, c0, kTcBQ, src + c0, scale, !valid);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t t_s = tmem, t_o = tmem + kTcBK;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int qrow = q0 + tid;
    const int last_q = min(q0 + kTcBQ, S) - 1;
    const int nblk = last_q / kTcBK + 1;
    uint32_t ph_s = 0, ph_o = 0;
    int issued = 0;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;

    // K block kb into sK (row j = key k0 + j); with_v: V transposed into sV.
    auto stage_kv = [&](int kb, bool with_v) {
        const int k0 = kb * kTcBK;
        const bool kvalid = k0 + tid < S;
        const float* ks = kbase + (size_t)(k0 + tid) * HD;
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 64) stage_row64(sK, tid, c0, kTcBK, ks + c0, 1.0f, !kvalid);
        if (with_v) {
            // Thread t: keys 2 (t % 64), + 1 and dims [hd/2 * (t / 64), + hd/2).
            const int kp = tid & 63, half = tid >> 6;
            const int j0 = 2 * kp;
            const bool v0 = k0 + j0 < S, v1 = k0 + j0 + 1 < S;
            const float* r0 = vbase + (size_t)(k0 + j0) * HD;
            const float* r1 = r0 + HD;
#pragma unroll 4
            for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 4) {
                const float4 a = v0 ? *reinterpret_cast<const float4*>(r0 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 e = v1 ? *reinterpret_cast<const float4*>(r1 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<uint32_t*>(sV + sw128_off(c + 0, j0, HD)) = pack_bf16x2(a.x, e.x);
                *reinterpret_cast<uint32_t*>(sV + sw128_off(c + 1, j0, HD)) = pack_bf16x2(a.y, e.y);
                *reinterpret_cast<uint32_t*>(sV + sw128_off(c + 2, j0, HD)) = pack_bf16x2(a.z, e.z);
                *reinterpret_cast<uint32_t*>(sV + sw128_off(c + 3, j0, HD)) = pack_bf16x2(a.w, e.w);
            }
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
    };
    // S = Q K^T into TMEM columns [0, 128), then wait for it.
    auto mma_s = [&]() -> bool {
        if (tid == 0) {
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK);
#pragma unroll
            for (int kb = 0; kb < HD / 64; ++kb)
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    tc_mma<false>(t_s, smem_desc_sw128(qa + kb * kTcBQ * 128) + 2 * ks,
                                  smem_desc_sw128(ka + kb * kTcBK * 128) + 2 * ks, L::kIdescS,
                                  (kb | ks) ? 1u : 0u);
            tc_commit(&bar[0]);
        }
        ++issued;
        const bool got = mbar_wait(&bar[0], ph_s, err, kDevErrTimeoutMma);
        ph_s ^= 1u;
        tc_fence_after();
        return __syncthreads_and(got);
    };
    // This thread's row of S (128 columns) in 4 loads of 32, scaled/masked.
    auto read_s = [&](int k0, float (&sv)[kTcBK]) {
#pragma unroll
        for (int c = 0; c < kTcBK; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_s + lane_base + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int key = k0 + c + j;
                sv[c + j] = (key > qrow || key >= S) ? -INFINITY : __uint_as_float(r[j]);
            }
        }
    };

    // ---------------------------------------------------------- pass 1
    for (int kb = 0; kb < nblk && ok; ++kb) {
        stage_kv(kb, false);
        if (!mma_s()) { ok = false; break; }
        float sv[kTcBK];
        read_s(kb * kTcBK, sv);
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < kTcBK; ++j) mt = fmaxf(mt, sv[j]);
        const float mn = fmaxf(m, mt);
        float ps = 0.0f;
#pragma unroll
        for (int j = 0; j < kTcBK; ++j) ps += sv[j] == -INFINITY ? 0.0f : expf(sv[j] - mn);
        l = (m == -INFINITY ? 0.0f : l * expf(m - mn)) + ps;
        m = mn;
        tc_fence_before();
        __syncthreads();   // every row of S read before the next block overwrites it
    }
    // ---------------------------------------------------------- pass 2
    const float il = l > 0.0f ? 1.0f / l : 0.0f;
    for (int kb = 0; kb < nblk && ok; ++kb) {
        stage_kv(kb, true);
        if (!mma_s()) { ok = false; break; }
        float sv[kTcBK];
        read_s(kb * kTcBK, sv);
#pragma unroll
        for (int c0 = 0; c0 < kTcBK; c0 += 8) {
            float p[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                p[j] = sv[c0 + j] == -INFINITY ? 0.0f : expf(sv[c0 + j] - m) * il;
            const uint4 u = make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]),
                                       pack_bf16x2(p[4], p[5]), pack_bf16x2(p[6], p[7]));
            *reinterpret_cast<uint4*>(sP + sw128_off(tid, c0, kTcBQ)) = u;
        }
        fence_async_shared();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = smem_u32(sP), va = smem_u32(sV);
#pragma unroll
            for (int kb2 = 0; kb2 < kTcBK / 64; ++kb2)
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    tc_mma<false>(t_o, smem_desc_sw128(pa + kb2 * kTcBQ * 128) + 2 * ks,
                                  smem_desc_sw128(va + kb2 * HD * 128) + 2 * ks, L::kIdescO,
                                  (kb | kb2 | ks) ? 1u : 0u);
            tc_commit(&bar[1]);
        }
        ++issued;
        const bool got = mbar_wait(&bar[1], ph_o, err, kDevErrTimeoutMma);
        ph_o ^= 1u;
        tc_fence_after();
        if (!__syncthreads_and(got)) { ok = false; break; }
    }
    if (ok) {   // CTA-uniform: the TMEM loads are warp-collective, only the stores are per row
        // O row -> the o projection's A operand (bf16), cols h * hd ..
        __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(a_out) + ((size_t)b * S + qrow) * d + h * HD;
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_o + lane_base + c, r);
            tmem_ld_wait();
            if (qrow < S) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    const uint4 u = make_uint4(
                        pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])),
                        pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                        pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5])),
                        pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7])));
                    *reinterpret_cast<uint4*>(orow + c + j) = u;
                }
            }
        }
    }
    if (!ok && tid == 0) {
        // Let every MMA this CTA issued finish before TMEM is released.
        tc_commit(&bar[2]);
        mbar_wait(&bar[2], 0, err, kDevErrTimeoutDrain);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// Decode: one query per (sequence, head) at position *pos_dev (a device
// counter, so a captured decode step replays at every position) over keys
// 0..pos, split over the keys: a CTA per (64-key chunk, head, sequence)
// writes its chunk's partial softmax -- running max m, sum l and the
// unnormalised output o [hd] -- and attn_decode_combine_kernel merges the
// chunks, o = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c.  The grid covers
// max_seq keys; chunks past the position exit at once.
constexpr int kDecThreads = 128;
constexpr int kDecChunk = 64;

// Rotate-half RoPE of one head vector held kPer values per lane (lane l has
// dims l * kPer ..): the partner of dim j < hd/2 is j + hd/2, held by lane
// l ^ 16.  Same expression as rope_kv_kernel.
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

// The decode step's RoPE and KV-cache write are fused in: every CTA rotates
// its query itself, and the CTA whose chunk holds the current position
// rotates that position's key and writes key and value to the cache before
// it scores.
template <int HD>
__global__ void __launch_bounds__(kDecThreads)
attn_decode_partial_kernel(const float* __restrict__ qkv, const int* __restrict__ pos_dev, int H,
                           float* __restrict__ kc, float* __restrict__ vc, int max_seq,
                           float scale, const float2* __restrict__ rope,
                           float* __restrict__ part, int nch) {
    constexpr int kPer = HD / 32;             // q values per lane
    constexpr int kParts = kDecThreads / HD;  // key classes of the value pass
    constexpr int kWarps = kDecThreads / 32;
    constexpr int kKeysPerWarp = kDecChunk / kWarps;
    __shared__ float sp[kDecChunk];
    __shared__ float sacc[kDecThreads];
    const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Dependent launch.  The position counter and the cached keys and values
    // before it were written by earlier decode steps, which completed before
    // the previous kernel started (it is launched only after the one before
    // it has passed its own wait): prefetch this chunk's cached rows into L2
    // now, while the q/k/v projection (the previous kernel) still runs.
    {
        const int pos0 = *pos_dev;
        const int kk0 = c * kDecChunk;
        if (tid < 2 && kk0 < pos0) {
            const int rows = min(kDecChunk, pos0 - kk0);
            const float* src = (tid == 0 ? kc : vc) + (((size_t)b * H + h) * max_seq + kk0) * HD;
            prefetch_l2_bulk(src, (uint32_t)(rows * HD * sizeof(float)));
        }
    }
    wait_predecessor_grid();   // q/k/v of this step
    launch_dependents();
    const int pos = *pos_dev;
    const int n = pos + 1;
    const int k0 = c * kDecChunk;
    if (k0 >= n) return;
    const int nk = min(kDecChunk, n - k0);
    const int d = H * HD;
    const float* q = qkv + (size_t)b * 3 * d + h * HD;
    const float* kb = kc + (((size_t)b * H + h) * max_seq + k0) * HD;
    const float* vb = vc + (((size_t)b * H + h) * max_seq + k0) * HD;
    const float2* cs_row = rope + (size_t)pos * (HD / 2);
    float qv[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) qv[i] = q[lane * kPer + i];
    rope_lane<HD>(qv, lane, cs_row);
#pragma unroll
    for (int i = 0; i < kPer; ++i) qv[i] *= scale;
    if (pos < k0 + kDecChunk) {
        // This chunk holds the new position: its key and value enter the cache.
        if (warp == 0) {
            float kv[kPer];
#pragma unroll
            for (int i = 0; i < kPer; ++i) kv[i] = q[d + lane * kPer + i];
            rope_lane<HD>(kv, lane, cs_row);
            float* kd = kc + (((size_t)b * H + h) * max_seq + pos) * HD;
#pragma unroll
            for (int i = 0; i < kPer; ++i) kd[lane * kPer + i] = kv[i];
        } else if (warp == 1) {
            float* vd = vc + (((size_t)b * H + h) * max_seq + pos) * HD;
#pragma unroll
            for (int i = 0; i < kPer; ++i) vd[lane * kPer + i] = q[2 * d + lane * kPer + i];
        }
        __syncthreads();
    }
    // Scores: warp w takes keys w, w + 4, ...; every K row load is issued
    // before the reductions.
    float dots[kKeysPerWarp];
#pragma unroll
    for (int i = 0; i < kKeysPerWarp; ++i) {
        const int j = warp + kWarps * i;
        float acc = 0.0f;
        if (j < nk) {
            // Plain (coherent) vector loads: this kernel itself may have
            // written row pos.
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
        const int j = warp + kWarps * i;
        if (lane == 0 && j < nk) sp[j] = v;
    }
    __syncthreads();
    float* out = part + (((size_t)b * H + h) * nch + c) * (HD + 2);
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
    __syncthreads();
    // Values: thread (class, column) takes keys class, class + kParts, ...;
    // all of its V loads are issued before the first FMA (one memory round
    // trip per chunk instead of one per group of keys).
    const int col = tid % HD, cls = tid / HD;
    constexpr int kKeysPerThread = kDecChunk / kParts;
    float vv[kKeysPerThread];
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
        const int j = cls + i * kParts;
        vv[i] = j < nk ? vb[(size_t)j * HD + col] : 0.0f;
    }
    float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < kKeysPerThread; ++i) {
        const int j = cls + i * kParts;
        if (j < nk) a[i & 3] = fmaf(sp[j], vv[i], a[i & 3]);
    }
    sacc[tid] = (a[0] + a[1]) + (a[2] + a[3]);
    __syncthreads();
    if (tid < HD) {
        float v = sacc[tid];
#pragma unroll
        for (int p = 1; p < kParts; ++p) v += sacc[tid + p * HD];
        out[tid] = v;
    }
}

constexpr int kAttnStagedChunks = 2048;   // 16 KB of staged maxima and sums

// Chunk maxima and sums are staged in shared memory (one load round trip),
// then every chunk's output value of this thread's dimension is loaded 16
// chunks at a time before it is used; the sums run in chunk order.
template <int HD, bool kTf>
__global__ void __launch_bounds__(HD)
attn_decode_combine_kernel(const float* __restrict__ part, const int* __restrict__ pos_dev, int H,
                           int nch, void* __restrict__ a_hi, void* __restrict__ a_lo) {
    extern __shared__ float s_ml[];   // [nch] maxima, then [nch] sums
    const int h = blockIdx.x, b = blockIdx.y, t = threadIdx.x;
    wait_predecessor_grid();   // dependent launch: the partials
    launch_dependents();
    const int used = (*pos_dev + kDecChunk) / kDecChunk;   // chunks holding keys 0..pos
    const float* base = part + ((size_t)b * H + h) * nch * (HD + 2);
    // Staged when the launch gave shared memory for them (nch <= kAttnStagedChunks).
    const bool staged = nch <= kAttnStagedChunks;
    if (staged) {
        for (int c = t; c < used; c += HD) {
            s_ml[c] = base[(size_t)c * (HD + 2) + HD];
            s_ml[nch + c] = base[(size_t)c * (HD + 2) + HD + 1];
        }
        __syncthreads();
    }
    auto mval = [&](int c) { return staged ? s_ml[c] : base[(size_t)c * (HD + 2) + HD]; };
    auto lval = [&](int c) { return staged ? s_ml[nch + c] : base[(size_t)c * (HD + 2) + HD + 1]; };
    float M = -INFINITY;
    for (int c = 0; c < used; ++c) M = fmaxf(M, mval(c));
    float L = 0.0f, o = 0.0f;
    constexpr int kU = 16;
    for (int c0 = 0; c0 < used; c0 += kU) {
        float pv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
            pv[u] = c0 + u < used ? base[(size_t)(c0 + u) * (HD + 2) + t] : 0.0f;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int c = c0 + u;
            if (c < used) {
                const float w = expf(mval(c) - M);
                L = fmaf(w, lval(c), L);
                o = fmaf(w, pv[u], o);
            }
        }
    }
    store_a1<kTf>(a_hi, a_lo, b, H * HD, h * HD + t, o / L);
}

// ------------------------------------------------------------ argmax
// Greedy choice per row of logits [B][V], as generate_decode picks it
// (src/model.cu:2081-2089): the first index holding the maximum, scanning
// with a strict '>' from index 0 -- so NaNs are never chosen, except that a
// NaN at index 0 yields 0.  Writes the id to ids[b] and, if `seq_out`, to
// seq_out[b * seq_ld + step] (-1 once the sequence has emitted eos); the
// step is *step_dev when given (a captured decode step).
__global__ void __launch_bounds__(1024)
argmax_kernel(const float* __restrict__ logits, int V, int* __restrict__ ids,
              int* __restrict__ seq_out, int seq_ld, int step, const int* __restrict__ step_dev,
              int eos, int* __restrict__ done) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* row = logits + (size_t)b * V;
    float best = -INFINITY;
    int bi = -1;
    // Each thread scans its indices in ascending order (groups of 4, 8 groups
    // loaded at once when the row is 16-byte aligned, then the tail), keeping
    // the first index of its maximum.
    auto see = [&](float x, int v) {
        if (x > best || (bi < 0 && x == best)) { best = x; bi = v; }
    };
    int v_tail = 0;
    if ((V & 3) == 0) {
        constexpr int kU = 8;
        const float4* row4 = reinterpret_cast<const float4*>(row);
        const int nv = V / 4;
        for (int v0 = tid; v0 < nv; v0 += kU * blockDim.x) {
            float4 q[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int v = v0 + u * blockDim.x;
                if (v < nv) q[u] = row4[v];
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int v = v0 + u * blockDim.x;
                if (v < nv) {
                    see(q[u].x, 4 * v);
                    see(q[u].y, 4 * v + 1);
                    see(q[u].z, 4 * v + 2);
                    see(q[u].w, 4 * v + 3);
                }
            }
        }
        v_tail = V;
    }
    for (int v = v_tail + tid; v < V; v += blockDim.x) see(row[v], v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        best = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
        bi = lane < (int)(blockDim.x >> 5) ? si[lane] : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) { best = ov; bi = oi; }
        }
        if (lane == 0) {
            int id = bi < 0 || row[0] != row[0] ? 0 : bi;
            if (done) {
                if (done[b]) id = -1;
                else if (id == eos) done[b] = 1;
            }
            ids[b] = id < 0 ? 0 : id;
            if (seq_out) seq_out[(size_t)b * seq_ld + (step_dev ? *step_dev : step)] = id;
        }
    }
}

// ------------------------------------------------------------ step counters
// The decode position and generation step live on the device, so that one
// captured decode step (a CUDA graph) serves every position.
__global__ void set_counters_kernel(int* pos_dev, int* step_dev, int pos, int step) {
    *pos_dev = pos;
    *step_dev = step;
}

__global__ void advance_kernel(int* pos_dev, int* step_dev) {
    ++*pos_dev;
    ++*step_dev;
}

// gen[b][*step_dev][:] = logits[b][:] (generate's logits output, [B][n][V]).
__global__ void __launch_bounds__(256)
save_logits_kernel(const float4* __restrict__ logits, float4* __restrict__ gen,
                   const int* __restrict__ step_dev, int V4, int n) {
    const int b = blockIdx.y;
    const size_t dst = ((size_t)b * n + *step_dev) * V4;
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V4; v += gridDim.x * blockDim.x)
        gen[dst + v] = logits[(size_t)b * V4 + v];
}

// ------------------------------------------------------------ dense GEMV
// Decode-sized dense projections (q/k/v, o, the output head at T <= 4 rows,
// BF16): y[t][n] (+)= W[n] . A[t] for t < T, W bf16 [N][K], A the bf16
// operand rows; `accumulate` adds into y (the o projection into the residual
// stream), else y is overwritten.  These are weight-streaming bound; 128-row tensor-core tiles would be
// 1-4 rows full and spread the N x K stream over few CTAs, so instead every
// warp of one CTA per SM owns an equal contiguous range of weight rows and
// streams them once with 128-bit loads, two rows at a time, all of a row
// pair's loads in flight.  Launched as a dependent grid: the weights do not
// depend on the previous kernel, so each warp starts an L2 prefetch of its
// first rows before it waits for that kernel; the activations and y are
// read after the wait.  Each y element is one warp's sum (no atomics).
constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxRows = 4;
constexpr uint32_t kGemvPrefetchBytes = 16384;   // per warp
constexpr int kGemvVecs = 8;                     // 16-byte loads per row per lane per pass

__device__ __forceinline__ uint4 gemv_stream_load(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& r, float (&v)[8]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

template <int TM>
__global__ void __launch_bounds__(kGemvThreads, 1)
dense_gemv_kernel(const __nv_bfloat16* __restrict__ W, const __nv_bfloat16* __restrict__ A,
                  int N, int K, int T, int accumulate, float* __restrict__ y) {
    const int lane = threadIdx.x & 31;
    const long long nw = (long long)gridDim.x * kGemvWarps;
    const long long gw = (long long)blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    const int r0 = (int)((long long)N * gw / nw), r1 = (int)((long long)N * (gw + 1) / nw);
    if (lane == 0 && r1 > r0) {
        const size_t bytes = (size_t)(r1 - r0) * K * sizeof(__nv_bfloat16);
        prefetch_l2_bulk(W + (size_t)r0 * K,
                         (uint32_t)(bytes < kGemvPrefetchBytes ? bytes : kGemvPrefetchBytes));
    }
    wait_predecessor_grid();
    launch_dependents();
    // The T activation rows, staged once per CTA through L2 (written by the
    // previous kernel) into shared memory, where every warp reads them.
    extern __shared__ __align__(16) uint4 s_a[];
    const int kv = K / 8;
    for (int i = threadIdx.x; i < T * kv; i += blockDim.x)
        s_a[i] = __ldcg(reinterpret_cast<const uint4*>(A) + i);
    __syncthreads();
    for (int r = r0; r < r1; r += 2) {
        const bool two = r + 1 < r1;
        const __nv_bfloat16* w0 = W + (size_t)r * K;
        const __nv_bfloat16* w1 = two ? w0 + K : w0;
        // This warp's outputs (through L2: the previous kernel may have just
        // written them), loaded now so their latency overlaps the stream.
        float yv[2][TM];
#pragma unroll
        for (int m = 0; m < TM; ++m) {
            yv[0][m] = (accumulate && lane == 0 && m < T) ? __ldcg(y + (size_t)m * N + r) : 0.0f;
            yv[1][m] = (accumulate && lane == 0 && m < T && two) ? __ldcg(y + (size_t)m * N + r + 1)
                                                                 : 0.0f;
        }
        float acc[2][TM];
#pragma unroll
        for (int m = 0; m < TM; ++m) acc[0][m] = acc[1][m] = 0.0f;
        for (int k0 = lane * 8; k0 < K; k0 += 32 * 8 * kGemvVecs) {
            uint4 raw[kGemvVecs][2];
#pragma unroll
            for (int u = 0; u < kGemvVecs; ++u) {
                const int kk = k0 + u * 256;
                if (kk < K) {
                    raw[u][0] = gemv_stream_load(w0 + kk);
                    raw[u][1] = gemv_stream_load(w1 + kk);
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvVecs; ++u) {
                const int kk = k0 + u * 256;
                if (kk >= K) break;
                float wv0[8], wv1[8];
                bf16x8_to_f32(raw[u][0], wv0);
                bf16x8_to_f32(raw[u][1], wv1);
#pragma unroll
                for (int m = 0; m < TM; ++m) {
                    if (m >= T) break;
                    float av[8];
                    bf16x8_to_f32(s_a[m * kv + kk / 8], av);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        acc[0][m] = fmaf(wv0[q], av[q], acc[0][m]);
                        acc[1][m] = fmaf(wv1[q], av[q], acc[1][m]);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < TM; ++m) {
            if (m >= T) break;
            const float v0 = warp_sum(acc[0][m]);
            const float v1 = warp_sum(acc[1][m]);
            if (lane == 0) {
                y[(size_t)m * N + r] = yv[0][m] + v0;
                if (two) y[(size_t)m * N + r + 1] = yv[1][m] + v1;
            }
        }
    }
}

// ------------------------------------------------------------ dense projection
// y [rows][N] (+)= A [rows][K] . W[N][K]^T on the expert GEMM: a Layer with
// one expert whose "down" weights are W (d = N, ffp = K), reading the shared
// A operand and tile list of the decoder.
struct Dense {
    Layer L;
};

void free_dense(Dense& D) {
    if (D.L.w2_hi) cudaFree(D.L.w2_hi);
    if (D.L.w2_lo) cudaFree(D.L.w2_lo);
    D.L.w2_hi = D.L.w2_lo = nullptr;
}

}  // namespace
}  // namespace moe

// ============================================================ the model
struct MoeDecoder {
    MoeDecoderConfig cfg{};
    int d = 0, H = 0, HD = 0, V = 0, nl = 0;
    int max_rows = 0;         // max_batch * max_seq
    int a_rows = 0;           // A operand rows (max_rows rounded up to 256)
    std::vector<float*> attn_norm;
    std::vector<moe::Dense> qkv, wo;
    std::vector<MoeHandle*> moe;
    moe::Dense head;
    float* embed = nullptr;
    float* final_norm = nullptr;
    float2* rope = nullptr;   // [max_seq][head_dim / 2] (cos, sin)
    float* kc = nullptr;      // [n_layers][max_batch][H][max_seq][head_dim]
    float* vc = nullptr;
    float* x = nullptr;       // [max_rows][d] residual stream (ping)
    float* x2 = nullptr;      // (pong)
    float* qkvbuf = nullptr;  // [max_rows][3d]
    float* logits = nullptr;  // [max_batch][vocab]
    float* gen_logits = nullptr;   // [max_batch][gen_cap][vocab] (generate)
    size_t gen_cap = 0;
    int* tok = nullptr;       // [max_rows]
    int* next = nullptr;      // [max_batch]
    int* seq_ids = nullptr;   // [max_batch][max_seq] generated ids
    int* done = nullptr;      // [max_batch]
    void* a_hi = nullptr;
    void* a_lo = nullptr;
    CUtensorMap tm_a_hi{}, tm_a_lo{};
    moe::MTile* mtiles = nullptr;
    moe::MTile* ptiles = nullptr;
    int* num_mtiles = nullptr;
    int* num_ptiles = nullptr;
    int* row_token = nullptr;
    float* row_weight = nullptr;
    int* dev_err = nullptr;
    float* attn_part = nullptr;   // decode attention partials [max_batch][H][chunks][hd + 2]
    int* pos_dev = nullptr;   // next decode position
    int* step_dev = nullptr;  // next generation step
    // The captured decode step of generate, for (batch, eos, logits buffer,
    // new tokens); re-captured when any of them changes.
    cudaGraphExec_t step_graph = nullptr;
    int g_B = -1, g_eos = 0, g_n = 0;
    float* g_logits = nullptr;
    int sm_count = 148;
    // The fused batch-1 decode step (decode_step.cu): available when the
    // configuration fits it (step_ok), used while step_on is set (off by
    // default: on B200 the kernel chain measured faster).
    bool step_ok = false, step_on = false;
    moe::StepLayer* step_layers = nullptr;   // [n_layers], device
    float* step_ws = nullptr;                // xm, router logits, h, part
    unsigned* step_sync = nullptr;           // grid-barrier words [3]
    size_t step_smem = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev[3] = {};
    float t_prefill = 0.0f, t_decode = 0.0f;
    int B = 0, pos = 0;       // sequences of the current batch, next position
    size_t bytes = 0;
};

namespace moe {
namespace {

#define DEC_CUDA(call)                                                                 \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return report_error(MOE_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

#define DEC_RC(call)              \
    do {                          \
        int rc_ = (call);         \
        if (rc_) return rc_;      \
    } while (0)

struct DecDeviceGuard {
    int prev = -1;
    explicit DecDeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DecDeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
cudaError_t dec_alloc(MoeDecoder& m, T** p, size_t bytes) {
    *p = nullptr;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes ? bytes : 256);
    if (e == cudaSuccess) m.bytes += bytes;
    return e;
}

int round_up(int v, int g) { return (v + g - 1) / g * g; }

// W = the listed fp32 row blocks stacked ([sum rows][K]), host or device
// pointers, converted into the projection's weight planes.
int make_dense(MoeDecoder& m, Dense& D, const float* const* parts, const int* part_rows,
               int nparts, int K) {
    Layer& L = D.L;
    int N = 0;
    for (int i = 0; i < nparts; ++i) N += part_rows[i];
    L.cfg.precision = m.cfg.precision;
    L.cfg.device = m.cfg.device;
    L.d = N;
    L.ff = K;
    L.ffp = K;
    L.E = 1;
    L.E_route = 1;
    L.k = 1;
    L.sm_count = m.sm_count;
    L.gemm_variant = MOE_GEMM_AUTO;
    L.profile = false;
    const bool tf = split_planes(L);   // 3xTF32 (the decoder's precisions: FP32, BF16)
    const size_t eb = plane_bytes(L);
    DEC_CUDA(dec_alloc(m, &L.w2_hi, eb * N * K));
    if (tf) DEC_CUDA(dec_alloc(m, &L.w2_lo, eb * N * K));
    float* stage = nullptr;
    DEC_CUDA(cudaMalloc(&stage, sizeof(float) * (size_t)N * K));
    size_t off = 0;
    int rc = MOE_OK;
    for (int i = 0; i < nparts && !rc; ++i) {
        const size_t n = (size_t)part_rows[i] * K;
        cudaError_t e = cudaMemcpyAsync(stage + off, parts[i], sizeof(float) * n, cudaMemcpyDefault,
                                        m.stream);
        if (e != cudaSuccess) rc = report_error(MOE_ERR_CUDA, std::string("weight copy: ") + cudaGetErrorString(e));
        off += n;
    }
    if (!rc) {
        cudaError_t e = convert_down(L, 0, stage, m.stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m.stream);
        if (e != cudaSuccess) rc = report_error(MOE_ERR_CUDA, std::string("weight conversion: ") + cudaGetErrorString(e));
    }
    cudaFree(stage);
    if (rc) return rc;
    const uint32_t box_k = tf ? 32 : 64;
    std::string err;
    const bool bf = !tf;
    if (!make_tmap_2d(&L.tm_w2_hi, L.w2_hi, bf, K, N, box_k, kTileN, &err) ||
        !make_tmap_2d(&L.tm_w2_hi2, L.w2_hi, bf, K, N, box_k, kTileN / 2, &err))
        return report_error(MOE_ERR_CUDA, err);
    if (tf) {
        if (!make_tmap_2d(&L.tm_w2_lo, L.w2_lo, false, K, N, box_k, kTileN, &err) ||
            !make_tmap_2d(&L.tm_w2_lo2, L.w2_lo, false, K, N, box_k, kTileN / 2, &err))
            return report_error(MOE_ERR_CUDA, err);
    } else {
        L.tm_w2_lo = L.tm_w2_hi;
        L.tm_w2_lo2 = L.tm_w2_hi2;
    }
    Workspace& W = L.ws;
    W.mtiles = m.mtiles;
    W.num_mtiles = m.num_mtiles;
    W.ptiles = m.ptiles;
    W.num_ptiles = m.num_ptiles;
    W.row_token = m.row_token;
    W.row_weight = m.row_weight;
    W.h_hi = m.a_hi;
    W.h_lo = m.a_lo;
    W.tm_h_hi = m.tm_a_hi;
    W.tm_h_lo = m.tm_a_lo;
    W.dev_err = m.dev_err;
    W.cap_rows = m.a_rows;
    return MOE_OK;
}

bool tf_mode(const MoeDecoder& m) { return m.cfg.precision == MOE_PREC_FP32; }

float* layer_kc(MoeDecoder& m, int l) {
    return m.kc + (size_t)l * m.cfg.max_batch * m.H * m.cfg.max_seq * m.HD;
}
float* layer_vc(MoeDecoder& m, int l) {
    return m.vc + (size_t)l * m.cfg.max_batch * m.H * m.cfg.max_seq * m.HD;
}

cudaError_t launch_tiles(MoeDecoder& m, int T) {
    const int rows_pad = round_up(T, 2 * kTileM);
    dense_tiles_kernel<<<std::min((rows_pad + 255) / 256, 4 * m.sm_count), 256, 0, m.stream>>>(
        T, rows_pad, m.mtiles, m.num_mtiles, m.ptiles, m.num_ptiles, m.row_token, m.row_weight);
    return cudaGetLastError();
}

// A kernel launched as a dependent grid of the previous one on m.stream (it
// calls wait_predecessor_grid() before touching earlier kernels' data).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(MoeDecoder& m, dim3 grid, dim3 block, size_t smem, void (*kern)(KArgs...),
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = m.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// The dense projections of T rows run as the GEMV (BF16, T <= 4, the
// activation rows fit the default shared memory) instead of the grouped GEMM.
bool use_gemv(const MoeDecoder& m, int T) {
    return T >= 1 && T <= kGemvMaxRows && !tf_mode(m) && m.d % 8 == 0 &&
           (size_t)T * m.d * sizeof(__nv_bfloat16) <= 48 * 1024;
}

// y (+)= A . W^T for the first T rows of the shared A operand (y [T][N]):
// the GEMV at decode-sized T (`accumulate` adds into y, else y is
// overwritten), the grouped GEMM otherwise (which always adds, into a y the
// caller zeroed unless it accumulates).
cudaError_t launch_dense(MoeDecoder& m, const Dense& D, int T, float* y, bool accumulate) {
    const Layer& L = D.L;
    if (!use_gemv(m, T)) return launch_expert_gemm_rows(L, T, y, m.stream, 1);
    const auto* W = static_cast<const __nv_bfloat16*>(L.w2_hi);
    const auto* A = static_cast<const __nv_bfloat16*>(m.a_hi);
    const size_t smem = (size_t)T * L.ffp * sizeof(__nv_bfloat16);
    const int acc = accumulate ? 1 : 0;
    const dim3 grid(m.sm_count), block(kGemvThreads);
    if (T == 1) return launch_pdl(m, grid, block, smem, dense_gemv_kernel<1>, W, A, L.d, L.ffp, T, acc, y);
    if (T == 2) return launch_pdl(m, grid, block, smem, dense_gemv_kernel<2>, W, A, L.d, L.ffp, T, acc, y);
    return launch_pdl(m, grid, block, smem, dense_gemv_kernel<4>, W, A, L.d, L.ffp, T, acc, y);
}

// rms_norm(rows src0 + r * stride of x, r < T) -> A, zeroing `zero` [zero_n]
// floats.  For the grouped GEMM, A's rows up to the next 256 are zeroed too;
// the GEMV reads only the T rows.
cudaError_t launch_rms_pack(MoeDecoder& m, const float* x, int src0, int stride, int T,
                            const float* w, float* zero, size_t zero_n) {
    const float eps = m.cfg.rms_eps;
    float4* z = reinterpret_cast<float4*>(zero);
    if (use_gemv(m, T) && m.d <= 4 * kPackThreads * kPackMaxVec)
        return launch_pdl(m, dim3(T), dim3(kPackThreads), 0, rms_pack_row_kernel<false>, x, src0,
                          stride, m.d, eps, w, m.a_hi, m.a_lo, z, zero_n / 4);
    const int rows_pad = use_gemv(m, T) ? T : round_up(T, 2 * kTileM);
    const int grid = (rows_pad + 7) / 8;
    if (tf_mode(m))
        return launch_pdl(m, dim3(grid), dim3(256), 0, rms_pack_kernel<true>, x, src0, stride, T,
                          rows_pad, m.d, eps, w, m.a_hi, m.a_lo, z, zero_n / 4);
    return launch_pdl(m, dim3(grid), dim3(256), 0, rms_pack_kernel<false>, x, src0, stride, T,
                      rows_pad, m.d, eps, w, m.a_hi, m.a_lo, z, zero_n / 4);
}

template <int HD>
cudaError_t launch_attention_t(MoeDecoder& m, int l, int B, int S, bool prefill) {
    const float scale = 1.0f / sqrtf((float)HD);
    if (prefill && !tf_mode(m)) {
        const size_t smem = TcAttn<HD>::kSmem;
        auto k = attn_prefill_tc_kernel<HD>;
        cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        k<<<dim3((S + kTcBQ - 1) / kTcBQ, m.H, B), 128, smem, m.stream>>>(
            m.qkvbuf, S, m.H, layer_kc(m, l), layer_vc(m, l), m.cfg.max_seq, scale, m.a_hi,
            m.dev_err);
    } else if (prefill) {
        const size_t smem = AttnSmem<HD>::kBytes;
        dim3 grid((S + kAttBQ - 1) / kAttBQ, m.H, B);
        if (tf_mode(m)) {
            auto k = attn_prefill_kernel<HD, true>;
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            k<<<grid, 256, smem, m.stream>>>(m.qkvbuf, S, m.H, layer_kc(m, l), layer_vc(m, l),
                                             m.cfg.max_seq, scale, m.a_hi, m.a_lo);
        } else {
            auto k = attn_prefill_kernel<HD, false>;
            cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            k<<<grid, 256, smem, m.stream>>>(m.qkvbuf, S, m.H, layer_kc(m, l), layer_vc(m, l),
                                             m.cfg.max_seq, scale, m.a_hi, m.a_lo);
        }
    } else {
        const int nch = (m.cfg.max_seq + kDecChunk - 1) / kDecChunk;
        cudaError_t e = launch_pdl(m, dim3(nch, m.H, B), dim3(kDecThreads), 0,
                                   attn_decode_partial_kernel<HD>, m.qkvbuf, m.pos_dev, m.H,
                                   layer_kc(m, l), layer_vc(m, l), m.cfg.max_seq, scale, m.rope,
                                   m.attn_part, nch);
        if (e != cudaSuccess) return e;
        const size_t smem = nch <= kAttnStagedChunks ? 2 * sizeof(float) * (size_t)nch : 0;
        if (tf_mode(m))
            return launch_pdl(m, dim3(m.H, B), dim3(HD), smem, attn_decode_combine_kernel<HD, true>,
                              m.attn_part, m.pos_dev, m.H, nch, m.a_hi, m.a_lo);
        return launch_pdl(m, dim3(m.H, B), dim3(HD), smem, attn_decode_combine_kernel<HD, false>,
                          m.attn_part, m.pos_dev, m.H, nch, m.a_hi, m.a_lo);
    }
    return cudaGetLastError();
}

cudaError_t launch_rope_kv(MoeDecoder& m, int l, int T, int rps, const int* pos_dev) {
    if (m.HD == 128)
        rope_kv_kernel<128><<<T, 256, 0, m.stream>>>(m.qkvbuf, rps, 0, pos_dev, m.H, m.rope,
                                                     layer_kc(m, l), layer_vc(m, l), m.cfg.max_seq);
    else
        rope_kv_kernel<64><<<T, 256, 0, m.stream>>>(m.qkvbuf, rps, 0, pos_dev, m.H, m.rope,
                                                    layer_kc(m, l), layer_vc(m, l), m.cfg.max_seq);
    return cudaGetLastError();
}

// One decoder layer over T rows: B sequences of rps rows each (prefill:
// rps = S from position 0; decode: rps = 1 at the device position).
int run_layer(MoeDecoder& m, int l, int B, int T, int rps, bool prefill) {
    // The GEMV overwrites q/k/v; the grouped GEMM adds into a zeroed buffer.
    const bool gemv = use_gemv(m, T);
    DEC_CUDA(launch_rms_pack(m, m.x, 0, 1, T, m.attn_norm[l], gemv ? nullptr : m.qkvbuf,
                             gemv ? 0 : (size_t)T * 3 * m.d));
    DEC_CUDA(launch_dense(m, m.qkv[l], T, m.qkvbuf, false));
    // Decode rotates q and k inside the attention kernel (and writes the cache there).
    if (prefill) DEC_CUDA(launch_rope_kv(m, l, T, rps, nullptr));
    if (m.HD == 128)
        DEC_CUDA(launch_attention_t<128>(m, l, B, rps, prefill));
    else
        DEC_CUDA(launch_attention_t<64>(m, l, B, rps, prefill));
    DEC_CUDA(launch_dense(m, m.wo[l], T, m.x, true));   // x += o . Wo^T
    DEC_RC(moe_block_forward_device(m.moe[l], m.x, m.x2, T, m.stream));
    std::swap(m.x, m.x2);
    return MOE_OK;
}

// Greedy ids of the B logits rows (see run_head).
int launch_argmax(MoeDecoder& m, int B, bool record, int step, const int* step_dev, int eos) {
    argmax_kernel<<<B, 1024, 0, m.stream>>>(m.logits, m.V, m.next, record ? m.seq_ids : nullptr,
                                            m.cfg.max_seq, step, step_dev, eos,
                                            record ? m.done : nullptr);
    DEC_CUDA(cudaGetLastError());
    return MOE_OK;
}

// Final norm of row src0 + b * stride (b < B), the output head into
// m.logits, and the greedy ids; with `record`, also into seq_ids[b][step]
// (step = *step_dev when step_dev is given) with the EOS bookkeeping.  Leaves
// the tile list at B rows.
int run_head(MoeDecoder& m, int B, int src0, int stride, bool record, int step,
             const int* step_dev, int eos) {
    const bool gemv = use_gemv(m, B);
    if (!gemv) DEC_CUDA(launch_tiles(m, B));
    DEC_CUDA(launch_rms_pack(m, m.x, src0, stride, B, m.final_norm, gemv ? nullptr : m.logits,
                             gemv ? 0 : (size_t)B * m.V));
    DEC_CUDA(launch_dense(m, m.head, B, m.logits, false));
    return launch_argmax(m, B, record, step, step_dev, eos);
}

// Prefill of B sequences of S tokens from m.tok; the device counters then
// point at position S, generation step 1.
int run_prefill(MoeDecoder& m, int B, int S, bool record, int eos) {
    const int T = B * S;
    DEC_CUDA(launch_tiles(m, T));
    embed_gather_kernel<<<T, 256, 0, m.stream>>>(m.tok, m.embed, m.V, m.d, m.x, m.dev_err);
    DEC_CUDA(cudaGetLastError());
    for (int l = 0; l < m.nl; ++l) DEC_RC(run_layer(m, l, B, T, S, true));
    DEC_RC(run_head(m, B, S - 1, S, record, 0, nullptr, eos));
    set_counters_kernel<<<1, 1, 0, m.stream>>>(m.pos_dev, m.step_dev, S, 1);
    DEC_CUDA(cudaGetLastError());
    m.B = B;
    m.pos = S;
    return MOE_OK;
}

StepArgs step_args(MoeDecoder& m, const int* tok);

// One decode step of the m.B sequences: token ids from `tok` (device, [B])
// at the device position, which it advances.  Enqueues only -- the host's
// m.pos is the caller's to advance -- so it can be captured as a graph.  With
// `record`, the ids go to seq_ids at the device step and, if `save`, the
// logits to save[b][step] ([B][n][V]).
int run_decode(MoeDecoder& m, const int* tok, bool record, int eos, float* save, int n) {
    const int B = m.B;
    if (B == 1 && m.step_ok && m.step_on) {
        // One sequence: the whole layer stack and the output head in one
        // cooperative launch, then the greedy id.
        DEC_CUDA(launch_step_fused(step_args(m, tok), m.HD, m.sm_count, m.step_smem, m.stream));
        DEC_RC(launch_argmax(m, 1, record, 0, m.step_dev, eos));
    } else {
        embed_gather_kernel<<<B, 256, 0, m.stream>>>(tok, m.embed, m.V, m.d, m.x, m.dev_err);
        DEC_CUDA(cudaGetLastError());
        for (int l = 0; l < m.nl; ++l) DEC_RC(run_layer(m, l, B, B, 1, false));
        DEC_RC(run_head(m, B, 0, 1, record, 0, m.step_dev, eos));
    }
    if (save) {
        save_logits_kernel<<<dim3(std::max(1, std::min(m.V / 4 / 256, 64)), B), 256, 0, m.stream>>>(
            reinterpret_cast<const float4*>(m.logits), reinterpret_cast<float4*>(save),
            m.step_dev, m.V / 4, n);
        DEC_CUDA(cudaGetLastError());
    }
    advance_kernel<<<1, 1, 0, m.stream>>>(m.pos_dev, m.step_dev);
    DEC_CUDA(cudaGetLastError());
    return MOE_OK;
}

void drop_graph(MoeDecoder& m) {
    if (m.step_graph) cudaGraphExecDestroy(m.step_graph);
    m.step_graph = nullptr;
    m.g_B = -1;
}

// generate's decode step as a CUDA graph (captured once per batch / eos /
// logits buffer / length), so that a step costs one launch instead of
// about ten per layer.
int step_graph(MoeDecoder& m, int eos, float* save, int n) {
    if (m.step_graph && m.g_B == m.B && m.g_eos == eos && m.g_logits == save && m.g_n == n)
        return MOE_OK;
    drop_graph(m);
    DEC_CUDA(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeRelaxed));
    const int rc = run_decode(m, m.next, true, eos, save, n);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(m.stream, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess)
        return report_error(MOE_ERR_CUDA, std::string("decode-step capture: ") + cudaGetErrorString(ce));
    const cudaError_t ie = cudaGraphInstantiate(&m.step_graph, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
        m.step_graph = nullptr;
        return report_error(MOE_ERR_CUDA, std::string("decode-step graph: ") + cudaGetErrorString(ie));
    }
    m.g_B = m.B;
    m.g_eos = eos;
    m.g_logits = save;
    m.g_n = n;
    return MOE_OK;
}

int check_dev_err(MoeDecoder& m) {
    int flag = 0;
    DEC_CUDA(cudaMemcpy(&flag, m.dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (!flag) return MOE_OK;
    cudaMemset(m.dev_err, 0, sizeof(int));
    // A fused step that gave up left its barrier words mid-step.
    if (m.step_sync) cudaMemset(m.step_sync, 0, 4 * sizeof(unsigned));
    if (flag & kDecErrToken) return report_error(MOE_ERR_INVALID, "a token id is outside [0, vocab)");
    char buf[96];
    std::snprintf(buf, sizeof buf, "a device-side wait timed out (flags 0x%x)", flag);
    return report_error(MOE_ERR_TIMEOUT, buf);
}

int validate(const MoeDecoderConfig& c) {
    auto bad = [](int code, const char* msg) { return report_error(code, msg); };
    if (c.n_layers < 1) return bad(MOE_ERR_INVALID, "n_layers must be >= 1");
    if (c.head_dim != 64 && c.head_dim != 128) return bad(MOE_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
    if (c.n_heads < 1 || c.d_model != c.n_heads * c.head_dim)
        return bad(MOE_ERR_UNSUPPORTED, "d_model must equal n_heads * head_dim");
    if (c.d_model % 128 != 0) return bad(MOE_ERR_UNSUPPORTED, "d_model must be a multiple of 128");
    if (c.vocab < 32 || c.vocab % 32 != 0) return bad(MOE_ERR_UNSUPPORTED, "vocab must be a positive multiple of 32");
    if (c.max_batch < 1 || c.max_seq < 1) return bad(MOE_ERR_INVALID, "max_batch and max_seq must be >= 1");
    if ((long long)c.max_batch * c.max_seq > (1 << 22)) return bad(MOE_ERR_UNSUPPORTED, "max_batch * max_seq too large");
    if (c.precision == MOE_PREC_FP32_BF16X3)
        return bad(MOE_ERR_UNSUPPORTED, "the decoder runs in FP32 (3xTF32) or BF16 precision");
    if (c.precision != MOE_PREC_FP32 && c.precision != MOE_PREC_BF16) return bad(MOE_ERR_INVALID, "unknown precision");
    if (!(c.rms_eps >= 0.0f) || !(c.rope_base > 0.0f)) return bad(MOE_ERR_INVALID, "rms_eps >= 0 and rope_base > 0 required");
    return MOE_OK;
}

// The fused batch-1 decode step: available in BF16 precision when one
// 512-thread CTA per SM fits the step's shared memory, every router expert
// has a CTA of its own (E <= SMs) and the MoE blocks use the RMSNorm with
// dense bf16 operands of row stride d.  Builds the per-layer operand table
// and the step's workspace.
int setup_fused_step(MoeDecoder& m) {
    if (tf_mode(m) || m.d > 8192 || m.d % 128 != 0) return MOE_OK;
    const Layer& L0 = m.moe[0]->L;
    if (L0.E > m.sm_count || L0.E > kMaxExperts || L0.k > kMaxTopK || L0.k < 1) return MOE_OK;
    for (int l = 0; l < m.nl; ++l) {
        const Layer& L = m.moe[l]->L;
        if (!L.norm_rms || !L.norm_w || !L.norm_b || !L.w13_hi || !L.w2_hi || L.ep) return MOE_OK;
        if (m.qkv[l].L.ffp != m.d || m.wo[l].L.ffp != m.d) return MOE_OK;
    }
    if (m.head.L.ffp != m.d) return MOE_OK;
    int coop = 0;
    DEC_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m.cfg.device));
    if (!coop) return MOE_OK;
    const int nch = (m.cfg.max_seq + kDecChunk - 1) / kDecChunk;
    const size_t smem = step_fused_smem(m.d, m.H, nch);
    if (smem > 200 * 1024 || step_fused_occupancy(m.HD, smem) < 1) {
        cudaGetLastError();
        return MOE_OK;
    }
    std::vector<StepLayer> tab(m.nl);
    for (int l = 0; l < m.nl; ++l) {
        const Layer& L = m.moe[l]->L;
        StepLayer& t = tab[l];
        t.attn_norm = m.attn_norm[l];
        t.wqkv = static_cast<const __nv_bfloat16*>(m.qkv[l].L.w2_hi);
        t.wo = static_cast<const __nv_bfloat16*>(m.wo[l].L.w2_hi);
        t.kc = layer_kc(m, l);
        t.vc = layer_vc(m, l);
        t.wg = L.wg;
        t.bias = L.bias;
        t.ffn_norm = L.norm_w;
        t.ffn_norm_b = L.norm_b;
        t.ffn_eps = L.norm_eps;
        t.w13 = static_cast<const __nv_bfloat16*>(L.w13_hi);
        t.w2 = static_cast<const __nv_bfloat16*>(L.w2_hi);
    }
    DEC_CUDA(dec_alloc(m, &m.step_layers, sizeof(StepLayer) * m.nl));
    DEC_CUDA(cudaMemcpy(m.step_layers, tab.data(), sizeof(StepLayer) * m.nl, cudaMemcpyHostToDevice));
    const size_t nk = (L0.ffp + kDownChunk - 1) / kDownChunk;
    const size_t ws = (size_t)m.d + 256 + (size_t)L0.k * L0.ffp + nk * L0.k * m.d;
    DEC_CUDA(dec_alloc(m, &m.step_ws, sizeof(float) * ws));
    DEC_CUDA(dec_alloc(m, &m.step_sync, 4 * sizeof(unsigned)));
    DEC_CUDA(cudaMemset(m.step_sync, 0, 4 * sizeof(unsigned)));
    m.step_smem = smem;
    m.step_ok = true;   // available; off until moe_decoder_set_fused_step enables it
    return MOE_OK;
}

// The step's operands for token ids `tok` (device, one id).
StepArgs step_args(MoeDecoder& m, const int* tok) {
    const Layer& L0 = m.moe[0]->L;
    StepArgs a{};
    a.layers = m.step_layers;
    a.nl = m.nl;
    a.d = m.d;
    a.H = m.H;
    a.E = L0.E;
    a.k = L0.k;
    a.ffp = L0.ffp;
    a.V = m.V;
    a.max_seq = m.cfg.max_seq;
    a.nch = (m.cfg.max_seq + kDecChunk - 1) / kDecChunk;
    a.policy = L0.cfg.router_policy;
    a.quantum = L0.cfg.router_quantum;
    a.tie_eps = L0.cfg.router_tie_eps;
    a.eps = m.cfg.rms_eps;
    a.scale = 1.0f / sqrtf((float)m.HD);
    a.tok = tok;
    a.embed = m.embed;
    a.final_norm = m.final_norm;
    a.head = static_cast<const __nv_bfloat16*>(m.head.L.w2_hi);
    a.rope = m.rope;
    a.pos_dev = m.pos_dev;
    a.qkv = m.qkvbuf;
    a.attn_part = m.attn_part;
    a.xm = m.step_ws;
    a.logits_e = a.xm + m.d;
    a.h = a.logits_e + 256;
    a.part = a.h + (size_t)L0.k * L0.ffp;
    a.logits = m.logits;
    a.sync = m.step_sync;
    a.err = m.dev_err;
    return a;
}

void destroy(MoeDecoder* m) {
    if (!m) return;
    DecDeviceGuard guard(m->cfg.device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    drop_graph(*m);
    for (MoeHandle* h : m->moe) moe_destroy(h);
    for (auto& D : m->qkv) free_dense(D);
    for (auto& D : m->wo) free_dense(D);
    free_dense(m->head);
    for (float* p : m->attn_norm) cudaFree(p);
    void* bufs[] = {m->embed, m->final_norm, m->rope, m->kc, m->vc, m->x, m->x2, m->qkvbuf,
                    m->logits, m->gen_logits, m->tok, m->next, m->seq_ids, m->done, m->a_hi,
                    m->a_lo, m->mtiles, m->ptiles, m->num_mtiles, m->num_ptiles, m->row_token,
                    m->row_weight, m->dev_err, m->pos_dev, m->step_dev, m->attn_part,
                    m->step_layers, m->step_ws, m->step_sync};
    for (void* p : bufs)
        if (p) cudaFree(p);
    for (cudaEvent_t e : m->ev)
        if (e) cudaEventDestroy(e);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int create(const MoeDecoderConfig* cfg, const MoeDecoderWeights* w, bool device_ptrs,
           MoeDecoder** out) {
    if (!cfg || !w || !out) return report_error(MOE_ERR_INVALID, "null argument");
    *out = nullptr;
    DEC_RC(validate(*cfg));
    if (!w->embed || !w->final_norm || !w->attn_norm || !w->wq || !w->wk || !w->wv || !w->wo ||
        !w->ffn_norm || !w->router || !w->w1 || !w->w3 || !w->w2)
        return report_error(MOE_ERR_INVALID, "missing weight pointers");
    int ndev = 0;
    DEC_CUDA(cudaGetDeviceCount(&ndev));
    if (cfg->device < 0 || cfg->device >= ndev) return report_error(MOE_ERR_INVALID, "no such device");
    DecDeviceGuard guard(cfg->device);
    int major = 0, minor = 0;
    DEC_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cfg->device));
    DEC_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, cfg->device));
    if (major != 10 || minor != 0)
        return report_error(MOE_ERR_UNSUPPORTED, "libmoe_b200 is built for sm_100a (B200) only");
    std::unique_ptr<MoeDecoder, void (*)(MoeDecoder*)> m(new MoeDecoder(), destroy);
    MoeDecoder& M = *m;
    M.cfg = *cfg;
    M.d = cfg->d_model;
    M.H = cfg->n_heads;
    M.HD = cfg->head_dim;
    M.V = cfg->vocab;
    M.nl = cfg->n_layers;
    M.max_rows = cfg->max_batch * cfg->max_seq;
    M.a_rows = round_up(std::max(M.max_rows, cfg->max_batch), 2 * kTileM);
    DEC_CUDA(cudaDeviceGetAttribute(&M.sm_count, cudaDevAttrMultiProcessorCount, cfg->device));
    DEC_CUDA(cudaStreamCreateWithFlags(&M.stream, cudaStreamNonBlocking));
    for (auto& e : M.ev) DEC_CUDA(cudaEventCreate(&e));
    const size_t d = M.d, V = M.V, rows = M.max_rows, B = cfg->max_batch, S = cfg->max_seq;
    const bool tf = tf_mode(M);
    const size_t eb = tf ? 4 : 2;
    // Activations, caches, A operand and tile list.
    DEC_CUDA(dec_alloc(M, &M.x, sizeof(float) * rows * d));
    DEC_CUDA(dec_alloc(M, &M.x2, sizeof(float) * rows * d));
    DEC_CUDA(dec_alloc(M, &M.qkvbuf, sizeof(float) * rows * 3 * d));
    DEC_CUDA(dec_alloc(M, &M.logits, sizeof(float) * B * V));
    DEC_CUDA(dec_alloc(M, &M.tok, sizeof(int) * rows));
    DEC_CUDA(dec_alloc(M, &M.next, sizeof(int) * B));
    DEC_CUDA(dec_alloc(M, &M.seq_ids, sizeof(int) * B * S));
    DEC_CUDA(dec_alloc(M, &M.done, sizeof(int) * B));
    const size_t cache = (size_t)M.nl * B * M.H * S * M.HD;
    DEC_CUDA(dec_alloc(M, &M.kc, sizeof(float) * cache));
    DEC_CUDA(dec_alloc(M, &M.vc, sizeof(float) * cache));
    DEC_CUDA(dec_alloc(M, &M.a_hi, eb * (size_t)M.a_rows * d));
    if (tf) DEC_CUDA(dec_alloc(M, &M.a_lo, (size_t)4 * M.a_rows * d));
    const int max_mt = M.a_rows / kTileM + 2;
    DEC_CUDA(dec_alloc(M, &M.mtiles, sizeof(MTile) * max_mt));
    DEC_CUDA(dec_alloc(M, &M.ptiles, sizeof(MTile) * max_mt));
    DEC_CUDA(dec_alloc(M, &M.num_mtiles, sizeof(int)));
    DEC_CUDA(dec_alloc(M, &M.num_ptiles, sizeof(int)));
    DEC_CUDA(dec_alloc(M, &M.row_token, sizeof(int) * M.a_rows));
    DEC_CUDA(dec_alloc(M, &M.row_weight, sizeof(float) * M.a_rows));
    DEC_CUDA(dec_alloc(M, &M.dev_err, sizeof(int)));
    DEC_CUDA(cudaMemset(M.dev_err, 0, sizeof(int)));
    DEC_CUDA(dec_alloc(M, &M.attn_part, sizeof(float) * B * M.H *
                                            ((S + kDecChunk - 1) / kDecChunk) * (M.HD + 2)));
    DEC_CUDA(dec_alloc(M, &M.pos_dev, sizeof(int)));
    DEC_CUDA(dec_alloc(M, &M.step_dev, sizeof(int)));
    DEC_CUDA(cudaMemset(M.pos_dev, 0, sizeof(int)));
    DEC_CUDA(cudaMemset(M.step_dev, 0, sizeof(int)));
    DEC_CUDA(cudaMemset(M.a_hi, 0, eb * (size_t)M.a_rows * d));
    if (tf) DEC_CUDA(cudaMemset(M.a_lo, 0, (size_t)4 * M.a_rows * d));
    {
        std::string err;
        const uint32_t box_k = tf ? 32 : 64;
        if (!make_tmap_2d(&M.tm_a_hi, M.a_hi, !tf, d, M.a_rows, box_k, kTileM, &err))
            return report_error(MOE_ERR_CUDA, err);
        if (tf) {
            if (!make_tmap_2d(&M.tm_a_lo, M.a_lo, false, d, M.a_rows, box_k, kTileM, &err))
                return report_error(MOE_ERR_CUDA, err);
        } else {
            M.tm_a_lo = M.tm_a_hi;
        }
    }
    // RoPE table, in double: (cos, sin) of p * base^(-2j / hd).
    {
        const int half = M.HD / 2;
        std::vector<float2> tab((size_t)S * half);
        for (size_t p = 0; p < S; ++p)
            for (int j = 0; j < half; ++j) {
                const double inv = std::pow((double)cfg->rope_base, -2.0 * j / (double)M.HD);
                const double a = (double)p * inv;
                tab[p * half + j] = make_float2((float)std::cos(a), (float)std::sin(a));
            }
        DEC_CUDA(dec_alloc(M, &M.rope, sizeof(float2) * tab.size()));
        DEC_CUDA(cudaMemcpy(M.rope, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice));
    }
    // Embedding (gather copy and output head) and norms.
    DEC_CUDA(dec_alloc(M, &M.embed, sizeof(float) * V * d));
    DEC_CUDA(cudaMemcpy(M.embed, w->embed, sizeof(float) * V * d, cudaMemcpyDefault));
    DEC_CUDA(dec_alloc(M, &M.final_norm, sizeof(float) * d));
    DEC_CUDA(cudaMemcpy(M.final_norm, w->final_norm, sizeof(float) * d, cudaMemcpyDefault));
    {
        const float* parts[1] = {M.embed};
        const int prow[1] = {M.V};
        DEC_RC(make_dense(M, M.head, parts, prow, 1, M.d));
    }
    M.attn_norm.assign(M.nl, nullptr);
    M.qkv.resize(M.nl);
    M.wo.resize(M.nl);
    M.moe.assign(M.nl, nullptr);
    const int E = cfg->num_experts;
    for (int l = 0; l < M.nl; ++l) {
        if (!w->attn_norm[l] || !w->wq[l] || !w->wk[l] || !w->wv[l] || !w->wo[l] ||
            !w->ffn_norm[l] || !w->router[l])
            return report_error(MOE_ERR_INVALID, "null layer weight");
        DEC_CUDA(dec_alloc(M, &M.attn_norm[l], sizeof(float) * d));
        DEC_CUDA(cudaMemcpy(M.attn_norm[l], w->attn_norm[l], sizeof(float) * d, cudaMemcpyDefault));
        const float* qkv_parts[3] = {w->wq[l], w->wk[l], w->wv[l]};
        const int qkv_rows[3] = {M.d, M.d, M.d};
        DEC_RC(make_dense(M, M.qkv[l], qkv_parts, qkv_rows, 3, M.d));
        const float* o_parts[1] = {w->wo[l]};
        const int o_rows[1] = {M.d};
        DEC_RC(make_dense(M, M.wo[l], o_parts, o_rows, 1, M.d));
        MoeConfig mc;
        moe_config_init(&mc);
        mc.d_model = M.d;
        mc.d_ff = cfg->d_ff;
        mc.num_experts = E;
        mc.top_k = cfg->top_k;
        mc.router_policy = MOE_ROUTER_SOFTMAX_TOPK;
        mc.precision = cfg->precision;
        mc.device = cfg->device;
        mc.max_tokens = M.max_rows;
        MoeWeightsHost mw{};
        mw.router_weight = w->router[l];
        mw.router_bias = nullptr;
        mw.w1 = w->w1 + (size_t)l * E;
        mw.w3 = w->w3 + (size_t)l * E;
        mw.w2 = w->w2 + (size_t)l * E;
        DEC_RC(device_ptrs ? moe_create_from_device(&mc, &mw, &M.moe[l])
                           : moe_create(&mc, &mw, &M.moe[l]));
        DEC_RC(moe_set_post_rms_norm(M.moe[l], w->ffn_norm[l], cfg->rms_eps));
        M.bytes += moe_device_bytes(M.moe[l]);
    }
    DEC_RC(setup_fused_step(M));
    DEC_CUDA(cudaDeviceSynchronize());
    *out = m.release();
    return MOE_OK;
}

int copy_tokens(MoeDecoder& m, const int32_t* tokens, size_t n) {
    DEC_CUDA(cudaMemcpyAsync(m.tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, m.stream));
    return MOE_OK;
}

int prefill_impl(MoeDecoder& m, const int32_t* tokens, int B, int S, float* logits,
                 int32_t* next_ids);
int decode_step_impl(MoeDecoder& m, const int32_t* tokens, float* logits, int32_t* next_ids);
int generate_impl(MoeDecoder& m, const int32_t* prompt, int B, int S, int max_new_tokens,
                  int eos_id, float* logits, int32_t* ids);

}  // namespace
}  // namespace moe

extern "C" {

void moe_decoder_config_init(MoeDecoderConfig* c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->n_layers = 8;
    c->d_model = 2048;
    c->n_heads = 16;
    c->head_dim = 128;
    c->vocab = 32000;
    c->num_experts = 16;
    c->top_k = 2;
    c->d_ff = 5632;
    c->rms_eps = 1.0e-5f;
    c->rope_base = 10000.0f;
    c->precision = MOE_PREC_BF16;
    c->max_batch = 16;
    c->max_seq = 640;
    c->device = 0;
}

int moe_decoder_create(const MoeDecoderConfig* cfg, const MoeDecoderWeights* w, MoeDecoder** out) {
    return moe::create(cfg, w, false, out);
}

int moe_decoder_create_from_device(const MoeDecoderConfig* cfg, const MoeDecoderWeights* w,
                                   MoeDecoder** out) {
    return moe::create(cfg, w, true, out);
}

void moe_decoder_destroy(MoeDecoder* m) { moe::destroy(m); }

size_t moe_decoder_device_bytes(const MoeDecoder* m) { return m ? m->bytes : 0; }

int moe_decoder_prefill(MoeDecoder* m, const int32_t* tokens, int32_t B, int32_t S, float* logits,
                        int32_t* next_ids) {
    using namespace moe;
    if (!m || !tokens) return report_error(MOE_ERR_INVALID, "null argument");
    if (B < 1 || B > m->cfg.max_batch || S < 1 || S > m->cfg.max_seq)
        return report_error(MOE_ERR_INVALID, "need 1 <= B <= max_batch and 1 <= S <= max_seq");
    DecDeviceGuard guard(m->cfg.device);
    m->B = 0;   // until this call succeeds there is no batch to decode
    const int rc = prefill_impl(*m, tokens, B, S, logits, next_ids);
    if (rc) m->B = 0;
    return rc;
}

int moe_decoder_decode_step(MoeDecoder* m, const int32_t* tokens, float* logits, int32_t* next_ids) {
    using namespace moe;
    if (!m || !tokens) return report_error(MOE_ERR_INVALID, "null argument");
    if (m->B < 1) return report_error(MOE_ERR_INVALID, "decode step before a prefill");
    if (m->pos >= m->cfg.max_seq) return report_error(MOE_ERR_INVALID, "the sequences reached max_seq");
    DecDeviceGuard guard(m->cfg.device);
    const int rc = decode_step_impl(*m, tokens, logits, next_ids);
    if (rc) m->B = 0;   // the caches may be half-written: a new prefill is needed
    return rc;
}

int moe_decoder_generate(MoeDecoder* m, const int32_t* prompt, int32_t B, int32_t S,
                         int32_t max_new_tokens, int32_t eos_id, float* logits, int32_t* ids) {
    using namespace moe;
    if (!m || !prompt || !ids) return report_error(MOE_ERR_INVALID, "null argument");
    if (max_new_tokens < 1) return report_error(MOE_ERR_INVALID, "max_new_tokens must be positive");
    if (B < 1 || B > m->cfg.max_batch || S < 1)
        return report_error(MOE_ERR_INVALID, "need 1 <= B <= max_batch and S >= 1");
    if ((long long)S + max_new_tokens - 1 > m->cfg.max_seq)
        return report_error(MOE_ERR_INVALID, "prompt + max_new_tokens - 1 exceeds max_seq");
    DecDeviceGuard guard(m->cfg.device);
    m->B = 0;
    const int rc = generate_impl(*m, prompt, B, S, max_new_tokens, eos_id, logits, ids);
    if (rc) m->B = 0;
    return rc;
}

int moe_decoder_last_timing(const MoeDecoder* m, float* prefill_ms, float* decode_ms) {
    using namespace moe;
    if (!m) return report_error(MOE_ERR_INVALID, "null decoder");
    if (prefill_ms) *prefill_ms = m->t_prefill;
    if (decode_ms) *decode_ms = m->t_decode;
    return MOE_OK;
}

int moe_decoder_set_fused_step(MoeDecoder* m, int32_t enable) {
    using namespace moe;
    if (!m) return report_error(MOE_ERR_INVALID, "null decoder");
    if (enable && !m->step_ok)
        return report_error(MOE_ERR_UNSUPPORTED,
                            "the fused decode step needs BF16 precision, experts <= SMs and "
                            "d_model <= 8192");
    if ((enable != 0) != m->step_on) {
        DecDeviceGuard guard(m->cfg.device);
        cudaStreamSynchronize(m->stream);
        drop_graph(*m);   // the captured step holds the other path
        m->step_on = enable != 0;
    }
    return MOE_OK;
}

int moe_decoder_fused_step_active(const MoeDecoder* m) { return m && m->step_ok && m->step_on ? 1 : 0; }

}  // extern "C"

namespace moe {
namespace {

int prefill_impl(MoeDecoder& M, const int32_t* tokens, int B, int S, float* logits,
                 int32_t* next_ids) {
    MoeDecoder* m = &M;
    DEC_RC(copy_tokens(*m, tokens, (size_t)B * S));
    DEC_RC(run_prefill(*m, B, S, false, -1));
    if (logits)
        DEC_CUDA(cudaMemcpyAsync(logits, m->logits, sizeof(float) * B * m->V, cudaMemcpyDeviceToHost, m->stream));
    if (next_ids)
        DEC_CUDA(cudaMemcpyAsync(next_ids, m->next, sizeof(int) * B, cudaMemcpyDeviceToHost, m->stream));
    DEC_CUDA(cudaStreamSynchronize(m->stream));
    return check_dev_err(*m);
}

int decode_step_impl(MoeDecoder& M, const int32_t* tokens, float* logits, int32_t* next_ids) {
    MoeDecoder* m = &M;
    DEC_RC(copy_tokens(*m, tokens, (size_t)m->B));
    DEC_RC(run_decode(*m, m->tok, false, -1, nullptr, 0));
    ++m->pos;
    if (logits)
        DEC_CUDA(cudaMemcpyAsync(logits, m->logits, sizeof(float) * m->B * m->V, cudaMemcpyDeviceToHost, m->stream));
    if (next_ids)
        DEC_CUDA(cudaMemcpyAsync(next_ids, m->next, sizeof(int) * m->B, cudaMemcpyDeviceToHost, m->stream));
    DEC_CUDA(cudaStreamSynchronize(m->stream));
    return check_dev_err(*m);
}

int generate_impl(MoeDecoder& M, const int32_t* prompt, int B, int S, int max_new_tokens,
                  int eos_id, float* logits, int32_t* ids) {
    MoeDecoder* m = &M;
    const size_t V = m->V, n = max_new_tokens;
    if (logits && m->gen_cap < (size_t)B * n) {
        drop_graph(*m);   // it writes into the old buffer
        if (m->gen_logits) {
            cudaFree(m->gen_logits);
            m->bytes -= sizeof(float) * m->gen_cap * V;
        }
        m->gen_logits = nullptr;
        m->gen_cap = 0;
        DEC_CUDA(dec_alloc(*m, &m->gen_logits, sizeof(float) * B * n * V));
        m->gen_cap = (size_t)B * n;
    }
    cudaStream_t s = m->stream;
    DEC_RC(copy_tokens(*m, prompt, (size_t)B * S));
    DEC_CUDA(cudaMemsetAsync(m->done, 0, sizeof(int) * B, s));
    DEC_CUDA(cudaEventRecord(m->ev[0], s));
    DEC_RC(run_prefill(*m, B, S, true, eos_id));
    if (logits)
        DEC_CUDA(cudaMemcpy2DAsync(m->gen_logits, n * V * sizeof(float), m->logits, V * sizeof(float),
                                   V * sizeof(float), B, cudaMemcpyDeviceToDevice, s));
    DEC_CUDA(cudaEventRecord(m->ev[1], s));
    if (max_new_tokens > 1) {
        float* save = logits ? m->gen_logits : nullptr;
        DEC_RC(step_graph(*m, eos_id, save, (int)n));
        for (int step = 1; step < max_new_tokens; ++step) {
            DEC_CUDA(cudaGraphLaunch(m->step_graph, s));
            ++m->pos;
        }
    }
    DEC_CUDA(cudaEventRecord(m->ev[2], s));
    DEC_CUDA(cudaMemcpy2DAsync(ids, n * sizeof(int), m->seq_ids, m->cfg.max_seq * sizeof(int),
                               n * sizeof(int), B, cudaMemcpyDeviceToHost, s));
    if (logits)
        DEC_CUDA(cudaMemcpyAsync(logits, m->gen_logits, sizeof(float) * B * n * V,
                                 cudaMemcpyDeviceToHost, s));
    DEC_CUDA(cudaStreamSynchronize(s));
    DEC_CUDA(cudaEventElapsedTime(&m->t_prefill, m->ev[0], m->ev[1]));
    DEC_CUDA(cudaEventElapsedTime(&m->t_decode, m->ev[1], m->ev[2]));
    // generate_decode leaves a stopped sequence's later logits at zero.
    if (logits)
        for (int b = 0; b < B; ++b)
            for (size_t t = 0; t < n; ++t)
                if (ids[(size_t)b * n + t] < 0)
                    std::memset(logits + ((size_t)b * n + t) * V, 0, sizeof(float) * V);
    return check_dev_err(*m);
}

}  // namespace
}  // namespace moe
