// Expert parallelism: one process and one B200 per rank; rank r holds experts
// r, r + G, r + 2G, ... (round-robin placement).  The reference has no
// multi-GPU path; this is the layer's scale-out.
//
// Fused, deduplicated transport (the default, MOE_EP_TRANSPORT_P2P): every
// rank allocates a receive buffer and a return buffer with one fixed segment
// per source rank ([G][cap] rows, cap = max_tokens: one row per token per
// source), a metadata buffer and count and flag words, and maps every other
// rank's through CUDA IPC (handles exchanged once, with an NCCL all-gather).
// Then, with no host synchronisation and no NCCL call:
//   1. router; compact scans of the expert positions and of the
//      destinations;
//   2. the push kernel stores one row per (token, destination rank) straight
//      into the destination's receive buffer over NVLink, with the token's
//      selections on that rank as metadata;
//   3. a signal kernel writes this rank's counts into each rank's count
//      words and raises its dispatch flag there (system-scope fence, release
//      store of the step's epoch);
//   4. a wait kernel spins (bounded) until every source's flag shows the
//      epoch; the arrival scan and the arrangement place each received row
//      in each of its experts' GEMM rows; both GEMMs run, the down GEMM
//      storing each expert's output at its (received row, selection) slot;
//   5. the return push adds each received row's expert outputs in ascending
//      expert order (the reference's fma combine) and stores the one summed
//      row into the source's return buffer; signal and wait again;
//   6. the combine adds the rows a token's ranks returned, in ascending rank
//      order.  Every sum has a fixed order, so a step is bit-reproducible.
// Buffers are never rewritten before their reader is done, by the data
// dependencies alone: a rank pushes step e + 1 only after its step-e combine,
// which needed every rank's step-e results, which those ranks computed after
// arranging (copying out) their step-e arrivals.  No load of another GPU's
// memory uses TMA; the peer traffic is plain stores.
//
// NCCL transport (MOE_EP_TRANSPORT_NCCL), the baseline; forward on rank r
// with T local tokens (every rank runs it collectively):
//   1. router over all E experts (router weights are replicated);
//   2. compact dispatch (granule 1): rows sorted by dispatch position, then
//      token, so the rows for rank j are one contiguous run; fp32 rows in
//      FP32 precision, bf16 rows in BF16 precision;
//   3. counts exchange: each rank sends rank j its E/G per-expert counts for
//      j's experts; one small device-to-host copy gives the split sizes;
//   4. payload exchange (grouped ncclSend / ncclRecv, self included);
//   5. the received [source][local expert][token] rows are arranged into the
//      grouped GEMM's expert blocks: the same scan kernel as the local
//      dispatch, run on the [source][local expert] count matrix, gives each
//      (source, expert) run its place; an arrange kernel converts the rows
//      (bf16, or tf32 hi + lo);
//   6. gate/up GEMM, then the down GEMM storing each row's result (fp32, or
//      bf16 in BF16 precision) at the row it arrived in;
//   7. return exchange (the reverse splits), so each rank gets its own rows
//      back in its compact dispatch order;
//   8. combine: y[token] = its k returned rows, weighted, in ascending expert
//      order.
#include <cuda_bf16.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {

// ------------------------------------------------------------------ NCCL
// Loaded at first use, so the library itself does not depend on NCCL being
// installed.  In a process that already loaded NCCL (e.g. through PyTorch),
// dlopen returns that same library.
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

namespace {

NcclApi g_nccl;
std::mutex g_nccl_mu;

bool load_nccl(std::string* err) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.ok) return true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        *err = std::string("cannot load NCCL: ") + dlerror();
        return false;
    }
#define MOE_SYM(field, name)                                                   \
    g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));  \
    if (!g_nccl.field) {                                                       \
        *err = std::string("NCCL symbol missing: ") + name;                   \
        return false;                                                          \
    }
    MOE_SYM(GetUniqueId, "ncclGetUniqueId")
    MOE_SYM(CommInitRank, "ncclCommInitRank")
    MOE_SYM(CommDestroy, "ncclCommDestroy")
    MOE_SYM(Send, "ncclSend")
    MOE_SYM(Recv, "ncclRecv")
    MOE_SYM(GroupStart, "ncclGroupStart")
    MOE_SYM(GroupEnd, "ncclGroupEnd")
    MOE_SYM(AllGather, "ncclAllGather")
    MOE_SYM(GetErrorString, "ncclGetErrorString")
#undef MOE_SYM
    g_nccl.ok = true;
    return true;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return report_error(MOE_ERR_NCCL, std::string(what) + ": " +
                                          (g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "?"));
}

}  // namespace

struct EpState {
    int rank = 0, world = 1;
    int e_local = 0;            // experts per rank
    ncclComm_t comm = nullptr;
    int cap_T = 0;              // local tokens the buffers hold
    size_t row_bytes = 0;       // bytes of one dispatched row
    void* send_rows = nullptr;  // [T*k][d] compact, expert-sorted
    int* send_tok = nullptr;    // compact row -> local token
    float* send_w = nullptr;    // compact row -> routing weight
    int* send_slot = nullptr;   // selection slot t * k + s -> compact row
    int* send_eoff = nullptr;   // [E+1] compact offsets
    void* recv_rows = nullptr;  // [G*T*k][d]
    float* ret_send = nullptr;  // [G*T*k][d] results (dispatch element type), by arrival row
    float* ret_recv = nullptr;  // [T*k][d] results, by compact row
    int* cnt_recv = nullptr;    // [G][E_local] device
    int* cnt_scan = nullptr;    // [G][E_local] device (scan in place)
    int* h_counts = nullptr;    // pinned [E]
    int* h_cnt_recv = nullptr;  // pinned [G][E_local]
    // Fused (P2P) transport.
    int transport = MOE_EP_TRANSPORT_P2P;
    int cap_src = 0;             // rows of one source segment
    uint32_t epoch = 0;          // forward steps run
    void* p2p_recv = nullptr;    // [G][cap_src] rows, written by the sources
    void* p2p_ret = nullptr;     // [G][cap_src] result rows, written by the expert ranks
    int* p2p_cnt = nullptr;      // [G][E_local], written by the sources
    unsigned* p2p_flag = nullptr;  // [2][G]: dispatch flag of source s, return flag of rank j
    // Deduplicated fused transport: one row per (token, destination rank).
    int kmax = 1;                // selections one row can carry: min(top_k, E_local)
    int2* p2p_meta = nullptr;    // [G][cap_src][kmax] {pos * 256 + local expert, weight bits}, x = -1 ends
    int* dest_hist = nullptr;    // [blocks][G] tokens per destination per 32-token block (scanned in place)
    int* dest_cnt = nullptr;     // [G] rows sent to each rank
    int* dest_off = nullptr;     // [G + 1]
    int* slot_dd = nullptr;      // [cap_T][G] row of token t at rank g (-1: none)
    int* rows_recv = nullptr;    // [G] rows received from each source this step
    void** d_peer_recv = nullptr;  // [G] every rank's p2p_recv (own included), device array
    void** d_peer_ret = nullptr;
    int** d_peer_cnt = nullptr;
    unsigned** d_peer_flag = nullptr;
    int2** d_peer_meta = nullptr;
    std::vector<void*> ipc_opened;  // mappings of the other ranks' buffers
    // Round-robin placement: rank r holds experts r, r + G, r + 2G, ...;
    // eperm[e] = (e % G) * E_local + e / G is expert e's dispatch position
    // (rank-major, so each rank's experts are one contiguous run).
    int* eperm = nullptr;
    // Failure of the fused transport: poison (device word) is set by a wait
    // that ran out and stops this rank's peer stores and flags; each forward
    // ends with a copy of the device error flags into h_err (pinned) and
    // err_ev; failed (host) is set once a completed copy shows a flag.
    unsigned long long wait_ns = 0;
    int* poison = nullptr;
    int* h_err = nullptr;
    cudaEvent_t err_ev = nullptr;
    bool err_recorded = false;
    bool failed = false;
};

namespace {

void ep_free_buffers(EpState& S) {
    for (void* p : S.ipc_opened) cudaIpcCloseMemHandle(p);
    S.ipc_opened.clear();
    for (void* p : {S.send_rows, (void*)S.send_tok, (void*)S.send_w, (void*)S.send_eoff,
                    S.recv_rows, (void*)S.ret_send, (void*)S.ret_recv, (void*)S.cnt_recv,
                    (void*)S.cnt_scan, S.p2p_recv, S.p2p_ret, (void*)S.p2p_cnt,
                    (void*)S.p2p_flag, (void*)S.d_peer_recv,
                    (void*)S.d_peer_ret, (void*)S.d_peer_cnt, (void*)S.d_peer_flag,
                    (void*)S.p2p_meta, (void*)S.dest_hist, (void*)S.dest_cnt, (void*)S.dest_off,
                    (void*)S.slot_dd, (void*)S.send_slot, (void*)S.rows_recv,
                    (void*)S.d_peer_meta})
        if (p) cudaFree(p);
    S.p2p_meta = nullptr;
    S.dest_hist = S.dest_cnt = S.dest_off = S.slot_dd = S.rows_recv = nullptr;
    S.send_slot = nullptr;
    S.d_peer_meta = nullptr;
    S.p2p_recv = S.p2p_ret = nullptr;
    S.p2p_cnt = nullptr;
    S.p2p_flag = nullptr;
    if (S.poison) cudaFree(S.poison);
    if (S.h_err) cudaFreeHost(S.h_err);
    if (S.err_ev) cudaEventDestroy(S.err_ev);
    S.poison = nullptr;
    S.h_err = nullptr;
    S.err_ev = nullptr;
    S.err_recorded = false;
    S.d_peer_recv = S.d_peer_ret = nullptr;
    S.d_peer_cnt = nullptr;
    S.d_peer_flag = nullptr;
    if (S.h_counts) cudaFreeHost(S.h_counts);
    if (S.h_cnt_recv) cudaFreeHost(S.h_cnt_recv);
    S.send_rows = S.recv_rows = nullptr;
    S.send_tok = S.send_eoff = S.cnt_recv = S.cnt_scan = S.h_counts = S.h_cnt_recv = nullptr;
    S.send_w = S.ret_send = S.ret_recv = nullptr;
    S.cap_T = 0;
}

int ep_ensure(Layer& L, int T) {
    EpState& S = *L.ep;
    if (T <= S.cap_T) return MOE_OK;
    cudaDeviceSynchronize();
    ep_free_buffers(S);
    const int capT = T > 64 ? T : 64;
    const size_t rows_local = (size_t)capT * L.k;
    const size_t rows_recv = rows_local * S.world;
    S.row_bytes = (size_t)L.d * wire_bytes(L);
    cudaError_t e = cudaSuccess;
    auto A = [&](void** p, size_t b) {
        if (e == cudaSuccess) e = cudaMalloc(p, b ? b : 256);
    };
    A(&S.send_rows, rows_local * S.row_bytes);
    A((void**)&S.send_tok, rows_local * sizeof(int));
    A((void**)&S.send_w, rows_local * sizeof(float));
    A((void**)&S.send_slot, rows_local * sizeof(int));
    A((void**)&S.send_eoff, (L.E_route + 1) * sizeof(int));
    A(&S.recv_rows, rows_recv * S.row_bytes);
    A((void**)&S.ret_send, rows_recv * L.d * sizeof(float));
    A((void**)&S.ret_recv, rows_local * L.d * sizeof(float));
    A((void**)&S.cnt_recv, (size_t)S.world * S.e_local * sizeof(int));
    A((void**)&S.cnt_scan, (size_t)S.world * S.e_local * sizeof(int));
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&S.h_counts, L.E_route * sizeof(int), 0);
    if (e == cudaSuccess)
        e = cudaHostAlloc((void**)&S.h_cnt_recv, (size_t)S.world * S.e_local * sizeof(int), 0);
    if (e != cudaSuccess) {
        ep_free_buffers(S);
        return report_error(MOE_ERR_OOM, std::string("expert-parallel buffers: ") +
                                             cudaGetErrorString(e));
    }
    S.cap_T = capT;
    // The receiving side runs the grouped GEMMs on up to world * T tokens' rows.
    return ensure_workspace(L, capT * S.world);
}

// One warp per received row: find its (source, local expert) run, place it in
// the expert's GEMM block and convert it to the operand format.
// cap_src > 0 (fused transport): source s's rows sit at rows
// [s * cap_src, ...) of recv, and row_token gets the return slot
// s * cap_src + q; else the sources' runs are contiguous and row_token gets
// the arrival row.  rows is a bound: rows past the received total exit.
// Received rows and counts were written by other GPUs: they are read through
// L2 only.
// One received row (fp32 on the wire for kFmt kActTf32x2 / kActBf16x2, bf16
// for kActBf16) into each of the n GEMM rows prow[0..n) of the operand
// planes, one warp, columns lane-strided.  Rows written by other GPUs are
// read through L2 only.
template <int kFmt>
__device__ __forceinline__ void convert_row(const void* src_row, int d, const int* prow, int n,
                                            void* a_hi, void* a_lo, int lane) {
    if constexpr (kFmt == kActBf16) {
        const uint4* src = static_cast<const uint4*>(src_row);
        for (int v = lane; v < d / 8; v += 32) {
            const uint4 u = __ldcg(src + v);
            for (int j = 0; j < n; ++j)
                reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a_hi) + (size_t)prow[j] * d)[v] = u;
        }
    } else {
        const float4* src = static_cast<const float4*>(src_row);
        for (int v = lane; v < d / 4; v += 32) {
            const float4 f = __ldcg(src + v);
            if constexpr (kFmt == kActTf32x2) {
                float4 h, l;
                h.x = to_tf32(f.x); l.x = to_tf32(f.x - h.x);
                h.y = to_tf32(f.y); l.y = to_tf32(f.y - h.y);
                h.z = to_tf32(f.z); l.z = to_tf32(f.z - h.z);
                h.w = to_tf32(f.w); l.w = to_tf32(f.w - h.w);
                for (int j = 0; j < n; ++j) {
                    reinterpret_cast<float4*>(static_cast<float*>(a_hi) + (size_t)prow[j] * d)[v] = h;
                    reinterpret_cast<float4*>(static_cast<float*>(a_lo) + (size_t)prow[j] * d)[v] = l;
                }
            } else {
                uint2 hp, lp;
                split_bf16x2(f.x, f.y, hp.x, lp.x);
                split_bf16x2(f.z, f.w, hp.y, lp.y);
                for (int j = 0; j < n; ++j) {
                    reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a_hi) + (size_t)prow[j] * d)[v] = hp;
                    reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a_lo) + (size_t)prow[j] * d)[v] = lp;
                }
            }
        }
    }
}

template <int kFmt>
__global__ void __launch_bounds__(256)
ep_arrange_kernel(const void* __restrict__ recv, int rows, int d, int G, int El, int cap_src,
                  const int* __restrict__ cnt, const int* __restrict__ base,
                  const int* __restrict__ eoff, int* __restrict__ row_token,
                  float* __restrict__ row_weight, void* __restrict__ a_hi,
                  void* __restrict__ a_lo) {
    extern __shared__ int sm[];
    int* src_off = sm;              // [G + 1] first arrival row of each source
    int* run_off = sm + G + 1;      // [G][El + 1] offsets inside each source
    if (threadIdx.x == 0) {
        int off = 0;
        for (int s = 0; s < G; ++s) {
            src_off[s] = off;
            int r = 0;
            for (int e = 0; e < El; ++e) {
                run_off[s * (El + 1) + e] = r;
                r += __ldcg(cnt + s * El + e);
            }
            run_off[s * (El + 1) + El] = r;
            off += r;
        }
        src_off[G] = off;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * 8 + warp;
    if (i >= rows || i >= src_off[G]) return;
    int s = 0;
    while (s + 1 < G && src_off[s + 1] <= i) ++s;
    const int q = i - src_off[s];
    int e = 0;
    while (e + 1 < El && run_off[s * (El + 1) + e + 1] <= q) ++e;
    const int prow = eoff[e] + base[s * El + e] + (q - run_off[s * (El + 1) + e]);
    const size_t src_row = cap_src > 0 ? (size_t)s * cap_src + q : (size_t)i;
    if (lane == 0) {
        row_token[prow] = (int)src_row;
        row_weight[prow] = 1.0f;
    }
    const size_t wb = kFmt == kActBf16 ? 2 : 4;
    convert_row<kFmt>(static_cast<const char*>(recv) + src_row * d * wb, d, &prow, 1, a_hi, a_lo,
                      lane);
}

// y[t] = token t's k returned rows (fp32 in FP32 precision, bf16 in BF16),
// each times its routing weight, added with the reference's fma in ascending
// expert order from 0.  Slot s's row is ret[slot_row[t * k + s]].  idx holds
// dispatch positions; under the round-robin placement position p is expert
// (p % El) * G + p / El.  One warp per token; every element of y[t] is
// written.
template <bool kF32>
__global__ void __launch_bounds__(256)
ep_combine_kernel(const void* __restrict__ ret, int T, int k, int d, int G, int El,
                  const int* __restrict__ idx, const float* __restrict__ w,
                  const int* __restrict__ slot_row, float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    int key = 0, row = 0;
    float wv = 0.0f;
    if (lane < k) {
        const int p = idx[(size_t)t * k + lane];
        key = (p % El) * G + p / El;
        wv = w[(size_t)t * k + lane];
        row = slot_row[(size_t)t * k + lane];
    }
    int ord[kMaxTopK];
    float ow[kMaxTopK];
    slot_order_keys<kMaxTopK>(key, wv, k, lane, ord, ow);
    int rows[kMaxTopK];
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) rows[r] = __shfl_sync(0xffffffffu, row, ord[r]);
    float4* dst = reinterpret_cast<float4*>(y + (size_t)t * d);
    for (int v = lane; v < d / 4; v += 32) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int r = 0; r < k; ++r) {
            const size_t rj = (size_t)rows[r];
            float4 f;
            if constexpr (kF32) {
                f = reinterpret_cast<const float4*>(static_cast<const float*>(ret) + rj * d)[v];
            } else {
                const uint2 u = reinterpret_cast<const uint2*>(
                    static_cast<const __nv_bfloat16*>(ret) + rj * d)[v];
                f = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
            }
            acc.x = __fmaf_rn(ow[r], f.x, acc.x);
            acc.y = __fmaf_rn(ow[r], f.y, acc.y);
            acc.z = __fmaf_rn(ow[r], f.z, acc.z);
            acc.w = __fmaf_rn(ow[r], f.w, acc.w);
        }
        dst[v] = acc;
    }
}

int ep_forward_nccl(Layer& L, const float* x, float* y, int T, cudaStream_t s) {
    EpState& S = *L.ep;
    int rc = ep_ensure(L, T);
    if (rc) return rc;
    Workspace& W = L.ws;
    const int G = S.world, El = S.e_local, Eg = L.E_route;
    const ncclDataType_t dt = fp32_faithful(L) ? ncclFloat32 : ncclBfloat16;
    const size_t d = L.d;
    auto cuda_err = [](cudaError_t e, const char* what) {
        return report_error(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    };
    cudaError_t ce;
    ncclResult_t nr;
    L.prof_n = 0;

    // 1-2: route and pack locally (compact, expert-sorted).
    prof_mark(L, 0, s);
    if (T > 0) {
        if ((ce = launch_router(L, x, T, W.logits, W.idx, W.wts, W.blockhist, s, NormRef{},
                                S.eperm)) != cudaSuccess)
            return cuda_err(ce, "router");
        prof_mark(L, 1, s);
        if ((ce = launch_scan_generic(W.blockhist, (T + kRouteTokens - 1) / kRouteTokens, Eg, 1,
                                      W.counts, S.send_eoff, nullptr, nullptr, nullptr, nullptr,
                                      nullptr, nullptr, s)) != cudaSuccess)
            return cuda_err(ce, "dispatch scan");
        prof_mark(L, 2, s);
        if ((ce = launch_dispatch_permute_to(L, x, T, Eg, S.send_eoff, S.send_tok, S.send_w,
                                             S.send_slot, S.send_rows, s)) != cudaSuccess)
            return cuda_err(ce, "dispatch permute");
    } else {
        if ((ce = cudaMemsetAsync(W.counts, 0, Eg * sizeof(int), s)) != cudaSuccess)
            return cuda_err(ce, "counts");
    }
    // 3: counts exchange.
    prof_mark(L, 5, s);
    if ((nr = g_nccl.GroupStart()) != ncclSuccess) return nccl_fail(nr, "ncclGroupStart");
    for (int j = 0; j < G; ++j) {
        g_nccl.Send(W.counts + j * El, El, ncclInt32, j, S.comm, s);
        g_nccl.Recv(S.cnt_recv + j * El, El, ncclInt32, j, S.comm, s);
    }
    if ((nr = g_nccl.GroupEnd()) != ncclSuccess) return nccl_fail(nr, "counts exchange");
    if ((ce = cudaMemcpyAsync(S.h_counts, W.counts, Eg * sizeof(int), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (ce = cudaMemcpyAsync(S.h_cnt_recv, S.cnt_recv, (size_t)G * El * sizeof(int),
                              cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (ce = cudaMemcpyAsync(S.cnt_scan, S.cnt_recv, (size_t)G * El * sizeof(int),
                              cudaMemcpyDeviceToDevice, s)) != cudaSuccess)
        return cuda_err(ce, "counts copy");
    if ((ce = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_err(ce, "counts sync");
    std::vector<int64_t> send_rows(G), send_off(G + 1), recv_rows(G), recv_off(G + 1);
    if ((rc = moe_ep_plan(S.h_counts, S.h_cnt_recv, G, El, send_rows.data(), send_off.data(),
                          recv_rows.data(), recv_off.data())) != MOE_OK)
        return rc;
    const int R = (int)recv_off[G];
    const size_t rb = S.row_bytes;
    // 4: payload exchange.
    if ((nr = g_nccl.GroupStart()) != ncclSuccess) return nccl_fail(nr, "ncclGroupStart");
    for (int j = 0; j < G; ++j) {
        if (send_rows[j])
            g_nccl.Send(static_cast<char*>(S.send_rows) + send_off[j] * rb, send_rows[j] * d, dt, j,
                        S.comm, s);
        if (recv_rows[j])
            g_nccl.Recv(static_cast<char*>(S.recv_rows) + recv_off[j] * rb, recv_rows[j] * d, dt, j,
                        S.comm, s);
    }
    if ((nr = g_nccl.GroupEnd()) != ncclSuccess) return nccl_fail(nr, "dispatch exchange");
    // 5-6: arrange and run the local experts.
    prof_mark(L, 2, s);
    if (R > 0) {
        if ((ce = launch_scan_generic(S.cnt_scan, G, El, kTileM, W.counts, W.eoff, W.mtiles,
                                      W.num_mtiles, W.ptiles, W.num_ptiles, W.row_token,
                                      W.row_weight, s)) != cudaSuccess)
            return cuda_err(ce, "arrival scan");
        const size_t smem = sizeof(int) * ((G + 1) + (size_t)G * (El + 1));
        const int grid = (R + 7) / 8;
        auto run = [&](auto kern) {
            kern<<<grid, 256, smem, s>>>(S.recv_rows, R, L.d, G, El, 0, S.cnt_recv, S.cnt_scan,
                                         W.eoff, W.row_token, W.row_weight, W.a_hi, W.a_lo);
        };
        switch (act_format(L, false)) {
            case kActTf32x2: run(ep_arrange_kernel<kActTf32x2>); break;
            case kActBf16x2: run(ep_arrange_kernel<kActBf16x2>); break;
            default: run(ep_arrange_kernel<kActBf16>); break;
        }
        if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "arrange");
        prof_mark(L, 3, s);
        if ((ce = launch_expert_gemm_rows(L, R, nullptr, s, 0)) != cudaSuccess)
            return cuda_err(ce, "gate/up GEMM");
        prof_mark(L, 4, s);
        if ((ce = launch_expert_gemm_rows(L, R, S.ret_send, s, 2)) != cudaSuccess)
            return cuda_err(ce, "down GEMM");
    }
    // 7: return exchange (same element type as the dispatch).
    prof_mark(L, 6, s);
    if ((nr = g_nccl.GroupStart()) != ncclSuccess) return nccl_fail(nr, "ncclGroupStart");
    for (int j = 0; j < G; ++j) {
        if (recv_rows[j])
            g_nccl.Send(reinterpret_cast<char*>(S.ret_send) + recv_off[j] * rb, recv_rows[j] * d, dt,
                        j, S.comm, s);
        if (send_rows[j])
            g_nccl.Recv(reinterpret_cast<char*>(S.ret_recv) + send_off[j] * rb, send_rows[j] * d, dt,
                        j, S.comm, s);
    }
    if ((nr = g_nccl.GroupEnd()) != ncclSuccess) return nccl_fail(nr, "combine exchange");
    // 8: weighted combine into y.
    prof_mark(L, 7, s);
    if (T > 0) {
        if (fp32_faithful(L))
            ep_combine_kernel<true><<<(T + 7) / 8, 256, 0, s>>>(S.ret_recv, T, L.k, L.d, G, El,
                                                                W.idx, W.wts, S.send_slot, y);
        else
            ep_combine_kernel<false><<<(T + 7) / 8, 256, 0, s>>>(S.ret_recv, T, L.k, L.d, G, El,
                                                                 W.idx, W.wts, S.send_slot, y);
        if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "combine");
    }
    prof_mark(L, kProfEnd, s);
    return MOE_OK;
}

// ------------------------------------------------------------ fused transport
constexpr unsigned long long kPeerWaitNs = 5000000000ull;   // 5 s: the default peer-wait bound

// Thread j: for rank j, copy this rank's counts for j's experts into j's
// count words (dispatch only), then -- after a system-scope fence that orders
// this step's earlier writes to j (the previous kernel's row stores
// included) -- raise flag [which][this rank] in j's flag words to `epoch`.
__global__ void ep_signal_kernel(int* const* peer_cnt, const int* __restrict__ counts,
                                 unsigned* const* peer_flag, int G, int El, int rank, int which,
                                 unsigned epoch, const int* poison,
                                 const int* __restrict__ rows = nullptr) {
    const int j = threadIdx.x;
    // A failed rank raises no flags: its peers' waits run out instead of
    // proceeding on a step it did not complete.
    if (j >= G || *reinterpret_cast<const volatile int*>(poison)) return;
    if (peer_cnt)
        for (int e = 0; e < El; ++e) peer_cnt[j][rank * El + e] = counts[j * El + e];
    if (peer_cnt && rows) peer_cnt[j][G * El + rank] = rows[j];   // rows this rank sends j
    __threadfence_system();
    st_release_sys(peer_flag[j] + which * G + rank, epoch);
}

// Wait until every rank's flag [which][s] shows `epoch` (bounded: on a
// timeout the error flag is set).  Then copy the n count words the sources
// wrote (read through L2) to cnt_a and cnt_b, each clamped to a segment's
// capacity -- or zeros after a timeout, so a failed step moves no rows.
__global__ void ep_wait_kernel(const unsigned* flag, int G, int which, unsigned epoch,
                               const int* cnt_src, int* __restrict__ cnt_a, int* __restrict__ cnt_b,
                               int n, int cap, int* err, int* poison, unsigned long long budget_ns,
                               int* __restrict__ rows_out = nullptr) {
    __shared__ int timed_out;
    // A rank that failed in an earlier step waits for nothing.
    if (threadIdx.x == 0) timed_out = *reinterpret_cast<volatile int*>(poison);
    __syncthreads();
    const int sidx = threadIdx.x;
    if (sidx < G && !timed_out) {
        const unsigned* f = flag + which * G + sidx;
        if (ld_acquire_sys(f) < epoch) {
            const unsigned long long t0 = global_timer_ns();
            while (ld_acquire_sys(f) < epoch) {
                if (global_timer_ns() - t0 > budget_ns) {
                    atomicOr(err, kDevErrTimeoutPeer);
                    timed_out = 1;
                    break;
                }
                __nanosleep(128);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && timed_out) *reinterpret_cast<volatile int*>(poison) = 1;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int c = timed_out ? 0 : min(max(__ldcg(cnt_src + i), 0), cap);
        cnt_a[i] = c;
        cnt_b[i] = c;
    }
    if (rows_out)   // the sources' row counts follow their n count words
        for (int i = threadIdx.x; i < G; i += blockDim.x)
            rows_out[i] = timed_out ? 0 : min(max(__ldcg(cnt_src + n + i), 0), cap);
}

// ------------------------------------------------------------ deduplicated transport
// A token whose k experts fall on the same rank crosses NVLink once for that
// rank: the source sends one row per (token, destination rank) with the
// token's selections on that rank as metadata; the rank runs the row through
// each of its experts, sums their weighted outputs into one fp32 row in
// ascending expert order (the return push), and returns that single row;
// the source adds its ranks' rows in ascending rank order.  Rows of one
// source keep ascending token order, so each selection also carries its
// position inside its expert's block from this source -- exactly the compact
// dispatch scan's -- and the receiver places it without a scan of its own.

// Per 32-token block: how many of its tokens send to each rank (G <= 32).
__global__ void __launch_bounds__(256)
ep_dest_hist_kernel(const int* __restrict__ idx, int T, int k, int El, int G,
                    int* __restrict__ dest_hist) {
    __shared__ unsigned s_mask[32];
    const int t0 = blockIdx.x * kRouteTokens;
    const int n_tok = min(kRouteTokens, T - t0);
    if (threadIdx.x < 32) s_mask[threadIdx.x] = 0u;
    __syncthreads();
    const int i = threadIdx.x;
    if (i < n_tok * k) {
        const int e = idx[(size_t)t0 * k + i];
        if (e >= 0 && e < El * G) atomicOr(&s_mask[e / El], 1u << (i / k));
    }
    __syncthreads();
    if (threadIdx.x < G) dest_hist[(size_t)blockIdx.x * G + threadIdx.x] = __popc(s_mask[threadIdx.x]);
}

// Rows and metadata into the destination ranks' receive buffers.  ebase /
// gbase: the scanned per-block bases of the expert positions and of the
// destinations (relative to each one's start).  kMode 0: bf16 rows, 2: fp32.
template <int kMode>
__global__ void __launch_bounds__(256)
ep_dedup_push_kernel(const float* __restrict__ x, int T, int d, int k, int El, int G, int kmax,
                     const int* __restrict__ idx, const float* __restrict__ wts,
                     const int* __restrict__ ebase, const int* __restrict__ gbase,
                     void* const* __restrict__ peer_recv, int2* const* __restrict__ peer_meta,
                     int cap, int rank, int* __restrict__ slot_dd, const int* poison) {
    // A failed rank stores nothing into other GPUs' buffers.
    if (*reinterpret_cast<const volatile int*>(poison)) return;
    __shared__ unsigned s_emask[kMaxExperts];
    __shared__ unsigned s_gmask[32];
    __shared__ int s_list[kRouteTokens * 32];   // (token << 16) | (g << 11)... packed below
    __shared__ int s_row[kRouteTokens * 32];
    __shared__ int s_n;
    const int Eg = El * G;
    const int blk = blockIdx.x;
    const int t0 = blk * kRouteTokens;
    const int n_tok = min(kRouteTokens, T - t0);
    for (int e = threadIdx.x; e < Eg; e += blockDim.x) s_emask[e] = 0u;
    if (threadIdx.x < 32) s_gmask[threadIdx.x] = 0u;
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_tok * k; i += blockDim.x) {
        const int e = idx[(size_t)t0 * k + i];
        if (e >= 0 && e < Eg) {
            atomicOr(&s_emask[e], 1u << (i / k));
            atomicOr(&s_gmask[e / El], 1u << (i / k));
        }
    }
    __syncthreads();
    // One thread per (token, destination): its row index, metadata and slot.
    for (int i = threadIdx.x; i < n_tok * G; i += blockDim.x) {
        const int tl = i / G, g = i % G;
        const unsigned below = (1u << tl) - 1u;
        const int t = t0 + tl;
        if (!((s_gmask[g] >> tl) & 1u)) {
            slot_dd[(size_t)t * G + g] = -1;
            continue;
        }
        const int r = gbase[(size_t)blk * G + g] + __popc(s_gmask[g] & below);
        slot_dd[(size_t)t * G + g] = r;
        int2* meta = peer_meta[g] + ((size_t)rank * cap + r) * kmax;
        int j = 0;
        for (int sl = 0; sl < k; ++sl) {
            const int e = idx[(size_t)t * k + sl];
            if (e < 0 || e >= Eg || e / El != g) continue;
            const int pos = ebase[(size_t)blk * Eg + e] + __popc(s_emask[e] & below);
            if (j < kmax) meta[j] = make_int2(pos * 256 + (e - g * El), __float_as_int(wts[(size_t)t * k + sl]));
            ++j;
        }
        for (; j < kmax; ++j) meta[j] = make_int2(-1, 0);
        const int n = atomicAdd(&s_n, 1);
        s_list[n] = tl * 32 + g;
        s_row[n] = r;
    }
    __syncthreads();
    // Row copies, one warp per (token, destination).
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int p = warp; p < s_n; p += nw) {
        const int tl = s_list[p] / 32, g = s_list[p] % 32;
        const float4* src = reinterpret_cast<const float4*>(x + (size_t)(t0 + tl) * d);
        const size_t row = (size_t)rank * cap + s_row[p];
        if constexpr (kMode == 0) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(peer_recv[g]) + row * d);
            for (int v = lane; v < d / 8; v += 32) {
                const float4 a = __ldg(src + 2 * v), b = __ldg(src + 2 * v + 1);
                __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
                __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
                dst[v] = make_uint4(*reinterpret_cast<uint32_t*>(&p0), *reinterpret_cast<uint32_t*>(&p1),
                                    *reinterpret_cast<uint32_t*>(&p2), *reinterpret_cast<uint32_t*>(&p3));
            }
        } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(peer_recv[g]) + row * d);
            for (int v = lane; v < d / 4; v += 32) dst[v] = __ldg(src + v);
        }
    }
}

// The selections received row i (source s) carries, from its metadata, in
// metadata order: local expert, routing weight and GEMM row of each.  An
// entry whose row would fall outside the expert blocks (inconsistent
// metadata: never expected) is dropped, by the arrangement and the return
// push alike.  Metadata was written by another GPU: read through L2 only.
struct DdSelections {
    int n;
    int e[kMaxTopK];
    float w[kMaxTopK];
    int prow[kMaxTopK];
};

__device__ __forceinline__ void dd_selections(const int2* __restrict__ meta, size_t i, int kmax,
                                              int s, int El, const int* __restrict__ base,
                                              const int* __restrict__ eoff, DdSelections& out) {
    out.n = 0;
    const int lim = eoff[El];
    for (int j = 0; j < kmax && j < kMaxTopK; ++j) {
        const int2 m = __ldcg(meta + i * kmax + j);
        if (m.x < 0) break;
        const int e = m.x & 255, pos = m.x >> 8;
        if (e >= El) break;
        const int pr = eoff[e] + base[s * El + e] + pos;
        if (pr >= lim) continue;
        out.e[out.n] = e;
        out.w[out.n] = __int_as_float(m.y);
        out.prow[out.n] = pr;
        ++out.n;
    }
}

// One warp per received row (source s, row r < rows_recv[s]): its metadata
// places it in each of its local experts' GEMM rows (row_token = the
// received slot i = s * cap + r, row_weight = the routing weight, row_slot =
// i * kmax + j for its j-th placed selection, where the down GEMM stores that
// expert's output), and the row is converted into each of those A rows.
// Rows were written by other GPUs: read through L2 only.
template <int kFmt>
__global__ void __launch_bounds__(256)
ep_dd_arrange_kernel(const void* __restrict__ recv, const int2* __restrict__ meta,
                     const int* __restrict__ rows_recv, int cap, int d, int G, int El, int kmax,
                     const int* __restrict__ base, const int* __restrict__ eoff,
                     int* __restrict__ row_token, float* __restrict__ row_weight,
                     int* __restrict__ row_slot, void* __restrict__ a_hi,
                     void* __restrict__ a_lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t i = (size_t)blockIdx.x * 8 + warp;
    if (i >= (size_t)G * cap) return;
    const int s = (int)(i / cap), r = (int)(i % cap);
    if (r >= rows_recv[s]) return;
    DdSelections sel;
    dd_selections(meta, i, kmax, s, El, base, eoff, sel);
    const int n = sel.n;
    if (lane < n) {
        row_token[sel.prow[lane]] = (int)i;
        row_weight[sel.prow[lane]] = sel.w[lane];
        row_slot[sel.prow[lane]] = (int)(i * kmax) + lane;
    }
    const size_t wb = kFmt == kActBf16 ? 2 : 4;
    convert_row<kFmt>(static_cast<const char*>(recv) + i * d * wb, d, sel.prow, n, a_hi, a_lo,
                      lane);
}

// One warp per received row i: the outputs of its experts (part row
// i * kmax + j for its j-th placed selection, unweighted fp32) are added with
// the reference's fma in ascending expert order from 0, and the one summed
// row goes back to the source's return buffer, row rank * cap + r (bf16 in
// BF16 precision, fp32 in FP32).  Local expert order is global expert order
// on one rank (rank + G * local).
template <bool kF32>
__global__ void __launch_bounds__(256)
ep_return_push_kernel(const float* __restrict__ part, const int2* __restrict__ meta,
                      const int* __restrict__ rows_recv, int cap, int d, int G, int El, int kmax,
                      const int* __restrict__ base, const int* __restrict__ eoff, int rank,
                      void* const* __restrict__ peer_ret, const int* poison) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t i = (size_t)blockIdx.x * 8 + warp;
    if (i >= (size_t)G * cap || *reinterpret_cast<const volatile int*>(poison)) return;
    const int s = (int)(i / cap), r = (int)(i % cap);
    if (r >= rows_recv[s]) return;
    DdSelections sel;
    dd_selections(meta, i, kmax, s, El, base, eoff, sel);
    // Placed index j of each selection, by ascending expert (insertion sort;
    // experts are distinct within a token).
    int ord[kMaxTopK];
    for (int j = 0; j < sel.n; ++j) {
        int q = j;
        while (q > 0 && sel.e[ord[q - 1]] > sel.e[j]) {
            ord[q] = ord[q - 1];
            --q;
        }
        ord[q] = j;
    }
    const float4* src = reinterpret_cast<const float4*>(part) + i * kmax * (d / 4);
    const size_t row = (size_t)rank * cap + r;
    auto sum4 = [&](int v) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int q = 0; q < sel.n; ++q) {
            const int j = ord[q];
            const float4 f = __ldcs(src + (size_t)j * (d / 4) + v);
            const float w = sel.w[j];
            acc.x = __fmaf_rn(w, f.x, acc.x);
            acc.y = __fmaf_rn(w, f.y, acc.y);
            acc.z = __fmaf_rn(w, f.z, acc.z);
            acc.w = __fmaf_rn(w, f.w, acc.w);
        }
        return acc;
    };
    if constexpr (kF32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(peer_ret[s]) + row * d);
        for (int v = lane; v < d / 4; v += 32) dst[v] = sum4(v);
    } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(peer_ret[s]) + row * d);
        for (int v = lane; v < d / 8; v += 32) {
            const float4 a = sum4(2 * v), b = sum4(2 * v + 1);
            __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
            __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
            dst[v] = make_uint4(*reinterpret_cast<uint32_t*>(&p0), *reinterpret_cast<uint32_t*>(&p1),
                                *reinterpret_cast<uint32_t*>(&p2), *reinterpret_cast<uint32_t*>(&p3));
        }
    }
}

// y[t] = sum over ranks g (ascending) of the row rank g returned for token t
// (written by other GPUs: read through L2 only).  One warp per token; every
// element of y[t] is written, so y needs no clearing.
template <bool kF32>
__global__ void __launch_bounds__(256)
ep_dd_combine_kernel(const void* __restrict__ ret, const int* __restrict__ slot_dd, int T, int G,
                     int cap, int d, float* __restrict__ y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    int rows[32];
    for (int g = 0; g < G; ++g) rows[g] = slot_dd[(size_t)t * G + g];
    float4* dst = reinterpret_cast<float4*>(y + (size_t)t * d);
    for (int v = lane; v < d / 4; v += 32) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int g = 0; g < G; ++g) {
            if (rows[g] < 0) continue;
            const size_t rr = (size_t)g * cap + rows[g];
            float4 f;
            if constexpr (kF32) {
                f = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(ret) + rr * d) + v);
            } else {
                const uint2 u = __ldcg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(ret) + rr * d) + v);
                f = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
            }
            acc.x += f.x; acc.y += f.y; acc.z += f.z; acc.w += f.w;
        }
        dst[v] = acc;
    }
}

// Collective (every rank of the group, once, at creation): allocate the
// buffers other ranks write into, export them through CUDA IPC, all-gather
// the handles over NCCL and map every other rank's.
int ep_p2p_setup(Layer& L, int capT, cudaStream_t s) {
    EpState& S = *L.ep;
    const int G = S.world, El = S.e_local;
    if (G > 32) return report_error(MOE_ERR_UNSUPPORTED, "the fused transport supports up to 32 ranks");
    S.cap_T = capT;
    S.cap_src = capT;   // one row per (token, destination)
    S.kmax = std::min(L.k, El);
    S.row_bytes = (size_t)L.d * wire_bytes(L);
    const size_t rows_local = (size_t)capT * L.k;
    const size_t seg_bytes = (size_t)G * S.cap_src * S.row_bytes;
    const int nblk = (capT + kRouteTokens - 1) / kRouteTokens;
    cudaError_t e = cudaSuccess;
    auto A = [&](void** p, size_t b) {
        if (e == cudaSuccess) e = cudaMalloc(p, b ? b : 256);
    };
    A((void**)&S.send_tok, rows_local * sizeof(int));
    A((void**)&S.send_w, rows_local * sizeof(float));
    A((void**)&S.send_eoff, (L.E_route + 1) * sizeof(int));
    A((void**)&S.cnt_recv, (size_t)G * El * sizeof(int));
    A((void**)&S.cnt_scan, (size_t)G * El * sizeof(int));
    A(&S.p2p_recv, seg_bytes);
    A(&S.p2p_ret, seg_bytes);
    // Count words: [G][El] per-expert rows from each source, then [G] rows.
    A((void**)&S.p2p_cnt, (size_t)G * (El + 1) * sizeof(int));
    A((void**)&S.p2p_flag, 2 * G * sizeof(unsigned));
    A((void**)&S.p2p_meta, (size_t)G * S.cap_src * S.kmax * sizeof(int2));
    A((void**)&S.dest_hist, (size_t)nblk * G * sizeof(int));
    A((void**)&S.dest_cnt, G * sizeof(int));
    A((void**)&S.dest_off, (G + 1) * sizeof(int));
    A((void**)&S.slot_dd, (size_t)capT * G * sizeof(int));
    A((void**)&S.rows_recv, G * sizeof(int));
    A((void**)&S.poison, sizeof(int));
    A((void**)&S.d_peer_recv, G * sizeof(void*));
    A((void**)&S.d_peer_ret, G * sizeof(void*));
    A((void**)&S.d_peer_cnt, G * sizeof(int*));
    A((void**)&S.d_peer_flag, G * sizeof(unsigned*));
    A((void**)&S.d_peer_meta, G * sizeof(int2*));
    if (e == cudaSuccess) e = cudaMemset(S.poison, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaHostAlloc((void**)&S.h_err, sizeof(int), 0);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&S.err_ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMemset(S.p2p_flag, 0, 2 * G * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(S.p2p_cnt, 0, (size_t)G * (El + 1) * sizeof(int));
    if (e != cudaSuccess)
        return report_error(MOE_ERR_OOM, std::string("expert-parallel buffers: ") +
                                             cudaGetErrorString(e));
    // Handles of this rank's five shared buffers, all-gathered.
    constexpr int kBufs = 5;
    void* mine[kBufs] = {S.p2p_recv, S.p2p_ret, S.p2p_cnt, S.p2p_flag, S.p2p_meta};
    std::vector<cudaIpcMemHandle_t> h_all((size_t)G * kBufs), h_mine(kBufs);
    for (int i = 0; i < kBufs && e == cudaSuccess; ++i) e = cudaIpcGetMemHandle(&h_mine[i], mine[i]);
    void* d_hbuf = nullptr;
    const size_t hb = kBufs * sizeof(cudaIpcMemHandle_t);
    if (e == cudaSuccess) e = cudaMalloc(&d_hbuf, hb * (G + 1));
    if (e == cudaSuccess) e = cudaMemcpy(d_hbuf, h_mine.data(), hb, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (d_hbuf) cudaFree(d_hbuf);
        return report_error(MOE_ERR_CUDA, std::string("IPC export: ") + cudaGetErrorString(e));
    }
    ncclResult_t nr = g_nccl.AllGather(d_hbuf, static_cast<char*>(d_hbuf) + hb, hb, ncclUint8,
                                       S.comm, s);
    if (nr != ncclSuccess) {
        cudaFree(d_hbuf);
        return nccl_fail(nr, "IPC handle all-gather");
    }
    e = cudaStreamSynchronize(s);
    if (e == cudaSuccess)
        e = cudaMemcpy(h_all.data(), static_cast<char*>(d_hbuf) + hb, hb * G, cudaMemcpyDeviceToHost);
    cudaFree(d_hbuf);
    std::vector<void*> ptr((size_t)G * kBufs);
    for (int j = 0; j < G && e == cudaSuccess; ++j)
        for (int i = 0; i < kBufs && e == cudaSuccess; ++i) {
            if (j == S.rank) {
                ptr[(size_t)j * kBufs + i] = mine[i];
            } else {
                void* p = nullptr;
                e = cudaIpcOpenMemHandle(&p, h_all[(size_t)j * kBufs + i],
                                         cudaIpcMemLazyEnablePeerAccess);
                if (e == cudaSuccess) {
                    S.ipc_opened.push_back(p);
                    ptr[(size_t)j * kBufs + i] = p;
                }
            }
        }
    if (e != cudaSuccess)
        return report_error(MOE_ERR_CUDA, std::string("IPC mapping of a peer's buffers: ") +
                                              cudaGetErrorString(e));
    std::vector<void*> col(G);
    void** dst[kBufs] = {S.d_peer_recv, S.d_peer_ret, reinterpret_cast<void**>(S.d_peer_cnt),
                         reinterpret_cast<void**>(S.d_peer_flag),
                         reinterpret_cast<void**>(S.d_peer_meta)};
    for (int i = 0; i < kBufs && e == cudaSuccess; ++i) {
        for (int j = 0; j < G; ++j) col[j] = ptr[(size_t)j * kBufs + i];
        e = cudaMemcpy(dst[i], col.data(), G * sizeof(void*), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) return report_error(MOE_ERR_CUDA, cudaGetErrorString(e));
    // The receiving side runs the grouped GEMMs on up to world * T tokens' rows.
    if (int rc = ensure_workspace(L, capT * G)) return rc;
    // No rank leaves setup before every rank has mapped its peers' buffers
    // (5 per peer; ranks take different times over them), so a first step
    // that follows creation at once does not spend its bounded peer wait on
    // a rank still mapping.
    char* d_sync = nullptr;
    e = cudaMalloc(&d_sync, 16 * (size_t)(G + 1));
    if (e != cudaSuccess) return report_error(MOE_ERR_OOM, cudaGetErrorString(e));
    nr = g_nccl.AllGather(d_sync, d_sync + 16, 16, ncclUint8, S.comm, s);
    const cudaError_t se = nr == ncclSuccess ? cudaStreamSynchronize(s) : cudaSuccess;
    cudaFree(d_sync);
    if (nr != ncclSuccess) return nccl_fail(nr, "setup barrier");
    if (se != cudaSuccess) return report_error(MOE_ERR_CUDA, cudaGetErrorString(se));
    return MOE_OK;
}

// MOE_ERR_TIMEOUT once the group has failed: a completed copy of the device
// error flags (taken at the end of every fused forward) shows a flag.  With
// wait, the last forward's copy is waited for first.
int ep_failure(EpState& S, bool wait) {
    if (!S.failed && S.err_recorded) {
        const cudaError_t q = wait ? cudaEventSynchronize(S.err_ev) : cudaEventQuery(S.err_ev);
        if (q == cudaSuccess) {
            if (*reinterpret_cast<volatile int*>(S.h_err) != 0) S.failed = true;
        } else if (q != cudaErrorNotReady) {
            return report_error(MOE_ERR_CUDA, std::string("expert-parallel status: ") +
                                                  cudaGetErrorString(q));
        }
    }
    if (S.failed)
        return report_error(MOE_ERR_TIMEOUT,
                            "an expert-parallel peer wait timed out (a rank missed a step or "
                            "stopped); the group is failed: destroy and recreate it on every rank");
    return MOE_OK;
}

int ep_forward_p2p(Layer& L, const float* x, float* y, int T, cudaStream_t s) {
    EpState& S = *L.ep;
    if (T > S.cap_T)
        return report_error(MOE_ERR_INVALID,
                            "T exceeds the expert-parallel capacity fixed at creation (max_tokens)");
    if (int rc = ep_failure(S, false)) return rc;
    Workspace& W = L.ws;
    const int G = S.world, El = S.e_local, Eg = L.E_route;
    const unsigned epoch = ++S.epoch;
    auto cuda_err = [](cudaError_t e, const char* what) {
        return report_error(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    };
    cudaError_t ce;
    L.prof_n = 0;
    // 1-2: route; per (token, destination rank) one row and its selections
    // straight into the destination's receive buffer.
    const int nblk = (T + kRouteTokens - 1) / kRouteTokens;
    prof_mark(L, 0, s);
    if (T > 0) {
        if ((ce = launch_router(L, x, T, W.logits, W.idx, W.wts, W.blockhist, s, NormRef{},
                                S.eperm)) != cudaSuccess)
            return cuda_err(ce, "router");
        prof_mark(L, 1, s);
        // Expert positions (compact): per-expert counts to the ranks, and each
        // selection's position inside its expert's block from this source.
        if ((ce = launch_scan_generic(W.blockhist, nblk, Eg, 1, W.counts, S.send_eoff, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, s)) != cudaSuccess)
            return cuda_err(ce, "dispatch scan");
        ep_dest_hist_kernel<<<nblk, 256, 0, s>>>(W.idx, T, L.k, El, G, S.dest_hist);
        if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "destination histogram");
        if ((ce = launch_scan_generic(S.dest_hist, nblk, G, 1, S.dest_cnt, S.dest_off, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, s)) != cudaSuccess)
            return cuda_err(ce, "destination scan");
        prof_mark(L, 5, s);
        if (fp32_faithful(L))
            ep_dedup_push_kernel<2><<<nblk, 256, 0, s>>>(x, T, L.d, L.k, El, G, S.kmax, W.idx,
                                                         W.wts, W.blockhist, S.dest_hist,
                                                         S.d_peer_recv, S.d_peer_meta, S.cap_src,
                                                         S.rank, S.slot_dd, S.poison);
        else
            ep_dedup_push_kernel<0><<<nblk, 256, 0, s>>>(x, T, L.d, L.k, El, G, S.kmax, W.idx,
                                                         W.wts, W.blockhist, S.dest_hist,
                                                         S.d_peer_recv, S.d_peer_meta, S.cap_src,
                                                         S.rank, S.slot_dd, S.poison);
        if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "dispatch push");
    } else {
        prof_mark(L, 5, s);
        if ((ce = cudaMemsetAsync(W.counts, 0, Eg * sizeof(int), s)) != cudaSuccess ||
            (ce = cudaMemsetAsync(S.dest_cnt, 0, G * sizeof(int), s)) != cudaSuccess)
            return cuda_err(ce, "counts");
    }
    // 3-4: counts, row counts and flags to every rank; wait for every source's.
    const int sig_threads = (G + 31) / 32 * 32;
    ep_signal_kernel<<<1, sig_threads, 0, s>>>(S.d_peer_cnt, W.counts, S.d_peer_flag, G, El,
                                               S.rank, 0, epoch, S.poison, S.dest_cnt);
    ep_wait_kernel<<<1, std::max(sig_threads, 128), 0, s>>>(S.p2p_flag, G, 0, epoch, S.p2p_cnt,
                                                            S.cnt_recv, S.cnt_scan, G * El,
                                                            S.cap_src, W.dev_err, S.poison,
                                                            S.wait_ns, S.rows_recv);
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "dispatch signal");
    prof_mark(L, 2, s);
    // Arrival scan (per-source bases inside each local expert's block) and
    // arrangement: each received row into each of its experts' GEMM rows.
    if ((ce = launch_scan_generic(S.cnt_scan, G, El, kTileM, W.counts, W.eoff, W.mtiles,
                                  W.num_mtiles, W.ptiles, W.num_ptiles, W.row_token,
                                  W.row_weight, s)) != cudaSuccess)
        return cuda_err(ce, "arrival scan");
    const size_t R_bound = (size_t)G * S.cap_src;
    const int grid = (int)((R_bound + 7) / 8);
    {
        auto run = [&](auto kern) {
            kern<<<grid, 256, 0, s>>>(S.p2p_recv, S.p2p_meta, S.rows_recv, S.cap_src, L.d, G, El,
                                      S.kmax, S.cnt_scan, W.eoff, W.row_token, W.row_weight,
                                      W.row_slot, W.a_hi, W.a_lo);
        };
        switch (act_format(L, false)) {
            case kActTf32x2: run(ep_dd_arrange_kernel<kActTf32x2>); break;
            case kActBf16x2: run(ep_dd_arrange_kernel<kActBf16x2>); break;
            default: run(ep_dd_arrange_kernel<kActBf16>); break;
        }
    }
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "arrange");
    // 5-6: the local experts; the down GEMM stores each expert's output at
    // its (received row, selection) slot, K whole.  The expected routed rows
    // (T * k, this rank's own) size the GEMM launch; any count is run
    // correctly.
    const int R_est = std::max(T, 1) * L.k;
    prof_mark(L, 3, s);
    if ((ce = launch_expert_gemm_rows(L, R_est, nullptr, s, 0)) != cudaSuccess)
        return cuda_err(ce, "gate/up GEMM");
    prof_mark(L, 4, s);
    if ((ce = launch_expert_gemm_rows(L, R_est, nullptr, s, 3)) != cudaSuccess)
        return cuda_err(ce, "down GEMM");
    // 7: one summed row per received row back to its source; return flags.
    prof_mark(L, 6, s);
    if (fp32_faithful(L))
        ep_return_push_kernel<true><<<grid, 256, 0, s>>>(W.part, S.p2p_meta, S.rows_recv,
                                                         S.cap_src, L.d, G, El, S.kmax,
                                                         S.cnt_scan, W.eoff, S.rank,
                                                         S.d_peer_ret, S.poison);
    else
        ep_return_push_kernel<false><<<grid, 256, 0, s>>>(W.part, S.p2p_meta, S.rows_recv,
                                                          S.cap_src, L.d, G, El, S.kmax,
                                                          S.cnt_scan, W.eoff, S.rank,
                                                          S.d_peer_ret, S.poison);
    ep_signal_kernel<<<1, sig_threads, 0, s>>>(nullptr, nullptr, S.d_peer_flag, G, El, S.rank, 1,
                                               epoch, S.poison);
    ep_wait_kernel<<<1, std::max(sig_threads, 128), 0, s>>>(S.p2p_flag, G, 1, epoch, nullptr,
                                                            nullptr, nullptr, 0, 0, W.dev_err,
                                                            S.poison, S.wait_ns);
    if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "return signal");
    // 8: y[t] = sum of its ranks' rows, ascending rank.
    prof_mark(L, 7, s);
    if (T > 0) {
        if (fp32_faithful(L))
            ep_dd_combine_kernel<true><<<(T + 7) / 8, 256, 0, s>>>(S.p2p_ret, S.slot_dd, T, G,
                                                                   S.cap_src, L.d, y);
        else
            ep_dd_combine_kernel<false><<<(T + 7) / 8, 256, 0, s>>>(S.p2p_ret, S.slot_dd, T, G,
                                                                    S.cap_src, L.d, y);
        if ((ce = cudaGetLastError()) != cudaSuccess) return cuda_err(ce, "combine");
    }
    prof_mark(L, kProfEnd, s);
    // The step's device error flags, read back without blocking; the next
    // forward (or moe_ep_check) looks at them once the copy has completed.
    if ((ce = cudaMemcpyAsync(S.h_err, W.dev_err, sizeof(int), cudaMemcpyDeviceToHost, s)) !=
            cudaSuccess ||
        (ce = cudaEventRecord(S.err_ev, s)) != cudaSuccess)
        return cuda_err(ce, "status copy");
    S.err_recorded = true;
    return MOE_OK;
}

int ep_forward(Layer& L, const float* x, float* y, int T, cudaStream_t s) {
    if (L.ep->transport == MOE_EP_TRANSPORT_NCCL) return ep_forward_nccl(L, x, y, T, s);
    return ep_forward_p2p(L, x, y, T, s);
}

struct DeviceGuardEp {
    int prev = -1;
    explicit DeviceGuardEp(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuardEp() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

void ep_destroy(Layer& L) {
    if (!L.ep) return;
    ep_free_buffers(*L.ep);
    if (L.ep->eperm) cudaFree(L.ep->eperm);
    if (L.ep->comm && g_nccl.ok) g_nccl.CommDestroy(L.ep->comm);
    delete L.ep;
    L.ep = nullptr;
}

}  // namespace moe

extern "C" {

int moe_ep_plan(const int32_t* counts, const int32_t* counts_in, int32_t world, int32_t e_local,
                int64_t* send_rows, int64_t* send_off, int64_t* recv_rows, int64_t* recv_off) {
    if (!counts || !counts_in || !send_rows || !send_off || !recv_rows || !recv_off || world < 1 ||
        e_local < 1)
        return moe::report_error(MOE_ERR_INVALID, "moe_ep_plan: bad argument");
    send_off[0] = recv_off[0] = 0;
    for (int j = 0; j < world; ++j) {
        int64_t a = 0, b = 0;
        for (int e = 0; e < e_local; ++e) {
            if (counts[j * e_local + e] < 0 || counts_in[j * e_local + e] < 0)
                return moe::report_error(MOE_ERR_INVALID, "moe_ep_plan: negative count");
            a += counts[j * e_local + e];
            b += counts_in[j * e_local + e];
        }
        send_rows[j] = a;
        recv_rows[j] = b;
        send_off[j + 1] = send_off[j] + a;
        recv_off[j + 1] = recv_off[j] + b;
    }
    return MOE_OK;
}

int moe_ep_unique_id(void* id_out) {
    std::string err;
    if (!id_out) return moe::report_error(MOE_ERR_INVALID, "null argument");
    if (!moe::load_nccl(&err)) return moe::report_error(MOE_ERR_NCCL, err);
    ncclUniqueId id;
    ncclResult_t r = moe::g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) return moe::nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof id);
    return MOE_OK;
}

static int ep_create(const MoeConfig* cfg, const MoeWeightsHost* w, bool device_ptrs, int rank,
                     int world, const void* nccl_id, MoeHandle** out) {
    using namespace moe;
    std::string err;
    if (!cfg || !w || !nccl_id || !out) return report_error(MOE_ERR_INVALID, "null argument");
    if (world < 1 || rank < 0 || rank >= world) return report_error(MOE_ERR_INVALID, "bad rank");
    if (cfg->num_experts % world != 0)
        return report_error(MOE_ERR_INVALID, "num_experts must be a multiple of the group size");
    if (!load_nccl(&err)) return report_error(MOE_ERR_NCCL, err);
    const int El = cfg->num_experts / world;
    // Round-robin placement (balances a skewed router, e.g. BASELINE config
    // 5's Zipf-like bias): dispatch position i holds expert
    // (i % El) * world + i / El, so this rank's slice [rank * El, ...) is
    // experts rank, rank + world, ...  The router weights keep the experts'
    // own order.
    const int Eg = cfg->num_experts;
    std::vector<const float*> w1p(Eg), w2p(Eg), w3p(Eg);
    std::vector<int> eperm(Eg);
    for (int i = 0; i < Eg; ++i) {
        const int e = (i % El) * world + i / El;
        w1p[i] = w->w1[e];
        w2p[i] = w->w2[e];
        w3p[i] = w->w3[e];
        eperm[e] = i;
    }
    MoeWeightsHost wp = *w;
    wp.w1 = w1p.data();
    wp.w2 = w2p.data();
    wp.w3 = w3p.data();
    MoeHandle* h = nullptr;
    int rc = create_slice(cfg, &wp, device_ptrs, rank * El, El, &h);
    if (rc) return rc;
    DeviceGuardEp guard(cfg->device);
    auto* S = new EpState();
    S->rank = rank;
    S->world = world;
    S->e_local = El;
    h->L.ep = S;
    cudaError_t ce = cudaMalloc(&S->eperm, Eg * sizeof(int));
    if (ce == cudaSuccess)
        ce = cudaMemcpy(S->eperm, eperm.data(), Eg * sizeof(int), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        rc = report_error(MOE_ERR_CUDA, std::string("expert placement: ") + cudaGetErrorString(ce));
        moe_destroy(h);
        return rc;
    }
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    ncclResult_t r = g_nccl.CommInitRank(&S->comm, world, id, rank);
    if (r != ncclSuccess) {
        rc = nccl_fail(r, "ncclCommInitRank");
        S->comm = nullptr;
        moe_destroy(h);
        return rc;
    }
    S->transport = cfg->ep_transport;
    S->wait_ns = (cfg->ep_wait_ms > 0 ? (unsigned long long)cfg->ep_wait_ms * 1000000ull
                                      : kPeerWaitNs);
    if (S->transport == MOE_EP_TRANSPORT_P2P) {
        // Fixed capacity: the buffers are mapped by every rank once.
        const int capT = cfg->max_tokens > 0 ? cfg->max_tokens : 4096;
        rc = ep_p2p_setup(h->L, capT, h->own_stream);
        if (rc) {
            moe_destroy(h);
            return rc;
        }
    }
    *out = h;
    return MOE_OK;
}

int moe_ep_create(const MoeConfig* cfg, const MoeWeightsHost* w, int rank, int world,
                  const void* nccl_id, MoeHandle** out) {
    return ep_create(cfg, w, false, rank, world, nccl_id, out);
}

int moe_ep_create_from_device(const MoeConfig* cfg, const MoeWeightsHost* w, int rank, int world,
                              const void* nccl_id, MoeHandle** out) {
    return ep_create(cfg, w, true, rank, world, nccl_id, out);
}

int moe_ep_check(MoeHandle* h) {
    using namespace moe;
    if (!h || !h->L.ep) return report_error(MOE_ERR_INVALID, "not an expert-parallel handle");
    if (h->L.ep->transport == MOE_EP_TRANSPORT_NCCL) return MOE_OK;
    DeviceGuardEp guard(h->L.cfg.device);
    return ep_failure(*h->L.ep, true);
}

int moe_ep_forward_device(MoeHandle* h, const float* x, float* y, int32_t T, void* stream) {
    using namespace moe;
    if (!h || !h->L.ep) return report_error(MOE_ERR_INVALID, "not an expert-parallel handle");
    if (T < 0) return report_error(MOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !y)) return report_error(MOE_ERR_INVALID, "null x or y");
    DeviceGuardEp guard(h->L.cfg.device);
    return ep_forward(h->L, x, y, T, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
