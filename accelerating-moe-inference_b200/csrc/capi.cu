// C ABI of libmoe_b200.so (declared in include/moe_b200.h): layer handles,
// weight upload, workspace management and the forward orchestration.
//
// forward on device buffers, all on the caller's stream, no host sync:
//   router_kernel -> dispatch_scan -> dispatch_permute
//   -> gate/up grouped GEMM (SwiGLU epilogue) -> down grouped GEMM (each
//   routed row's output at its selection slot) -> ordered combine into y
// or, for T <= decode_max_tokens, router -> scan -> the weight-streaming
// decode kernels -> ordered combine.
#include <cudaTypedefs.h>

#include <algorithm>
#include <array>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "moe_internal.h"
#include "ptx.cuh"

namespace moe {
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(MOE_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define MOE_CUDA(call)                                            \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);       \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool load_encode(std::string* err) {
    if (g_encode) return true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        *err = "cuTensorMapEncodeTiled is not available from the driver";
        return false;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return true;
}

void free_ptr(void* p) {
    if (p) cudaFree(p);
}

template <typename T>
cudaError_t dalloc(T** p, size_t bytes, size_t* counter) {
    *p = nullptr;
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), bytes);
    if (e == cudaSuccess && counter) *counter += bytes;
    return e;
}

void free_workspace(Workspace& W) {
    free_ptr(W.logits); free_ptr(W.idx); free_ptr(W.wts); free_ptr(W.blockhist);
    free_ptr(W.counts); free_ptr(W.eoff); free_ptr(W.mtiles); free_ptr(W.num_mtiles);
    free_ptr(W.ptiles); free_ptr(W.num_ptiles);
    free_ptr(W.row_token); free_ptr(W.row_weight); free_ptr(W.row_slot); free_ptr(W.part);
    free_ptr(W.a_hi); free_ptr(W.a_lo);
    free_ptr(W.h_hi); free_ptr(W.h_lo); free_ptr(W.x_stage); free_ptr(W.y_stage);
    free_ptr(W.dev_err); free_ptr(W.h_dec); free_ptr(W.dec_counter);
    free_ptr(W.row_mean); free_ptr(W.row_inv);
    W = Workspace{};
}

}  // namespace

int ensure_workspace(Layer& L, int T) {
    Workspace& W = L.ws;
    if (T <= W.cap_T && W.dev_err) return MOE_OK;
    // Grow-only.  Work queued on the previous buffers must finish first.
    if (W.dev_err) MOE_CUDA(cudaDeviceSynchronize());
    const int capT = std::max({T, W.cap_T + W.cap_T / 2, 64});
    free_workspace(W);
    const size_t k = L.k, E = L.E_route > L.E ? L.E_route : L.E;
    const int nblk = (capT + kRouteTokens - 1) / kRouteTokens;
    const int cap_mtiles = (int)((size_t)capT * k / kTileM) + L.E + 1;
    const size_t cap_rows = (size_t)cap_mtiles * kTileM;
    const size_t eb = plane_bytes(L);
    const bool two = split_planes(L);
    size_t bytes = 0;
    MOE_CUDA(dalloc(&W.logits, sizeof(float) * capT * E, &bytes));
    MOE_CUDA(dalloc(&W.idx, sizeof(int) * capT * k, &bytes));
    MOE_CUDA(dalloc(&W.wts, sizeof(float) * capT * k, &bytes));
    MOE_CUDA(dalloc(&W.blockhist, sizeof(int) * nblk * E, &bytes));
    MOE_CUDA(dalloc(&W.counts, sizeof(int) * E, &bytes));
    MOE_CUDA(dalloc(&W.eoff, sizeof(int) * (E + 1), &bytes));
    MOE_CUDA(dalloc(&W.mtiles, sizeof(MTile) * cap_mtiles, &bytes));
    MOE_CUDA(dalloc(&W.num_mtiles, sizeof(int), &bytes));
    MOE_CUDA(dalloc(&W.ptiles, sizeof(MTile) * cap_mtiles, &bytes));
    MOE_CUDA(dalloc(&W.num_ptiles, sizeof(int), &bytes));
    MOE_CUDA(dalloc(&W.row_token, sizeof(int) * cap_rows, &bytes));
    MOE_CUDA(dalloc(&W.row_weight, sizeof(float) * cap_rows, &bytes));
    MOE_CUDA(dalloc(&W.row_slot, sizeof(int) * cap_rows, &bytes));
    // Expert output rows for the ordered combine: one per selection slot, or
    // per (slot, K split) at decode sizes -- the down GEMM splits K only for
    // at most kSplitMaxRows routed rows, into at most k_blocks / kSplitMinBlocks
    // parts, and the decode kernel into decode_chunks() parts for T <= 64.
    {
        const size_t gemm_splits = (size_t)L.ffp / 32 / kSplitMinBlocks + 1;
        const size_t dec_rows = (size_t)decode_max_supported_tokens() * k * decode_chunks(L);
        W.part_rows = std::max({(size_t)capT * k, (size_t)kSplitMaxRows * gemm_splits, dec_rows});
        MOE_CUDA(dalloc(&W.part, sizeof(float) * W.part_rows * L.d, &bytes));
    }
    // A holds the dispatched rows in the GEMM operand format or, for the
    // decode kernels, as fp32 rows in the fp32-faithful precisions (at the
    // same padded row positions).
    MOE_CUDA(dalloc(&W.a_hi, (fp32_faithful(L) ? 4 : eb) * cap_rows * L.d, &bytes));
    MOE_CUDA(dalloc(&W.h_hi, eb * cap_rows * L.ffp, &bytes));
    if (two) {
        MOE_CUDA(dalloc(&W.a_lo, eb * cap_rows * L.d, &bytes));
        MOE_CUDA(dalloc(&W.h_lo, eb * cap_rows * L.ffp, &bytes));
    }
    MOE_CUDA(dalloc(&W.h_dec, sizeof(float) * (size_t)decode_max_supported_tokens() * k * L.ffp,
                    &bytes));
    MOE_CUDA(dalloc(&W.dec_counter, 2 * sizeof(int), &bytes));
    MOE_CUDA(dalloc(&W.row_mean, sizeof(float) * capT, &bytes));
    MOE_CUDA(dalloc(&W.row_inv, sizeof(float) * capT, &bytes));
    MOE_CUDA(dalloc(&W.dev_err, sizeof(int), &bytes));
    MOE_CUDA(cudaMemset(W.dev_err, 0, sizeof(int)));
    MOE_CUDA(cudaMemset(W.num_mtiles, 0, sizeof(int)));
    MOE_CUDA(cudaMemset(W.num_ptiles, 0, sizeof(int)));
    W.cap_T = capT;
    W.cap_rows = (int)cap_rows;
    W.cap_mtiles = cap_mtiles;
    W.bytes = bytes;
    const bool bf = planes_bf16(L);
    const uint32_t box_k = kblock_elems(L);
    std::string err;
    if (!make_tmap_2d(&W.tm_a_hi, W.a_hi, bf, L.d, cap_rows, box_k, kTileM, &err) ||
        !make_tmap_2d(&W.tm_h_hi, W.h_hi, bf, L.ffp, cap_rows, box_k, kTileM, &err))
        return fail(MOE_ERR_CUDA, err);
    if (two) {
        if (!make_tmap_2d(&W.tm_a_lo, W.a_lo, bf, L.d, cap_rows, box_k, kTileM, &err) ||
            !make_tmap_2d(&W.tm_h_lo, W.h_lo, bf, L.ffp, cap_rows, box_k, kTileM, &err))
            return fail(MOE_ERR_CUDA, err);
    } else {
        W.tm_a_lo = W.tm_a_hi;
        W.tm_h_lo = W.tm_h_hi;
    }
    return MOE_OK;
}

namespace {

int ensure_stage(Layer& L, int T) {
    int rc = ensure_workspace(L, T);
    if (rc) return rc;
    Workspace& W = L.ws;
    if (!W.x_stage) {
        MOE_CUDA(dalloc(&W.x_stage, sizeof(float) * (size_t)W.cap_T * L.d, &W.bytes));
        MOE_CUDA(dalloc(&W.y_stage, sizeof(float) * (size_t)W.cap_T * L.d, &W.bytes));
    }
    return MOE_OK;
}

}  // namespace

// The decode-kernel threshold MOE_DECODE_AUTO resolves to, from the measured
// crossover with the grouped GEMMs on B200 (C2 weights): in BF16 the grouped
// GEMMs stream as fast as the decode kernels from T = 2 on and faster from
// T = 4; in FP32 the decode kernels read 4 bytes per weight against the
// 3xTF32 GEMMs' 8 and stay ahead up to about T = 14.
int auto_decode_max_tokens(int precision) { return precision == MOE_PREC_BF16 ? 1 : 14; }

namespace {

int validate_config(const MoeConfig& c) {
    if (c.d_model <= 0 || c.d_model % 64 != 0)
        return fail(MOE_ERR_UNSUPPORTED, "d_model must be a positive multiple of 64");
    if (c.d_ff <= 0) return fail(MOE_ERR_INVALID, "d_ff must be positive");
    if (c.num_experts < 1 || c.num_experts > kMaxExperts)
        return fail(MOE_ERR_UNSUPPORTED, "num_experts must be in 1..256");
    if (c.top_k < 1 || c.top_k > kMaxTopK || c.top_k > c.num_experts)
        return fail(MOE_ERR_INVALID, "top_k must be in 1..min(8, num_experts)");
    if (c.router_policy != MOE_ROUTER_PHI_QUANTISED && c.router_policy != MOE_ROUTER_SOFTMAX_TOPK)
        return fail(MOE_ERR_INVALID, "unknown router_policy");
    if (c.router_policy == MOE_ROUTER_PHI_QUANTISED && (c.top_k != 2 || c.num_experts < 2))
        return fail(MOE_ERR_INVALID, "the PHI_QUANTISED router selects exactly 2 experts");
    if (c.router_policy == MOE_ROUTER_PHI_QUANTISED && !(c.router_quantum > 0.0f))
        return fail(MOE_ERR_INVALID, "router_quantum must be positive");
    if (c.precision != MOE_PREC_FP32 && c.precision != MOE_PREC_BF16 &&
        c.precision != MOE_PREC_FP32_BF16X3)
        return fail(MOE_ERR_INVALID, "unknown precision");
    if (c.decode_max_tokens < -1 || c.decode_max_tokens > decode_max_supported_tokens())
        return fail(MOE_ERR_INVALID, "decode_max_tokens must be in -1..64");
    if (c.max_tokens < 0) return fail(MOE_ERR_INVALID, "max_tokens < 0");
    if (c.gemm_variant < MOE_GEMM_AUTO || c.gemm_variant > MOE_GEMM_CTA_PAIR)
        return fail(MOE_ERR_INVALID, "unknown gemm_variant");
    if (c.ep_transport != MOE_EP_TRANSPORT_P2P && c.ep_transport != MOE_EP_TRANSPORT_NCCL)
        return fail(MOE_ERR_INVALID, "unknown ep_transport");
    if (c.ep_wait_ms < 0) return fail(MOE_ERR_INVALID, "ep_wait_ms < 0");
    return MOE_OK;
}

int check_device_errors(Layer& L) {
    int flag = 0;
    if (!L.ws.dev_err) return MOE_OK;
    MOE_CUDA(cudaMemcpy(&flag, L.ws.dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (flag) {
        cudaMemset(L.ws.dev_err, 0, sizeof(int));
        char buf[128];
        std::snprintf(buf, sizeof buf, "a device-side wait timed out (flags 0x%x)", flag);
        return fail(MOE_ERR_TIMEOUT, buf);
    }
    return MOE_OK;
}

// block: the decoder layer's MoE half -- x is the attention output, the
// post-attention LayerNorm is applied on load and x is added after the
// combine (stages: norm statistics count as router time, the residual as
// down time).
int forward_impl(Layer& L, const float* x, float* y, int T, cudaStream_t s, bool block = false) {
    int rc = ensure_workspace(L, T);
    if (rc) return rc;
    Workspace& W = L.ws;
    L.last_stream = s;
    L.last_T = T;
    L.prof_n = 0;
    NormRef nr;
    if (block) {
        nr.mean = W.row_mean;
        nr.inv = W.row_inv;
        nr.w = L.norm_w;
        nr.b = L.norm_b;
    }
    const bool decode = T <= L.cfg.decode_max_tokens;
    // A decode-sized batch is routed and dispatched by one single-CTA launch.
    int kc = 0, stages = 0;
    const bool small = route_small_geometry(L, T, block, &kc, &stages);
    // The small-batch router computes RMSNorm statistics itself when every
    // K chunk is resident in its shared memory (one launch fewer per block).
    const bool rms_inline = small && block && L.norm_rms && route_small_resident(L, kc, stages);
    prof_mark(L, 0, s);
    if (block && L.norm_rms && !rms_inline)
        MOE_CUDA(launch_rms_stats(x, T, L.d, L.norm_eps, W.row_mean, W.row_inv, s));
    else if (block && !L.norm_rms)
        MOE_CUDA(launch_row_stats(x, T, L.d, L.norm_eps, W.row_mean, W.row_inv, W.dev_err, s));
    if (small) {
        MOE_CUDA(launch_route_small(L, x, T, nr, decode, s, rms_inline));
    } else {
        MOE_CUDA(launch_router(L, x, T, W.logits, W.idx, W.wts, W.blockhist, s, nr));
    }
    prof_mark(L, 1, s);
    // A batch that fits one router block is scanned inside the permute kernel.
    if (T > kRouteTokens) MOE_CUDA(launch_dispatch_scan(L, T, s));
    prof_mark(L, 2, s);
    int nsplit = 1;
    if (decode) {
        // marks stages 3 and 4 between its kernels
        MOE_CUDA(launch_decode(L, x, T, &nsplit, s, nr, /*packed=*/small));
    } else {
        if (!small) MOE_CUDA(launch_dispatch_permute(L, x, T, s, nr));
        prof_mark(L, 3, s);
        MOE_CUDA(launch_expert_gemm_rows(L, T * L.k, nullptr, s, 0));
        prof_mark(L, 4, s);
        MOE_CUDA(launch_expert_gemm_rows(L, T * L.k, nullptr, s, 3,
                                         (size_t)T * L.k * L.d, &nsplit));
    }
    // The combine (and the block's residual, y = moe + x) counts as down time.
    MOE_CUDA(launch_combine(L, T, nsplit, block ? x : nullptr, y, s));
    prof_mark(L, kProfEnd, s);
    return MOE_OK;
}

// ------------------------------------------------------------ model.bin
struct BinEntry {
    std::vector<uint64_t> shape;
    uint64_t offset = 0, bytes = 0;
};

// The index format of ModelLoader (src/model_loader.cu:14-30): u32 count; per
// entry u32 name_len, name bytes, u32 ndim, u32 dims[ndim], u64 offset,
// u64 bytes; payloads are fp32.
int read_index(const std::string& path, std::unordered_map<std::string, BinEntry>* out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail(MOE_ERR_IO, "cannot open model: " + path);
    auto rd32 = [&](uint32_t* v) { return bool(f.read(reinterpret_cast<char*>(v), 4)); };
    auto rd64 = [&](uint64_t* v) { return bool(f.read(reinterpret_cast<char*>(v), 8)); };
    uint32_t count = 0;
    if (!rd32(&count)) return fail(MOE_ERR_IO, "truncated model.bin");
    for (uint32_t i = 0; i < count; ++i) {
        uint32_t nl = 0, nd = 0;
        if (!rd32(&nl) || nl > (1u << 20)) return fail(MOE_ERR_IO, "truncated model.bin");
        std::string name(nl, '\0');
        if (!f.read(name.data(), nl) || !rd32(&nd) || nd > 8)
            return fail(MOE_ERR_IO, "truncated model.bin");
        BinEntry e;
        e.shape.resize(nd);
        for (uint32_t j = 0; j < nd; ++j) {
            uint32_t v;
            if (!rd32(&v)) return fail(MOE_ERR_IO, "truncated model.bin");
            e.shape[j] = v;
        }
        if (!rd64(&e.offset) || !rd64(&e.bytes)) return fail(MOE_ERR_IO, "truncated model.bin");
        (*out)[name] = std::move(e);
    }
    return MOE_OK;
}

int load_tensor(const std::string& path, const std::unordered_map<std::string, BinEntry>& idx,
                const std::string& name, std::vector<float>* out, std::vector<uint64_t>* shape) {
    auto it = idx.find(name);
    if (it == idx.end()) return fail(MOE_ERR_IO, "missing tensor: " + name);
    uint64_t n = 1;
    for (uint64_t dd : it->second.shape) n *= dd;
    if (it->second.bytes != n * sizeof(float))
        return fail(MOE_ERR_IO, "tensor is not float32: " + name);
    out->resize(n);
    std::ifstream f(path, std::ios::binary);
    if (!f) return fail(MOE_ERR_IO, "cannot reopen model: " + path);
    f.seekg(static_cast<std::streamoff>(it->second.offset));
    if (!f.read(reinterpret_cast<char*>(out->data()), static_cast<std::streamsize>(n * 4)))
        return fail(MOE_ERR_IO, "truncated tensor: " + name);
    if (shape) *shape = it->second.shape;
    return MOE_OK;
}

}  // namespace

int report_error(int code, const std::string& msg) { return fail(code, msg); }

bool make_tmap_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer,
                  uint32_t box_inner, uint32_t box_outer, std::string* err) {
    if (!load_encode(err)) return false;
    const size_t es = bf16 ? 2 : 4;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * es};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        std::snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) for a %llux%llu map",
                      (int)r, (unsigned long long)outer, (unsigned long long)inner);
        *err = buf;
        return false;
    }
    return true;
}

}  // namespace moe

using moe::Layer;

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

const char* moe_last_error(void) { return moe::g_last_error.c_str(); }

void moe_config_init(MoeConfig* c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->d_model = 4096;
    c->d_ff = 448;
    c->num_experts = 16;
    c->top_k = 2;
    c->router_policy = MOE_ROUTER_PHI_QUANTISED;
    c->precision = MOE_PREC_FP32;
    c->router_quantum = 1.0e-3f;
    c->router_tie_eps = 2.0e-2f;
    c->decode_max_tokens = MOE_DECODE_AUTO;
    c->device = 0;
    c->max_tokens = 0;
}

}  // extern "C"

namespace moe {
namespace {
int create_impl(const MoeConfig* cfg, const MoeWeightsHost* w, bool device_ptrs, MoeHandle** out);
}
}  // namespace moe

extern "C" {

int moe_create(const MoeConfig* cfg, const MoeWeightsHost* w, MoeHandle** out) {
    return moe::create_impl(cfg, w, false, out);
}

int moe_create_from_device(const MoeConfig* cfg, const MoeWeightsHost* w, MoeHandle** out) {
    return moe::create_impl(cfg, w, true, out);
}

}  // extern "C"

namespace moe {
namespace {
int create_impl(const MoeConfig* cfg, const MoeWeightsHost* w, bool device_ptrs, MoeHandle** out) {
    return create_slice(cfg, w, device_ptrs, 0, cfg ? cfg->num_experts : 0, out);
}
}  // namespace

// Build a handle that routes over cfg->num_experts experts and holds experts
// [e_first, e_first + e_count) (all of them unless expert-parallel).
int create_slice(const MoeConfig* cfg, const MoeWeightsHost* w, bool device_ptrs, int e_first,
                 int e_count, MoeHandle** out, ExpertReader* reader) {
    if (!cfg || !w || !out) return fail(MOE_ERR_INVALID, "null argument");
    *out = nullptr;
    int rc = validate_config(*cfg);
    if (rc) return rc;
    if (reader && device_ptrs) return fail(MOE_ERR_INVALID, "an expert reader supplies host weights");
    if (!w->router_weight || (!reader && (!w->w1 || !w->w2 || !w->w3)))
        return fail(MOE_ERR_INVALID, "missing weight pointers");
    if (e_first < 0 || e_count < 1 || e_first + e_count > cfg->num_experts)
        return fail(MOE_ERR_INVALID, "bad expert slice");
    for (int e = e_first; !reader && e < e_first + e_count; ++e)
        if (!w->w1[e] || !w->w2[e] || !w->w3[e]) return fail(MOE_ERR_INVALID, "null expert weight");
    int ndev = 0;
    MOE_CUDA(cudaGetDeviceCount(&ndev));
    if (cfg->device < 0 || cfg->device >= ndev) return fail(MOE_ERR_INVALID, "no such device");
    DeviceGuard guard(cfg->device);
    int major = 0, minor = 0;
    MOE_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cfg->device));
    MOE_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, cfg->device));
    if (major != 10 || minor != 0)
        return fail(MOE_ERR_UNSUPPORTED, "libmoe_b200 is built for sm_100a (B200) only");

    std::unique_ptr<MoeHandle> h(new MoeHandle());
    Layer& L = h->L;
    L.cfg = *cfg;
    if (L.cfg.decode_max_tokens < 0) L.cfg.decode_max_tokens = auto_decode_max_tokens(cfg->precision);
    L.d = cfg->d_model;
    L.ff = cfg->d_ff;
    L.ffp = (cfg->d_ff + kFfBlock - 1) / kFfBlock * kFfBlock;
    L.E = e_count;
    L.E_route = cfg->num_experts;
    L.e_first = e_first;
    L.k = cfg->top_k;
    MOE_CUDA(cudaDeviceGetAttribute(&L.sm_count, cudaDevAttrMultiProcessorCount, cfg->device));
    MOE_CUDA(cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking));
    MOE_CUDA(cudaStreamCreateWithFlags(&h->h2d_stream, cudaStreamNonBlocking));
    MOE_CUDA(cudaStreamCreateWithFlags(&h->d2h_stream, cudaStreamNonBlocking));
    for (int c = 0; c < MoeHandle::kMaxChunks; ++c) {
        MOE_CUDA(cudaEventCreateWithFlags(&h->in_ev[c], cudaEventDisableTiming));
        MOE_CUDA(cudaEventCreateWithFlags(&h->out_ev[c], cudaEventDisableTiming));
    }
    cudaStream_t s = h->own_stream;

    const size_t d = L.d, E = L.E, ffp = L.ffp, ff = L.ff;
    const bool two = split_planes(L);
    const size_t eb = plane_bytes(L);
    size_t& wb = L.weight_bytes;
    auto cleanup_and_fail = [&](int code) {
        moe_destroy(h.release());
        return code;
    };
#define MOE_CUDA_C(call)                                                 \
    do {                                                                 \
        cudaError_t e_ = (call);                                         \
        if (e_ != cudaSuccess) return cleanup_and_fail(cuda_fail(e_, #call)); \
    } while (0)
    const cudaMemcpyKind kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const size_t Er = L.E_route;
    MOE_CUDA_C(dalloc(&L.wg, sizeof(float) * Er * d, &wb));
    MOE_CUDA_C(cudaMemcpy(L.wg, w->router_weight, sizeof(float) * Er * d, kind));
    if (w->router_bias) {
        MOE_CUDA_C(dalloc(&L.bias, sizeof(float) * Er, &wb));
        MOE_CUDA_C(cudaMemcpy(L.bias, w->router_bias, sizeof(float) * Er, kind));
    }
    MOE_CUDA_C(dalloc(&L.w13_hi, eb * E * 2 * ffp * d, &wb));
    MOE_CUDA_C(dalloc(&L.w2_hi, eb * E * d * ffp, &wb));
    if (two) {
        MOE_CUDA_C(dalloc(&L.w13_lo, eb * E * 2 * ffp * d, &wb));
        MOE_CUDA_C(dalloc(&L.w2_lo, eb * E * d * ffp, &wb));
    }
    if (fp32_faithful(L)) {
        MOE_CUDA_C(dalloc(&L.w13_f32, 4 * E * 2 * ffp * d, &wb));
        MOE_CUDA_C(dalloc(&L.w2_f32, 4 * E * d * ffp, &wb));
    }
    if (device_ptrs) {
        // The caller's device copies serve directly as the converters' input.
        MOE_CUDA_C(cudaDeviceSynchronize());
        for (int e = 0; e < L.E; ++e) {
            MOE_CUDA_C(convert_gateup(L, e, w->w1[e_first + e], w->w3[e_first + e], s));
            MOE_CUDA_C(convert_down(L, e, w->w2[e_first + e], s));
        }
        MOE_CUDA_C(cudaStreamSynchronize(s));
    } else {
        // Device staging for one expert's three fp32 tensors; with a reader,
        // two pinned host buffers in turn: tensor i is read into buffer
        // i % 2 while the copy of tensor i - 1 runs (event-gated reuse).
        struct Staging {
            float* dev[3] = {};
            float* pin[2] = {};
            cudaEvent_t ev[2] = {};
            ~Staging() {
                for (float* p : dev) if (p) cudaFree(p);
                for (float* p : pin) if (p) cudaFreeHost(p);
                for (cudaEvent_t e : ev) if (e) cudaEventDestroy(e);
            }
        } st;
        const size_t n = ff * d;
        for (float*& p : st.dev) MOE_CUDA_C(dalloc(&p, sizeof(float) * n, nullptr));
        if (reader)
            for (int i = 0; i < 2; ++i) {
                MOE_CUDA_C(cudaHostAlloc(reinterpret_cast<void**>(&st.pin[i]), sizeof(float) * n, 0));
                MOE_CUDA_C(cudaEventCreateWithFlags(&st.ev[i], cudaEventDisableTiming));
            }
        long long issued = 0;
        for (int e = 0; e < L.E; ++e) {
            const float* host[3] = {reader ? nullptr : w->w1[e_first + e],
                                    reader ? nullptr : w->w3[e_first + e],
                                    reader ? nullptr : w->w2[e_first + e]};
            for (int which = 0; which < 3; ++which) {
                const float* src = host[which];
                if (reader) {
                    const int b = static_cast<int>(issued & 1);
                    if (issued >= 2) MOE_CUDA_C(cudaEventSynchronize(st.ev[b]));
                    const int rrc = reader->read(e_first + e, which, st.pin[b], n);
                    if (rrc) {
                        cudaStreamSynchronize(s);
                        return cleanup_and_fail(rrc);
                    }
                    src = st.pin[b];
                }
                MOE_CUDA_C(cudaMemcpyAsync(st.dev[which], src, sizeof(float) * n, kind, s));
                if (reader) MOE_CUDA_C(cudaEventRecord(st.ev[issued & 1], s));
                ++issued;
            }
            MOE_CUDA_C(convert_gateup(L, e, st.dev[0], st.dev[1], s));
            MOE_CUDA_C(convert_down(L, e, st.dev[2], s));
            if (!reader) MOE_CUDA_C(cudaStreamSynchronize(s));
        }
        MOE_CUDA_C(cudaStreamSynchronize(s));
    }
    const uint32_t box_k = kblock_elems(L);
    std::string err;
    const bool bf = planes_bf16(L);
    if (!make_tmap_2d(&L.tm_w13_hi, L.w13_hi, bf, d, E * 2 * ffp, box_k, kTileN, &err) ||
        !make_tmap_2d(&L.tm_w2_hi, L.w2_hi, bf, ffp, E * d, box_k, kTileN, &err))
        return cleanup_and_fail(fail(MOE_ERR_CUDA, err));
    if (two) {
        if (!make_tmap_2d(&L.tm_w13_lo, L.w13_lo, bf, d, E * 2 * ffp, box_k, kTileN, &err) ||
            !make_tmap_2d(&L.tm_w2_lo, L.w2_lo, bf, ffp, E * d, box_k, kTileN, &err))
            return cleanup_and_fail(fail(MOE_ERR_CUDA, err));
    } else {
        L.tm_w13_lo = L.tm_w13_hi;
        L.tm_w2_lo = L.tm_w2_hi;
    }
    if (!make_tmap_2d(&L.tm_w13_hi2, L.w13_hi, bf, d, E * 2 * ffp, box_k, kTileN / 2, &err) ||
        !make_tmap_2d(&L.tm_w2_hi2, L.w2_hi, bf, ffp, E * d, box_k, kTileN / 2, &err))
        return cleanup_and_fail(fail(MOE_ERR_CUDA, err));
    if (two) {
        if (!make_tmap_2d(&L.tm_w13_lo2, L.w13_lo, bf, d, E * 2 * ffp, box_k, kTileN / 2, &err) ||
            !make_tmap_2d(&L.tm_w2_lo2, L.w2_lo, bf, ffp, E * d, box_k, kTileN / 2, &err))
            return cleanup_and_fail(fail(MOE_ERR_CUDA, err));
    } else {
        L.tm_w13_lo2 = L.tm_w13_hi2;
        L.tm_w2_lo2 = L.tm_w2_hi2;
    }
    L.gemm_variant = cfg->gemm_variant;
    rc = ensure_workspace(L, std::max(cfg->max_tokens, 1));
    if (rc) return cleanup_and_fail(rc);
#undef MOE_CUDA_C
    *out = h.release();
    return MOE_OK;
}
}  // namespace moe

extern "C" {

int moe_create_from_model_bin(const MoeConfig* cfg_in, const char* path, int layer_idx,
                              MoeHandle** out) {
    using namespace moe;
    if (!cfg_in || !path || !out) return fail(MOE_ERR_INVALID, "null argument");
    std::unordered_map<std::string, BinEntry> index;
    int rc = read_index(path, &index);
    if (rc) return rc;
    MoeConfig cfg = *cfg_in;
    const std::string base = "model.layers." + std::to_string(layer_idx) + ".block_sparse_moe";
    std::vector<float> gate;
    std::vector<uint64_t> gshape;
    rc = load_tensor(path, index, base + ".gate.weight", &gate, &gshape);
    if (rc) return rc;
    if (gshape.size() != 2) return fail(MOE_ERR_IO, "router weight is not 2-D");
    if (cfg.num_experts == 0) cfg.num_experts = (int)gshape[0];
    if (cfg.d_model == 0) cfg.d_model = (int)gshape[1];
    if ((int)gshape[0] != cfg.num_experts || (int)gshape[1] != cfg.d_model)
        return fail(MOE_ERR_INVALID, "router weight shape does not match the config");
    // Expert tensors: shapes checked from the index now, data streamed from
    // the file one tensor at a time during the upload (ExpertReader).
    std::vector<std::array<const BinEntry*, 3>> ent(cfg.num_experts);
    for (int e = 0; e < cfg.num_experts; ++e) {
        const std::string pre = base + ".experts." + std::to_string(e);
        const char* names[3] = {".w1.weight", ".w3.weight", ".w2.weight"};
        for (int which = 0; which < 3; ++which) {
            auto it = index.find(pre + names[which]);
            if (it == index.end()) return fail(MOE_ERR_IO, "missing tensor: " + pre + names[which]);
            ent[e][which] = &it->second;
        }
        const auto& s1 = ent[e][0]->shape;
        const auto& s3 = ent[e][1]->shape;
        const auto& s2 = ent[e][2]->shape;
        if (s1.size() != 2 || s2.size() != 2 || s3.size() != 2)
            return fail(MOE_ERR_IO, "expert weight is not 2-D");
        if (cfg.d_ff == 0) cfg.d_ff = (int)s1[0];
        if ((int)s1[0] != cfg.d_ff || (int)s1[1] != cfg.d_model || s3 != s1 ||
            (int)s2[0] != cfg.d_model || (int)s2[1] != cfg.d_ff)
            return fail(MOE_ERR_INVALID, "expert weight shapes do not match the config");
        for (int which = 0; which < 3; ++which)
            if (ent[e][which]->bytes != (uint64_t)cfg.d_ff * cfg.d_model * sizeof(float))
                return fail(MOE_ERR_IO, "tensor is not float32: " + pre + names[which]);
    }
    struct FileReader : ExpertReader {
        std::ifstream f;
        const std::vector<std::array<const BinEntry*, 3>>* ent = nullptr;
        int read(int e, int which, float* dst, size_t n) override {
            const BinEntry* be = (*ent)[e][which];
            f.seekg(static_cast<std::streamoff>(be->offset));
            if (!f.read(reinterpret_cast<char*>(dst), static_cast<std::streamsize>(n * 4)))
                return fail(MOE_ERR_IO, "truncated expert tensor of expert " + std::to_string(e));
            return MOE_OK;
        }
    } reader;
    reader.f.open(path, std::ios::binary);
    if (!reader.f) return fail(MOE_ERR_IO, std::string("cannot reopen model: ") + path);
    reader.ent = &ent;
    std::vector<float> bias;
    MoeWeightsHost wh{};
    wh.router_weight = gate.data();
    if (index.count(base + ".gate.bias")) {
        rc = load_tensor(path, index, base + ".gate.bias", &bias, nullptr);
        if (rc) return rc;
        if ((int)bias.size() != cfg.num_experts) return fail(MOE_ERR_IO, "router bias shape");
        wh.router_bias = bias.data();
    }
    // The decoder layer's post-attention LayerNorm, when the file has it.
    const std::string pn = "model.layers." + std::to_string(layer_idx) + ".post_attention_layernorm";
    std::vector<float> nw, nb;
    if (index.count(pn + ".weight") && index.count(pn + ".bias")) {
        if ((rc = load_tensor(path, index, pn + ".weight", &nw, nullptr)) ||
            (rc = load_tensor(path, index, pn + ".bias", &nb, nullptr)))
            return rc;
        if ((int)nw.size() != cfg.d_model || (int)nb.size() != cfg.d_model)
            return fail(MOE_ERR_IO, "post_attention_layernorm shape");
    }
    rc = create_slice(&cfg, &wh, false, 0, cfg.num_experts, out, &reader);
    if (rc || nw.empty()) return rc;
    rc = moe_set_post_norm(*out, nw.data(), nb.data(), 1.0e-5f);
    if (rc) {
        moe_destroy(*out);
        *out = nullptr;
    }
    return rc;
}

void moe_destroy(MoeHandle* h) {
    if (!h) return;
    moe::DeviceGuard guard(h->L.cfg.device);
    cudaDeviceSynchronize();
    Layer& L = h->L;
    if (L.ep) moe::ep_destroy(L);
    moe::free_workspace(L.ws);
    moe::free_ptr(L.wg); moe::free_ptr(L.bias); moe::free_ptr(L.w13_hi); moe::free_ptr(L.w13_lo);
    moe::free_ptr(L.w2_hi); moe::free_ptr(L.w2_lo); moe::free_ptr(L.w13_f32); moe::free_ptr(L.w2_f32);
    moe::free_ptr(L.norm_w); moe::free_ptr(L.norm_b);
    for (cudaEvent_t& e : L.prof_ev)
        if (e) cudaEventDestroy(e);
    for (int c = 0; c < MoeHandle::kMaxChunks; ++c) {
        if (h->in_ev[c]) cudaEventDestroy(h->in_ev[c]);
        if (h->out_ev[c]) cudaEventDestroy(h->out_ev[c]);
    }
    if (h->h2d_stream) cudaStreamDestroy(h->h2d_stream);
    if (h->d2h_stream) cudaStreamDestroy(h->d2h_stream);
    if (h->own_stream) cudaStreamDestroy(h->own_stream);
    delete h;
}

int moe_get_config(const MoeHandle* h, MoeConfig* cfg) {
    if (!h || !cfg) return moe::fail(MOE_ERR_INVALID, "null argument");
    *cfg = h->L.cfg;
    return MOE_OK;
}

size_t moe_device_bytes(const MoeHandle* h) {
    return h ? h->L.weight_bytes + h->L.ws.bytes : 0;
}

int moe_set_decode_max_tokens(MoeHandle* h, int32_t n) {
    if (!h || n < -1 || n > moe::decode_max_supported_tokens())
        return moe::fail(MOE_ERR_INVALID, "decode_max_tokens must be in -1..64");
    h->L.cfg.decode_max_tokens = n < 0 ? moe::auto_decode_max_tokens(h->L.cfg.precision) : n;
    return MOE_OK;
}

int moe_profile_enable(MoeHandle* h, int enable) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    if (enable && !L.prof_ev[0])
        for (cudaEvent_t& e : L.prof_ev) MOE_CUDA(cudaEventCreate(&e));
    L.profile = enable != 0;
    return MOE_OK;
}

int moe_profile_read(MoeHandle* h, float* stage_ms, int32_t n) {
    using namespace moe;
    if (!h || !stage_ms || n < 0) return fail(MOE_ERR_INVALID, "bad argument");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    if (!L.prof_ev[0]) return fail(MOE_ERR_INVALID, "profiling was never enabled");
    for (int i = 0; i < n && i < kProfileStages; ++i) stage_ms[i] = 0.0f;
    if (L.prof_n > 0) MOE_CUDA(cudaEventSynchronize(L.prof_ev[L.prof_n - 1]));
    for (int j = 0; j + 1 < L.prof_n; ++j) {
        const int st = L.prof_stage[j];
        if (st < 0 || st >= n || st >= kProfileStages) continue;
        float ms = 0.0f;
        MOE_CUDA(cudaEventElapsedTime(&ms, L.prof_ev[j], L.prof_ev[j + 1]));
        stage_ms[st] += ms;
    }
    return kProfileStages;
}

int moe_forward_device(MoeHandle* h, const float* x, float* y, int32_t T, void* stream) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    if (T < 0) return fail(MOE_ERR_INVALID, "T < 0");
    if (T == 0) return MOE_OK;
    if (!x || !y) return fail(MOE_ERR_INVALID, "null x or y");
    if (x == y) return fail(MOE_ERR_INVALID, "y must not alias x");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)
        return fail(MOE_ERR_INVALID, "x and y must be 16-byte aligned");
    DeviceGuard guard(h->L.cfg.device);
    return forward_impl(h->L, x, y, T, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace moe {
namespace {
int forward_host_impl(MoeHandle* h, const float* x, float* y, int32_t T, bool block) {
    if (T < 0) return fail(MOE_ERR_INVALID, "T < 0");
    if (T == 0) return MOE_OK;
    if (!x || !y) return fail(MOE_ERR_INVALID, "null x or y");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    int rc = ensure_stage(L, T);
    if (rc) return rc;
    cudaStream_t s = h->own_stream;
    const size_t row = sizeof(float) * (size_t)L.d;
    // Rows are independent, so large batches run as a pipeline of chunks: the
    // copy-in of chunk c + 1 and the copy-out of chunk c - 1 overlap chunk c's
    // compute (and each other: the link is full duplex).  Chunks stay at
    // least 2048 tokens so the grouped GEMMs keep their weight reuse (at
    // config 2, 1024-token chunks made the fp32-faithful e2e slower).
    int nch = T / 2048;
    if (nch > MoeHandle::kMaxChunks) nch = MoeHandle::kMaxChunks;
    if (nch < 2 || !h->h2d_stream) nch = 1;
    if (nch == 1) {
        MOE_CUDA(cudaMemcpyAsync(L.ws.x_stage, x, row * T, cudaMemcpyHostToDevice, s));
        rc = forward_impl(L, L.ws.x_stage, L.ws.y_stage, T, s, block);
        if (rc) return rc;
        MOE_CUDA(cudaMemcpyAsync(y, L.ws.y_stage, row * T, cudaMemcpyDeviceToHost, s));
        MOE_CUDA(cudaStreamSynchronize(s));
        return check_device_errors(L);
    }
    int off = 0;
    for (int c = 0; c < nch; ++c) {
        const int n = (int)((long long)T * (c + 1) / nch) - off;
        const size_t b = row * n, o = (size_t)off * L.d;
        MOE_CUDA(cudaMemcpyAsync(L.ws.x_stage + o, x + o, b, cudaMemcpyHostToDevice, h->h2d_stream));
        MOE_CUDA(cudaEventRecord(h->in_ev[c], h->h2d_stream));
        MOE_CUDA(cudaStreamWaitEvent(s, h->in_ev[c], 0));
        rc = forward_impl(L, L.ws.x_stage + o, L.ws.y_stage + o, n, s, block);
        if (rc) return rc;
        MOE_CUDA(cudaEventRecord(h->out_ev[c], s));
        MOE_CUDA(cudaStreamWaitEvent(h->d2h_stream, h->out_ev[c], 0));
        MOE_CUDA(cudaMemcpyAsync(y + o, L.ws.y_stage + o, b, cudaMemcpyDeviceToHost, h->d2h_stream));
        off += n;
    }
    MOE_CUDA(cudaStreamSynchronize(h->d2h_stream));
    MOE_CUDA(cudaStreamSynchronize(s));
    return check_device_errors(L);
}

int check_block(const MoeHandle* h) {
    if (!h->L.norm_w) return fail(MOE_ERR_INVALID, "no post-attention norm attached (moe_set_post_norm)");
    return MOE_OK;
}
}  // namespace
}  // namespace moe

extern "C" {

int moe_forward_host(MoeHandle* h, const float* x, float* y, int32_t T) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    return forward_host_impl(h, x, y, T, false);
}

int moe_block_forward_host(MoeHandle* h, const float* attn, float* y, int32_t T) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    if (int rc = check_block(h)) return rc;
    return forward_host_impl(h, attn, y, T, true);
}

int moe_block_forward_device(MoeHandle* h, const float* attn, float* y, int32_t T, void* stream) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    if (int rc = check_block(h)) return rc;
    if (T < 0) return fail(MOE_ERR_INVALID, "T < 0");
    if (T == 0) return MOE_OK;
    if (!attn || !y) return fail(MOE_ERR_INVALID, "null attn or y");
    if (attn == y) return fail(MOE_ERR_INVALID, "y must not alias attn");
    if ((reinterpret_cast<uintptr_t>(attn) | reinterpret_cast<uintptr_t>(y)) & 15)
        return fail(MOE_ERR_INVALID, "attn and y must be 16-byte aligned");
    DeviceGuard guard(h->L.cfg.device);
    return forward_impl(h->L, attn, y, T, static_cast<cudaStream_t>(stream), true);
}

int moe_set_post_norm(MoeHandle* h, const float* weight, const float* bias, float eps) {
    using namespace moe;
    if (!h || !weight || !bias) return fail(MOE_ERR_INVALID, "null argument");
    if (!(eps >= 0.0f)) return fail(MOE_ERR_INVALID, "eps must be >= 0");
    if (!norm_supported(h->L.d))
        return fail(MOE_ERR_UNSUPPORTED, "the fused LayerNorm needs d_model a multiple of 128");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    const size_t bytes = sizeof(float) * L.d;
    if (!L.norm_w) {
        MOE_CUDA(dalloc(&L.norm_w, bytes, &L.weight_bytes));
        MOE_CUDA(dalloc(&L.norm_b, bytes, &L.weight_bytes));
    }
    MOE_CUDA(cudaDeviceSynchronize());   // no forward may still read the old values
    MOE_CUDA(cudaMemcpy(L.norm_w, weight, bytes, cudaMemcpyHostToDevice));
    MOE_CUDA(cudaMemcpy(L.norm_b, bias, bytes, cudaMemcpyHostToDevice));
    L.norm_eps = eps;
    L.norm_rms = false;
    return MOE_OK;
}

int moe_set_post_rms_norm(MoeHandle* h, const float* weight, float eps) {
    using namespace moe;
    if (!h || !weight) return fail(MOE_ERR_INVALID, "null argument");
    if (!(eps >= 0.0f)) return fail(MOE_ERR_INVALID, "eps must be >= 0");
    if (!norm_supported(h->L.d))
        return fail(MOE_ERR_UNSUPPORTED, "the fused norm needs d_model a multiple of 128");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    const size_t bytes = sizeof(float) * L.d;
    if (!L.norm_w) {
        MOE_CUDA(dalloc(&L.norm_w, bytes, &L.weight_bytes));
        MOE_CUDA(dalloc(&L.norm_b, bytes, &L.weight_bytes));
    }
    MOE_CUDA(cudaDeviceSynchronize());   // no forward may still read the old values
    MOE_CUDA(cudaMemcpy(L.norm_w, weight, bytes, cudaMemcpyDefault));
    MOE_CUDA(cudaMemset(L.norm_b, 0, bytes));
    L.norm_eps = eps;
    L.norm_rms = true;
    return MOE_OK;
}

int moe_layer_norm_device(const float* x, const float* weight, const float* bias, float eps,
                          int32_t rows, int32_t cols, float* y, void* stream) {
    using namespace moe;
    if (rows < 0 || !norm_supported(cols))
        return fail(MOE_ERR_INVALID, "rows >= 0 and cols a positive multiple of 128 required");
    if (rows == 0) return MOE_OK;
    if (!x || !weight || !bias || !y) return fail(MOE_ERR_INVALID, "null argument");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
         reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(bias)) & 15)
        return fail(MOE_ERR_INVALID, "pointers must be 16-byte aligned");
    if (!(eps >= 0.0f)) return fail(MOE_ERR_INVALID, "eps must be >= 0");
    MOE_CUDA(launch_layer_norm(x, rows, cols, eps, weight, bias, y,
                               static_cast<cudaStream_t>(stream)));
    return MOE_OK;
}

int moe_route_device(MoeHandle* h, const float* x, int32_t T, float* logits, int32_t* idx,
                     float* weights, void* stream) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    if (T < 0) return fail(MOE_ERR_INVALID, "T < 0");
    if (T == 0) return MOE_OK;
    if (!x || !idx || !weights) return fail(MOE_ERR_INVALID, "null argument");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    int rc = ensure_workspace(L, T);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    L.last_stream = s;
    L.last_T = T;
    MOE_CUDA(launch_router(L, x, T, logits, idx, weights, L.ws.blockhist, s));
    // The scan reads the histogram the router just wrote, so counts and the
    // layout queries below describe this call.
    MOE_CUDA(launch_dispatch_scan(L, T, s));
    return MOE_OK;
}

int moe_route_host(MoeHandle* h, const float* x, int32_t T, float* logits, int32_t* idx,
                   float* weights) {
    using namespace moe;
    if (!h) return fail(MOE_ERR_INVALID, "null handle");
    if (T < 0) return fail(MOE_ERR_INVALID, "T < 0");
    if (T == 0) return MOE_OK;
    if (!x || !idx || !weights) return fail(MOE_ERR_INVALID, "null argument");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    int rc = ensure_stage(L, T);
    if (rc) return rc;
    cudaStream_t s = h->own_stream;
    Workspace& W = L.ws;
    MOE_CUDA(cudaMemcpyAsync(W.x_stage, x, sizeof(float) * (size_t)T * L.d, cudaMemcpyHostToDevice, s));
    L.last_stream = s;
    L.last_T = T;
    MOE_CUDA(launch_router(L, W.x_stage, T, W.logits, W.idx, W.wts, W.blockhist, s));
    MOE_CUDA(launch_dispatch_scan(L, T, s));
    if (logits)
        MOE_CUDA(cudaMemcpyAsync(logits, W.logits, sizeof(float) * (size_t)T * L.E,
                                 cudaMemcpyDeviceToHost, s));
    MOE_CUDA(cudaMemcpyAsync(idx, W.idx, sizeof(int) * (size_t)T * L.k, cudaMemcpyDeviceToHost, s));
    MOE_CUDA(cudaMemcpyAsync(weights, W.wts, sizeof(float) * (size_t)T * L.k,
                             cudaMemcpyDeviceToHost, s));
    MOE_CUDA(cudaStreamSynchronize(s));
    return check_device_errors(L);
}

int moe_selftest_wait_timeout(int device, int32_t budget_us) {
    using namespace moe;
    if (budget_us < 1 || budget_us > 2000000) return fail(MOE_ERR_INVALID, "budget_us out of range");
    int ndev = 0;
    MOE_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(MOE_ERR_INVALID, "no such device");
    DeviceGuard guard(device);
    int* flag = nullptr;
    MOE_CUDA(cudaMalloc(&flag, sizeof(int)));
    MOE_CUDA(cudaMemset(flag, 0, sizeof(int)));
    cudaError_t e = launch_selftest_wait(flag, (unsigned long long)budget_us * 1000ull);
    int h_flag = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h_flag, flag, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(flag);
    if (e != cudaSuccess) return cuda_fail(e, "selftest kernel");
    if (h_flag & kDevErrTimeoutSelftest) {
        char buf[96];
        std::snprintf(buf, sizeof buf, "a device-side wait timed out (flags 0x%x)", h_flag);
        return fail(MOE_ERR_TIMEOUT, buf);
    }
    return fail(MOE_ERR_CUDA, "selftest: the wait that nothing completes did not time out");
}

int moe_host_alloc(size_t bytes, void** out) {
    using namespace moe;
    if (!out) return fail(MOE_ERR_INVALID, "null argument");
    *out = nullptr;
    cudaError_t e = cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocDefault);
    if (e != cudaSuccess) return fail(MOE_ERR_OOM, std::string("cudaHostAlloc: ") + cudaGetErrorString(e));
    return MOE_OK;
}

int moe_host_free(void* p) {
    using namespace moe;
    if (!p) return MOE_OK;
    MOE_CUDA(cudaFreeHost(p));
    return MOE_OK;
}

int moe_expert_counts(MoeHandle* h, int32_t* counts) {
    using namespace moe;
    if (!h || !counts) return fail(MOE_ERR_INVALID, "null argument");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    MOE_CUDA(cudaStreamSynchronize(L.last_stream));
    MOE_CUDA(cudaMemcpy(counts, L.ws.counts, sizeof(int) * L.E, cudaMemcpyDeviceToHost));
    return check_device_errors(L);
}

int moe_dispatch_layout(MoeHandle* h, int32_t* row_token, float* row_weight, int32_t rows_cap,
                        int32_t* rows_out, int32_t* expert_offsets) {
    using namespace moe;
    if (!h || !rows_out) return fail(MOE_ERR_INVALID, "null argument");
    DeviceGuard guard(h->L.cfg.device);
    Layer& L = h->L;
    MOE_CUDA(cudaStreamSynchronize(L.last_stream));
    std::vector<int> eoff(L.E + 1);
    MOE_CUDA(cudaMemcpy(eoff.data(), L.ws.eoff, sizeof(int) * (L.E + 1), cudaMemcpyDeviceToHost));
    const int rows = eoff[L.E];
    *rows_out = rows;
    if (expert_offsets) std::copy(eoff.begin(), eoff.end(), expert_offsets);
    if (rows > rows_cap) return fail(MOE_ERR_INVALID, "rows_cap is smaller than the packed rows");
    if (row_token)
        MOE_CUDA(cudaMemcpy(row_token, L.ws.row_token, sizeof(int) * rows, cudaMemcpyDeviceToHost));
    if (row_weight)
        MOE_CUDA(cudaMemcpy(row_weight, L.ws.row_weight, sizeof(float) * rows,
                            cudaMemcpyDeviceToHost));
    return check_device_errors(L);
}

}  // extern "C"
