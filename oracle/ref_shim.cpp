// TEST INFRASTRUCTURE ONLY.
//
// A C entry layer over the reference's own host MoE classes, compiled from
// the reference sources where they lie (src/tensor.cu, src/layer.cu,
// src/model_loader.cu) by oracle/Makefile into oracle/_ref/libref_e<E>.so,
// one library per expert count because the reference fixes NUM_EXPERTS at
// compile time (include/config.h:13).  Tests use it to pin the CPU
// restatement in moe_oracle.c; bench.py's reference arm times it.
//
// PhiMoE::route is private in the reference (include/layer.h:35); the test
// shim opens it so the reference's own routing decisions can be compared
// token by token.  Nothing else in the reference is changed.
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <fstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

// Standard headers come first so the access override below reaches only the
// reference's own headers.
#define private public
#include "tensor.h"
#include "model_loader.h"
#include "layer.h"
#undef private

namespace {
thread_local std::string g_err;

struct RefMoe {
    ModelLoader loader;
    PhiMoE moe;
    RefMoe(const char* path, std::size_t layer) : loader(path), moe(loader, layer) {}
};

int fail(const std::exception& e) {
    g_err = e.what();
    return -1;
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_num_experts() { return static_cast<int>(apss26::NUM_EXPERTS); }

int ref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

void* ref_moe_create(const char* model_bin, int layer_idx) {
    try {
        return new RefMoe(model_bin, static_cast<std::size_t>(layer_idx));
    } catch (const std::exception& e) {
        fail(e);
        return nullptr;
    }
}

void ref_moe_destroy(void* h) { delete static_cast<RefMoe*>(h); }

// y[T][d] = PhiMoE::forward(x[T][d])  (src/layer.cu:80-103).
int ref_moe_forward(void* h, const float* x, int T, int d, float* y) {
    try {
        auto* r = static_cast<RefMoe*>(h);
        Tensor xt({static_cast<std::size_t>(T), static_cast<std::size_t>(d)});
        std::memcpy(xt.data(), x, sizeof(float) * static_cast<std::size_t>(T) * d);
        Tensor yt;
        r->moe.forward(xt, yt);
        if (yt.size() != static_cast<std::size_t>(T) * d) {
            g_err = "reference output has an unexpected size";
            return -1;
        }
        std::memcpy(y, yt.data(), sizeof(float) * yt.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// logits[T][E] = x . gate^T, then the reference route per token
// (src/layer.cu:84, 47-70).  idx/w are [T][2] in selection order.
int ref_moe_route(void* h, const float* x, int T, int d, float* logits, int* idx, float* w) {
    try {
        auto* r = static_cast<RefMoe*>(h);
        const std::size_t E = apss26::NUM_EXPERTS;
        Tensor xt({static_cast<std::size_t>(T), static_cast<std::size_t>(d)});
        std::memcpy(xt.data(), x, sizeof(float) * static_cast<std::size_t>(T) * d);
        Tensor router({static_cast<std::size_t>(T), E});
        tensor_ops::matmul_transposed(xt, r->moe.gate_, router);
        std::memcpy(logits, router.data(), sizeof(float) * router.size());
        for (int t = 0; t < T; ++t) {
            Tensor one({E});
            for (std::size_t e = 0; e < E; ++e) one[e] = router.at(t, e);
            std::vector<std::pair<int, float>> routes;
            r->moe.route(one, routes);
            for (int s = 0; s < 2; ++s) {
                idx[2 * t + s] = routes[s].first;
                w[2 * t + s] = routes[s].second;
            }
        }
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// tensor_ops::layer_norm on raw buffers (src/tensor.cu:174-189).
int ref_layer_norm(const float* x, const float* w, const float* b, float eps, int T, int d,
                   float* y) {
    try {
        Tensor xt({static_cast<std::size_t>(T), static_cast<std::size_t>(d)});
        Tensor wt({static_cast<std::size_t>(d)}), bt({static_cast<std::size_t>(d)});
        Tensor yt({static_cast<std::size_t>(T), static_cast<std::size_t>(d)});
        std::memcpy(xt.data(), x, sizeof(float) * xt.size());
        std::memcpy(wt.data(), w, sizeof(float) * wt.size());
        std::memcpy(bt.data(), b, sizeof(float) * bt.size());
        tensor_ops::layer_norm(xt, wt, bt, eps, yt);
        std::memcpy(y, yt.data(), sizeof(float) * yt.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// tensor_ops::matmul_transposed on raw buffers (src/tensor.cu:136-148).
int ref_matmul_transposed(const float* a, const float* b, float* c, int m, int k, int n) {
    try {
        Tensor at({static_cast<std::size_t>(m), static_cast<std::size_t>(k)});
        Tensor bt({static_cast<std::size_t>(n), static_cast<std::size_t>(k)});
        Tensor ct({static_cast<std::size_t>(m), static_cast<std::size_t>(n)});
        std::memcpy(at.data(), a, sizeof(float) * at.size());
        std::memcpy(bt.data(), b, sizeof(float) * bt.size());
        tensor_ops::matmul_transposed(at, bt, ct);
        std::memcpy(c, ct.data(), sizeof(float) * ct.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// tensor_ops::apply_rope on raw buffers (src/tensor.cu:191-210): q [seq][q_heads *
// head_dim] and k [seq][kv_heads * head_dim] rotated in place, position = row.
int ref_apply_rope(float* q, float* k, int seq, int q_heads, int kv_heads, int head_dim,
                   float theta) {
    try {
        const std::size_t S = static_cast<std::size_t>(seq), hd = static_cast<std::size_t>(head_dim);
        Tensor qt({S, static_cast<std::size_t>(q_heads) * hd});
        Tensor kt({S, static_cast<std::size_t>(kv_heads) * hd});
        std::memcpy(qt.data(), q, sizeof(float) * qt.size());
        std::memcpy(kt.data(), k, sizeof(float) * kt.size());
        tensor_ops::apply_rope(qt, kt, S, static_cast<std::size_t>(q_heads),
                               static_cast<std::size_t>(kv_heads), hd, theta);
        std::memcpy(q, qt.data(), sizeof(float) * qt.size());
        std::memcpy(k, kt.data(), sizeof(float) * kt.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

// PhiAttention::forward (src/layer.cu:110-147) of layer `layer` of a
// model.bin: x [S][d] -> y [S][heads * head_dim projected by o_proj], with the
// heads, head_dim, sliding window and RoPE base of this build's config.h.
int ref_attention(const char* model_bin, int layer, const float* x, int S, int d, float* y,
                  int y_cols) {
    try {
        ModelLoader loader(model_bin);
        PhiAttention att(loader, static_cast<std::size_t>(layer));
        Tensor xt({static_cast<std::size_t>(S), static_cast<std::size_t>(d)}), yt;
        std::memcpy(xt.data(), x, sizeof(float) * xt.size());
        att.forward(xt, yt);
        if (yt.size() != static_cast<std::size_t>(S) * static_cast<std::size_t>(y_cols))
            throw std::invalid_argument("ref_attention: unexpected output size");
        std::memcpy(y, yt.data(), sizeof(float) * yt.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

int ref_attention_heads() { return static_cast<int>(apss26::NUM_ATTENTION_HEADS); }

// PhiDecoderLayer::forward (src/layer.cu:152-162) of layer `layer` of a
// model.bin: x [S][d] -> y [S][d] (input LayerNorm, attention, residual,
// post-attention LayerNorm, PhiMoE, residual), with this build's config.h.
int ref_decoder_layer(const char* model_bin, int layer, const float* x, int S, int d, float* y) {
    try {
        ModelLoader loader(model_bin);
        PhiDecoderLayer dl(loader, static_cast<std::size_t>(layer));
        Tensor xt({static_cast<std::size_t>(S), static_cast<std::size_t>(d)}), yt;
        std::memcpy(xt.data(), x, sizeof(float) * xt.size());
        dl.forward(xt, yt);
        if (yt.size() != xt.size()) throw std::invalid_argument("ref_decoder_layer: output size");
        std::memcpy(y, yt.data(), sizeof(float) * yt.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(e);
    }
}

}  // extern "C"
