// MoE layer classes of the drop-in (include/layer.h) over the C ABI.
#include "layer.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <vector>
#include <stdexcept>
#include <string>

namespace {

[[noreturn]] void throw_status(int rc, const char* what) {
    const std::string msg = std::string(what) + ": " + moe_last_error();
    if (rc == MOE_ERR_INVALID) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

std::shared_ptr<MoeHandle> make_handle(const MoeConfig& cfg, const Tensor& gate,
                                       const Tensor* bias, const std::vector<Tensor>& w1,
                                       const std::vector<Tensor>& w3,
                                       const std::vector<Tensor>& w2) {
    std::vector<const float*> p1, p2, p3;
    for (std::size_t e = 0; e < w1.size(); ++e) {
        p1.push_back(w1[e].data());
        p2.push_back(w2[e].data());
        p3.push_back(w3[e].data());
    }
    MoeWeightsHost w{};
    w.router_weight = gate.data();
    w.router_bias = bias ? bias->data() : nullptr;
    w.w1 = p1.data();
    w.w2 = p2.data();
    w.w3 = p3.data();
    MoeHandle* h = nullptr;
    const int rc = moe_create(&cfg, &w, &h);
    if (rc != MOE_OK) throw_status(rc, "moe_create");
    return std::shared_ptr<MoeHandle>(h, moe_destroy);
}

void check_2d(const Tensor& x, std::size_t d) {
    if (x.ndim() != 2 || x.size(1) != d) throw std::invalid_argument("MoE input shape");
}

}  // namespace

// ---------------------------------------------------------------- Linear
Linear::Linear(const ModelLoader& loader, const std::string& weight, const std::string& bias)
    : weight_(loader.load(weight)) {
    if (!bias.empty() && loader.has(bias)) bias_ = loader.load(bias);
}

void Linear::forward(const Tensor& x, Tensor& y) const {
    const std::size_t in = x.size(x.ndim() - 1), rows = x.size() / in;
    Tensor flat = x;
    flat.reshape({rows, in});
    y = Tensor({rows, weight_.size(0)});
    tensor_ops::matmul_transposed(flat, weight_, y);
    if (bias_.size()) tensor_ops::add_bias_inplace(y, bias_);
}

// ---------------------------------------------------------------- PhiMLP
// One expert is a layer with a single expert, top-1 softmax routing and an
// all-zero router: every token goes to expert 0 with weight exactly 1.
PhiMLP::PhiMLP(const ModelLoader& loader, const std::string& prefix, int precision, int device) {
    std::vector<Tensor> w1, w2, w3;
    w1.push_back(loader.load(prefix + ".w1.weight"));
    w2.push_back(loader.load(prefix + ".w2.weight"));
    w3.push_back(loader.load(prefix + ".w3.weight"));
    d_ = w1[0].size(1);
    MoeConfig cfg;
    moe_config_init(&cfg);
    cfg.d_model = static_cast<int32_t>(d_);
    cfg.d_ff = static_cast<int32_t>(w1[0].size(0));
    cfg.num_experts = 1;
    cfg.top_k = 1;
    cfg.router_policy = MOE_ROUTER_SOFTMAX_TOPK;
    cfg.precision = precision;
    cfg.device = device;
    Tensor gate({1, d_});
    h_ = make_handle(cfg, gate, nullptr, w1, w3, w2);
}

void PhiMLP::forward(const Tensor& x, Tensor& y) const {
    const std::size_t rows = x.size() / x.size(x.ndim() - 1);
    if (x.size(x.ndim() - 1) != d_) throw std::invalid_argument("PhiMLP input shape");
    Tensor out(x.shape());
    const int rc = moe_forward_host(h_.get(), x.data(), out.data(), static_cast<int32_t>(rows));
    if (rc != MOE_OK) throw_status(rc, "PhiMLP::forward");
    y = std::move(out);
}

// ---------------------------------------------------------------- PhiMoE
namespace {
MoeConfig reference_config() {
    MoeConfig c;
    moe_config_init(&c);
    c.d_model = c.d_ff = c.num_experts = 0;  // taken from the file
    return c;
}
}  // namespace

PhiMoE::PhiMoE(const ModelLoader& loader, std::size_t layer_idx)
    : PhiMoE(loader, layer_idx, reference_config()) {}

namespace {

// The MoE layer `layer_idx` of a model file (src/layer.cu:73-77 names).
std::shared_ptr<MoeHandle> load_moe(const ModelLoader& loader, std::size_t layer_idx,
                                    const MoeConfig& cfg_in) {
    const std::string base = "model.layers." + std::to_string(layer_idx) + ".block_sparse_moe";
    Tensor gate = loader.load(base + ".gate.weight");
    if (gate.ndim() != 2) throw std::runtime_error("router weight is not 2-D: " + base);
    MoeConfig cfg = cfg_in;
    if (cfg.num_experts == 0) {
        int e = 0;
        while (loader.has(base + ".experts." + std::to_string(e) + ".w1.weight")) ++e;
        cfg.num_experts = e;
    }
    if (cfg.d_model == 0) cfg.d_model = static_cast<int32_t>(gate.size(1));
    std::vector<Tensor> w1, w2, w3;
    for (int e = 0; e < cfg.num_experts; ++e) {
        const std::string pre = base + ".experts." + std::to_string(e);
        w1.push_back(loader.load(pre + ".w1.weight"));
        w2.push_back(loader.load(pre + ".w2.weight"));
        w3.push_back(loader.load(pre + ".w3.weight"));
    }
    if (cfg.d_ff == 0 && !w1.empty()) cfg.d_ff = static_cast<int32_t>(w1[0].size(0));
    Tensor bias;
    const bool has_bias = loader.has(base + ".gate.bias");
    if (has_bias) bias = loader.load(base + ".gate.bias");
    return make_handle(cfg, gate, has_bias ? &bias : nullptr, w1, w3, w2);
}

}  // namespace

PhiMoE::PhiMoE(const ModelLoader& loader, std::size_t layer_idx, const MoeConfig& cfg_in)
    : h_(load_moe(loader, layer_idx, cfg_in)) {
    moe_get_config(h_.get(), &cfg_);
}

void PhiMoE::forward(const Tensor& x, Tensor& y) const {
    check_2d(x, static_cast<std::size_t>(cfg_.d_model));
    Tensor out({x.size(0), x.size(1)});
    const int rc = moe_forward_host(h_.get(), x.data(), out.data(), static_cast<int32_t>(x.size(0)));
    if (rc != MOE_OK) throw_status(rc, "PhiMoE::forward");
    y = std::move(out);
}

void PhiMoE::forward_device(const float* x_dev, float* y_dev, std::size_t rows, void* stream) const {
    const int rc = moe_forward_device(h_.get(), x_dev, y_dev, static_cast<int32_t>(rows), stream);
    if (rc != MOE_OK) throw_status(rc, "PhiMoE::forward_device");
}

void PhiMoE::route(const Tensor& x, std::vector<std::pair<int, float>>& routes) const {
    check_2d(x, static_cast<std::size_t>(cfg_.d_model));
    const std::size_t rows = x.size(0), k = static_cast<std::size_t>(cfg_.top_k);
    std::vector<int32_t> idx(rows * k);
    std::vector<float> w(rows * k);
    const int rc = moe_route_host(h_.get(), x.data(), static_cast<int32_t>(rows), nullptr,
                                  idx.data(), w.data());
    if (rc != MOE_OK) throw_status(rc, "PhiMoE::route");
    routes.clear();
    for (std::size_t i = 0; i < rows * k; ++i) routes.emplace_back(idx[i], w[i]);
}

// ---------------------------------------------------------------- PhiMoEBlock
PhiMoEBlock::PhiMoEBlock(const ModelLoader& loader, std::size_t layer_idx)
    : PhiMoEBlock(loader, layer_idx, reference_config()) {}

PhiMoEBlock::PhiMoEBlock(const ModelLoader& loader, std::size_t layer_idx, const MoeConfig& cfg)
    : h_(load_moe(loader, layer_idx, cfg)) {
    moe_get_config(h_.get(), &cfg_);
    const std::string pn =
        "model.layers." + std::to_string(layer_idx) + ".post_attention_layernorm";
    const Tensor w = loader.load(pn + ".weight");
    const Tensor b = loader.load(pn + ".bias");
    if (w.size() != static_cast<std::size_t>(cfg_.d_model) || b.size() != w.size())
        throw std::runtime_error("post_attention_layernorm shape: " + pn);
    const int rc = moe_set_post_norm(h_.get(), w.data(), b.data(), 1.0e-5f);
    if (rc != MOE_OK) throw_status(rc, "moe_set_post_norm");
}

void PhiMoEBlock::forward(const Tensor& attn, Tensor& y) const {
    check_2d(attn, static_cast<std::size_t>(cfg_.d_model));
    Tensor out({attn.size(0), attn.size(1)});
    const int rc = moe_block_forward_host(h_.get(), attn.data(), out.data(),
                                          static_cast<int32_t>(attn.size(0)));
    if (rc != MOE_OK) throw_status(rc, "PhiMoEBlock::forward");
    y = std::move(out);
}

void PhiMoEBlock::forward_device(const float* attn_dev, float* y_dev, std::size_t rows,
                                 void* stream) const {
    const int rc = moe_block_forward_device(h_.get(), attn_dev, y_dev, static_cast<int32_t>(rows),
                                            stream);
    if (rc != MOE_OK) throw_status(rc, "PhiMoEBlock::forward_device");
}

// ---------------------------------------------------------------- PhiAttention
namespace {

std::string attn_name(std::size_t layer_idx, const char* proj, const char* what) {
    return "model.layers." + std::to_string(layer_idx) + ".self_attn." + proj + "." + what;
}

}  // namespace

PhiAttention::PhiAttention(const ModelLoader& loader, std::size_t layer_idx)
    : PhiAttention(loader, layer_idx, PhiAttentionGeometry{}) {}

PhiAttention::PhiAttention(const ModelLoader& loader, std::size_t layer_idx,
                           const PhiAttentionGeometry& g)
    : q_proj_(loader, attn_name(layer_idx, "q_proj", "weight"), attn_name(layer_idx, "q_proj", "bias")),
      k_proj_(loader, attn_name(layer_idx, "k_proj", "weight"), attn_name(layer_idx, "k_proj", "bias")),
      v_proj_(loader, attn_name(layer_idx, "v_proj", "weight"), attn_name(layer_idx, "v_proj", "bias")),
      o_proj_(loader, attn_name(layer_idx, "o_proj", "weight"), attn_name(layer_idx, "o_proj", "bias")),
      g_(g) {
    if (g_.heads == 0 || g_.kv_heads == 0 || g_.heads % g_.kv_heads || g_.head_dim % 2)
        throw std::invalid_argument("PhiAttention geometry");
}

// Causal attention with the reference's arithmetic per score (a
// d-ascending fused multiply-add chain, scaled by 1/sqrt(head_dim) in
// float), its max-subtracted exp in double, its running denominator and its
// probability-times-value chain; scores are computed once per (query, key)
// rather than three times, with the same values.
void PhiAttention::forward(const Tensor& x, Tensor& y) const {
    const std::size_t S = x.size(0);
    const std::size_t H = g_.heads, KVH = g_.kv_heads, hd = g_.head_dim;
    Tensor q, k, v;
    q_proj_.forward(x, q);
    k_proj_.forward(x, k);
    v_proj_.forward(x, v);
    if (q.size(1) != H * hd || k.size(1) != KVH * hd || v.size(1) != KVH * hd)
        throw std::invalid_argument("PhiAttention: projection widths do not match the geometry");
    tensor_ops::apply_rope(q, k, S, H, KVH, hd, g_.rope_theta);
    Tensor out({S, H * hd});
    const std::size_t group = H / KVH;
    const float scale = std::sqrt(static_cast<float>(hd));
    const float* Q = q.data();
    const float* K = k.data();
    const float* V = v.data();
    float* O = out.data();
    const std::size_t qw = H * hd, kw = KVH * hd;
#pragma omp parallel for
    for (long long w = 0; w < static_cast<long long>(S * H); ++w) {
        const std::size_t qi = static_cast<std::size_t>(w) / H, qh = static_cast<std::size_t>(w) % H;
        const std::size_t kh = qh / group;
        const std::size_t k0 = qi + 1 > g_.sliding_window ? qi + 1 - g_.sliding_window : 0;
        std::vector<float> sc(qi + 1 - k0);
        float maxv = -std::numeric_limits<float>::infinity();
        for (std::size_t ki = k0; ki <= qi; ++ki) {
            const float* qr = Q + qi * qw + qh * hd;
            const float* kr = K + ki * kw + kh * hd;
            float s = 0.0f;
            for (std::size_t d = 0; d < hd; ++d) s = std::fma(qr[d], kr[d], s);
            sc[ki - k0] = s / scale;
            maxv = std::max(maxv, sc[ki - k0]);
        }
        float denom = 0.0f;
        for (float& s : sc) {
            s = static_cast<float>(std::exp(static_cast<double>(s - maxv)));
            denom += s;
        }
        for (std::size_t d = 0; d < hd; ++d) {
            float value = 0.0f;
            for (std::size_t ki = k0; ki <= qi; ++ki)
                value = std::fma(sc[ki - k0] / denom, V[ki * kw + kh * hd + d], value);
            O[qi * qw + qh * hd + d] = value;
        }
    }
    o_proj_.forward(out, y);
}

// ---------------------------------------------------------------- PhiDecoderLayer
PhiDecoderLayer::PhiDecoderLayer(const ModelLoader& loader, std::size_t layer_idx)
    : PhiDecoderLayer(loader, layer_idx, PhiAttentionGeometry{}, reference_config()) {}

PhiDecoderLayer::PhiDecoderLayer(const ModelLoader& loader, std::size_t layer_idx,
                                 const PhiAttentionGeometry& g, const MoeConfig& moe_cfg)
    : input_norm_weight_(loader.load("model.layers." + std::to_string(layer_idx) +
                                     ".input_layernorm.weight")),
      input_norm_bias_(loader.load("model.layers." + std::to_string(layer_idx) +
                                   ".input_layernorm.bias")),
      attention_(loader, layer_idx, g),
      moe_(loader, layer_idx, moe_cfg),
      eps_(g.norm_eps) {}

void PhiDecoderLayer::forward(const Tensor& x, Tensor& y) const {
    Tensor normed(x.shape()), attn;
    tensor_ops::layer_norm(x, input_norm_weight_, input_norm_bias_, eps_, normed);
    attention_.forward(normed, attn);
    tensor_ops::add_inplace(attn, x);
    moe_.forward(attn, y);
}
