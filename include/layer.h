// layer.h -- the MoE layer classes of the drop-in, over libmoe_b200.so.
//
// Mirrors the reference's include/layer.h:11-36 (songsnim/accelerating-MoE-
// inference) for the MoE hot path:
//   Linear   y = x W^T (+ b)                    host, reference arithmetic
//   PhiMLP   SwiGLU expert, src/layer.cu:32-45  on the GPU (a 1-expert layer)
//   PhiMoE   router + experts + combine,        on the GPU
//            src/layer.cu:80-103
// Constructors take the same (ModelLoader, index / prefix) arguments and load
// the same tensor names; forward(const Tensor& x, Tensor& y) allocates y like
// the reference does.  Errors keep the reference's exception types:
// std::invalid_argument for shape mismatches, std::runtime_error for I/O and
// device failures (carrying moe_last_error()).
//
//   PhiMoEBlock  the MoE half of PhiDecoderLayer::forward (src/layer.cu:
//            157-161): post-attention LayerNorm, PhiMoE, residual add, on the
//            GPU with the norm fused into the MoE's input
//   PhiAttention  src/layer.cu:105-147 on the host, with the reference's
//            arithmetic (the attention is not on this library's GPU path)
//   PhiDecoderLayer  src/layer.cu:149-162: input LayerNorm and attention on
//            the host, then PhiMoEBlock on the GPU
//
// Layers share their device handle between copies; a handle runs one forward
// at a time, so copies must not run forward concurrently.
#pragma once

#include "model_loader.h"
#include "moe_b200.h"
#include "tensor.h"

#include <cstddef>
#include <memory>
#include <string>
#include <utility>
#include <vector>

class Linear {
public:
    Linear() = default;
    Linear(const ModelLoader& loader, const std::string& weight, const std::string& bias = "");
    void forward(const Tensor& x, Tensor& y) const;

private:
    Tensor weight_;
    Tensor bias_;
};

class PhiMLP {
public:
    PhiMLP(const ModelLoader& loader, const std::string& prefix, int precision = MOE_PREC_FP32,
           int device = 0);
    void forward(const Tensor& x, Tensor& y) const;

private:
    std::shared_ptr<MoeHandle> h_;
    std::size_t d_ = 0;
};

class PhiMoE {
public:
    // The reference's configuration: its quantised top-2 router
    // (include/config.h:13-23), expert count and sizes taken from the file,
    // fp32-faithful expert arithmetic.
    PhiMoE(const ModelLoader& loader, std::size_t layer_idx);
    // Any configuration; zero d_model / d_ff / num_experts come from the file.
    PhiMoE(const ModelLoader& loader, std::size_t layer_idx, const MoeConfig& cfg);

    void forward(const Tensor& x, Tensor& y) const;
    // Device-resident variant for an engine that keeps activations on the GPU
    // (the reference's DeviceMoE segment, src/model.cu:1976-2019).
    void forward_device(const float* x_dev, float* y_dev, std::size_t rows,
                        void* stream = nullptr) const;
    // Expert indices / weights [rows][top_k] of x (host), in selection order.
    void route(const Tensor& x, std::vector<std::pair<int, float>>& routes) const;

    const MoeConfig& config() const { return cfg_; }

private:
    std::shared_ptr<MoeHandle> h_;
    MoeConfig cfg_{};
};

// y = attn + PhiMoE(layer_norm(attn)) with the layer's
// post_attention_layernorm.{weight,bias} and NORM_EPS 1e-5 (include/config.h:
// 19).  In PhiDecoderLayer::forward this replaces
//     layer_norm(attn, post_norm_weight_, post_norm_bias_, NORM_EPS, post);
//     moe_.forward(post, ff);  add_inplace(ff, attn);  y = std::move(ff);
class PhiMoEBlock {
public:
    PhiMoEBlock(const ModelLoader& loader, std::size_t layer_idx);
    PhiMoEBlock(const ModelLoader& loader, std::size_t layer_idx, const MoeConfig& cfg);

    void forward(const Tensor& attn, Tensor& y) const;
    void forward_device(const float* attn_dev, float* y_dev, std::size_t rows,
                        void* stream = nullptr) const;

    const MoeConfig& config() const { return cfg_; }

private:
    std::shared_ptr<MoeHandle> h_;
    MoeConfig cfg_{};
};

// Attention geometry.  The defaults are the reference's constants
// (include/config.h:10-19: 16 query heads, 4 KV heads of 128, sliding window
// 2047, RoPE base 1e4, LayerNorm eps 1e-5), which its PhiAttention compiles
// in; the overloads below take another geometry.
struct PhiAttentionGeometry {
    std::size_t heads = 16;
    std::size_t kv_heads = 4;
    std::size_t head_dim = 128;
    std::size_t sliding_window = 2047;
    float rope_theta = 10000.0f;
    float norm_eps = 1.0e-5f;
};

class PhiAttention {
public:
    PhiAttention(const ModelLoader& loader, std::size_t layer_idx);
    PhiAttention(const ModelLoader& loader, std::size_t layer_idx, const PhiAttentionGeometry& g);
    void forward(const Tensor& x, Tensor& y) const;

private:
    Linear q_proj_, k_proj_, v_proj_, o_proj_;
    PhiAttentionGeometry g_;
};

// y = h + PhiMoE(layer_norm(h)), h = x + attention(layer_norm(x)) -- the
// reference's PhiDecoderLayer::forward with its MoE half (post-attention
// LayerNorm, router, experts, combine, residual) on the GPU.
class PhiDecoderLayer {
public:
    PhiDecoderLayer(const ModelLoader& loader, std::size_t layer_idx);
    PhiDecoderLayer(const ModelLoader& loader, std::size_t layer_idx,
                    const PhiAttentionGeometry& g, const MoeConfig& moe_cfg);
    void forward(const Tensor& x, Tensor& y) const;

private:
    Tensor input_norm_weight_, input_norm_bias_;
    PhiAttention attention_;
    PhiMoEBlock moe_;
    float eps_;
};
