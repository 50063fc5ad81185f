// tensor.h -- host fp32 tensor of the MoE drop-in layer.
//
// Source-compatible with the reference's Tensor (include/tensor.h:7-57 of
// songsnim/accelerating-MoE-inference): row-major fp32 storage, Host or
// Pinned allocation, bounds-checked at(), reshape / reshape_within_capacity,
// fill / zero, and the same exceptions (std::out_of_range for bad indices,
// std::invalid_argument for rank or size mismatches, std::runtime_error when
// pinned allocation fails).  Pinned tensors make moe_forward_host's copies
// run at full PCIe / C2C speed.
#pragma once

#include <cstddef>
#include <initializer_list>
#include <string>
#include <vector>

class Tensor {
public:
    enum class Alloc { Host, Pinned };

    Tensor() = default;
    explicit Tensor(std::vector<std::size_t> shape, Alloc alloc = Alloc::Host);
    ~Tensor();
    Tensor(const Tensor& other);
    Tensor& operator=(const Tensor& other);
    Tensor(Tensor&& other) noexcept;
    Tensor& operator=(Tensor&& other) noexcept;

    std::size_t ndim() const { return shape_.size(); }
    std::size_t size() const { return size_; }
    std::size_t capacity() const { return capacity_; }
    Alloc alloc() const { return alloc_; }
    std::size_t size(std::size_t dim) const;
    const std::vector<std::size_t>& shape() const { return shape_; }

    float* data() { return data_; }
    const float* data() const { return data_; }
    float& operator[](std::size_t i) { return data_[i]; }
    const float& operator[](std::size_t i) const { return data_[i]; }

    float& at(std::size_t i);
    float& at(std::size_t i, std::size_t j);
    float& at(std::size_t i, std::size_t j, std::size_t k);
    float& at(std::size_t i, std::size_t j, std::size_t k, std::size_t l);
    const float& at(std::size_t i) const;
    const float& at(std::size_t i, std::size_t j) const;
    const float& at(std::size_t i, std::size_t j, std::size_t k) const;
    const float& at(std::size_t i, std::size_t j, std::size_t k, std::size_t l) const;

    void reshape(std::vector<std::size_t> shape);
    void reshape_within_capacity(std::vector<std::size_t> shape);
    void fill(float value);
    void zero() { fill(0.0f); }

private:
    std::vector<std::size_t> shape_;
    float* data_ = nullptr;
    std::size_t size_ = 0, capacity_ = 0;
    Alloc alloc_ = Alloc::Host;
    void release();
    std::size_t offset(std::initializer_list<std::size_t> indices) const;
};

// Host ops on the MoE path (src/tensor.cu:136-172 of the reference), with the
// reference's arithmetic: matmul_transposed is a k-ascending fused
// multiply-add chain per output, silu uses a double-precision exp.
namespace tensor_ops {
void matmul(const Tensor& a, const Tensor& b, Tensor& c);              // [M,K] x [K,N]
void matmul_transposed(const Tensor& a, const Tensor& b, Tensor& c);   // [M,K] x [N,K]
void add_inplace(Tensor& a, const Tensor& b);
void add_bias_inplace(Tensor& a, const Tensor& bias);
void mul(const Tensor& a, const Tensor& b, Tensor& c);
void silu(const Tensor& x, Tensor& y);
// src/tensor.cu:174-189, with the reference build's arithmetic: serial
// j-ascending sums, unfused variance terms, fused output expression.
void layer_norm(const Tensor& x, const Tensor& weight, const Tensor& bias, float eps, Tensor& y);
// Softmax over the last dimension (declared by the reference, include/
// tensor.h:67, with no definition there): max-subtracted, exp in double.
void softmax_last_dim(const Tensor& x, Tensor& y);
// Rotary embedding in rotate-half form, in place, position = row
// (src/tensor.cu:191-210): q [seq][q_heads * head_dim], k [seq][kv_heads *
// head_dim].
void apply_rope(Tensor& q, Tensor& k, std::size_t seq_len, std::size_t q_heads,
                std::size_t kv_heads, std::size_t head_dim, float theta);
}
