// Host Tensor and the MoE-path tensor_ops of the drop-in layer (include/tensor.h).
#include "tensor.h"

#include "moe_b200.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <limits>
#include <stdexcept>
#include <string>

Tensor::Tensor(std::vector<std::size_t> shape, Alloc alloc) : shape_(std::move(shape)), alloc_(alloc) {
    std::size_t n = 1;
    for (std::size_t d : shape_) n *= d;
    if (alloc_ == Alloc::Pinned) {
        void* p = nullptr;
        if (moe_host_alloc(n * sizeof(float), &p) != MOE_OK)
            throw std::runtime_error(std::string("pinned tensor allocation: ") + moe_last_error());
        data_ = static_cast<float*>(p);
    } else {
        data_ = new float[n > 0 ? n : 1];
    }
    size_ = capacity_ = n;
    std::fill(data_, data_ + n, 0.0f);
}

void Tensor::release() {
    if (!data_) return;
    if (alloc_ == Alloc::Pinned) {
        if (moe_host_free(data_) != MOE_OK)
            std::fprintf(stderr, "pinned tensor free: %s\n", moe_last_error());
    } else {
        delete[] data_;
    }
    data_ = nullptr;
    size_ = capacity_ = 0;
}

Tensor::~Tensor() { release(); }

Tensor::Tensor(const Tensor& other) : shape_(other.shape_) {
    if (other.size_) {
        data_ = new float[other.size_];
        std::copy(other.data_, other.data_ + other.size_, data_);
        size_ = capacity_ = other.size_;
    }
}

Tensor& Tensor::operator=(const Tensor& other) {
    if (this != &other) {
        Tensor tmp(other);
        *this = std::move(tmp);
    }
    return *this;
}

Tensor::Tensor(Tensor&& o) noexcept
    : shape_(std::move(o.shape_)), data_(o.data_), size_(o.size_), capacity_(o.capacity_),
      alloc_(o.alloc_) {
    o.shape_.clear();
    o.data_ = nullptr;
    o.size_ = o.capacity_ = 0;
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this != &o) {
        release();
        shape_ = std::move(o.shape_);
        data_ = o.data_;
        size_ = o.size_;
        capacity_ = o.capacity_;
        alloc_ = o.alloc_;
        o.shape_.clear();
        o.data_ = nullptr;
        o.size_ = o.capacity_ = 0;
    }
    return *this;
}

std::size_t Tensor::size(std::size_t dim) const {
    if (dim >= shape_.size()) throw std::out_of_range("Tensor dimension");
    return shape_[dim];
}

std::size_t Tensor::offset(std::initializer_list<std::size_t> idx) const {
    if (idx.size() != shape_.size()) throw std::invalid_argument("Tensor rank mismatch");
    std::size_t off = 0;
    std::size_t d = 0;
    for (std::size_t i : idx) {
        if (i >= shape_[d]) throw std::out_of_range("Tensor index");
        off = off * shape_[d] + i;
        ++d;
    }
    return off;
}

float& Tensor::at(std::size_t i) { return data_[offset({i})]; }
float& Tensor::at(std::size_t i, std::size_t j) { return data_[offset({i, j})]; }
float& Tensor::at(std::size_t i, std::size_t j, std::size_t k) { return data_[offset({i, j, k})]; }
float& Tensor::at(std::size_t i, std::size_t j, std::size_t k, std::size_t l) {
    return data_[offset({i, j, k, l})];
}
const float& Tensor::at(std::size_t i) const { return data_[offset({i})]; }
const float& Tensor::at(std::size_t i, std::size_t j) const { return data_[offset({i, j})]; }
const float& Tensor::at(std::size_t i, std::size_t j, std::size_t k) const {
    return data_[offset({i, j, k})];
}
const float& Tensor::at(std::size_t i, std::size_t j, std::size_t k, std::size_t l) const {
    return data_[offset({i, j, k, l})];
}

void Tensor::reshape(std::vector<std::size_t> shape) {
    std::size_t n = 1;
    for (std::size_t d : shape) n *= d;
    if (n != size_) throw std::invalid_argument("reshape changes tensor size");
    shape_ = std::move(shape);
}

void Tensor::reshape_within_capacity(std::vector<std::size_t> shape) {
    std::size_t n = 1;
    for (std::size_t d : shape) n *= d;
    if (n > capacity_) throw std::invalid_argument("reshape exceeds tensor capacity");
    shape_ = std::move(shape);
    size_ = n;
}

void Tensor::fill(float v) { std::fill(data_, data_ + size_, v); }

namespace tensor_ops {

void matmul_transposed(const Tensor& a, const Tensor& b, Tensor& c) {
    if (a.ndim() != 2 || b.ndim() != 2 || c.ndim() != 2)
        throw std::invalid_argument("matmul_transposed shape");
    const std::size_t m = a.size(0), k = a.size(1), n = b.size(0);
    if (b.size(1) != k || c.size(0) != m || c.size(1) != n)
        throw std::invalid_argument("matmul_transposed shape");
    const float* A = a.data();
    const float* B = b.data();
    float* C = c.data();
#pragma omp parallel for
    for (long long i = 0; i < static_cast<long long>(m); ++i)
        for (std::size_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (std::size_t p = 0; p < k; ++p) s = std::fma(A[i * k + p], B[j * k + p], s);
            C[i * n + j] = s;
        }
}

// c[i][j] = sum_p a[i][p] * b[p][j], a p-ascending fused multiply-add chain
// per output, as matmul_transposed.
void matmul(const Tensor& a, const Tensor& b, Tensor& c) {
    if (a.ndim() != 2 || b.ndim() != 2 || c.ndim() != 2)
        throw std::invalid_argument("matmul shape");
    const std::size_t m = a.size(0), k = a.size(1), n = b.size(1);
    if (b.size(0) != k || c.size(0) != m || c.size(1) != n)
        throw std::invalid_argument("matmul shape");
    const float* A = a.data();
    const float* B = b.data();
    float* C = c.data();
#pragma omp parallel for
    for (long long i = 0; i < static_cast<long long>(m); ++i)
        for (std::size_t j = 0; j < n; ++j) {
            float s = 0.0f;
            for (std::size_t p = 0; p < k; ++p) s = std::fma(A[i * k + p], B[p * n + j], s);
            C[i * n + j] = s;
        }
}

void softmax_last_dim(const Tensor& x, Tensor& y) {
    if (x.ndim() == 0 || y.size() != x.size()) throw std::invalid_argument("softmax shape");
    const std::size_t h = x.size(x.ndim() - 1), rows = x.size() / h;
    const float* X = x.data();
    float* Y = y.data();
    for (std::size_t r = 0; r < rows; ++r) {
        const float* xr = X + r * h;
        float* yr = Y + r * h;
        float m = -std::numeric_limits<float>::infinity();
        for (std::size_t j = 0; j < h; ++j) m = std::max(m, xr[j]);
        double sum = 0.0;
        for (std::size_t j = 0; j < h; ++j) sum += std::exp(static_cast<double>(xr[j] - m));
        for (std::size_t j = 0; j < h; ++j)
            yr[j] = static_cast<float>(std::exp(static_cast<double>(xr[j] - m)) / sum);
    }
}

// Pair (j, j + head_dim / 2) of every head of row s turns by the angle
// s * theta^(-2j / head_dim), computed in float as the reference does.
void apply_rope(Tensor& q, Tensor& k, std::size_t seq_len, std::size_t q_heads,
                std::size_t kv_heads, std::size_t head_dim, float theta) {
    if (head_dim % 2 || q.ndim() != 2 || k.ndim() != 2 || q.size(0) < seq_len ||
        k.size(0) < seq_len || q.size(1) != q_heads * head_dim || k.size(1) != kv_heads * head_dim)
        throw std::invalid_argument("apply_rope shape");
    const std::size_t half = head_dim / 2;
    auto rotate = [&](Tensor& t, std::size_t heads, std::size_t s) {
        float* row = t.data() + s * t.size(1);
        for (std::size_t j = 0; j < half; ++j) {
            const float inv = std::pow(theta, -2.0f * static_cast<float>(j) /
                                                  static_cast<float>(head_dim));
            const float ang = static_cast<float>(s) * inv;
            const float c = std::cos(ang), sn = std::sin(ang);
            for (std::size_t hh = 0; hh < heads; ++hh) {
                float* p = row + hh * head_dim;
                const float x0 = p[j], x1 = p[j + half];
                // (x0 * c - x1 * sn, x1 * c + x0 * sn), each contracted to one
                // fma around the second product's rounding.
                p[j] = std::fma(x0, c, -(x1 * sn));
                p[j + half] = std::fma(x1, c, x0 * sn);
            }
        }
    };
    for (std::size_t s = 0; s < seq_len; ++s) {
        rotate(q, q_heads, s);
        rotate(k, kv_heads, s);
    }
}

void layer_norm(const Tensor& x, const Tensor& weight, const Tensor& bias, float eps, Tensor& y) {
    if (x.ndim() == 0) throw std::invalid_argument("layer norm shape");
    const std::size_t h = x.size(x.ndim() - 1), rows = x.size() / h;
    if (weight.size() != h || bias.size() != h || y.size() != x.size())
        throw std::invalid_argument("layer norm shape");
    const float* X = x.data();
    const float* W = weight.data();
    const float* B = bias.data();
    float* Y = y.data();
#pragma omp parallel for
    for (long long r = 0; r < static_cast<long long>(rows); ++r) {
        const float* xr = X + static_cast<std::size_t>(r) * h;
        float* yr = Y + static_cast<std::size_t>(r) * h;
        float mean = 0.0f;
        for (std::size_t j = 0; j < h; ++j) mean += xr[j];
        mean /= static_cast<float>(h);
        float var = 0.0f;
        for (std::size_t j = 0; j < h; ++j) {
            const float dv = xr[j] - mean;
            var += dv * dv;
        }
        const float inv = 1.0f / std::sqrt(var / static_cast<float>(h) + eps);
        for (std::size_t j = 0; j < h; ++j) yr[j] = std::fma((xr[j] - mean) * inv, W[j], B[j]);
    }
}

void add_inplace(Tensor& a, const Tensor& b) {
    if (a.size() != b.size()) throw std::invalid_argument("add shape");
    for (std::size_t i = 0; i < a.size(); ++i) a[i] += b[i];
}

void add_bias_inplace(Tensor& a, const Tensor& bias) {
    if (bias.ndim() != 1 || a.ndim() == 0 || a.size(a.ndim() - 1) != bias.size(0))
        throw std::invalid_argument("bias shape");
    const std::size_t h = bias.size(0);
    for (std::size_t i = 0; i < a.size(); ++i) a[i] += bias[i % h];
}

void mul(const Tensor& a, const Tensor& b, Tensor& c) {
    if (a.size() != b.size() || c.size() != a.size()) throw std::invalid_argument("mul shape");
    for (std::size_t i = 0; i < a.size(); ++i) c[i] = a[i] * b[i];
}

void silu(const Tensor& x, Tensor& y) {
    if (x.size() != y.size()) throw std::invalid_argument("silu shape");
    for (std::size_t i = 0; i < x.size(); ++i)
        y[i] = x[i] / (1.0f + static_cast<float>(std::exp(static_cast<double>(-x[i]))));
}

}  // namespace tensor_ops
