// Drives the drop-in C++ layer the way the reference's code uses its own
// classes (include/layer.h, include/model_loader.h, include/tensor.h):
//
//   test_phimoe errors <dir>                       exception types, no GPU
//   test_phimoe forward <model.bin> <x.bin> <T> <d> <out_prefix>
//       PhiMoE(loader, 0).forward(x, y)  -> <out_prefix>.moe.bin
//       PhiMLP(loader, "...experts.0")   -> <out_prefix>.mlp.bin
//       PhiMoE::route                    -> <out_prefix>.route.bin (int idx, float w)
//       a wrong-width input must throw std::invalid_argument
//   test_phimoe layernorm <model.bin> <x.bin> <T> <d> <out_prefix>   no GPU
//       tensor_ops::layer_norm with post_attention_layernorm -> <out_prefix>.ln.bin
//   test_phimoe block <model.bin> <x.bin> <T> <d> <out_prefix>
//       PhiMoEBlock(loader, 0).forward(attn, y)          -> <out_prefix>.block.bin
//   test_phimoe rope <q.bin> <k.bin> <S> <heads> <kv_heads> <head_dim> <out_prefix>   no GPU
//       tensor_ops::apply_rope (base 1e4)                -> <out_prefix>.q.bin / .k.bin
//   test_phimoe attention <model.bin> <x.bin> <S> <d> <heads> <kv_heads> <out_prefix>   no GPU
//       PhiAttention(loader, 0, geometry: head_dim 128, no effective window)
//                                                        -> <out_prefix>.attn.bin
//   test_phimoe decoder <model.bin> <x.bin> <S> <d> <heads> <kv_heads> <out_prefix>
//       PhiDecoderLayer(loader, 0, same geometry, the reference's MoE
//       configuration with sizes from the file)           -> <out_prefix>.dec.bin
#include "layer.h"
#include "model_loader.h"
#include "tensor.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

static int failures = 0;
#define CHECK(cond, msg)                                  \
    do {                                                  \
        if (!(cond)) {                                    \
            std::fprintf(stderr, "FAIL: %s\n", msg);      \
            ++failures;                                   \
        }                                                 \
    } while (0)

template <typename Ex, typename F>
static bool throws(F f, const char* needle) {
    try {
        f();
    } catch (const Ex& e) {
        return std::strstr(e.what(), needle) != nullptr;
    } catch (...) {
        return false;
    }
    return false;
}

static void write_file(const std::string& p, const void* data, size_t n) {
    std::ofstream f(p, std::ios::binary);
    f.write(static_cast<const char*>(data), static_cast<std::streamsize>(n));
}

static int errors(const std::string& dir) {
    CHECK(throws<std::runtime_error>([&] { ModelLoader l(dir + "/does_not_exist.bin"); },
                                     "cannot open model"),
          "missing file");
    {
        const std::string p = dir + "/trunc.bin";
        const unsigned char bytes[6] = {3, 0, 0, 0, 9, 0};
        write_file(p, bytes, sizeof bytes);
        CHECK(throws<std::runtime_error>([&] { ModelLoader l(p); }, "truncated model.bin"),
              "truncated index");
    }
    {
        const std::string p = dir + "/empty.bin";
        const unsigned char zero[4] = {0, 0, 0, 0};
        write_file(p, zero, sizeof zero);
        ModelLoader l(p);
        CHECK(!l.has("x"), "has() on an empty index");
        CHECK(throws<std::runtime_error>([&] { l.load("model.layers.0.block_sparse_moe.gate.weight"); },
                                         "missing tensor"),
              "missing tensor");
        CHECK(throws<std::runtime_error>([&] { PhiMoE m(l, 0); }, "missing tensor"),
              "PhiMoE on a file without the layer");
    }
    Tensor t({2, 3});
    CHECK(throws<std::out_of_range>([&] { t.at(2, 0); }, "Tensor index"), "at() bounds");
    CHECK(throws<std::invalid_argument>([&] { t.at(1); }, "rank"), "at() rank");
    CHECK(throws<std::invalid_argument>([&] { t.reshape({4, 2}); }, "reshape"), "reshape size");
    Tensor a({2, 4}), b({3, 4}), c({2, 3});
    for (size_t i = 0; i < a.size(); ++i) a[i] = 0.5f * float(i);
    for (size_t i = 0; i < b.size(); ++i) b[i] = 0.25f * float(i) - 1.0f;
    tensor_ops::matmul_transposed(a, b, c);
    CHECK(c.at(1, 2) == 0.5f * (4 * 1.0f + 5 * 1.25f + 6 * 1.5f + 7 * 1.75f), "matmul_transposed");
    Tensor bad({2, 5});
    CHECK(throws<std::invalid_argument>([&] { tensor_ops::matmul_transposed(bad, b, c); },
                                        "matmul_transposed shape"),
          "matmul shape");
    // matmul: [M,K] x [K,N]
    Tensor bt({4, 3}), c2({2, 3});
    for (size_t p = 0; p < 4; ++p)
        for (size_t j = 0; j < 3; ++j) bt.at(p, j) = b.at(j, p);
    tensor_ops::matmul(a, bt, c2);
    CHECK(std::memcmp(c.data(), c2.data(), c.size() * 4) == 0, "matmul == matmul_transposed");
    CHECK(throws<std::invalid_argument>([&] { tensor_ops::matmul(a, b, c2); }, "matmul shape"),
          "matmul inner size");
    // softmax_last_dim: rows sum to 1, order kept, max-subtracted (large inputs finite)
    Tensor sx({2, 3}), sy({2, 3});
    const float vals[6] = {1.0f, 2.0f, 3.0f, 1000.0f, 1001.0f, 999.0f};
    std::memcpy(sx.data(), vals, sizeof vals);
    tensor_ops::softmax_last_dim(sx, sy);
    CHECK(std::abs(sy.at(0, 0) + sy.at(0, 1) + sy.at(0, 2) - 1.0f) < 1e-6f, "softmax sums to 1");
    CHECK(sy.at(1, 1) > sy.at(1, 0) && sy.at(1, 0) > sy.at(1, 2), "softmax order");
    CHECK(std::abs(sy.at(0, 2) - sy.at(1, 1)) < 1e-6f, "softmax shift invariance");
    Tensor q1({1, 4}), k1({1, 4});
    CHECK(throws<std::invalid_argument>(
              [&] { tensor_ops::apply_rope(q1, k1, 1, 1, 1, 3, 10000.0f); }, "apply_rope shape"),
          "apply_rope odd head_dim");
    std::printf("%s\n", failures ? "errors: FAILED" : "errors: ok");
    return failures ? 1 : 0;
}

static int forward(const std::string& model, const std::string& xpath, size_t T, size_t d,
                   const std::string& out) {
    ModelLoader loader(model);
    PhiMoE moe(loader, 0);
    Tensor x({T, d});
    {
        std::ifstream f(xpath, std::ios::binary);
        f.read(reinterpret_cast<char*>(x.data()), static_cast<std::streamsize>(T * d * 4));
        if (!f) throw std::runtime_error("cannot read x");
    }
    Tensor y;
    moe.forward(x, y);
    CHECK(y.ndim() == 2 && y.size(0) == T && y.size(1) == d, "PhiMoE output shape");
    write_file(out + ".moe.bin", y.data(), y.size() * 4);

    PhiMLP mlp(loader, "model.layers.0.block_sparse_moe.experts.0");
    Tensor ym;
    mlp.forward(x, ym);
    write_file(out + ".mlp.bin", ym.data(), ym.size() * 4);

    std::vector<std::pair<int, float>> routes;
    moe.route(x, routes);
    std::vector<int> idx;
    std::vector<float> w;
    for (auto& r : routes) {
        idx.push_back(r.first);
        w.push_back(r.second);
    }
    write_file(out + ".route_idx.bin", idx.data(), idx.size() * 4);
    write_file(out + ".route_w.bin", w.data(), w.size() * 4);

    Tensor wrong({T, d + 64});
    CHECK(throws<std::invalid_argument>([&] { Tensor yy; moe.forward(wrong, yy); }, "shape"),
          "wrong width input");
    Tensor pinned({T, d}, Tensor::Alloc::Pinned);
    std::memcpy(pinned.data(), x.data(), T * d * 4);
    Tensor yp;
    moe.forward(pinned, yp);
    CHECK(std::memcmp(yp.data(), y.data(), T * d * 4) == 0, "pinned input gives the same y");
    std::printf("%s\n", failures ? "forward: FAILED" : "forward: ok");
    return failures ? 1 : 0;
}

static Tensor read_x(const std::string& xpath, size_t T, size_t d) {
    Tensor x({T, d});
    std::ifstream f(xpath, std::ios::binary);
    f.read(reinterpret_cast<char*>(x.data()), static_cast<std::streamsize>(T * d * 4));
    if (!f) throw std::runtime_error("cannot read x");
    return x;
}

static int layernorm(const std::string& model, const std::string& xpath, size_t T, size_t d,
                     const std::string& out) {
    ModelLoader loader(model);
    const Tensor x = read_x(xpath, T, d);
    const Tensor w = loader.load("model.layers.0.post_attention_layernorm.weight");
    const Tensor b = loader.load("model.layers.0.post_attention_layernorm.bias");
    Tensor y({T, d});
    tensor_ops::layer_norm(x, w, b, 1.0e-5f, y);
    write_file(out + ".ln.bin", y.data(), y.size() * 4);
    Tensor bad({T, d + 1});
    CHECK(throws<std::invalid_argument>([&] { tensor_ops::layer_norm(x, w, b, 1e-5f, bad); },
                                        "layer norm shape"),
          "layer_norm shape");
    std::printf("%s\n", failures ? "layernorm: FAILED" : "layernorm: ok");
    return failures ? 1 : 0;
}

static int block(const std::string& model, const std::string& xpath, size_t T, size_t d,
                 const std::string& out) {
    ModelLoader loader(model);
    PhiMoEBlock blk(loader, 0);
    const Tensor attn = read_x(xpath, T, d);
    Tensor y;
    blk.forward(attn, y);
    CHECK(y.ndim() == 2 && y.size(0) == T && y.size(1) == d, "PhiMoEBlock output shape");
    write_file(out + ".block.bin", y.data(), y.size() * 4);
    std::printf("%s\n", failures ? "block: FAILED" : "block: ok");
    return failures ? 1 : 0;
}

static Tensor read_mat(const std::string& path, size_t rows, size_t cols) { return read_x(path, rows, cols); }

static PhiAttentionGeometry test_geometry(size_t heads, size_t kv_heads) {
    PhiAttentionGeometry g;
    g.heads = heads;
    g.kv_heads = kv_heads;
    g.head_dim = 128;
    g.sliding_window = 1000000;   // beyond any test sequence
    return g;
}

static int rope(const std::string& qp, const std::string& kp, size_t S, size_t H, size_t KVH,
                size_t hd, const std::string& out) {
    Tensor q = read_mat(qp, S, H * hd), k = read_mat(kp, S, KVH * hd);
    tensor_ops::apply_rope(q, k, S, H, KVH, hd, 10000.0f);
    write_file(out + ".q.bin", q.data(), q.size() * 4);
    write_file(out + ".k.bin", k.data(), k.size() * 4);
    std::printf("rope: ok\n");
    return 0;
}

static int attention(const std::string& model, const std::string& xpath, size_t S, size_t d,
                     size_t H, size_t KVH, const std::string& out) {
    ModelLoader loader(model);
    PhiAttention att(loader, 0, test_geometry(H, KVH));
    const Tensor x = read_x(xpath, S, d);
    Tensor y;
    att.forward(x, y);
    write_file(out + ".attn.bin", y.data(), y.size() * 4);
    std::printf("attention: ok\n");
    return 0;
}

static int decoder(const std::string& model, const std::string& xpath, size_t S, size_t d,
                   size_t H, size_t KVH, const std::string& out) {
    ModelLoader loader(model);
    MoeConfig cfg;
    moe_config_init(&cfg);              // the reference's router and precision
    cfg.d_model = cfg.d_ff = cfg.num_experts = 0;   // sizes from the file
    PhiDecoderLayer layer(loader, 0, test_geometry(H, KVH), cfg);
    const Tensor x = read_x(xpath, S, d);
    Tensor y;
    layer.forward(x, y);
    CHECK(y.ndim() == 2 && y.size(0) == S && y.size(1) == d, "PhiDecoderLayer output shape");
    write_file(out + ".dec.bin", y.data(), y.size() * 4);
    std::printf("%s\n", failures ? "decoder: FAILED" : "decoder: ok");
    return failures ? 1 : 0;
}

int main(int argc, char** argv) {
    try {
        if (argc >= 3 && std::string(argv[1]) == "errors") return errors(argv[2]);
        if (argc >= 7 && std::string(argv[1]) == "forward")
            return forward(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]), argv[6]);
        if (argc >= 7 && std::string(argv[1]) == "layernorm")
            return layernorm(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]), argv[6]);
        if (argc >= 7 && std::string(argv[1]) == "block")
            return block(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]), argv[6]);
        if (argc >= 9 && std::string(argv[1]) == "rope")
            return rope(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]),
                        std::stoul(argv[6]), std::stoul(argv[7]), argv[8]);
        if (argc >= 9 && std::string(argv[1]) == "attention")
            return attention(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]),
                             std::stoul(argv[6]), std::stoul(argv[7]), argv[8]);
        if (argc >= 9 && std::string(argv[1]) == "decoder")
            return decoder(argv[2], argv[3], std::stoul(argv[4]), std::stoul(argv[5]),
                           std::stoul(argv[6]), std::stoul(argv[7]), argv[8]);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "uncaught: %s\n", e.what());
        return 2;
    }
    std::fprintf(stderr, "usage: test_phimoe errors <dir> | forward <model> <x> <T> <d> <out>\n");
    return 2;
}
