// model.bin reader of the drop-in layer (include/model_loader.h).
#include "model_loader.h"

#include <fstream>
#include <stdexcept>

namespace {
template <typename T>
T read_pod(std::ifstream& f) {
    T v{};
    f.read(reinterpret_cast<char*>(&v), sizeof(T));
    if (!f) throw std::runtime_error("truncated model.bin");
    return v;
}
}  // namespace

ModelLoader::ModelLoader(const std::string& path) : path_(path) {
    std::ifstream f(path_, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open model: " + path_);
    const auto count = read_pod<std::uint32_t>(f);
    for (std::uint32_t i = 0; i < count; ++i) {
        const auto name_len = read_pod<std::uint32_t>(f);
        if (name_len > (1u << 20)) throw std::runtime_error("truncated model.bin");
        std::string name(name_len, '\0');
        f.read(name.data(), name_len);
        if (!f) throw std::runtime_error("truncated model.bin");
        const auto ndim = read_pod<std::uint32_t>(f);
        if (ndim > 8) throw std::runtime_error("truncated model.bin");
        Entry e;
        e.shape.resize(ndim);
        for (auto& d : e.shape) d = read_pod<std::uint32_t>(f);
        e.offset = read_pod<std::uint64_t>(f);
        e.bytes = read_pod<std::uint64_t>(f);
        entries_[std::move(name)] = std::move(e);
    }
}

std::vector<std::size_t> ModelLoader::shape(const std::string& name) const {
    const auto it = entries_.find(name);
    if (it == entries_.end()) throw std::runtime_error("missing tensor: " + name);
    return it->second.shape;
}

Tensor ModelLoader::load(const std::string& name) const {
    const auto it = entries_.find(name);
    if (it == entries_.end()) throw std::runtime_error("missing tensor: " + name);
    const Entry& e = it->second;
    std::size_t n = 1;
    for (std::size_t d : e.shape) n *= d;
    if (e.bytes != n * sizeof(float)) throw std::runtime_error("tensor is not float32: " + name);
    Tensor out(e.shape);
    std::ifstream f(path_, std::ios::binary);
    if (!f) throw std::runtime_error("cannot reopen model: " + path_);
    f.seekg(static_cast<std::streamoff>(e.offset));
    f.read(reinterpret_cast<char*>(out.data()), static_cast<std::streamsize>(e.bytes));
    if (!f) throw std::runtime_error("truncated tensor: " + name);
    return out;
}
