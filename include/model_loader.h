// model_loader.h -- reads the reference's model.bin (include/model_loader.h
// and src/model_loader.cu:14-50 of songsnim/accelerating-MoE-inference):
// u32 count; per tensor u32 name_len, name, u32 ndim, u32 dims[ndim],
// u64 offset, u64 bytes; fp32 payloads.  Same interface and the same
// std::runtime_error messages ("cannot open model: ", "truncated model.bin",
// "missing tensor: ", "tensor is not float32: ", "truncated tensor: ").
#pragma once

#include "tensor.h"

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

class ModelLoader {
public:
    explicit ModelLoader(const std::string& path);
    Tensor load(const std::string& name) const;
    bool has(const std::string& name) const { return entries_.count(name) != 0; }
    const std::string& path() const { return path_; }
    // Shape of a tensor without reading its payload (std::runtime_error if absent).
    std::vector<std::size_t> shape(const std::string& name) const;

private:
    struct Entry {
        std::vector<std::size_t> shape;
        std::uint64_t offset = 0;
        std::uint64_t bytes = 0;
    };
    std::string path_;
    std::unordered_map<std::string, Entry> entries_;
};
