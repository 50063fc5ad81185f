// model.bin reader of the drop-in layer (include/model_loader.h).
//
// The index is parsed from a buffered positional reader (pread into a 64 KB
// window), with every field bounds-checked before use; tensor payloads are
// read with one pread loop straight into the tensor's storage.  The file is
// opened per operation, so a loader holds no descriptor between calls.  The
// exception messages are the reference's (src/model_loader.cu:14-50), which
// callers of the drop-in may match on.
#include "model_loader.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>

namespace {

// An open file, closed on scope exit.
struct File {
    int fd = -1;
    explicit File(const std::string& path) : fd(::open(path.c_str(), O_RDONLY | O_CLOEXEC)) {}
    ~File() {
        if (fd >= 0) ::close(fd);
    }
    File(const File&) = delete;
    File& operator=(const File&) = delete;
};

// Reads exactly n bytes at offset off; false on a short file or an error.
bool pread_all(int fd, void* dst, std::size_t n, std::uint64_t off) {
    auto* p = static_cast<char*>(dst);
    while (n > 0) {
        const ssize_t r = ::pread(fd, p, n, static_cast<off_t>(off));
        if (r <= 0) return false;
        p += r;
        n -= static_cast<std::size_t>(r);
        off += static_cast<std::uint64_t>(r);
    }
    return true;
}

// Sequential little-endian fields over a pread window.  Any read past the
// end of the file throws "truncated model.bin".
class IndexReader {
public:
    explicit IndexReader(int fd) : fd_(fd) {}

    template <typename T>
    T field() {
        T v{};
        take(&v, sizeof(T));
        return v;
    }
    std::string text(std::size_t n) {
        std::string s(n, '\0');
        take(s.data(), n);
        return s;
    }

private:
    void take(void* dst, std::size_t n) {
        auto* out = static_cast<char*>(dst);
        while (n > 0) {
            if (pos_ == len_) refill();
            const std::size_t k = std::min(n, len_ - pos_);
            std::memcpy(out, buf_ + pos_, k);
            pos_ += k;
            out += k;
            n -= k;
        }
    }
    void refill() {
        const ssize_t r = ::pread(fd_, buf_, sizeof buf_, static_cast<off_t>(file_off_));
        if (r <= 0) throw std::runtime_error("truncated model.bin");
        file_off_ += static_cast<std::uint64_t>(r);
        len_ = static_cast<std::size_t>(r);
        pos_ = 0;
    }
    int fd_;
    char buf_[1 << 16];
    std::size_t len_ = 0, pos_ = 0;
    std::uint64_t file_off_ = 0;
};

constexpr std::uint32_t kMaxNameBytes = 1u << 20;
constexpr std::uint32_t kMaxRank = 8;

}  // namespace

ModelLoader::ModelLoader(const std::string& path) : path_(path) {
    File f(path_);
    if (f.fd < 0) throw std::runtime_error("cannot open model: " + path_);
    IndexReader in(f.fd);
    const auto count = in.field<std::uint32_t>();
    for (std::uint32_t i = 0; i < count; ++i) {
        const auto name_len = in.field<std::uint32_t>();
        if (name_len > kMaxNameBytes) throw std::runtime_error("truncated model.bin");
        std::string name = in.text(name_len);
        const auto rank = in.field<std::uint32_t>();
        if (rank > kMaxRank) throw std::runtime_error("truncated model.bin");
        Entry e;
        e.shape.reserve(rank);
        for (std::uint32_t r = 0; r < rank; ++r) e.shape.push_back(in.field<std::uint32_t>());
        e.offset = in.field<std::uint64_t>();
        e.bytes = in.field<std::uint64_t>();
        entries_.insert_or_assign(std::move(name), std::move(e));
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
    std::size_t count = 1;
    for (std::size_t extent : e.shape) count *= extent;
    if (e.bytes != count * sizeof(float)) throw std::runtime_error("tensor is not float32: " + name);
    Tensor out(e.shape);
    File f(path_);
    if (f.fd < 0) throw std::runtime_error("cannot reopen model: " + path_);
    if (!pread_all(f.fd, out.data(), static_cast<std::size_t>(e.bytes), e.offset))
        throw std::runtime_error("truncated tensor: " + name);
    return out;
}
