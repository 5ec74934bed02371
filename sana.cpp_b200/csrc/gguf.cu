// GGUF reader (see gguf.h): host code only.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace sana {
namespace {

// Metadata value types of the GGUF layout.
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};

// Bounds-checked little-endian cursor over the mapping.
struct Cursor {
    const uint8_t* base;
    size_t size, pos = 0;
    const std::string& path;

    [[noreturn]] void fail(const std::string& what) const {
        throw std::runtime_error("malformed gguf weight file " + path + ": " + what);
    }
    void need(size_t n) const {
        if (n > size || pos > size - n) fail("truncated");
    }
    template <class T>
    T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > (1u << 20)) fail("string longer than 1 MiB");
        need(static_cast<size_t>(n));
        std::string s(reinterpret_cast<const char*>(base + pos), static_cast<size_t>(n));
        pos += static_cast<size_t>(n);
        return s;
    }
    void skip_value(uint32_t type, int depth = 0) {
        switch (type) {
            case kU8: case kI8: case kBool: need(1); pos += 1; return;
            case kU16: case kI16: need(2); pos += 2; return;
            case kU32: case kI32: case kF32: need(4); pos += 4; return;
            case kU64: case kI64: case kF64: need(8); pos += 8; return;
            case kString: str(); return;
            case kArray: {
                if (depth > 4) fail("nested arrays deeper than 4");
                const uint32_t et = get<uint32_t>();
                const uint64_t n = get<uint64_t>();
                if (n > size) fail("array longer than the file");
                for (uint64_t i = 0; i < n; ++i) skip_value(et, depth + 1);
                return;
            }
            default: fail("unknown metadata value type " + std::to_string(type));
        }
    }
};

}  // namespace

int64_t GgufTensor::elements() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
}

GgufFile::GgufFile(const std::string& path) : path_(path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("failed to open gguf weight file: " + path);
    struct stat st;
    if (::fstat(fd, &st) != 0 || st.st_size <= 0) {
        ::close(fd);
        throw std::runtime_error("failed to open gguf weight file: " + path);
    }
    size_ = static_cast<size_t>(st.st_size);
    map_ = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) {
        map_ = nullptr;
        throw std::runtime_error("failed to map gguf weight file: " + path);
    }
    try {
        Cursor c{static_cast<const uint8_t*>(map_), size_, 0, path_};
        if (c.get<uint32_t>() != 0x46554747u) c.fail("bad magic");  // "GGUF"
        version_ = c.get<uint32_t>();
        if (version_ != 2 && version_ != 3) c.fail("unsupported version " + std::to_string(version_));
        const uint64_t n_tensors = c.get<uint64_t>();
        const uint64_t n_kv = c.get<uint64_t>();
        if (n_tensors > size_ || n_kv > size_) c.fail("implausible counts");
        for (uint64_t i = 0; i < n_kv; ++i) {
            const std::string key = c.str();
            const uint32_t type = c.get<uint32_t>();
            if (key == "general.alignment" && type == kU32) {
                alignment_ = c.get<uint32_t>();
                if (alignment_ == 0 || (alignment_ & (alignment_ - 1)) != 0) c.fail("alignment not a power of two");
            } else {
                c.skip_value(type);
            }
        }
        struct Rec {
            std::string name;
            uint32_t type;
            std::vector<int64_t> shape;
            uint64_t offset;
        };
        std::vector<Rec> recs;
        recs.reserve(static_cast<size_t>(n_tensors));
        for (uint64_t i = 0; i < n_tensors; ++i) {
            Rec r;
            r.name = c.str();
            const uint32_t nd = c.get<uint32_t>();
            if (nd > 8) c.fail("tensor rank above 8: " + r.name);
            std::vector<int64_t> ne(nd);
            for (uint32_t d = 0; d < nd; ++d) {
                const uint64_t e = c.get<uint64_t>();
                if (e > (1ull << 40)) c.fail("implausible extent in " + r.name);
                ne[d] = static_cast<int64_t>(e);
            }
            r.shape.assign(ne.rbegin(), ne.rend());
            r.type = c.get<uint32_t>();
            r.offset = c.get<uint64_t>();
            recs.push_back(std::move(r));
        }
        const uint64_t data_start = (c.pos + alignment_ - 1) / alignment_ * alignment_;
        if (data_start > size_) c.fail("data section past the end of the file");
        tensors_.reserve(recs.size());
        for (auto& r : recs) {
            GgufTensor t;
            t.name = r.name;
            t.type = r.type;
            t.shape = r.shape;
            const int esize = r.type == kGgufF32 ? 4 : (r.type == kGgufF16 || r.type == kGgufBF16) ? 2 : 0;
            t.nbytes = esize ? static_cast<uint64_t>(t.elements()) * esize : 0;
            if (r.offset % alignment_ != 0) c.fail("misaligned tensor data: " + r.name);
            if (r.offset > size_ - data_start || t.nbytes > size_ - data_start - r.offset)
                c.fail("tensor data past the end of the file: " + r.name);
            t.data = static_cast<const uint8_t*>(map_) + data_start + r.offset;
            t.file_offset = data_start + r.offset;
            if (!by_name_.emplace(t.name, tensors_.size()).second) c.fail("duplicate tensor name " + t.name);
            tensors_.push_back(std::move(t));
        }
    } catch (...) {
        ::munmap(map_, size_);
        map_ = nullptr;
        throw;
    }
}

GgufFile::~GgufFile() {
    if (map_) ::munmap(map_, size_);
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    const auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

}  // namespace sana
