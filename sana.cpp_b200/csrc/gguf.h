// GGUF weight files (the container the reference's loader reads through ggml's gguf API,
// weights_io.cpp:134-164): a memory-mapped reader of the published GGUF layout, versions 2
// and 3, keeping each tensor's name, element type, shape and a pointer into the mapping.
//
// Layout read here: "GGUF" magic, u32 version, u64 tensor count, u64 metadata count; the
// metadata key/value pairs (skipped except general.alignment); one record per tensor (name,
// u32 rank, u64 extents fastest-first, u32 element type, u64 offset); then the data section
// at the next multiple of the alignment (default 32), each tensor at its offset from there.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace sana {

// Element types of the tensor records (ggml's numbering).
enum GgufType : uint32_t { kGgufF32 = 0, kGgufF16 = 1, kGgufBF16 = 30 };

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    std::vector<int64_t> shape;  // slowest-varying first (numpy / PyTorch order: extents reversed)
    const uint8_t* data = nullptr;
    uint64_t file_offset = 0;    // of the first data byte from the start of the file
    uint64_t nbytes = 0;         // 0 for element types without a fixed size here
    int64_t elements() const;
};

class GgufFile {
public:
    // Maps and parses `path`; throws std::runtime_error (the reference's error for a weight
    // file it cannot open or parse) when the file is missing, truncated or malformed.
    explicit GgufFile(const std::string& path);
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    const std::string& path() const { return path_; }
    uint32_t version() const { return version_; }
    uint64_t alignment() const { return alignment_; }
    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    // nullptr when absent
    const GgufTensor* find(const std::string& name) const;

private:
    std::string path_;
    void* map_ = nullptr;
    size_t size_ = 0;
    uint32_t version_ = 0;
    uint64_t alignment_ = 32;
    std::vector<GgufTensor> tensors_;
    std::unordered_map<std::string, size_t> by_name_;
};

}  // namespace sana
