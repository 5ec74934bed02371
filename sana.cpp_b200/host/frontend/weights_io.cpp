// weights_io.h over this repository's readers: GGUF files indexed with the C ABI's sana_gguf_*
// (the reference goes through ggml's gguf API, weights_io.cpp:134-164), the npy format and the
// JSON index parsed here. Behaviour follows weights_io.cpp: the same names, the same error
// types and messages, payloads read as little-endian fp32. One deliberate difference: a GGUF
// tensor stored as fp16 / bf16 is indexed with that dtype, so load_weight_tensor refuses it
// ("only float32 saved weights are supported") instead of reading its bytes as fp32.
#include <algorithm>
#include <cctype>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <limits>
#include <sstream>
#include <stdexcept>
#include <string>

#include "sana_cuda.h"
#include "weights_io.h"

namespace {

using Index = std::unordered_map<std::string, SavedWeightInfo>;

std::unordered_map<std::string, SavedWeightInfo> gguf_index(const std::string& path) {
    char err[512] = {0};
    sana_gguf* f = nullptr;
    if (sana_gguf_open(path.c_str(), &f, err, sizeof err) != SANA_OK)
        throw std::runtime_error("failed to open gguf weight file: " + path);
    Index index;
    const int n = sana_gguf_tensor_count(f);
    for (int i = 0; i < n; ++i) {
        const char* name = nullptr;
        int type = 0, rank = 0;
        int64_t shape[8] = {0};
        uint64_t offset = 0;
        sana_gguf_tensor_info(f, i, &name, &type, &rank, shape, 8, nullptr, nullptr);
        sana_gguf_tensor_offset(f, i, &offset);
        SavedWeightInfo info;
        info.file = path;
        for (int d = 0; d < rank; ++d) info.shape.push_back(static_cast<size_t>(shape[d]));
        info.dtype = type == 0 ? "float32" : type == 1 ? "float16" : type == 30 ? "bfloat16" : "gguf type " + std::to_string(type);
        info.format = WeightFormat::Gguf;
        info.offset = static_cast<size_t>(offset);
        index[name] = std::move(info);
    }
    sana_gguf_close(f);
    return index;
}

// --- the JSON index: {"name": {"file": "...", "shape": [..], "dtype": "..."}, ...} ----------

class JsonCursor {
public:
    explicit JsonCursor(const std::string& text) : s_(text) {}

    void skip() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    bool peek(char c) {
        skip();
        return i_ < s_.size() && s_[i_] == c;
    }
    void expect(char c) {
        if (!peek(c)) throw std::runtime_error("invalid weight index json");
        ++i_;
    }
    bool at_end() {
        skip();
        return i_ >= s_.size();
    }
    // a quoted string; a backslash takes the next character literally
    std::string string() {
        skip();
        if (i_ >= s_.size() || s_[i_] != '"') throw std::runtime_error("expected quoted json string");
        ++i_;
        std::string out;
        while (i_ < s_.size() && s_[i_] != '"') {
            if (s_[i_] == '\\' && ++i_ >= s_.size()) throw std::runtime_error("invalid json escape");
            out.push_back(s_[i_++]);
        }
        if (i_ >= s_.size()) throw std::runtime_error("unterminated json string");
        ++i_;
        return out;
    }
    std::vector<size_t> dims() {
        expect('[');
        std::vector<size_t> out;
        if (peek(']')) {
            ++i_;
            return out;
        }
        for (;;) {
            skip();
            size_t used = 0;
            unsigned long long v = 0;
            try {
                v = std::stoull(s_.substr(i_, 32), &used);
            } catch (const std::exception&) {
                used = 0;
            }
            if (used == 0 || v > std::numeric_limits<size_t>::max())
                throw std::runtime_error("invalid shape dimension in weight index");
            out.push_back(static_cast<size_t>(v));
            i_ += used;
            if (at_end()) throw std::runtime_error("unterminated shape array");
            if (peek(']')) {
                ++i_;
                return out;
            }
            if (!peek(',')) throw std::runtime_error("invalid shape array separator");
            ++i_;
        }
    }
    // after an object member: true at the closing brace (consumed), false after a comma
    bool member_end(const char* unterminated, const char* bad_separator) {
        if (at_end()) throw std::runtime_error(unterminated);
        if (peek('}')) {
            ++i_;
            return true;
        }
        if (!peek(',')) throw std::runtime_error(bad_separator);
        ++i_;
        return false;
    }

private:
    const std::string& s_;
    size_t i_ = 0;
};

Index json_index(const std::string& path) {
    std::ifstream in(path);
    if (!in) throw std::runtime_error("failed to open weight index");
    const std::string text((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    JsonCursor c(text);
    Index index;
    c.expect('{');
    if (c.peek('}')) return index;
    for (;;) {
        const std::string name = c.string();
        c.expect(':');
        c.expect('{');
        SavedWeightInfo info;
        for (;;) {
            const std::string field = c.string();
            c.expect(':');
            if (field == "file")
                info.file = c.string();
            else if (field == "shape")
                info.shape = c.dims();
            else if (field == "dtype")
                info.dtype = c.string();
            else
                throw std::runtime_error("unexpected field in weight index");
            if (c.member_end("unterminated weight info object", "invalid weight info separator")) break;
        }
        index[name] = std::move(info);
        if (c.member_end("unterminated weight index object", "invalid top-level weight index separator")) break;
    }
    return index;
}

// --- npy -------------------------------------------------------------------------------------

// The header dictionary of an .npy file (format versions 1-3), leaving `in` at the payload.
std::string npy_header(std::ifstream& in) {
    char magic[6];
    in.read(magic, 6);
    if (!in || std::memcmp(magic, "\x93NUMPY", 6) != 0) throw std::runtime_error("invalid npy magic header");
    unsigned char version[2];
    in.read(reinterpret_cast<char*>(version), 2);
    if (!in) throw std::runtime_error("failed to read npy version");
    size_t length = 0;
    if (version[0] == 1) {
        unsigned char b[2];
        in.read(reinterpret_cast<char*>(b), 2);
        length = b[0] | (size_t{b[1]} << 8);
    } else if (version[0] == 2 || version[0] == 3) {
        unsigned char b[4];
        in.read(reinterpret_cast<char*>(b), 4);
        length = b[0] | (size_t{b[1]} << 8) | (size_t{b[2]} << 16) | (size_t{b[3]} << 24);
    } else {
        throw std::runtime_error("unsupported npy version");
    }
    if (!in) throw std::runtime_error("failed to read npy header size");
    std::string header(length, '\0');
    in.read(&header[0], static_cast<std::streamsize>(length));
    if (!in) throw std::runtime_error("failed to read npy header");
    return header;
}

bool npy_fortran(const std::string& h) {
    const size_t key = h.find("fortran_order");
    if (key == std::string::npos) throw std::runtime_error("npy header missing fortran_order");
    const size_t colon = h.find(':', key);
    if (colon == std::string::npos) throw std::runtime_error("invalid fortran_order entry");
    const size_t v = h.find_first_not_of(' ', colon + 1);
    if (v == std::string::npos) throw std::runtime_error("invalid fortran_order entry");
    if (h.compare(v, 4, "True") == 0) return true;
    if (h.compare(v, 5, "False") == 0) return false;
    throw std::runtime_error("invalid fortran_order value");
}

std::vector<size_t> npy_shape(const std::string& h) {
    const size_t open = h.find('(');
    const size_t close = open == std::string::npos ? std::string::npos : h.find(')', open);
    if (open == std::string::npos || close == std::string::npos) throw std::runtime_error("invalid shape entry");
    std::vector<size_t> shape;
    std::string token;
    std::istringstream items(h.substr(open + 1, close - open - 1));
    while (std::getline(items, token, ',')) {
        size_t a = token.find_first_not_of(' '), b = token.find_last_not_of(' ');
        if (a == std::string::npos) continue;
        token = token.substr(a, b - a + 1);
        if (!std::all_of(token.begin(), token.end(), [](char ch) { return std::isdigit(static_cast<unsigned char>(ch)); }))
            throw std::runtime_error("invalid shape dimension");
        shape.push_back(static_cast<size_t>(std::stoull(token)));
    }
    if (shape.empty()) throw std::runtime_error("empty shape is not supported in npy loader");
    return shape;
}

}  // namespace

bool ends_with(const std::string& value, const std::string& suffix) {
    return value.size() >= suffix.size() && value.compare(value.size() - suffix.size(), suffix.size(), suffix) == 0;
}

Index load_weight_index(const std::string& path) { return ends_with(path, ".gguf") ? gguf_index(path) : json_index(path); }

Tensor load_weight_tensor(const std::string& weights_dir, const Index& index, const std::string& name) {
    const auto it = index.find(name);
    if (it == index.end()) throw std::invalid_argument("weight name not found in weight index");
    const SavedWeightInfo& info = it->second;
    if (info.dtype != "float32") throw std::runtime_error("only float32 saved weights are supported");
    if (info.format == WeightFormat::Npy) {
        Tensor t = load_npy_tensor(weights_dir + "/" + info.file);
        if (t.shape() != info.shape) throw std::runtime_error("loaded weight tensor shape does not match index metadata");
        return t;
    }
    Tensor t(info.shape);
    std::ifstream in(info.file, std::ios::binary);
    if (!in) throw std::runtime_error("failed to open gguf weight file: " + info.file);
    in.seekg(static_cast<std::streamoff>(info.offset));
    in.read(reinterpret_cast<char*>(t.data().data()), static_cast<std::streamsize>(t.numel() * sizeof(float)));
    if (!in) throw std::runtime_error("failed to read gguf tensor payload for: " + name);
    return t;
}

Tensor load_linear_weight_tensor(const std::string& weights_dir, const Index& index, const std::string& name) {
    Tensor w = load_weight_tensor(weights_dir, index, name);
    if (w.rank() != 2) throw std::invalid_argument("linear weight must be rank 2");
    return w.transpose_2d();
}

Tensor load_npy_tensor(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error("failed to open npy file");
    const std::string header = npy_header(in);
    if (header.find("'descr': '<f4'") == std::string::npos && header.find("\"descr\": \"<f4\"") == std::string::npos)
        throw std::runtime_error("only little-endian float32 npy tensors are supported");
    if (npy_fortran(header)) throw std::runtime_error("fortran-order npy tensors are not supported");
    Tensor t(npy_shape(header));
    in.read(reinterpret_cast<char*>(t.data().data()), static_cast<std::streamsize>(t.numel() * sizeof(float)));
    if (!in) throw std::runtime_error("failed to read tensor payload");
    return t;
}

// Format 1.0 with the payload starting on a 16-byte boundary, as numpy writes it.
void save_npy_tensor(const Tensor& tensor, const std::string& path) {
    std::string dims;
    for (size_t i = 0; i < tensor.rank(); ++i) dims += std::to_string(tensor.dim_size(i)) + (i + 1 < tensor.rank() ? ", " : ",");
    std::string header = "{'descr': '<f4', 'fortran_order': False, 'shape': (" + dims + "), }";
    const size_t unpadded = 10 + header.size() + 1;
    header.append((16 - unpadded % 16) % 16, ' ');
    header.push_back('\n');
    std::ofstream out(path, std::ios::binary);
    if (!out) throw std::runtime_error("failed to open npy file for writing: " + path);
    const unsigned char prefix[10] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0, static_cast<unsigned char>(header.size() & 0xff),
                                      static_cast<unsigned char>(header.size() >> 8)};
    out.write(reinterpret_cast<const char*>(prefix), 10);
    out.write(header.data(), static_cast<std::streamsize>(header.size()));
    out.write(reinterpret_cast<const char*>(tensor.data().data()), static_cast<std::streamsize>(tensor.numel() * sizeof(float)));
    if (!out) throw std::runtime_error("failed to write npy payload: " + path);
}

TensorComparison compare_tensor_to_reference(const Tensor& actual, const std::string& path) {
    const Tensor ref = load_npy_tensor(path);
    if (ref.shape() != actual.shape())
        throw std::invalid_argument("reference tensor shape does not match the actual tensor shape");
    return {actual.max_abs_diff(ref), actual.mean_abs_diff(ref)};
}

Tensor slice_batch_3d(const Tensor& input, size_t batch_index) {
    if (input.rank() != 3) throw std::invalid_argument("input must be rank 3");
    if (batch_index >= input.dim_size(0)) throw std::invalid_argument("batch_index out of range");
    const size_t n = input.dim_size(1) * input.dim_size(2);
    Tensor out({1, input.dim_size(1), input.dim_size(2)});
    const float* src = input.data().data() + batch_index * n;
    std::copy(src, src + n, out.data().begin());
    return out;
}

TensorComparison compare_batch_slice_to_reference(const Tensor& actual, const std::string& path, size_t batch_index) {
    const Tensor ref = slice_batch_3d(load_npy_tensor(path), batch_index);
    if (ref.shape() != actual.shape())
        throw std::invalid_argument("reference tensor slice shape does not match the actual tensor shape");
    return {actual.max_abs_diff(ref), actual.mean_abs_diff(ref)};
}

TensorComparison compare_block_output_to_reference(const Tensor& actual, const std::string& path, size_t batch_index) {
    const Tensor ref = slice_batch_3d(load_npy_tensor(path), batch_index);
    if (ref.shape() != actual.shape())
        throw std::invalid_argument("reference block output slice shape does not match the actual tensor shape");
    return {actual.max_abs_diff(ref), actual.mean_abs_diff(ref)};
}
