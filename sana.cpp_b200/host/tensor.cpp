// A self-contained implementation of the reference's Tensor (include/tensor.h) for programs
// that use the CUDA host layer without the rest of sana.cpp (this repository's C++ tests).
// A sana.cpp build links its own tensor.cpp instead and leaves this file out. The norms and
// modulation run on the GPU through the C ABI; the layout helpers are host copies.
#include "tensor.h"

#include <cmath>
#include <stdexcept>

#include "shim.h"

Tensor::Tensor(std::vector<size_t> shape) : shape_(std::move(shape)) { data_.assign(numel(), 0.0f); }

const std::vector<size_t>& Tensor::shape() const { return shape_; }
std::vector<float>& Tensor::data() { return data_; }
const std::vector<float>& Tensor::data() const { return data_; }

float& Tensor::at(size_t i) {
    if (i >= data_.size()) throw std::out_of_range("index out of range");
    return data_[i];
}
const float& Tensor::at(size_t i) const {
    if (i >= data_.size()) throw std::out_of_range("index out of range");
    return data_[i];
}
float& Tensor::at(const std::vector<size_t>& idx) { return at(flat_index(idx)); }
const float& Tensor::at(const std::vector<size_t>& idx) const { return at(flat_index(idx)); }

void Tensor::fill(float v) { std::fill(data_.begin(), data_.end(), v); }
bool Tensor::same_shape(const Tensor& o) const { return shape_ == o.shape_; }

size_t Tensor::flat_index(const std::vector<size_t>& idx) const {
    if (idx.size() > shape_.size()) throw std::out_of_range("indices size is greater than rank");
    size_t f = 0;
    for (size_t a = 0; a < shape_.size(); ++a) {
        const size_t i = a < idx.size() ? idx[a] : 0;
        if (i >= shape_[a]) throw std::out_of_range("index out of range");
        f = f * shape_[a] + i;
    }
    return f;
}

size_t Tensor::rank() const { return shape_.size(); }
size_t Tensor::numel() const {
    size_t n = 1;
    for (size_t d : shape_) n *= d;
    return n;
}
size_t Tensor::dim_size(size_t axis) const {
    if (axis >= shape_.size()) throw std::out_of_range("tensor dimension axis out of range");
    return shape_[axis];
}

void Tensor::add_inplace(const Tensor& o) {
    if (!same_shape(o)) throw std::invalid_argument("tensor shapes must match");
    for (size_t i = 0; i < data_.size(); ++i) data_[i] += o.data_[i];
}
void Tensor::mul_inplace_scalar(float s) {
    for (float& v : data_) v *= s;
}
void Tensor::mul_inplace_broadcast_lastdim(const Tensor& gate) {
    if (rank() != 3 || gate.rank() != 3 || gate.dim_size(0) != dim_size(0) || gate.dim_size(1) != 1 ||
        gate.dim_size(2) != dim_size(2))
        throw std::invalid_argument("gate must have shape {batch, 1, hidden}");
    const size_t B = dim_size(0), T = dim_size(1), C = dim_size(2);
    for (size_t b = 0; b < B; ++b)
        for (size_t t = 0; t < T; ++t)
            for (size_t c = 0; c < C; ++c) data_[(b * T + t) * C + c] *= gate.data_[b * C + c];
}
Tensor Tensor::transpose_2d() const {
    if (rank() != 2) throw std::invalid_argument("transpose_2d requires rank 2");
    Tensor out({shape_[1], shape_[0]});
    for (size_t r = 0; r < shape_[0]; ++r)
        for (size_t c = 0; c < shape_[1]; ++c) out.data_[c * shape_[0] + r] = data_[r * shape_[1] + c];
    return out;
}

Tensor Tensor::layer_norm_3d_lastdim(float eps, const Tensor* gamma, const Tensor* beta) const {
    if (rank() != 3) throw std::invalid_argument("input must be rank 3");
    const size_t C = dim_size(2), rows = numel() / (C ? C : 1);
    Tensor out(shape_);
    if (!numel()) return out;
    sana_shim::check(sana_op_layer_norm(sana_shim::handle(), data_.data(), sana_shim::as_int(rows, "rows"),
                                        sana_shim::as_int(C, "hidden"), eps, sana_shim::opt(gamma),
                                        sana_shim::opt(beta), out.data_.data()));
    return out;
}
Tensor Tensor::rms_norm_3d_lastdim(float eps, const Tensor* weight) const {
    if (rank() != 3) throw std::invalid_argument("input must be rank 3");
    const size_t C = dim_size(2), rows = numel() / (C ? C : 1);
    Tensor out(shape_);
    if (!numel()) return out;
    sana_shim::check(sana_op_rms_norm(sana_shim::handle(), data_.data(), sana_shim::as_int(rows, "rows"),
                                      sana_shim::as_int(C, "hidden"), eps, sana_shim::opt(weight), out.data_.data()));
    return out;
}
Tensor Tensor::modulate_3d_lastdim(const Tensor& shift, const Tensor& scale) const {
    if (rank() != 3) throw std::invalid_argument("input must be rank 3");
    const size_t B = dim_size(0), T = dim_size(1), C = dim_size(2);
    if (shift.numel() != B * C || scale.numel() != B * C)
        throw std::invalid_argument("shift and scale must have shape {batch, 1, hidden}");
    Tensor out(shape_);
    if (!numel()) return out;
    sana_shim::check(sana_op_modulate(sana_shim::handle(), data_.data(), sana_shim::as_int(B, "batch"),
                                      sana_shim::as_int(T, "tokens"), sana_shim::as_int(C, "hidden"), shift.data_.data(),
                                      scale.data_.data(), out.data_.data()));
    return out;
}

Tensor Tensor::tokens_to_grid_4d(size_t height, size_t width) const {
    if (rank() != 3 || dim_size(1) != height * width) throw std::invalid_argument("tokens must equal height * width");
    const size_t B = dim_size(0), HW = dim_size(1), C = dim_size(2);
    Tensor out({B, C, height, width});
    for (size_t b = 0; b < B; ++b)
        for (size_t t = 0; t < HW; ++t)
            for (size_t c = 0; c < C; ++c) out.data_[(b * C + c) * HW + t] = data_[(b * HW + t) * C + c];
    return out;
}
Tensor Tensor::grid_to_tokens_3d() const {
    if (rank() != 4) throw std::invalid_argument("input must be rank 4");
    const size_t B = dim_size(0), C = dim_size(1), HW = dim_size(2) * dim_size(3);
    Tensor out({B, HW, C});
    for (size_t b = 0; b < B; ++b)
        for (size_t c = 0; c < C; ++c)
            for (size_t t = 0; t < HW; ++t) out.data_[(b * HW + t) * C + c] = data_[(b * C + c) * HW + t];
    return out;
}
std::pair<Tensor, Tensor> Tensor::split_channels_4d() const {
    if (rank() != 4 || dim_size(1) % 2) throw std::invalid_argument("channels must be even");
    const size_t B = dim_size(0), C = dim_size(1) / 2, HW = dim_size(2) * dim_size(3);
    Tensor a({B, C, dim_size(2), dim_size(3)}), b2({B, C, dim_size(2), dim_size(3)});
    for (size_t b = 0; b < B; ++b) {
        std::copy(data_.begin() + b * 2 * C * HW, data_.begin() + (b * 2 * C + C) * HW, a.data_.begin() + b * C * HW);
        std::copy(data_.begin() + (b * 2 * C + C) * HW, data_.begin() + (b + 1) * 2 * C * HW,
                  b2.data_.begin() + b * C * HW);
    }
    return {a, b2};
}
std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor> Tensor::split_six_way_3d() const {
    if (rank() != 3 || dim_size(1) != 6) throw std::invalid_argument("input must have shape {batch, 6, hidden}");
    const size_t B = dim_size(0), C = dim_size(2);
    std::vector<Tensor> parts(6, Tensor({B, 1, C}));
    for (size_t k = 0; k < 6; ++k)
        for (size_t b = 0; b < B; ++b)
            std::copy(data_.begin() + (b * 6 + k) * C, data_.begin() + (b * 6 + k + 1) * C,
                      parts[k].data_.begin() + b * C);
    return {parts[0], parts[1], parts[2], parts[3], parts[4], parts[5]};
}
void Tensor::silu_inplace() {
    for (float& v : data_) v = v / (1.0f + std::exp(-v));
}
void Tensor::relu_inplace() {
    for (float& v : data_) v = v > 0.0f ? v : 0.0f;
}
float Tensor::max_abs_diff(const Tensor& o) const {
    if (!same_shape(o)) throw std::invalid_argument("tensor shapes must match");
    float m = 0.0f;
    for (size_t i = 0; i < data_.size(); ++i) m = std::max(m, std::fabs(data_[i] - o.data_[i]));
    return m;
}
float Tensor::mean_abs_diff(const Tensor& o) const {
    if (!same_shape(o)) throw std::invalid_argument("tensor shapes must match");
    double s = 0.0;
    for (size_t i = 0; i < data_.size(); ++i) s += std::fabs(data_[i] - o.data_[i]);
    return data_.empty() ? 0.0f : static_cast<float>(s / data_.size());
}
