// tensor.cpp -- the shim's host tensor (see core/tensor.h).
#include "core/tensor.h"

#include <stdexcept>

Tensor::Tensor(std::vector<size_t> shape, scalar_t fill_value) : shape_(std::move(shape)) {
    data_ = std::make_shared<std::vector<scalar_t>>(init_strides(), fill_value);
}

Tensor::Tensor(std::vector<size_t> shape, std::vector<scalar_t> data) : shape_(std::move(shape)) {
    if (init_strides() != data.size()) throw std::invalid_argument("Tensor: data size does not match shape");
    data_ = std::make_shared<std::vector<scalar_t>>(std::move(data));
}

Tensor::Tensor(std::shared_ptr<std::vector<scalar_t>> data, std::vector<size_t> shape, std::vector<size_t> strides,
               size_t offset)
    : data_(std::move(data)), shape_(std::move(shape)), strides_(std::move(strides)), offset_(offset) {}

size_t Tensor::init_strides() {
    strides_.assign(shape_.size(), 1);
    size_t n = 1;
    for (size_t i = shape_.size(); i-- > 0;) {
        strides_[i] = n;
        n *= shape_[i];
    }
    return n;
}

size_t Tensor::numel() const {
    size_t n = 1;
    for (size_t s : shape_) n *= s;
    return n;
}

bool Tensor::is_contiguous() const {
    size_t n = 1;
    for (size_t i = shape_.size(); i-- > 0;) {
        if (shape_[i] != 1 && strides_[i] != n) return false;
        n *= shape_[i];
    }
    return true;
}

namespace {
template <typename It>
size_t flat_index(const std::vector<size_t>& shape, const std::vector<size_t>& strides, size_t offset, It b, It e) {
    if ((size_t)(e - b) != shape.size()) throw std::out_of_range("Tensor::at: wrong number of indices");
    size_t pos = offset, i = 0;
    for (It it = b; it != e; ++it, ++i) {
        if (*it >= shape[i]) throw std::out_of_range("Tensor::at: index out of bounds");
        pos += *it * strides[i];
    }
    return pos;
}
}  // namespace

scalar_t& Tensor::at(std::initializer_list<size_t> idx) {
    return (*data_)[flat_index(shape_, strides_, offset_, idx.begin(), idx.end())];
}
scalar_t Tensor::at(std::initializer_list<size_t> idx) const {
    return (*data_)[flat_index(shape_, strides_, offset_, idx.begin(), idx.end())];
}
scalar_t& Tensor::at(const std::vector<size_t>& idx) {
    return (*data_)[flat_index(shape_, strides_, offset_, idx.begin(), idx.end())];
}
scalar_t Tensor::at(const std::vector<size_t>& idx) const {
    return (*data_)[flat_index(shape_, strides_, offset_, idx.begin(), idx.end())];
}

TensorPtr Tensor::reshape(std::vector<size_t> new_shape) const {
    if (!is_contiguous()) throw std::invalid_argument("Tensor::reshape: tensor is not contiguous");
    size_t n = 1;
    for (size_t s : new_shape) n *= s;
    if (n != numel()) throw std::invalid_argument("Tensor::reshape: element count changes");
    std::vector<size_t> st(new_shape.size(), 1);
    size_t acc = 1;
    for (size_t i = new_shape.size(); i-- > 0;) {
        st[i] = acc;
        acc *= new_shape[i];
    }
    return std::make_shared<Tensor>(data_, std::move(new_shape), std::move(st), offset_);
}

TensorPtr Tensor::contiguous() const {
    auto out = std::make_shared<Tensor>(shape_);
    std::vector<size_t> idx(shape_.size(), 0);
    auto& dst = out->mutable_data();
    for (size_t flat = 0; flat < dst.size(); flat++) {
        dst[flat] = at(idx);
        for (size_t i = idx.size(); i-- > 0;) {
            if (++idx[i] < shape_[i]) break;
            idx[i] = 0;
        }
    }
    return out;
}

TensorPtr Tensor::create(std::vector<size_t> shape, scalar_t fill) { return std::make_shared<Tensor>(std::move(shape), fill); }
TensorPtr Tensor::zeros(std::vector<size_t> shape) { return create(std::move(shape), 0.0f); }
TensorPtr Tensor::from_vector(std::vector<scalar_t> data) {
    size_t n = data.size();
    return std::make_shared<Tensor>(std::vector<size_t>{n}, std::move(data));
}
