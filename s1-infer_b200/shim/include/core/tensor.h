// core/tensor.h -- host tensor of the reference-interface shim.
//
// A strided fp32 host container with the names and signatures that the
// KV-cache path of s1-infer uses (include/core/tensor.h:5-69 of the
// reference: scalar_t, TensorPtr, shape/strides/at/data/reshape/contiguous
// and the factories).  It is only the I/O type of the shim; the KV storage
// and all compute live on the GPU behind include/s1kv.h.
#pragma once
#include <initializer_list>
#include <memory>
#include <vector>

using scalar_t = float;
class Tensor;
using TensorPtr = std::shared_ptr<Tensor>;

class Tensor : public std::enable_shared_from_this<Tensor> {
   public:
    Tensor(std::vector<size_t> shape, scalar_t fill_value = 0.0f);
    Tensor(std::vector<size_t> shape, std::vector<scalar_t> data);
    Tensor(std::shared_ptr<std::vector<scalar_t>> data, std::vector<size_t> shape, std::vector<size_t> strides,
           size_t offset);

    const std::vector<size_t>& shape() const { return shape_; }
    const std::vector<size_t>& strides() const { return strides_; }
    size_t rank() const { return shape_.size(); }
    size_t numel() const;
    bool is_contiguous() const;

    scalar_t& at(std::initializer_list<size_t> idx);
    scalar_t at(std::initializer_list<size_t> idx) const;
    scalar_t& at(const std::vector<size_t>& idx);
    scalar_t at(const std::vector<size_t>& idx) const;

    const std::vector<scalar_t>& data() const { return *data_; }
    std::vector<scalar_t>& mutable_data() { return *data_; }
    size_t offset() const { return offset_; }

    TensorPtr reshape(std::vector<size_t> new_shape) const;  // view; needs a contiguous tensor
    TensorPtr contiguous() const;                            // fresh contiguous copy

    static TensorPtr create(std::vector<size_t> shape, scalar_t fill = 0.0f);
    static TensorPtr zeros(std::vector<size_t> shape);
    static TensorPtr from_vector(std::vector<scalar_t> data);

   private:
    std::shared_ptr<std::vector<scalar_t>> data_;
    std::vector<size_t> shape_;
    std::vector<size_t> strides_;
    size_t offset_ = 0;
    size_t init_strides();
};
