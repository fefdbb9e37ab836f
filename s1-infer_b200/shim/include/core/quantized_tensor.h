// core/quantized_tensor.h -- the reference's int8 weight interface
// (include/core/quantized_tensor.h:7-23 of s1-infer) computed by the B200
// engine: quantize_tensor and the products run on the GPU (s1kv.h:
// s1kv_quantize_rows, s1kv_matmul_int8).  Same names, members and meaning;
// one addition: a cached device copy of data/scales, made on first use by a
// product and remade when data or scales change size or address.
#pragma once
#include <cstdint>
#include <memory>
#include <vector>

#include "core/tensor.h"

struct QuantizedTensor {
    std::vector<int8_t> data;
    std::vector<float> scales;  // one scale per row
    size_t rows;
    size_t cols;
    mutable std::shared_ptr<void> device;  // engine-side copy (not in the reference)
};

QuantizedTensor quantize_tensor(const Tensor& t);

float dequantize(const QuantizedTensor& qt, size_t row, size_t col);

void matmul_quantized_range_blocked(const scalar_t* a, const QuantizedTensor& b, scalar_t* out, size_t M, size_t K,
                                    size_t N, size_t col_start, size_t col_end);

TensorPtr matmul_quantized(const TensorPtr& x, const QuantizedTensor& w);
