// quantized_tensor.cpp -- quantize_tensor / dequantize /
// matmul_quantized_range_blocked / matmul_quantized of s1-infer
// (src/quantized_tensor.cpp:9-122) on the B200 engine.  Synchronous, host
// data in and out like the reference; quantization is bit-exact, products
// agree within 2e-5 of the output scale (the engine sums over k in a tree).
#include "core/quantized_tensor.h"

#include <cuda_runtime.h>

#include <stdexcept>

#include "s1kv.h"
#include "shim_internal.h"

using namespace s1kv_shim;

namespace {

// Device copy of a QuantizedTensor's data and scales.
struct DeviceWeights {
    int8_t* q = nullptr;
    float* scales = nullptr;
    const void* host_q = nullptr;
    const void* host_s = nullptr;
    size_t n = 0, rows = 0;
    ~DeviceWeights() {
        cudaFree(q);
        cudaFree(scales);
    }
};

DeviceWeights& device_weights(const QuantizedTensor& w) {
    if (w.data.size() != w.rows * w.cols || w.scales.size() != w.rows)
        throw std::runtime_error("QuantizedTensor: data/scales do not match rows x cols");
    auto* d = static_cast<DeviceWeights*>(w.device.get());
    if (!d || d->host_q != w.data.data() || d->host_s != w.scales.data() || d->n != w.data.size() || d->rows != w.rows) {
        auto fresh = std::make_shared<DeviceWeights>();
        cuda_check(cudaMalloc(&fresh->q, w.data.size() + 16), "matmul_quantized");
        cuda_check(cudaMalloc(&fresh->scales, w.rows * sizeof(float) + 16), "matmul_quantized");
        cuda_check(cudaMemcpy(fresh->q, w.data.data(), w.data.size(), cudaMemcpyHostToDevice), "matmul_quantized");
        cuda_check(cudaMemcpy(fresh->scales, w.scales.data(), w.rows * sizeof(float), cudaMemcpyHostToDevice),
                   "matmul_quantized");
        fresh->host_q = w.data.data();
        fresh->host_s = w.scales.data();
        fresh->n = w.data.size();
        fresh->rows = w.rows;
        w.device = fresh;
        d = fresh.get();
    }
    return *d;
}

// out_dev [M][N] = a_dev [M][K] * w on the default stream, synchronised.
void product(const float* a_dev, const QuantizedTensor& w, float* out_dev, size_t M) {
    DeviceWeights& d = device_weights(w);
    check(s1kv_matmul_int8(a_dev, (int64_t)M, (int64_t)w.rows, d.q, d.scales, (int64_t)w.cols, out_dev, nullptr),
          "matmul_quantized");
    cuda_check(cudaDeviceSynchronize(), "matmul_quantized");
}

}  // namespace

QuantizedTensor quantize_tensor(const Tensor& t) {
    if (t.shape().size() != 2) throw std::runtime_error("quantize_tensor: a 2-D tensor is needed");
    TensorPtr copy = t.is_contiguous() ? nullptr : t.contiguous();  // t may live outside a shared_ptr
    const float* src = copy ? copy->data().data() : t.data().data() + t.offset();
    QuantizedTensor r;
    r.rows = t.shape()[0];
    r.cols = t.shape()[1];
    r.data.resize(r.rows * r.cols);
    r.scales.resize(r.rows);
    const size_t n = r.rows * r.cols;
    thread_local DeviceBuffer buf;
    char* d = (char*)buf.get(n * 4 + n + r.rows * 4 + 64);
    float* dw = (float*)d;
    int8_t* dq = (int8_t*)(d + n * 4);
    float* ds = (float*)(d + ((n * 4 + n + 15) / 16) * 16);
    cuda_check(cudaMemcpy(dw, src, n * 4, cudaMemcpyHostToDevice), "quantize_tensor");
    check(s1kv_quantize_rows(dw, (int64_t)r.rows, (int64_t)r.cols, dq, ds, nullptr), "quantize_tensor");
    cuda_check(cudaMemcpy(r.data.data(), dq, n, cudaMemcpyDeviceToHost), "quantize_tensor");
    cuda_check(cudaMemcpy(r.scales.data(), ds, r.rows * 4, cudaMemcpyDeviceToHost), "quantize_tensor");
    return r;
}

float dequantize(const QuantizedTensor& qt, size_t row, size_t col) {
    return static_cast<float>(qt.data[row * qt.cols + col]) * qt.scales[row];
}

void matmul_quantized_range_blocked(const scalar_t* a, const QuantizedTensor& b, scalar_t* out, size_t M, size_t K,
                                    size_t N, size_t col_start, size_t col_end) {
    if (K != b.rows || N != b.cols || col_start > col_end || col_end > N)
        throw std::runtime_error("matmul_quantized_range_blocked: shape mismatch");
    if (M == 0 || col_start == col_end) return;
    thread_local DeviceBuffer buf;
    char* d = (char*)buf.get(M * K * 4 + M * N * 4 + 64);
    float* da = (float*)d;
    float* dout = (float*)(d + ((M * K * 4 + 15) / 16) * 16);
    cuda_check(cudaMemcpy(da, a, M * K * 4, cudaMemcpyHostToDevice), "matmul_quantized_range_blocked");
    product(da, b, dout, M);
    // columns [col_start, col_end) of every row, as the reference writes them
    cuda_check(cudaMemcpy2D(out + col_start, N * 4, dout + col_start, N * 4, (col_end - col_start) * 4, M,
                            cudaMemcpyDeviceToHost),
               "matmul_quantized_range_blocked");
}

TensorPtr matmul_quantized(const TensorPtr& x, const QuantizedTensor& w) {
    auto c = x->is_contiguous() ? x : x->contiguous();
    const size_t M = c->shape()[0], K = c->shape()[1];
    if (K != w.rows) throw std::runtime_error("matmul_quantized: x columns do not match the weight rows");
    auto out = Tensor::create({M, w.cols});
    matmul_quantized_range_blocked(c->data().data() + c->offset(), w, out->mutable_data().data(), M, K, w.cols, 0,
                                   w.cols);
    return out;
}
