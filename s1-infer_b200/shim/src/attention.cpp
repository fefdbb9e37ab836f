// attention.cpp -- reshape_to_heads, GQA_attention, GQA_attention_paged and
// apply_rope of s1-infer (src/nn/attention.cpp:7-239, src/nn/RoPE.cpp:6-39)
// computed by the B200 engine.  Synchronous, host tensors in and out.
#include "nn/attention.h"

#include <cuda_runtime.h>

#include <stdexcept>

#include "nn/RoPE.h"
#include "s1kv.h"
#include "shim_internal.h"

using namespace s1kv_shim;

namespace {

TensorPtr contiguous(const TensorPtr& t) { return t->is_contiguous() ? t : t->contiguous(); }

const float* host_data(const TensorPtr& t) { return t->data().data() + t->offset(); }

}  // namespace

TensorPtr reshape_to_heads(const TensorPtr& input, size_t num_heads, size_t head_dim) {
    return input->reshape({input->shape()[0], num_heads, head_dim});
}

TensorPtr GQA_attention(const TensorPtr& Q, const TensorPtr& K, const TensorPtr& V, size_t num_q_heads,
                        size_t num_kv_heads, size_t head_dim) {
    auto q = contiguous(Q), k = contiguous(K), v = contiguous(V);
    const size_t q_len = q->shape()[0], kv_len = k->shape()[0];
    auto out = Tensor::create({q_len, num_q_heads, head_dim});
    const size_t qb = q->numel() * 4, kb = k->numel() * 4, vb = v->numel() * 4;
    thread_local DeviceBuffer buf;
    char* d = (char*)buf.get(2 * qb + kb + vb + 64);
    cuda_check(cudaMemcpy(d, host_data(q), qb, cudaMemcpyHostToDevice), "GQA_attention");
    cuda_check(cudaMemcpy(d + qb, host_data(k), kb, cudaMemcpyHostToDevice), "GQA_attention");
    cuda_check(cudaMemcpy(d + qb + kb, host_data(v), vb, cudaMemcpyHostToDevice), "GQA_attention");
    float* dout = (float*)(d + qb + kb + vb);
    check(s1kv_attention_contig((const float*)d, (const float*)(d + qb), (const float*)(d + qb + kb), (int64_t)q_len,
                                (int64_t)kv_len, (int32_t)num_q_heads, (int32_t)num_kv_heads, (int32_t)head_dim, dout,
                                nullptr),
          "GQA_attention");
    cuda_check(cudaMemcpy(out->mutable_data().data(), dout, qb, cudaMemcpyDeviceToHost), "GQA_attention");
    return out;
}

TensorPtr GQA_attention_paged(const TensorPtr& Q, const KVView& k_view, const KVView& v_view, size_t num_q_heads,
                              size_t num_kv_heads, size_t head_dim) {
    const KVBlockPool* pool = pool_of(k_view.base);
    size_t seq = 0, seq_v = 0;
    if (!pool || pool != pool_of(v_view.base) || !pool->sequence_of(k_view.block_table, &seq) ||
        !pool->sequence_of(v_view.block_table, &seq_v) || seq != seq_v)
        throw std::runtime_error("GQA_attention_paged: views do not belong to one live sequence of a pool");
    if (num_kv_heads != pool->num_heads() || head_dim != pool->head_dim())
        throw std::runtime_error("GQA_attention_paged: head shape does not match the pool");
    auto q = contiguous(Q);
    const size_t q_len = q->shape()[0];
    auto out = Tensor::create({q_len, num_q_heads, head_dim});
    const size_t qb = q->numel() * 4;
    thread_local DeviceBuffer buf;
    char* d = (char*)buf.get(2 * qb + 64);
    cuda_check(cudaMemcpy(d, host_data(q), qb, cudaMemcpyHostToDevice), "GQA_attention_paged");
    const uint64_t s = seq;
    const int32_t ql = (int32_t)q_len;
    float* dout = (float*)(d + qb);
    check(s1kv_attention(pool->handle(), 0, &s, &ql, 1, (const float*)d, dout, (int32_t)num_q_heads, nullptr),
          "GQA_attention_paged");
    cuda_check(cudaMemcpy(out->mutable_data().data(), dout, qb, cudaMemcpyDeviceToHost), "GQA_attention_paged");
    return out;
}

TensorPtr apply_rope(const TensorPtr& input, size_t start_pos) {
    auto x = contiguous(input);
    const auto& shape = x->shape();
    const size_t T = shape[0], D = shape.back(), H = shape.size() == 3 ? shape[1] : 1;
    auto out = Tensor::create(shape);
    const size_t bytes = x->numel() * 4;
    if (!bytes) return out;
    thread_local DeviceBuffer buf;
    char* d = (char*)buf.get(2 * bytes + 64);
    cuda_check(cudaMemcpy(d, host_data(x), bytes, cudaMemcpyHostToDevice), "apply_rope");
    check(s1kv_apply_rope((const float*)d, (float*)(d + bytes), (int64_t)start_pos, (int64_t)T, (int32_t)H,
                          (int32_t)D, 0.0f, nullptr),
          "apply_rope");
    cuda_check(cudaMemcpy(out->mutable_data().data(), d + bytes, bytes, cudaMemcpyDeviceToHost), "apply_rope");
    return out;
}
