// ref_capi.cpp -- TEST INFRASTRUCTURE ONLY.  A C-ABI wrapper around the
// reference's own CPU implementation of the KV-cache path, compiled from the
// reference's sources where they lie (oracle/Makefile).  The parity tests use
// it to pin the C restatement (kvoracle.c) and the bench uses it as the timed
// CPU baseline ("kind": "reference").  Nothing in the product links it.
//
// Wrapped reference entry points:
//   KVBlockPool (include/infer/kv_block_pool.h:13-45)
//   apply_rope (include/nn/RoPE.h:4)
//   rmsnorm (include/nn/rmsnorm.h:4)
//   GQA_attention / GQA_attention_paged (include/nn/attention.h:8-10)
//   ThreadPool::parallel_for (include/infer/thread_pool.h:14)
//   quantize_tensor / matmul_quantized_range_blocked / matmul_quantized
//     (include/core/quantized_tensor.h:14-23)
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <vector>

#include "core/quantized_tensor.h"
#include "infer/kv_block_pool.h"
#include "infer/thread_pool.h"
#include "nn/RoPE.h"
#include "nn/attention.h"
#include "nn/rmsnorm.h"

namespace {

TensorPtr make_tensor(const float* data, std::vector<size_t> shape) {
    size_t n = 1;
    for (size_t s : shape) n *= s;
    return std::make_shared<Tensor>(shape, std::vector<scalar_t>(data, data + n));
}

void copy_out(const TensorPtr& t, float* out) {
    const auto& d = t->is_contiguous() ? t->data() : t->contiguous()->data();
    std::memcpy(out, d.data(), d.size() * sizeof(float));
}

}  // namespace

extern "C" {

// Status: 0 ok, 1 std::runtime_error thrown (the reference's only error).
void* ref_pool_new(int64_t H, int64_t D, int64_t max_blocks, int64_t bs) {
    return new KVBlockPool((size_t)H, (size_t)D, (size_t)max_blocks, (size_t)bs);
}

void ref_pool_free(void* p) { delete static_cast<KVBlockPool*>(p); }

int ref_append(void* p, uint64_t seq, const float* k, const float* v, int64_t T, int64_t H, int64_t D) {
    try {
        static_cast<KVBlockPool*>(p)->append(seq, make_tensor(k, {(size_t)T, (size_t)H, (size_t)D}),
                                             make_tensor(v, {(size_t)T, (size_t)H, (size_t)D}));
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

int64_t ref_length(void* p, uint64_t seq) { return (int64_t) static_cast<KVBlockPool*>(p)->length(seq); }

int ref_remove(void* p, uint64_t seq) {
    try {
        static_cast<KVBlockPool*>(p)->remove(seq);
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

int ref_truncate(void* p, uint64_t seq, int64_t keep) {
    try {
        static_cast<KVBlockPool*>(p)->truncate(seq, (size_t)keep);
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

int ref_get(void* p, uint64_t seq, int which, float* out) {
    try {
        auto* pool = static_cast<KVBlockPool*>(p);
        copy_out(which ? pool->get_v(seq) : pool->get_k(seq), out);
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

// Block table through the public KVView (kv_block_pool.h:6-11).
int ref_block_table(void* p, uint64_t seq, int32_t* out, int64_t cap, int64_t* n) {
    try {
        KVView kv = static_cast<KVBlockPool*>(p)->get_k_view(seq);
        int64_t m = (int64_t)kv.block_table->size();
        for (int64_t i = 0; i < m && i < cap; i++) out[i] = (int32_t)(*kv.block_table)[i];
        *n = m;
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

// Raw pool storage ([max_blocks * bs, H, D] fp32) through the view base.
const float* ref_pool_base(void* p, uint64_t seq, int which) {
    try {
        auto* pool = static_cast<KVBlockPool*>(p);
        return which ? pool->get_v_view(seq).base : pool->get_k_view(seq).base;
    } catch (const std::runtime_error&) {
        return nullptr;
    }
}

void ref_apply_rope(const float* x, int64_t T, int64_t H, int64_t D, int64_t start_pos, float* out) {
    TensorPtr in = H > 0 ? make_tensor(x, {(size_t)T, (size_t)H, (size_t)D}) : make_tensor(x, {(size_t)T, (size_t)D});
    copy_out(apply_rope(in, (size_t)start_pos), out);
}

void ref_rmsnorm(const float* x, int64_t rows, int64_t D, const float* w, float eps, float* out) {
    copy_out(rmsnorm(make_tensor(x, {(size_t)rows, (size_t)D}), make_tensor(w, {(size_t)D}), eps), out);
}

void ref_gqa_attention(const float* q, const float* k, const float* v, int64_t q_len, int64_t kv_len, int64_t Hq,
                       int64_t Hkv, int64_t D, float* out) {
    auto Q = make_tensor(q, {(size_t)q_len, (size_t)Hq, (size_t)D});
    auto K = make_tensor(k, {(size_t)kv_len, (size_t)Hkv, (size_t)D});
    auto V = make_tensor(v, {(size_t)kv_len, (size_t)Hkv, (size_t)D});
    copy_out(GQA_attention(Q, K, V, (size_t)Hq, (size_t)Hkv, (size_t)D), out);
}

int ref_gqa_attention_paged(void* p, uint64_t seq, const float* q, int64_t q_len, int64_t Hq, int64_t Hkv, int64_t D,
                            float* out) {
    try {
        auto* pool = static_cast<KVBlockPool*>(p);
        auto Q = make_tensor(q, {(size_t)q_len, (size_t)Hq, (size_t)D});
        copy_out(GQA_attention_paged(Q, pool->get_k_view(seq), pool->get_v_view(seq), (size_t)Hq, (size_t)Hkv,
                                     (size_t)D),
                 out);
        return 0;
    } catch (const std::runtime_error&) {
        return 1;
    }
}

// Decode attention for a batch of sequences over several layer pools, fanned
// out over (layer, sequence) tasks with the reference's ThreadPool.  Every
// task runs GQA_attention_paged for one decode query (q_len 1).  q and out
// are [n_layers][n_seqs][Hq][D].  Attention only reads the pools, so the
// tasks are independent.
void ref_decode_batch(void** pools, int64_t n_layers, const uint64_t* seqs, int64_t n_seqs, const float* q,
                      int64_t Hq, int64_t Hkv, int64_t D, int64_t n_threads, float* out) {
    ThreadPool tp((size_t)n_threads);
    size_t per = (size_t)(Hq * D);
    tp.parallel_for((size_t)(n_layers * n_seqs), [&](size_t start, size_t end) {
        for (size_t t = start; t < end; t++) {
            size_t l = t / (size_t)n_seqs, s = t % (size_t)n_seqs;
            auto* pool = static_cast<KVBlockPool*>(pools[l]);
            auto Q = make_tensor(q + t * per, {1, (size_t)Hq, (size_t)D});
            auto O = GQA_attention_paged(Q, pool->get_k_view(seqs[s]), pool->get_v_view(seqs[s]), (size_t)Hq,
                                         (size_t)Hkv, (size_t)D);
            copy_out(O, out + t * per);
        }
    });
}

// quantize_tensor on a [rows][cols] matrix: q (int8) and one scale per row.
void ref_quantize_tensor(const float* w, int64_t rows, int64_t cols, int8_t* q, float* scales) {
    Tensor t({(size_t)rows, (size_t)cols}, std::vector<scalar_t>(w, w + rows * cols));
    QuantizedTensor qt = quantize_tensor(t);
    std::memcpy(q, qt.data.data(), qt.data.size());
    std::memcpy(scales, qt.scales.data(), qt.scales.size() * sizeof(float));
}

static QuantizedTensor make_qt(const int8_t* q, const float* s, int64_t K, int64_t N) {
    QuantizedTensor qt;
    qt.data.assign(q, q + K * N);
    qt.scales.assign(s, s + K);
    qt.rows = (size_t)K;
    qt.cols = (size_t)N;
    return qt;
}

// matmul_quantized_range_blocked over all columns, on the calling thread.
void ref_matmul_quantized_blocked(const float* x, int64_t M, int64_t K, const int8_t* q, const float* s, int64_t N,
                                  float* out) {
    QuantizedTensor qt = make_qt(q, s, K, N);
    matmul_quantized_range_blocked(x, qt, out, (size_t)M, (size_t)K, (size_t)N, 0, (size_t)N);
}

// matmul_quantized: the reference's public entry, fanned out over its
// ThreadPool (get_pool()) when N >= 512.  `qt` is built once by
// ref_qt_new so that a timed loop measures the multiply alone.
void* ref_qt_new(const int8_t* q, const float* s, int64_t K, int64_t N) {
    return new QuantizedTensor(make_qt(q, s, K, N));
}
void ref_qt_free(void* qt) { delete static_cast<QuantizedTensor*>(qt); }
void ref_matmul_quantized(const float* x, int64_t M, int64_t K, void* qt, float* out) {
    auto* w = static_cast<QuantizedTensor*>(qt);
    copy_out(matmul_quantized(make_tensor(x, {(size_t)M, (size_t)K}), *w), out);
}

}  // extern "C"
