// infer/kv_block_pool.h -- KVBlockPool / KVView of s1-infer backed by the
// B200 engine (include/s1kv.h).
//
// Same names, signatures and error behaviour as the reference's
// include/infer/kv_block_pool.h:6-45: append / get_k / get_v / length /
// remove / truncate / get_k_view / get_v_view, std::runtime_error on an
// exhausted free list (after the tokens that fit are stored) and on unknown
// sequence ids.  Storage is a device-resident fp32 pool; calls are
// synchronous like the reference's.
//
// KVView::base is the DEVICE address of the pool's K (or V) storage and
// block_table points at a host mirror of the sequence's table; both stay
// valid until the next mutation of that sequence, as in the reference.
// Views are meant for GQA_attention_paged (include/nn/attention.h), which
// finds the pool and sequence from them; do not dereference base on the host.
#pragma once
#include <cstdint>
#include <unordered_map>
#include <vector>

#include "core/tensor.h"

struct s1kv_pool;

struct KVView {
    const scalar_t* base;
    const std::vector<size_t>* block_table;
    size_t block_size;
    size_t total_tokens;
};

class KVBlockPool {
   public:
    KVBlockPool(size_t num_heads, size_t head_dim, size_t max_blocks, size_t block_size = 16);
    ~KVBlockPool();
    KVBlockPool(KVBlockPool&& other) noexcept;
    KVBlockPool& operator=(KVBlockPool&&) = delete;
    KVBlockPool(const KVBlockPool&) = delete;
    KVBlockPool& operator=(const KVBlockPool&) = delete;

    void append(size_t sequence_id, const TensorPtr& k, const TensorPtr& v);
    TensorPtr get_k(size_t sequence_id) const;
    TensorPtr get_v(size_t sequence_id) const;
    size_t length(size_t sequence_id) const;

    void remove(size_t sequence_id);

    void truncate(size_t sequence_id, size_t keep_length);

    KVView get_k_view(size_t sequence_id) const;
    KVView get_v_view(size_t sequence_id) const;

    // Engine handle, for callers that want the C ABI (batched steps).
    s1kv_pool* handle() const { return pool_; }
    // The sequence whose view block_table points at (false if none).
    bool sequence_of(const std::vector<size_t>* block_table, size_t* sequence_id) const;
    size_t num_heads() const { return num_heads_; }
    size_t head_dim() const { return head_dim_; }

   private:
    s1kv_pool* pool_ = nullptr;
    size_t num_heads_, head_dim_, block_size_;
    mutable std::unordered_map<size_t, std::vector<size_t>> tables_;  // host mirrors behind KVView
    void refresh(size_t sequence_id) const;
    TensorPtr gather(size_t sequence_id, int which) const;
    KVView view(size_t sequence_id, int which) const;
};
