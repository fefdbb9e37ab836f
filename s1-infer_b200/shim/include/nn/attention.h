// nn/attention.h -- the attention entry points of s1-infer's KV path
// (reference include/nn/attention.h:6-10), computed on the GPU.
//
// GQA_attention_paged reads K/V through the block-table views of a
// KVBlockPool of this shim; GQA_attention takes contiguous host K/V.  Both
// return a fresh host tensor [q_len, num_q_heads, head_dim] and follow the
// reference's causal rule: row i attends to tokens 0 .. (kv_len - q_len) + i.
// The projection wrappers self_attention / self_attention_quantized are not
// part of this shim (they belong to the weight path).
#pragma once
#include "core/tensor.h"
#include "infer/kv_block_pool.h"

TensorPtr reshape_to_heads(const TensorPtr& input, size_t num_heads, size_t head_dim);

TensorPtr GQA_attention(const TensorPtr& Q, const TensorPtr& K, const TensorPtr& V, size_t num_q_heads,
                        size_t num_kv_heads, size_t head_dim);

TensorPtr GQA_attention_paged(const TensorPtr& Q, const KVView& k_view, const KVView& v_view, size_t num_q_heads,
                              size_t num_kv_heads, size_t head_dim);
