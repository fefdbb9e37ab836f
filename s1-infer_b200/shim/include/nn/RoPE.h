// nn/RoPE.h -- apply_rope of s1-infer (reference include/nn/RoPE.h:4) on the
// GPU: input [seq_len, emb_dim] or [seq_len, num_heads, head_dim]; token i
// rotates at start_pos + i with base 1e6.  Bit-identical to the reference.
#pragma once
#include "core/tensor.h"

TensorPtr apply_rope(const TensorPtr& input, size_t start_pos);
