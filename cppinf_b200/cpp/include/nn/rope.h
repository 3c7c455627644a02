#pragma once

#include <cstddef>
#include <utility>

#include "tensors/tensor.h"
#include "tensors/tensor_view.h"

namespace cppinf::nn {

// Drop-in for the reference's src/nn/rope.h:12-13.
// Applies split-half RoPE to a rank-3 tensor with head dim in the last axis and the sequence axis at dim 0 or 1.
// Positions start at sequence_position_offset, and the result returns in the input dtype.
tensors::Tensor apply_rope(const tensors::TensorView& input, std::size_t sequence_position_offset = 0,
                           float rope_base = 1000000.0f, std::size_t sequence_dimension = 1);

// Per-head RMSNorm of q [tokens, q_heads, head_dim] and k [tokens, k_heads, head_dim] followed by RoPE at positions
// sequence_position_offset + t, the sequence of src/nn/qwen_attention.cpp:383-390, in one kernel.
std::pair<tensors::Tensor, tensors::Tensor> qk_norm_rope(const tensors::TensorView& query,
                                                         const tensors::TensorView& key,
                                                         const tensors::TensorView& query_norm_weight,
                                                         const tensors::TensorView& key_norm_weight, float epsilon,
                                                         std::size_t sequence_position_offset = 0,
                                                         float rope_base = 1000000.0f);

} // namespace cppinf::nn
