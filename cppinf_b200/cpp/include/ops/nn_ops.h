#pragma once

#include <cstdint>
#include <utility>
#include <vector>

#include "tensors/tensor.h"
#include "tensors/tensor_view.h"

namespace cppinf::ops {

// Drop-ins for the reference's src/ops/nn_ops.h:9-22, with the same device rules as elementwise_ops.h.

// Applies SiLU elementwise and preserves the input shape and dtype.
tensors::Tensor silu(const tensors::TensorView& input);

// Applies softmax over the last dimension and preserves the dtype.
// Shapes: [d0, ..., dn] -> [d0, ..., dn].
tensors::Tensor softmax_last_dim(const tensors::TensorView& input);

// Applies f32 scale, causal masking over the last two dimensions, and softmax over the last dimension.
// Shapes: [batch..., query, key] -> [batch..., query, key].
tensors::Tensor scaled_causal_softmax_last_dim(const tensors::TensorView& input, float scale);

// Applies RMSNorm over the last dimension using a rank-1 weight tensor of matching width.
// Shapes: [d0, ..., width], [width] -> [d0, ..., width].
// BF16 inputs are computed in f32 and cast back to bf16 for the result.
tensors::Tensor rms_norm(const tensors::TensorView& input, const tensors::TensorView& weight, float epsilon);

// Fused forms used by the Qwen3 decoder block.

// Residual add then RMSNorm (src/nn/qwen_decoder_block.cpp:80-84): returns {lhs + rhs, rms_norm(lhs + rhs)}.
std::pair<tensors::Tensor, tensors::Tensor> add_rms_norm(const tensors::TensorView& lhs, const tensors::TensorView& rhs,
                                                         const tensors::TensorView& weight, float epsilon);

// mul(silu(gate), up) in one pass (src/nn/qwen_mlp.cpp:65-66), with the silu result rounded to the dtype first.
tensors::Tensor silu_mul(const tensors::TensorView& gate, const tensors::TensorView& up);

// Greedy pick of src/cli/cli_app.cpp:72-94 for every row of rank-2 logits [rows, vocab]: int64 ids are returned as a
// host std::vector (the only value the decode loop reads back).
std::vector<std::int64_t> row_argmax(const tensors::TensorView& logits);

} // namespace cppinf::ops
