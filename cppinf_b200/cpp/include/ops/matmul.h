#pragma once

#include <optional>

#include "tensors/dtype.h"
#include "tensors/tensor.h"
#include "tensors/tensor_view.h"

namespace cppinf::ops {

// Drop-in for the reference's src/ops/matmul.h.
struct MatmulOptions {
    std::optional<tensors::DType> output_dtype = std::nullopt;
};

// Multiplies rank-2 [m, k] and [k, n] tensors or rank-3 [b, m, k] and [b, k, n] tensors on the GPU (cppinf_matmul:
// the device decoder's fixed accumulation order). Supports f32 and bf16 inputs. Same-dtype inputs default to the
// same output dtype, while mixed f32/bf16 inputs default to f32 output. BF16 inputs may request an F32 result.
// Strided device views are read in place (a transposed [n, k] weight view takes the vector kernels).
tensors::Tensor matmul(const tensors::TensorView& lhs, const tensors::TensorView& rhs, MatmulOptions options = {});

} // namespace cppinf::ops
