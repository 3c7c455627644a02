#pragma once

#include "tensors/tensor.h"
#include "tensors/tensor_view.h"

namespace cppinf::ops {

// Drop-ins for the reference's src/ops/elementwise_ops.h:10,14. Inputs on the same GPU run there and return a device
// tensor; host inputs are staged to the current GPU and the result comes back to the host. Mixing host and device
// inputs throws std::invalid_argument.

// Adds two tensors with matching shape and f32 or bf16 dtype.
// Preserves the input dtype.
tensors::Tensor add(const tensors::TensorView& lhs, const tensors::TensorView& rhs);

// Multiplies two tensors with matching shape and f32 or bf16 dtype.
// Preserves the input dtype.
tensors::Tensor mul(const tensors::TensorView& lhs, const tensors::TensorView& rhs);

} // namespace cppinf::ops
