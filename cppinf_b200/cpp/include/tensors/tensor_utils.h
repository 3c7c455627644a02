#pragma once

#include <cstdint>
#include <span>
#include <string_view>

#include "tensors/shape.h"
#include "tensors/tensor.h"
#include "tensors/tensor_info.h"

namespace cppinf::tensors {

// Tensor factories of the reference's src/tensors/tensor_utils.h:20-93 (host tensors).

// Returns zero-offset metadata for a newly created output tensor.
TensorInfo make_result_tensor_info(std::string_view name, DType dtype, const Shape& shape);

// Returns an owned float tensor with bytes encoded in the requested model dtype.
Tensor make_float_tensor(std::string_view name, DType dtype, const Shape& shape, std::span<const float> values);

// Returns an owned f32 tensor from literal float values.
Tensor make_f32_tensor(std::string_view name, const Shape& shape, std::span<const float> values);

// Returns an owned bf16 tensor from literal float values.
Tensor make_bf16_tensor(std::string_view name, const Shape& shape, std::span<const float> values);

// Returns an owned bf16 tensor from already-quantized bf16 bit patterns.
Tensor make_bf16_bits_tensor(std::string_view name, const Shape& shape, std::span<const std::uint16_t> values);

// Returns an owned tensor copy with the same bytes and a different tensor name (same device).
Tensor rename_tensor(std::string_view name, const Tensor& tensor);

// Returns an owned dense copy of a view, on the view's device. Strided device views are gathered by a device kernel.
Tensor materialize_tensor(std::string_view name, const TensorView& tensor_view);

} // namespace cppinf::tensors
