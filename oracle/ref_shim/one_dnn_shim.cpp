// Scalar stand-ins for the helpers declared in the reference's src/ops/one_dnn_utils.h, so that the reference's own
// op sources (src/ops/*.cpp, src/nn/rope.cpp, src/nn/qwen_attention.cpp) link and run without the oneDNN library.
// TEST INFRASTRUCTURE ONLY (oracle/_ref build).
//
// What each stand-in computes is the documented semantics of the oneDNN primitive the reference configures:
//  - reorder (cast_with_one_dnn): f32 <-> bf16 with round-to-nearest-even, strided source, dense destination;
//  - binary add/sub/mul/div: f32 arithmetic on inputs already in the output dtype, numpy-style broadcast of size-1
//    dims, result stored in the output dtype;
//  - eltwise swish (x / (1 + exp(-alpha x))) and sqrt, computed in f32, stored in the output dtype.
// Functions that would hand oneDNN memory descriptors or engines to a primitive (make_desc, make_memory,
// cpu_engine, ...) throw: reference code that needs a real primitive (rms_norm's reduction, softmax_last_dim,
// matmul, transposes) reports "unavailable" instead of computing anything.
#include <cmath>
#include <cstring>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "ops/one_dnn_utils.h"
#include "ops/op_utils.h"
#include "tensors/tensor_utils.h"

namespace cppinf::ops::detail {
namespace {

[[noreturn]] void unavailable(const char* what) {
    throw std::runtime_error(std::string("oneDNN is not available in this build: ") + what);
}

// Flat index of the broadcast source element for output coordinate `index`.
std::size_t broadcast_index(const tensors::Shape& out_shape, const tensors::Shape& in_shape, std::size_t index) {
    const auto& od = out_shape.dims();
    const auto& id = in_shape.dims();
    std::size_t src = 0;
    std::size_t src_stride = 1;
    std::size_t rem = index;
    for (std::size_t k = od.size(); k-- > 0;) {
        const auto dim = static_cast<std::size_t>(od[k]);
        const auto coord = rem % dim;
        rem /= dim;
        const std::size_t in_axis = k + id.size() - od.size();
        const auto in_dim = static_cast<std::size_t>(id[in_axis]);
        src += (in_dim == 1 ? 0 : coord) * src_stride;
        src_stride *= in_dim;
    }
    return src;
}

float apply_binary(dnnl::algorithm algorithm, float a, float b) {
    switch (algorithm) {
    case dnnl::algorithm::binary_add:
        return a + b;
    case dnnl::algorithm::binary_sub:
        return a - b;
    case dnnl::algorithm::binary_mul:
        return a * b;
    case dnnl::algorithm::binary_div:
        return a / b;
    default:
        unavailable("binary algorithm");
    }
}

float apply_unary(dnnl::algorithm algorithm, float x, float alpha) {
    switch (algorithm) {
    case dnnl::algorithm::eltwise_swish:
        return x / (1.0f + std::exp(-alpha * x));
    case dnnl::algorithm::eltwise_sqrt:
        return std::sqrt(x);
    default:
        unavailable("eltwise algorithm");
    }
}

}  // namespace

const dnnl::engine& cpu_engine() {
    unavailable("cpu_engine");
}

tensors::Tensor make_result_tensor(std::string_view name, tensors::DType dtype, const tensors::Shape& shape) {
    return tensors::Tensor::zeros(tensors::make_result_tensor_info(name, dtype, shape));
}

dnnl::memory::data_type to_dnnl_dtype(tensors::DType dtype) {
    return dtype == tensors::DType::BF16 ? dnnl::memory::data_type::bf16 : dnnl::memory::data_type::f32;
}

dnnl::memory::desc make_dense_desc(const tensors::Shape&, tensors::DType, std::string_view) {
    unavailable("make_dense_desc");
}

dnnl::memory::desc make_desc(const tensors::TensorView&, std::string_view) {
    unavailable("make_desc");
}

dnnl::memory make_memory(const dnnl::memory::desc&, std::span<const std::byte>) {
    unavailable("make_memory");
}

dnnl::memory make_memory(const dnnl::memory::desc&, std::span<std::byte>) {
    unavailable("make_memory");
}

tensors::Tensor cast_with_one_dnn(const tensors::TensorView& input, tensors::DType dtype,
                                  std::string_view result_name) {
    auto result = make_result_tensor(result_name, dtype, input.tensor_info().shape);
    const auto count = input.tensor_info().shape.num_elements();
    for (std::size_t i = 0; i < count; ++i) {
        store_float_value(dtype, result.mutable_data(), i, load_float_value(input, i));
    }
    return result;
}

tensors::TensorView maybe_cast_to_dtype(const tensors::TensorView& input, tensors::DType dtype,
                                        std::optional<tensors::Tensor>& storage, std::string_view result_name) {
    if (input.tensor_info().dtype != dtype) {
        storage = cast_with_one_dnn(input, dtype, result_name);
        return storage->view();
    }
    return input;
}

tensors::Tensor maybe_cast_result(tensors::Tensor tensor, tensors::DType dtype, std::string_view result_name) {
    if (tensor.tensor_info().dtype != dtype) {
        return cast_with_one_dnn(tensor.view(), dtype, result_name);
    }
    return tensor;
}

tensors::Tensor binary_with_one_dnn(std::string_view result_name, const tensors::TensorView& lhs,
                                    const tensors::TensorView& rhs, dnnl::algorithm algorithm,
                                    tensors::DType output_dtype) {
    std::optional<tensors::Tensor> lhs_storage;
    std::optional<tensors::Tensor> rhs_storage;
    const auto a = maybe_cast_to_dtype(lhs, output_dtype, lhs_storage, result_name);
    const auto b = maybe_cast_to_dtype(rhs, output_dtype, rhs_storage, result_name);
    const auto& out_shape = a.tensor_info().shape;
    auto result = make_result_tensor(result_name, output_dtype, out_shape);
    const auto count = out_shape.num_elements();
    for (std::size_t i = 0; i < count; ++i) {
        const float av = load_float_value(a, i);
        const float bv = load_float_value(b, broadcast_index(out_shape, b.tensor_info().shape, i));
        store_float_value(output_dtype, result.mutable_data(), i, apply_binary(algorithm, av, bv));
    }
    return result;
}

tensors::Tensor unary_with_one_dnn(std::string_view result_name, const tensors::TensorView& input,
                                   dnnl::algorithm algorithm, tensors::DType output_dtype, float alpha, float) {
    std::optional<tensors::Tensor> storage;
    const auto x = maybe_cast_to_dtype(input, output_dtype, storage, result_name);
    auto result = make_result_tensor(result_name, output_dtype, x.tensor_info().shape);
    const auto count = x.tensor_info().shape.num_elements();
    for (std::size_t i = 0; i < count; ++i) {
        store_float_value(output_dtype, result.mutable_data(), i, apply_unary(algorithm, load_float_value(x, i), alpha));
    }
    return result;
}

}  // namespace cppinf::ops::detail
