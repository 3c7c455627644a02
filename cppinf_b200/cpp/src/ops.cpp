// Drop-in implementations of cppinf's op API (src/ops/elementwise_ops.h, src/ops/nn_ops.h, src/ops/tensor_ops.h,
// src/nn/rope.h) on the sm_100a kernels of the C ABI (include/cppinf_b200.h).
//
// Every op validates its arguments with the reference's checks and messages first, then runs on a GPU:
//  - inputs on one GPU: the op enqueues on the calling thread's current stream and returns a device tensor;
//  - host inputs: they are copied to the current GPU, the op runs there, and the result is copied back, so existing
//    host callers get the same values without a CPU code path;
//  - mixing host and device inputs, or two GPUs, throws std::invalid_argument.
// Result tensors carry the reference's result names ("rms_norm_result", "add_result", ...).
#include <cuda_runtime.h>

#include <cmath>
#include <format>
#include <limits>
#include <map>
#include <mutex>
#include <array>
#include <optional>
#include <stdexcept>
#include <string_view>
#include <tuple>
#include <vector>

#include "common/checked.h"
#include "cppinf_b200.h"
#include "cuda/runtime.h"
#include "nn/rope.h"
#include "ops/elementwise_ops.h"
#include "ops/nn_ops.h"
#include "ops/matmul.h"
#include "ops/tensor_ops.h"
#include "tensors/tensor_utils.h"

namespace cppinf {
namespace {

using tensors::Device;
using tensors::DType;
using tensors::Shape;
using tensors::Tensor;
using tensors::TensorInfo;
using tensors::TensorView;

cppinf_dtype abi_dtype(DType dtype) {
    return dtype == DType::BF16 ? CPPINF_DTYPE_BF16 : CPPINF_DTYPE_F32;
}

// ops::detail::validate_supported_float_dtype, src/ops/op_utils.h:18-27
void validate_supported_float_dtype(DType dtype, std::string_view op_name) {
    if (dtype == DType::BF16 || dtype == DType::F32) {
        return;
    }
    throw std::invalid_argument(std::format("{} received an unsupported dtype.", op_name));
}

int current_device() {
    int device = 0;
    cuda::check(cudaGetDevice(&device), "cudaGetDevice");
    return device;
}

// Where an op runs: the GPU all device inputs share, or the current GPU for all-host inputs.
struct Placement {
    bool host_inputs;
    Device device;
};

Placement place(std::initializer_list<const TensorView*> inputs, std::string_view op_name) {
    const Device first = (*inputs.begin())->device();
    for (const auto* input : inputs) {
        if (!(input->device() == first)) {
            throw std::invalid_argument(std::format("{} requires all inputs on the same device.", op_name));
        }
    }
    if (first.is_cuda()) {
        return {false, first};
    }
    return {true, Device::cuda(current_device())};
}

// A dense copy of an input on the op's GPU (or the input itself when it already is one).
class DeviceOperand {
  public:
    DeviceOperand(const TensorView& view, const Device& device) {
        if (view.device().is_cuda()) {
            if (view.is_contiguous()) {
                ptr_ = view.data().data();
            } else {
                owned_ = tensors::materialize_tensor(view.tensor_info().name, view);
                ptr_ = owned_->data().data();
            }
            return;
        }
        const auto host = view.is_contiguous()
                              ? std::optional<Tensor>()
                              : std::optional<Tensor>(tensors::materialize_tensor(view.tensor_info().name, view));
        const auto* src = host ? host->data().data() : view.data().data();
        owned_ = Tensor::empty(tensors::make_result_tensor_info(view.tensor_info().name, view.tensor_info().dtype,
                                                                view.tensor_info().shape),
                               device);
        if (owned_->byte_size() != 0) {
            cuda::check(cudaMemcpyAsync(owned_->mutable_data().data(), src, owned_->byte_size(),
                                        cudaMemcpyHostToDevice, cuda::current_stream()),
                        "cudaMemcpyAsync(host to device)");
            cuda::check(cudaStreamSynchronize(cuda::current_stream()), "cudaStreamSynchronize");
        }
        ptr_ = owned_->data().data();
    }

    const void* get() const { return ptr_; }

  private:
    std::optional<Tensor> owned_;
    const void* ptr_ = nullptr;
};

// Switches to the op's GPU for the duration of a call.
class DeviceScope {
  public:
    explicit DeviceScope(const Device& device) {
        cuda::check(cudaGetDevice(&previous_), "cudaGetDevice");
        if (previous_ != device.index) {
            cuda::check(cudaSetDevice(device.index), "cudaSetDevice");
        }
    }
    ~DeviceScope() { cudaSetDevice(previous_); }
    DeviceScope(const DeviceScope&) = delete;
    DeviceScope& operator=(const DeviceScope&) = delete;

  private:
    int previous_ = 0;
};

Tensor finish(Tensor result, const Placement& placement) {
    return placement.host_inputs ? result.to(Device::host()) : result;
}

void* out_ptr(Tensor& t) {
    return t.mutable_data().data();
}

// validate_elementwise_inputs, src/ops/elementwise_ops.cpp:14-24
void validate_elementwise_inputs(const TensorView& lhs, const TensorView& rhs, std::string_view op_name) {
    if (lhs.tensor_info().dtype != rhs.tensor_info().dtype) {
        throw std::invalid_argument(std::format("{} requires matching tensor dtypes.", op_name));
    }
    if (!(lhs.tensor_info().shape == rhs.tensor_info().shape)) {
        throw std::invalid_argument(std::format("{} requires matching tensor shapes.", op_name));
    }
    validate_supported_float_dtype(lhs.tensor_info().dtype, op_name);
}

// validate_last_dim_operation_input, src/ops/nn_ops.cpp:30-40
void validate_last_dim_operation_input(const TensorView& input, std::string_view op_name) {
    validate_supported_float_dtype(input.tensor_info().dtype, op_name);
    if (input.tensor_info().shape.rank() == 0) {
        throw std::invalid_argument(std::format("{} requires a tensor with rank at least 1.", op_name));
    }
    if (common::checked_non_negative_dim_to_size(input.tensor_info().shape.dims().back(),
                                                 std::format("{} last dim", op_name)) == 0) {
        throw std::invalid_argument(std::format("{} requires a non-empty last dimension.", op_name));
    }
}

// Checks of src/ops/nn_ops.cpp:140-159.
void validate_rms_norm(const TensorView& input, const TensorView& weight, float epsilon) {
    validate_last_dim_operation_input(input, "rms_norm");
    if (epsilon < 0.0f) {
        throw std::invalid_argument("rms_norm requires a non-negative epsilon.");
    }
    if (input.tensor_info().dtype != weight.tensor_info().dtype) {
        throw std::invalid_argument("rms_norm requires matching tensor dtypes.");
    }
    if (weight.tensor_info().shape.rank() != 1) {
        throw std::invalid_argument("rms_norm requires a rank-1 weight tensor.");
    }
    const auto last_dim =
        common::checked_non_negative_dim_to_size(input.tensor_info().shape.dims().back(), "rms_norm last dim");
    if (common::checked_non_negative_dim_to_size(weight.tensor_info().shape.dims()[0], "rms_norm weight size") !=
        last_dim) {
        throw std::invalid_argument("rms_norm weight size must match the input last dimension.");
    }
}

using BinaryEntry = int (*)(cppinf_dtype, const void*, const void*, void*, int64_t, void*);

Tensor binary_op(const TensorView& lhs, const TensorView& rhs, std::string_view op_name, std::string_view result_name,
                 BinaryEntry entry) {
    validate_elementwise_inputs(lhs, rhs, op_name);
    const auto placement = place({&lhs, &rhs}, op_name);
    DeviceScope scope(placement.device);
    const DeviceOperand a(lhs, placement.device);
    const DeviceOperand b(rhs, placement.device);
    const auto& info = lhs.tensor_info();
    auto result = Tensor::empty(tensors::make_result_tensor_info(result_name, info.dtype, info.shape),
                                placement.device);
    cuda::check_status(entry(abi_dtype(info.dtype), a.get(), b.get(), out_ptr(result),
                             static_cast<int64_t>(info.shape.num_elements()), cuda::current_stream()),
                       std::string(op_name).c_str());
    return finish(std::move(result), placement);
}

// Device RoPE angle tables (cppinf_rope_table), cached per (device, base, head_dim) and grown on demand.
const float* rope_table_for(const Device& device, float base, std::int64_t head_dim, std::int64_t positions,
                        std::int64_t& table_positions) {
    static std::mutex mutex;
    static std::map<std::tuple<int, float, std::int64_t>, std::pair<Tensor, std::int64_t>> tables;
    std::lock_guard<std::mutex> lock(mutex);
    const auto key = std::make_tuple(device.index, base, head_dim);
    auto it = tables.find(key);
    if (it == tables.end() || it->second.second < positions) {
        std::int64_t n = 64;
        while (n < positions) {
            n *= 2;
        }
        std::vector<float> host(static_cast<std::size_t>(n * head_dim));
        cuda::check_status(cppinf_rope_table(base, head_dim, n, host.data()), "rope_table");
        auto info = tensors::make_result_tensor_info("rope_table", DType::F32,
                                                     Shape({n, head_dim}));
        auto table = Tensor::empty(std::move(info), device);
        cuda::check(cudaMemcpy(out_ptr(table), host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice),
                    "cudaMemcpy(rope table)");
        it = tables.insert_or_assign(key, std::make_pair(std::move(table), n)).first;
    }
    table_positions = it->second.second;
    return static_cast<const float*>(static_cast<const void*>(it->second.first.data().data()));
}

// A strided device gather producing `out_shape` from `view` with the given element strides.
Tensor gather(const TensorView& input, const Placement& placement, std::string_view result_name,
              const std::vector<std::int64_t>& dims, const std::vector<std::int64_t>& elem_strides,
              const Shape& out_shape) {
    const auto& info = input.tensor_info();
    // A host input is staged whole (dense) first; its dense strides then apply.
    const DeviceOperand src(input, placement.device);
    auto result = Tensor::empty(tensors::make_result_tensor_info(result_name, info.dtype, out_shape),
                                placement.device);
    if (result.byte_size() != 0) {
        cuda::check_status(cppinf_strided_copy(abi_dtype(info.dtype), src.get(), static_cast<int64_t>(dims.size()),
                                               dims.data(), elem_strides.data(), out_ptr(result),
                                               cuda::current_stream()),
                           std::string(result_name).c_str());
    }
    return finish(std::move(result), placement);
}

// Element strides of the input as the gather kernel will see it (dense for staged host inputs or materialised
// device views).
std::vector<std::int64_t> operand_strides(const TensorView& input) {
    const auto element = tensors::element_size_bytes(input.tensor_info().dtype);
    const auto strides = (input.device().is_cuda() && input.is_contiguous()) || !input.device().is_cuda()
                             ? tensors::dense_strides_bytes(input.tensor_info())
                             : input.strides_bytes();
    std::vector<std::int64_t> out;
    for (const auto s : strides) {
        out.push_back(static_cast<std::int64_t>(s / element));
    }
    return out;
}

} // namespace

namespace ops {

// ---- elementwise_ops.h -------------------------------------------------------------------------------------------

tensors::Tensor add(const tensors::TensorView& lhs, const tensors::TensorView& rhs) {
    return binary_op(lhs, rhs, "add", "add_result", &cppinf_add);
}

tensors::Tensor mul(const tensors::TensorView& lhs, const tensors::TensorView& rhs) {
    return binary_op(lhs, rhs, "mul", "mul_result", &cppinf_mul);
}

// ---- nn_ops.h ----------------------------------------------------------------------------------------------------

tensors::Tensor silu(const tensors::TensorView& input) {
    validate_supported_float_dtype(input.tensor_info().dtype, "silu");
    const auto placement = place({&input}, "silu");
    DeviceScope scope(placement.device);
    const DeviceOperand x(input, placement.device);
    const auto& info = input.tensor_info();
    auto result = Tensor::empty(tensors::make_result_tensor_info("silu_result", info.dtype, info.shape),
                                placement.device);
    cuda::check_status(cppinf_silu(abi_dtype(info.dtype), x.get(), out_ptr(result),
                                   static_cast<int64_t>(info.shape.num_elements()), cuda::current_stream()),
                       "silu");
    return finish(std::move(result), placement);
}

tensors::Tensor softmax_last_dim(const tensors::TensorView& input) {
    validate_last_dim_operation_input(input, "softmax_last_dim");
    const auto placement = place({&input}, "softmax_last_dim");
    DeviceScope scope(placement.device);
    const DeviceOperand x(input, placement.device);
    const auto& info = input.tensor_info();
    const auto width = info.shape.dims().back();
    auto result = Tensor::empty(tensors::make_result_tensor_info("softmax_last_dim_result", info.dtype, info.shape),
                                placement.device);
    cuda::check_status(cppinf_softmax_last_dim(abi_dtype(info.dtype), x.get(), out_ptr(result),
                                               static_cast<int64_t>(info.shape.num_elements()) / width, width,
                                               cuda::current_stream()),
                       "softmax_last_dim");
    return finish(std::move(result), placement);
}

tensors::Tensor scaled_causal_softmax_last_dim(const tensors::TensorView& input, float scale) {
    // src/ops/nn_ops.cpp:77-98
    validate_last_dim_operation_input(input, "scaled_causal_softmax_last_dim");
    if (input.tensor_info().shape.rank() < 2) {
        throw std::invalid_argument("scaled_causal_softmax_last_dim requires a tensor with rank at least 2.");
    }
    if (!std::isfinite(scale)) {
        throw std::invalid_argument("scaled_causal_softmax_last_dim requires a finite scale.");
    }
    const auto& dims = input.tensor_info().shape.dims();
    const auto query_length = common::checked_non_negative_dim_to_size(
        dims[dims.size() - 2], "scaled_causal_softmax_last_dim query length");
    const auto key_length = common::checked_non_negative_dim_to_size(dims[dims.size() - 1],
                                                                     "scaled_causal_softmax_last_dim key length");
    if (query_length == 0 || key_length == 0) {
        throw std::invalid_argument("scaled_causal_softmax_last_dim requires non-empty attention dimensions.");
    }
    if (query_length != key_length) {
        throw std::invalid_argument("scaled_causal_softmax_last_dim requires square attention score matrices.");
    }
    const auto placement = place({&input}, "scaled_causal_softmax_last_dim");
    DeviceScope scope(placement.device);
    const auto& info = input.tensor_info();
    std::optional<Tensor> f32_input;
    const DeviceOperand staged(input, placement.device);
    const void* x = staged.get();
    const auto count = static_cast<int64_t>(info.shape.num_elements());
    if (info.dtype != DType::F32) {
        // maybe_cast_to_dtype(input, F32): the reference computes in f32 (src/ops/nn_ops.cpp:100-102).
        f32_input = Tensor::empty(tensors::make_result_tensor_info("scaled_causal_softmax_last_dim_result",
                                                                   DType::F32, info.shape),
                                  placement.device);
        cuda::check_status(cppinf_cast(abi_dtype(info.dtype), x, CPPINF_DTYPE_F32, out_ptr(*f32_input), count,
                                       cuda::current_stream()),
                           "cast");
        x = f32_input->data().data();
    }
    auto result = Tensor::empty(
        tensors::make_result_tensor_info("scaled_causal_softmax_last_dim_result", DType::F32, info.shape),
        placement.device);
    const auto n = static_cast<int64_t>(query_length);
    cuda::check_status(cppinf_scaled_causal_softmax_f32(static_cast<const float*>(x),
                                                        static_cast<float*>(out_ptr(result)), count / (n * n), n, n,
                                                        scale, cuda::current_stream()),
                       "scaled_causal_softmax_last_dim");
    return finish(std::move(result), placement);
}

tensors::Tensor rms_norm(const tensors::TensorView& input, const tensors::TensorView& weight, float epsilon) {
    validate_rms_norm(input, weight, epsilon);
    const auto placement = place({&input, &weight}, "rms_norm");
    DeviceScope scope(placement.device);
    const auto& info = input.tensor_info();
    const auto width = info.shape.dims().back();
    const auto rows = width == 0 ? 0 : static_cast<int64_t>(info.shape.num_elements()) / width;
    const auto element = tensors::element_size_bytes(info.dtype);

    // A device view whose rows are dense and evenly spaced is read in place; anything else is gathered first.
    std::int64_t row_stride = width;
    std::optional<DeviceOperand> dense;
    const void* x = nullptr;
    const auto& strides = input.strides_bytes();
    if (input.device().is_cuda() && !input.is_contiguous() && info.shape.rank() == 2 && strides[1] == element &&
        strides[0] % element == 0) {
        row_stride = static_cast<std::int64_t>(strides[0] / element);
        x = input.data().data();
    } else {
        dense.emplace(input, placement.device);
        x = dense->get();
    }
    const DeviceOperand w(weight, placement.device);
    auto result = Tensor::empty(tensors::make_result_tensor_info("rms_norm_result", info.dtype, info.shape),
                                placement.device);
    cuda::check_status(cppinf_rms_norm(abi_dtype(info.dtype), x, row_stride, w.get(), out_ptr(result), rows, width,
                                       epsilon, cuda::current_stream()),
                       "rms_norm");
    return finish(std::move(result), placement);
}

std::pair<tensors::Tensor, tensors::Tensor> add_rms_norm(const tensors::TensorView& lhs, const tensors::TensorView& rhs,
                                                         const tensors::TensorView& weight, float epsilon) {
    validate_elementwise_inputs(lhs, rhs, "add");
    validate_rms_norm(lhs, weight, epsilon);
    const auto placement = place({&lhs, &rhs, &weight}, "add_rms_norm");
    DeviceScope scope(placement.device);
    const DeviceOperand a(lhs, placement.device);
    const DeviceOperand b(rhs, placement.device);
    const DeviceOperand w(weight, placement.device);
    const auto& info = lhs.tensor_info();
    const auto width = info.shape.dims().back();
    auto sum = Tensor::empty(tensors::make_result_tensor_info("add_result", info.dtype, info.shape), placement.device);
    auto y = Tensor::empty(tensors::make_result_tensor_info("rms_norm_result", info.dtype, info.shape),
                           placement.device);
    cuda::check_status(cppinf_add_rms_norm(abi_dtype(info.dtype), a.get(), b.get(), w.get(), out_ptr(sum), out_ptr(y),
                                           static_cast<int64_t>(info.shape.num_elements()) / width, width, epsilon,
                                           cuda::current_stream()),
                       "add_rms_norm");
    return {finish(std::move(sum), placement), finish(std::move(y), placement)};
}

tensors::Tensor silu_mul(const tensors::TensorView& gate, const tensors::TensorView& up) {
    validate_supported_float_dtype(gate.tensor_info().dtype, "silu");
    validate_elementwise_inputs(gate, up, "mul");
    const auto placement = place({&gate, &up}, "mul");
    DeviceScope scope(placement.device);
    const DeviceOperand g(gate, placement.device);
    const DeviceOperand u(up, placement.device);
    const auto& info = gate.tensor_info();
    auto result = Tensor::empty(tensors::make_result_tensor_info("mul_result", info.dtype, info.shape),
                                placement.device);
    cuda::check_status(cppinf_silu_mul(abi_dtype(info.dtype), g.get(), u.get(), out_ptr(result),
                                       static_cast<int64_t>(info.shape.num_elements()), cuda::current_stream()),
                       "silu_mul");
    return finish(std::move(result), placement);
}

std::vector<std::int64_t> row_argmax(const tensors::TensorView& logits) {
    validate_supported_float_dtype(logits.tensor_info().dtype, "row_argmax");
    if (logits.tensor_info().shape.rank() != 2) {
        throw std::invalid_argument("CLI generation requires rank-2 logits.");
    }
    const auto& dims = logits.tensor_info().shape.dims();
    const auto rows = common::checked_positive_dim_to_size(dims[0], "logits sequence length");
    const auto cols = common::checked_positive_dim_to_size(dims[1], "logits vocab size");
    const auto placement = place({&logits}, "row_argmax");
    DeviceScope scope(placement.device);
    const DeviceOperand x(logits, placement.device);
    auto ids = Tensor::empty(tensors::make_result_tensor_info("row_argmax_result", DType::F32,
                                                              Shape({static_cast<std::int64_t>(rows) * 2})),
                             placement.device);
    cuda::check_status(cppinf_row_argmax(abi_dtype(logits.tensor_info().dtype), x.get(), static_cast<int64_t>(rows),
                                         static_cast<int64_t>(cols), static_cast<int64_t>(cols),
                                         static_cast<int64_t*>(out_ptr(ids)), cuda::current_stream()),
                       "row_argmax");
    std::vector<std::int64_t> out(rows);
    cuda::check(cudaMemcpyAsync(out.data(), ids.data().data(), rows * sizeof(std::int64_t), cudaMemcpyDeviceToHost,
                                cuda::current_stream()),
                "cudaMemcpyAsync(argmax)");
    cuda::check(cudaStreamSynchronize(cuda::current_stream()), "cudaStreamSynchronize");
    return out;
}

// ---- matmul.h ----------------------------------------------------------------------------------------------------

namespace {

// resolve_output_dtype and validate_matmul_inputs, src/ops/matmul.cpp:13-60
tensors::DType resolve_matmul_dtype(const TensorView& lhs, const TensorView& rhs, const MatmulOptions& options) {
    if (options.output_dtype.has_value()) {
        return *options.output_dtype;
    }
    if (lhs.tensor_info().dtype == rhs.tensor_info().dtype) {
        return lhs.tensor_info().dtype;
    }
    return DType::F32;
}

void validate_matmul(const TensorView& lhs, const TensorView& rhs, DType output_dtype) {
    validate_supported_float_dtype(lhs.tensor_info().dtype, "matmul");
    validate_supported_float_dtype(rhs.tensor_info().dtype, "matmul");
    validate_supported_float_dtype(output_dtype, "matmul");
    if (lhs.tensor_info().dtype == rhs.tensor_info().dtype) {
        if (output_dtype != lhs.tensor_info().dtype &&
            (lhs.tensor_info().dtype != DType::BF16 || output_dtype != DType::F32)) {
            throw std::invalid_argument(
                "matmul output dtype must match the input dtype, except BF16 inputs may request an F32 result.");
        }
    } else if (output_dtype != DType::F32) {
        throw std::invalid_argument("matmul requires an F32 result when input dtypes differ.");
    }
    const auto& ls = lhs.tensor_info().shape;
    const auto& rs = rhs.tensor_info().shape;
    if (ls.rank() != rs.rank()) {
        throw std::invalid_argument("matmul requires tensors with matching rank.");
    }
    if (ls.rank() != 2 && ls.rank() != 3) {
        throw std::invalid_argument("matmul requires rank-2 or rank-3 tensors.");
    }
    if (ls.rank() == 3 && ls.dims()[0] != rs.dims()[0]) {
        throw std::invalid_argument("matmul requires matching batch dimensions.");
    }
    if (ls.dims().back() != rs.dims()[rs.rank() - 2]) {
        throw std::invalid_argument("matmul inner dimensions must match.");
    }
}

// A matmul operand on the op's GPU with its element strides {batch, row, column}: device views are read in place,
// host tensors are staged dense.
struct MatmulOperand {
    std::optional<DeviceOperand> staged;
    const void* ptr = nullptr;
    std::array<std::int64_t, 3> strides{};
};

MatmulOperand matmul_operand(const TensorView& view, const Device& device) {
    MatmulOperand op;
    const auto rank = view.tensor_info().shape.rank();
    std::vector<std::int64_t> s;
    if (view.device().is_cuda()) {
        op.ptr = view.data().data();
        const auto element = tensors::element_size_bytes(view.tensor_info().dtype);
        for (const auto b : view.strides_bytes()) {
            s.push_back(static_cast<std::int64_t>(b / element));
        }
    } else {
        op.staged.emplace(view, device);
        op.ptr = op.staged->get();
        s = operand_strides(view);
    }
    op.strides = rank == 3 ? std::array<std::int64_t, 3>{s[0], s[1], s[2]} : std::array<std::int64_t, 3>{0, s[0], s[1]};
    return op;
}

} // namespace

tensors::Tensor matmul(const tensors::TensorView& lhs, const tensors::TensorView& rhs, MatmulOptions options) {
    const auto output_dtype = resolve_matmul_dtype(lhs, rhs, options);
    validate_matmul(lhs, rhs, output_dtype);
    const auto placement = place({&lhs, &rhs}, "matmul");
    DeviceScope scope(placement.device);
    const auto& ld = lhs.tensor_info().shape.dims();
    const auto& rd = rhs.tensor_info().shape.dims();
    const bool batched = ld.size() == 3;
    const std::int64_t batch = batched ? ld[0] : 1;
    const std::int64_t m = ld[ld.size() - 2];
    const std::int64_t k = ld.back();
    const std::int64_t n = rd.back();
    const auto shape = batched ? tensors::Shape({batch, m, n}) : tensors::Shape({m, n});
    auto result = Tensor::empty(tensors::make_result_tensor_info("matmul_result", output_dtype, shape),
                                placement.device);
    if (batch * m * n != 0) {
        const auto x = matmul_operand(lhs, placement.device);
        const auto w = matmul_operand(rhs, placement.device);
        cuda::check_status(cppinf_matmul(abi_dtype(lhs.tensor_info().dtype), x.ptr, x.strides.data(),
                                         abi_dtype(rhs.tensor_info().dtype), w.ptr, w.strides.data(),
                                         abi_dtype(output_dtype), out_ptr(result), batch, m, k, n,
                                         cuda::current_stream()),
                           "matmul");
    }
    return finish(std::move(result), placement);
}


// ---- tensor_ops.h ------------------------------------------------------------------------------------------------

tensors::Tensor cast(const tensors::TensorView& input, tensors::DType dtype) {
    validate_supported_float_dtype(input.tensor_info().dtype, "cast");
    validate_supported_float_dtype(dtype, "cast");
    const auto placement = place({&input}, "cast");
    DeviceScope scope(placement.device);
    const DeviceOperand x(input, placement.device);
    const auto& info = input.tensor_info();
    auto result =
        Tensor::empty(tensors::make_result_tensor_info("cast_result", dtype, info.shape), placement.device);
    cuda::check_status(cppinf_cast(abi_dtype(info.dtype), x.get(), abi_dtype(dtype), out_ptr(result),
                                   static_cast<int64_t>(info.shape.num_elements()), cuda::current_stream()),
                       "cast");
    return finish(std::move(result), placement);
}

tensors::TensorView reshape(const tensors::TensorView& input, tensors::Shape shape) {
    if (!input.is_contiguous()) {
        throw std::invalid_argument("reshape requires a contiguous tensor view.");
    }
    TensorInfo info{.name = input.tensor_info().name,
                    .dtype = input.tensor_info().dtype,
                    .shape = std::move(shape),
                    .byte_offset = input.tensor_info().byte_offset};
    if (info.byte_size() != input.byte_size()) {
        throw std::invalid_argument("reshape requires the same total byte size.");
    }
    return TensorView(std::move(info), input.data(), {}, 0, input.device());
}

tensors::TensorView squeeze(const tensors::TensorView& input, std::size_t dim) {
    const auto& shape = input.tensor_info().shape;
    if (shape.rank() == 0) {
        throw std::invalid_argument("squeeze requires a tensor with rank at least 1.");
    }
    if (dim >= shape.rank()) {
        throw std::out_of_range("squeeze dimension is out of bounds.");
    }
    if (common::checked_non_negative_dim_to_size(shape.dims()[dim], "squeeze dim size") != 1) {
        throw std::invalid_argument("squeeze requires the selected dimension to have size 1.");
    }
    std::vector<std::int64_t> dims;
    std::vector<std::size_t> strides;
    for (std::size_t k = 0; k < shape.rank(); ++k) {
        if (k != dim) {
            dims.push_back(shape.dims()[k]);
            strides.push_back(input.strides_bytes()[k]);
        }
    }
    TensorInfo info{.name = input.tensor_info().name,
                    .dtype = input.tensor_info().dtype,
                    .shape = Shape(std::move(dims)),
                    .byte_offset = input.tensor_info().byte_offset};
    return TensorView(std::move(info), input.data(), std::move(strides), 0, input.device());
}

tensors::TensorView narrow(const tensors::TensorView& input, std::size_t dim, std::size_t start, std::size_t length) {
    const auto& shape = input.tensor_info().shape;
    if (shape.rank() == 0) {
        throw std::invalid_argument("narrow requires a tensor with rank at least 1.");
    }
    if (dim >= shape.rank()) {
        throw std::out_of_range("narrow dimension is out of bounds.");
    }
    const auto dim_size = common::checked_non_negative_dim_to_size(shape.dims()[dim], "narrow dim size");
    if (start > dim_size || length > dim_size - start) {
        throw std::out_of_range("narrow range is out of bounds.");
    }
    const auto byte_start = start * input.strides_bytes()[dim];
    auto dims = shape.dims();
    dims[dim] = common::checked_size_to_dim(length, "narrow length");
    TensorInfo info{.name = input.tensor_info().name,
                    .dtype = input.tensor_info().dtype,
                    .shape = Shape(std::move(dims)),
                    .byte_offset = input.tensor_info().byte_offset + byte_start};
    return TensorView(std::move(info), input.data(), input.strides_bytes(), byte_start, input.device());
}

tensors::Tensor permute(const tensors::TensorView& input, std::span<const std::size_t> axes) {
    const auto rank = input.tensor_info().shape.rank();
    // validate_permutation_axes, src/ops/tensor_ops.cpp:53-69
    if (axes.size() != rank) {
        throw std::invalid_argument("permute requires one axis per input dimension.");
    }
    std::vector<bool> used(rank, false);
    for (const auto axis : axes) {
        if (axis >= rank) {
            throw std::out_of_range("permute axis is out of bounds.");
        }
        if (used[axis]) {
            throw std::invalid_argument("permute axes must be unique.");
        }
        used[axis] = true;
    }
    validate_supported_float_dtype(input.tensor_info().dtype, "permute");
    const auto placement = place({&input}, "permute");
    DeviceScope scope(placement.device);
    const auto src_strides = operand_strides(input);
    std::vector<std::int64_t> dims;
    std::vector<std::int64_t> strides;
    for (const auto axis : axes) {
        dims.push_back(input.tensor_info().shape.dims()[axis]);
        strides.push_back(src_strides[axis]);
    }
    return gather(input, placement, "permute_result", dims, strides, Shape(dims));
}

namespace {

using tensors::Shape;

Tensor transpose_last_two(const tensors::TensorView& input, std::string_view result_name) {
    const auto rank = input.tensor_info().shape.rank();
    if (rank != 2 && rank != 3) {
        throw std::invalid_argument("transpose_last_two_dims requires a rank-2 or rank-3 tensor.");
    }
    validate_supported_float_dtype(input.tensor_info().dtype, result_name);
    const auto placement = place({&input}, result_name);
    DeviceScope scope(placement.device);
    auto dims = input.tensor_info().shape.dims();
    auto strides = operand_strides(input);
    std::swap(dims[rank - 1], dims[rank - 2]);
    std::swap(strides[rank - 1], strides[rank - 2]);
    return gather(input, placement, result_name, dims, strides, Shape(dims));
}

} // namespace

tensors::Tensor transpose_2d(const tensors::TensorView& input) {
    if (input.tensor_info().shape.rank() != 2) {
        throw std::invalid_argument("transpose_2d requires a rank-2 tensor.");
    }
    return transpose_last_two(input, "transpose_2d_result");
}

tensors::Tensor transpose_last_two_dims(const tensors::TensorView& input) {
    return transpose_last_two(input, "transpose_last_two_dims_result");
}

tensors::Tensor repeat_interleave(const tensors::TensorView& input, std::size_t dim, std::size_t repeats) {
    const auto& shape = input.tensor_info().shape;
    if (dim >= shape.rank()) {
        throw std::out_of_range("repeat_interleave dimension is out of bounds.");
    }
    common::checked_positive_size(repeats, "repeat_interleave repeats");
    const auto dim_size = common::checked_non_negative_dim_to_size(shape.dims()[dim], "repeat_interleave dim size");
    if (dim_size > std::numeric_limits<std::size_t>::max() / repeats) {
        throw std::overflow_error("repeat_interleave output dimension overflowed.");
    }
    auto out_dims = shape.dims();
    out_dims[dim] = common::checked_size_to_dim(dim_size * repeats, "repeat_interleave output dim");
    if (shape.rank() + 1 > 8) {
        throw std::invalid_argument("repeat_interleave supports tensors of rank at most 7 on the device.");
    }
    validate_supported_float_dtype(input.tensor_info().dtype, "repeat_interleave");
    const auto placement = place({&input}, "repeat_interleave");
    DeviceScope scope(placement.device);
    // Gather through a rank+1 view [.., d, repeats, ..] whose repeat axis has stride 0.
    const auto src_strides = operand_strides(input);
    std::vector<std::int64_t> dims;
    std::vector<std::int64_t> strides;
    for (std::size_t k = 0; k < shape.rank(); ++k) {
        dims.push_back(shape.dims()[k]);
        strides.push_back(src_strides[k]);
        if (k == dim) {
            dims.push_back(static_cast<std::int64_t>(repeats));
            strides.push_back(0);
        }
    }
    return gather(input, placement, "repeat_interleave_result", dims, strides, Shape(out_dims));
}

} // namespace ops

namespace nn {

tensors::Tensor apply_rope(const tensors::TensorView& input, std::size_t sequence_position_offset, float rope_base,
                           std::size_t sequence_dimension) {
    // validate_rope_input, src/nn/rope.cpp:33-54
    const auto& info = input.tensor_info();
    if (info.dtype != DType::BF16 && info.dtype != DType::F32) {
        throw std::invalid_argument("apply_rope received an unsupported dtype.");
    }
    if (info.shape.rank() != 3) {
        throw std::invalid_argument("apply_rope requires a rank-3 tensor.");
    }
    if (!std::isfinite(rope_base) || rope_base <= 0.0f) {
        throw std::invalid_argument("apply_rope requires a positive finite rope base.");
    }
    if (sequence_dimension > 1) {
        throw std::invalid_argument("apply_rope requires the sequence dimension to be 0 or 1.");
    }
    const auto& dims = info.shape.dims();
    common::checked_positive_dim_to_size(dims[0], "rope dim 0");
    common::checked_positive_dim_to_size(dims[1], "rope dim 1");
    const auto head_size = common::checked_positive_dim_to_size(dims[2], "rope head size");
    if (head_size % 2 != 0) {
        throw std::invalid_argument("apply_rope requires an even head size.");
    }

    int previous = 0;
    cuda::check(cudaGetDevice(&previous), "cudaGetDevice");
    const bool host_input = !input.device().is_cuda();
    const Device device = host_input ? Device::cuda(previous) : input.device();
    if (device.index != previous) {
        cuda::check(cudaSetDevice(device.index), "cudaSetDevice");
    }
    const auto element = tensors::element_size_bytes(info.dtype);
    std::optional<Tensor> staged;
    const void* x = input.data().data();
    std::vector<std::int64_t> strides;
    if (host_input) {
        staged = tensors::materialize_tensor(info.name, input).to(device);
        x = staged->data().data();
        strides = {dims[1] * dims[2], dims[2], 1};
    } else {
        for (const auto s : input.strides_bytes()) {
            strides.push_back(static_cast<std::int64_t>(s / element));
        }
    }
    const auto seq_len = dims[sequence_dimension];
    std::int64_t table_positions = 0;
    const float* table = rope_table_for(device, rope_base, dims[2],
                                             static_cast<std::int64_t>(sequence_position_offset) + seq_len,
                                             table_positions);
    auto result = Tensor::empty(tensors::make_result_tensor_info("rope_result", info.dtype, info.shape), device);
    const auto status = cppinf_rope(info.dtype == DType::BF16 ? CPPINF_DTYPE_BF16 : CPPINF_DTYPE_F32, x, dims[0],
                                    dims[1], dims[2], strides[0], strides[1], strides[2],
                                    static_cast<std::int64_t>(sequence_dimension),
                                    static_cast<std::int64_t>(sequence_position_offset), table, table_positions,
                                    result.mutable_data().data(), cuda::current_stream());
    if (device.index != previous) {
        cudaSetDevice(previous);
    }
    cuda::check_status(status, "apply_rope");
    return host_input ? result.to(Device::host()) : result;
}

std::pair<tensors::Tensor, tensors::Tensor> qk_norm_rope(const tensors::TensorView& query,
                                                         const tensors::TensorView& key,
                                                         const tensors::TensorView& query_norm_weight,
                                                         const tensors::TensorView& key_norm_weight, float epsilon,
                                                         std::size_t sequence_position_offset, float rope_base) {
    const auto& qi = query.tensor_info();
    const auto& ki = key.tensor_info();
    // The two ops::rms_norm calls of src/nn/qwen_attention.cpp:383-384 validate first.
    validate_rms_norm(query, query_norm_weight, epsilon);
    validate_rms_norm(key, key_norm_weight, epsilon);
    if (qi.shape.rank() != 3 || ki.shape.rank() != 3 || qi.shape.dims()[0] != ki.shape.dims()[0] ||
        qi.shape.dims()[2] != ki.shape.dims()[2]) {
        throw std::invalid_argument("qk_norm_rope requires query [T, Hq, D] and key [T, Hk, D].");
    }
    if (!std::isfinite(rope_base) || rope_base <= 0.0f) {
        throw std::invalid_argument("apply_rope requires a positive finite rope base.");
    }
    const auto placement = place({&query, &key, &query_norm_weight, &key_norm_weight}, "qk_norm_rope");
    const bool dense = query.is_contiguous() && key.is_contiguous() && query_norm_weight.is_contiguous() &&
                       key_norm_weight.is_contiguous();
    if (!placement.host_inputs && dense) {
        DeviceScope scope(placement.device);
        const auto tokens = qi.shape.dims()[0];
        const auto head_dim = qi.shape.dims()[2];
        std::int64_t table_positions = 0;
        const float* table = rope_table_for(placement.device, rope_base, head_dim,
                                            static_cast<std::int64_t>(sequence_position_offset) + tokens,
                                            table_positions);
        auto q_out = Tensor::empty(tensors::make_result_tensor_info("rope_result", qi.dtype, qi.shape),
                                   placement.device);
        auto k_out = Tensor::empty(tensors::make_result_tensor_info("rope_result", ki.dtype, ki.shape),
                                   placement.device);
        const auto status = cppinf_qk_norm_rope(
            abi_dtype(qi.dtype), query.data().data(), key.data().data(), query_norm_weight.data().data(),
            key_norm_weight.data().data(), out_ptr(q_out), out_ptr(k_out), tokens, qi.shape.dims()[1],
            ki.shape.dims()[1], head_dim, static_cast<std::int64_t>(sequence_position_offset), epsilon, table,
            table_positions, cuda::current_stream());
        if (status == CPPINF_OK) {
            return {std::move(q_out), std::move(k_out)};
        }
        if (status != CPPINF_ERR_UNSUPPORTED) {
            cuda::check_status(status, "qk_norm_rope");
        }
    }
    // The reference's own two-step sequence on the device ops: host inputs, strided views, and head sizes the fused
    // kernel does not cover.
    const auto q_norm = ops::rms_norm(query, query_norm_weight, epsilon);
    const auto k_norm = ops::rms_norm(key, key_norm_weight, epsilon);
    return {apply_rope(q_norm.view(), sequence_position_offset, rope_base, 0),
            apply_rope(k_norm.view(), sequence_position_offset, rope_base, 0)};
}

} // namespace nn
} // namespace cppinf
