// cppinf tensors API (src/tensors/*) with host or device storage, plus the checked conversions of src/common and the
// per-thread CUDA stream the ops enqueue on.
#include <cuda_runtime.h>

#include <cstring>
#include <format>
#include <limits>
#include <stdexcept>
#include <utility>

#include "common/checked.h"
#include "cppinf_b200.h"
#include "cuda/runtime.h"
#include "tensors/bfloat16.h"
#include "tensors/device.h"
#include "tensors/dtype.h"
#include "tensors/shape.h"
#include "tensors/tensor.h"
#include "tensors/tensor_info.h"
#include "tensors/tensor_utils.h"
#include "tensors/tensor_view.h"

// ---- common ------------------------------------------------------------------------------------------------------

namespace cppinf::common {

std::size_t checked_non_negative_dim_to_size(std::int64_t dim, std::string_view field_name) {
    if (dim >= 0) {
        return static_cast<std::size_t>(dim);
    }
    throw std::invalid_argument(std::format("{} must be non-negative.", field_name));
}

std::size_t checked_positive_dim_to_size(std::int64_t dim, std::string_view field_name) {
    const auto size = checked_non_negative_dim_to_size(dim, field_name);
    return checked_positive_size(size, field_name);
}

std::size_t checked_positive_size(std::size_t value, std::string_view field_name) {
    if (value != 0) {
        return value;
    }
    throw std::invalid_argument(std::format("{} must be non-zero.", field_name));
}

std::int64_t checked_size_to_dim(std::size_t value, std::string_view field_name) {
    if (value <= static_cast<std::size_t>(std::numeric_limits<std::int64_t>::max())) {
        return static_cast<std::int64_t>(value);
    }
    throw std::overflow_error(std::format("{} does not fit in int64_t.", field_name));
}

} // namespace cppinf::common

// ---- cuda --------------------------------------------------------------------------------------------------------

namespace cppinf::cuda {
namespace {
thread_local cudaStream_t g_stream = cudaStreamPerThread;
}

cudaStream_t current_stream() {
    return g_stream;
}

void set_current_stream(cudaStream_t stream) {
    g_stream = stream;
}

StreamGuard::StreamGuard(cudaStream_t stream) : previous_(g_stream) {
    g_stream = stream;
}

StreamGuard::~StreamGuard() {
    g_stream = previous_;
}

void check(cudaError_t err, const char* what) {
    if (err != cudaSuccess) {
        throw std::runtime_error(std::format("{} failed: {}", what, cudaGetErrorString(err)));
    }
}

void check_status(int status, const char* what) {
    if (status == CPPINF_OK) {
        return;
    }
    const std::string message = cppinf_last_error();
    switch (status) {
    case CPPINF_ERR_INVALID_ARGUMENT:
        throw std::invalid_argument(message);
    case CPPINF_ERR_OUT_OF_RANGE:
        throw std::out_of_range(message);
    case CPPINF_ERR_OVERFLOW:
        throw std::overflow_error(message);
    default:
        throw std::runtime_error(std::format("{}: {} ({})", what, message, cppinf_status_name(status)));
    }
}

} // namespace cppinf::cuda

// ---- tensors -----------------------------------------------------------------------------------------------------

namespace cppinf::tensors {

std::size_t element_size_bytes(DType dtype) {
    switch (dtype) {
    case DType::BF16:
        return 2;
    case DType::F32:
        return 4;
    }
    throw std::invalid_argument("Unsupported DType.");
}

DType parse_dtype(std::string_view dtype_name) {
    if (dtype_name == "F32") {
        return DType::F32;
    }
    if (dtype_name == "BF16") {
        return DType::BF16;
    }
    throw std::invalid_argument("Unsupported safetensors dtype. Only BF16 and F32 are supported.");
}

std::string_view to_string(DType dtype) {
    switch (dtype) {
    case DType::BF16:
        return "bf16";
    case DType::F32:
        return "f32";
    }
    throw std::invalid_argument("Unsupported DType.");
}

std::uint16_t float_to_bfloat16_bits(float value) {
    std::uint32_t u = 0;
    std::memcpy(&u, &value, sizeof(u));
    // Round half to even on the 16 dropped bits.
    const std::uint32_t rounding = 0x7fffU + ((u >> 16U) & 1U);
    return static_cast<std::uint16_t>((u + rounding) >> 16U);
}

float bfloat16_bits_to_float(std::uint16_t bits) {
    const auto u = static_cast<std::uint32_t>(bits) << 16U;
    float value = 0.0f;
    std::memcpy(&value, &u, sizeof(value));
    return value;
}

Shape::Shape(std::vector<std::int64_t> dims) : dims_(std::move(dims)) {
    for (const auto dim : dims_) {
        if (dim < 0) {
            throw std::invalid_argument("Shape dimensions must be non-negative.");
        }
    }
}

const std::vector<std::int64_t>& Shape::dims() const {
    return dims_;
}

std::size_t Shape::rank() const {
    return dims_.size();
}

std::size_t Shape::num_elements() const {
    std::size_t count = 1;
    for (const auto dim : dims_) {
        const auto d = static_cast<std::size_t>(dim);
        if (d != 0 && count > std::numeric_limits<std::size_t>::max() / d) {
            throw std::overflow_error("Shape element count overflowed.");
        }
        count *= d;
    }
    return count;
}

std::string to_string(const Shape& shape) {
    std::string out = "[";
    for (std::size_t i = 0; i < shape.dims().size(); ++i) {
        out += (i == 0 ? "" : ", ") + std::to_string(shape.dims()[i]);
    }
    return out + "]";
}

std::size_t TensorInfo::byte_size() const {
    const auto count = shape.num_elements();
    const auto size = element_size_bytes(dtype);
    if (count > std::numeric_limits<std::size_t>::max() / size) {
        throw std::overflow_error("Tensor byte size overflowed.");
    }
    return count * size;
}

std::string to_string(const TensorInfo& tensor_info) {
    return std::format("TensorInfo(name=\"{}\", dtype={}, shape={}, offset={}, bytes={})", tensor_info.name,
                       to_string(tensor_info.dtype), to_string(tensor_info.shape), tensor_info.byte_offset,
                       tensor_info.byte_size());
}

std::string to_string(const Device& device) {
    return device.is_cuda() ? std::format("cuda:{}", device.index) : std::string("host");
}

// ---- TensorView --------------------------------------------------------------------------------------------------

std::vector<std::size_t> dense_strides_bytes(const TensorInfo& tensor_info) {
    const auto& dims = tensor_info.shape.dims();
    std::vector<std::size_t> strides(dims.size());
    std::size_t stride = element_size_bytes(tensor_info.dtype);
    for (std::size_t k = dims.size(); k-- > 0;) {
        strides[k] = stride;
        const auto d = static_cast<std::size_t>(dims[k]);
        if (d != 0 && stride > std::numeric_limits<std::size_t>::max() / d) {
            throw std::overflow_error("TensorView strides overflowed.");
        }
        stride *= d;
    }
    return strides;
}

namespace {

// Bytes from the view's first element to one past its last element.
std::size_t covered_bytes(const TensorInfo& info, const std::vector<std::size_t>& strides) {
    const auto& dims = info.shape.dims();
    std::size_t last = 0;
    for (std::size_t k = 0; k < dims.size(); ++k) {
        if (dims[k] == 0) {
            return 0;
        }
        const auto extent = (static_cast<std::size_t>(dims[k]) - 1) * strides[k];
        if (extent > std::numeric_limits<std::size_t>::max() - last) {
            throw std::overflow_error("TensorView covered byte size overflowed.");
        }
        last += extent;
    }
    const auto element = element_size_bytes(info.dtype);
    if (element > std::numeric_limits<std::size_t>::max() - last) {
        throw std::overflow_error("TensorView covered byte size overflowed.");
    }
    return last + element;
}

} // namespace

TensorView::TensorView(TensorInfo tensor_info, std::span<const std::byte> data, std::vector<std::size_t> strides_bytes,
                       std::size_t data_offset_bytes, Device device)
    : tensor_info_(std::move(tensor_info)), data_(data), strides_bytes_(std::move(strides_bytes)),
      data_offset_bytes_(data_offset_bytes), device_(device) {
    if (strides_bytes_.empty()) {
        strides_bytes_ = dense_strides_bytes(tensor_info_);
    }
    if (strides_bytes_.size() != tensor_info_.shape.rank()) {
        throw std::invalid_argument("TensorView strides must match tensor rank.");
    }
    if (data_offset_bytes_ > data_.size()) {
        throw std::invalid_argument("TensorView data offset is out of bounds.");
    }
    if (covered_bytes(tensor_info_, strides_bytes_) > data_.size() - data_offset_bytes_) {
        throw std::invalid_argument("TensorView backing bytes do not cover the requested view.");
    }
}

const TensorInfo& TensorView::tensor_info() const {
    return tensor_info_;
}

std::span<const std::byte> TensorView::data() const {
    return data_.subspan(data_offset_bytes_);
}

const std::vector<std::size_t>& TensorView::strides_bytes() const {
    return strides_bytes_;
}

bool TensorView::is_contiguous() const {
    return strides_bytes_ == dense_strides_bytes(tensor_info_);
}

std::size_t TensorView::byte_size() const {
    return tensor_info_.byte_size();
}

const Device& TensorView::device() const {
    return device_;
}

std::string to_string(const TensorView& tensor_view) {
    return std::format("TensorView(name=\"{}\", dtype={}, shape={}, bytes={})", tensor_view.tensor_info().name,
                       to_string(tensor_view.tensor_info().dtype), to_string(tensor_view.tensor_info().shape),
                       tensor_view.byte_size());
}

// ---- Tensor ------------------------------------------------------------------------------------------------------

// Stream-ordered device allocation, released on the stream it was allocated on.
class DeviceBuffer {
  public:
    DeviceBuffer(std::size_t bytes, int device) : bytes_(bytes), device_(device), stream_(cuda::current_stream()) {
        if (bytes_ == 0) {
            return;
        }
        int previous = 0;
        cuda::check(cudaGetDevice(&previous), "cudaGetDevice");
        cuda::check(cudaSetDevice(device_), "cudaSetDevice");
        const auto err = cudaMallocAsync(&ptr_, bytes_, stream_);
        cudaSetDevice(previous);
        cuda::check(err, "cudaMallocAsync");
    }

    ~DeviceBuffer() {
        if (ptr_ != nullptr) {
            int previous = 0;
            if (cudaGetDevice(&previous) == cudaSuccess) {
                cudaSetDevice(device_);
                cudaFreeAsync(ptr_, stream_);
                cudaSetDevice(previous);
            }
        }
    }

    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;

    std::byte* data() const { return static_cast<std::byte*>(ptr_); }
    std::size_t size() const { return bytes_; }

  private:
    void* ptr_ = nullptr;
    std::size_t bytes_;
    int device_;
    cudaStream_t stream_;
};

Tensor::Tensor(TensorInfo tensor_info, std::vector<std::byte> data)
    : tensor_info_(std::move(tensor_info)), data_(std::move(data)) {
    if (tensor_info_.byte_offset != 0) {
        throw std::invalid_argument("Owning Tensor byte offset must be zero.");
    }
    if (data_.size() != tensor_info_.byte_size()) {
        throw std::invalid_argument("Tensor byte size does not match TensorInfo.");
    }
}

Tensor::Tensor(TensorInfo tensor_info, std::shared_ptr<DeviceBuffer> buffer, Device device)
    : tensor_info_(std::move(tensor_info)), device_data_(std::move(buffer)), device_(device) {
    if (tensor_info_.byte_offset != 0) {
        throw std::invalid_argument("Owning Tensor byte offset must be zero.");
    }
}

Tensor Tensor::zeros(TensorInfo tensor_info) {
    const auto size = tensor_info.byte_size();
    return Tensor(std::move(tensor_info), std::vector<std::byte>(size));
}

Tensor Tensor::empty(TensorInfo tensor_info, Device device) {
    if (!device.is_cuda()) {
        return zeros(std::move(tensor_info));
    }
    const auto size = tensor_info.byte_size();
    return Tensor(std::move(tensor_info), std::make_shared<DeviceBuffer>(size, device.index), device);
}

Tensor Tensor::zeros(TensorInfo tensor_info, Device device) {
    auto tensor = empty(std::move(tensor_info), device);
    if (device.is_cuda() && tensor.byte_size() != 0) {
        cuda::check(cudaMemsetAsync(tensor.mutable_data().data(), 0, tensor.byte_size(), cuda::current_stream()),
                    "cudaMemsetAsync");
    }
    return tensor;
}

const TensorInfo& Tensor::tensor_info() const {
    return tensor_info_;
}

const std::vector<std::byte>& Tensor::bytes() const {
    if (device_.is_cuda()) {
        throw std::logic_error("Tensor::bytes() is host-only; copy device tensors with to(Device::host()).");
    }
    return data_;
}

std::span<const std::byte> Tensor::data() const {
    if (device_.is_cuda()) {
        return {device_data_->data(), device_data_->size()};
    }
    return data_;
}

std::span<std::byte> Tensor::mutable_data() {
    if (device_.is_cuda()) {
        return {device_data_->data(), device_data_->size()};
    }
    return data_;
}

std::size_t Tensor::byte_size() const {
    return device_.is_cuda() ? device_data_->size() : data_.size();
}

TensorView Tensor::view() const {
    return TensorView(tensor_info_, data(), {}, 0, device_);
}

const Device& Tensor::device() const {
    return device_;
}

Tensor Tensor::to(Device device) const {
    const auto stream = cuda::current_stream();
    if (!device.is_cuda()) {
        if (!device_.is_cuda()) {
            return *this;
        }
        std::vector<std::byte> host(byte_size());
        if (!host.empty()) {
            cuda::check(cudaMemcpyAsync(host.data(), data().data(), host.size(), cudaMemcpyDeviceToHost, stream),
                        "cudaMemcpyAsync(device to host)");
            cuda::check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        }
        return Tensor(tensor_info_, std::move(host));
    }
    auto out = empty(tensor_info_, device);
    if (byte_size() != 0) {
        const auto kind = device_.is_cuda() ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
        cuda::check(cudaMemcpyAsync(out.mutable_data().data(), data().data(), byte_size(), kind, stream),
                    "cudaMemcpyAsync(to device)");
        if (!device_.is_cuda()) {
            // The host source may be released as soon as this returns.
            cuda::check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
        }
    }
    return out;
}

bool Tensor::operator==(const Tensor& other) const {
    if (!(tensor_info_ == other.tensor_info_) || !(device_ == other.device_)) {
        return false;
    }
    if (!device_.is_cuda()) {
        return data_ == other.data_;
    }
    return to(Device::host()).data_ == other.to(Device::host()).data_;
}

std::string to_string(const Tensor& tensor) {
    return std::format("Tensor(name=\"{}\", dtype={}, shape={}, bytes={})", tensor.tensor_info().name,
                       to_string(tensor.tensor_info().dtype), to_string(tensor.tensor_info().shape),
                       tensor.byte_size());
}

// ---- tensor_utils ------------------------------------------------------------------------------------------------

TensorInfo make_result_tensor_info(std::string_view name, DType dtype, const Shape& shape) {
    return TensorInfo{.name = std::string(name), .dtype = dtype, .shape = shape, .byte_offset = 0};
}

Tensor make_float_tensor(std::string_view name, DType dtype, const Shape& shape, std::span<const float> values) {
    if (values.size() != shape.num_elements()) {
        throw std::invalid_argument("Tensor values must match the requested shape.");
    }
    const auto element = element_size_bytes(dtype);
    std::vector<std::byte> bytes(values.size() * element);
    for (std::size_t i = 0; i < values.size(); ++i) {
        if (dtype == DType::BF16) {
            const auto bits = float_to_bfloat16_bits(values[i]);
            std::memcpy(bytes.data() + i * element, &bits, element);
        } else {
            std::memcpy(bytes.data() + i * element, &values[i], element);
        }
    }
    return Tensor(make_result_tensor_info(name, dtype, shape), std::move(bytes));
}

Tensor make_f32_tensor(std::string_view name, const Shape& shape, std::span<const float> values) {
    return make_float_tensor(name, DType::F32, shape, values);
}

Tensor make_bf16_tensor(std::string_view name, const Shape& shape, std::span<const float> values) {
    return make_float_tensor(name, DType::BF16, shape, values);
}

Tensor make_bf16_bits_tensor(std::string_view name, const Shape& shape, std::span<const std::uint16_t> values) {
    if (values.size() != shape.num_elements()) {
        throw std::invalid_argument("Tensor values must match the requested shape.");
    }
    std::vector<std::byte> bytes(values.size() * sizeof(std::uint16_t));
    if (!values.empty()) {
        std::memcpy(bytes.data(), values.data(), bytes.size());
    }
    return Tensor(make_result_tensor_info(name, DType::BF16, shape), std::move(bytes));
}

Tensor rename_tensor(std::string_view name, const Tensor& tensor) {
    auto info = make_result_tensor_info(name, tensor.tensor_info().dtype, tensor.tensor_info().shape);
    if (!tensor.device().is_cuda()) {
        return Tensor(std::move(info), tensor.bytes());
    }
    auto out = Tensor::empty(std::move(info), tensor.device());
    if (out.byte_size() != 0) {
        cuda::check(cudaMemcpyAsync(out.mutable_data().data(), tensor.data().data(), out.byte_size(),
                                    cudaMemcpyDeviceToDevice, cuda::current_stream()),
                    "cudaMemcpyAsync(rename)");
    }
    return out;
}

Tensor materialize_tensor(std::string_view name, const TensorView& tensor_view) {
    const auto& info = tensor_view.tensor_info();
    auto result_info = make_result_tensor_info(name, info.dtype, info.shape);
    const auto element = element_size_bytes(info.dtype);
    const auto count = info.shape.num_elements();
    const auto& dims = info.shape.dims();
    const auto& strides = tensor_view.strides_bytes();
    if (tensor_view.device().is_cuda()) {
        auto out = Tensor::empty(std::move(result_info), tensor_view.device());
        if (count == 0) {
            return out;
        }
        std::vector<std::int64_t> elem_strides(strides.size());
        for (std::size_t k = 0; k < strides.size(); ++k) {
            if (strides[k] % element != 0) {
                throw std::invalid_argument("materialize_tensor requires element-aligned tensor strides.");
            }
            elem_strides[k] = static_cast<std::int64_t>(strides[k] / element);
        }
        const auto dtype = info.dtype == DType::BF16 ? CPPINF_DTYPE_BF16 : CPPINF_DTYPE_F32;
        cuda::check_status(cppinf_strided_copy(dtype, tensor_view.data().data(), static_cast<std::int64_t>(dims.size()),
                                               dims.data(), elem_strides.data(), out.mutable_data().data(),
                                               cuda::current_stream()),
                           "materialize_tensor");
        return out;
    }
    std::vector<std::byte> bytes(count * element);
    const auto src = tensor_view.data();
    for (std::size_t i = 0; i < count; ++i) {
        std::size_t rem = i;
        std::size_t offset = 0;
        for (std::size_t k = dims.size(); k-- > 0;) {
            const auto d = static_cast<std::size_t>(dims[k]);
            offset += (rem % d) * strides[k];
            rem /= d;
        }
        std::memcpy(bytes.data() + i * element, src.data() + offset, element);
    }
    return Tensor(std::move(result_info), std::move(bytes));
}

} // namespace cppinf::tensors
