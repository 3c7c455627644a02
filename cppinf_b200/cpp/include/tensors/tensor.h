#pragma once

#include <cstddef>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "device.h"
#include "tensor_info.h"
#include "tensor_view.h"

namespace cppinf::tensors {

class DeviceBuffer;

// Owning tensor (src/tensors/tensor.h:13-31) with host or device storage.
//
// Host tensors behave exactly like the reference's. Device tensors own stream-ordered device memory
// (cudaMallocAsync on the calling thread's current stream, released with cudaFreeAsync on the same stream); their
// data() spans hold device addresses. bytes() is host-only; to(Device) copies between host and device.
class Tensor {
  public:
    Tensor(TensorInfo tensor_info, std::vector<std::byte> data);

    static Tensor zeros(TensorInfo tensor_info);
    // Uninitialised device storage for `tensor_info` on GPU `device.index` (host: zero-filled).
    static Tensor empty(TensorInfo tensor_info, Device device);
    // Zero-filled storage on `device`.
    static Tensor zeros(TensorInfo tensor_info, Device device);

    const TensorInfo& tensor_info() const;
    const std::vector<std::byte>& bytes() const;
    std::span<const std::byte> data() const;
    std::span<std::byte> mutable_data();
    std::size_t byte_size() const;
    TensorView view() const;
    const Device& device() const;

    // Copy of this tensor on `device` (same name and metadata). Waits for the copy when the target is the host.
    Tensor to(Device device) const;

    // Metadata, device and bytes equal. Device tensors are compared through host copies.
    bool operator==(const Tensor& other) const;

  private:
    Tensor(TensorInfo tensor_info, std::shared_ptr<DeviceBuffer> buffer, Device device);

    TensorInfo tensor_info_;
    std::vector<std::byte> data_;
    std::shared_ptr<DeviceBuffer> device_data_;
    Device device_;
};

std::string to_string(const Tensor& tensor);

} // namespace cppinf::tensors
