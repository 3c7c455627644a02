#pragma once

#include <cstddef>
#include <span>
#include <string>
#include <vector>

#include "device.h"
#include "tensor_info.h"

namespace cppinf::tensors {

// Non-owning strided view (src/tensors/tensor_view.h:12-27). Strides are in bytes; an empty stride list means dense.
// The trailing `device` argument is the one addition: a view of device memory carries Device::cuda(i) and its span
// holds device addresses.
class TensorView {
  public:
    TensorView(TensorInfo tensor_info, std::span<const std::byte> data, std::vector<std::size_t> strides_bytes = {},
               std::size_t data_offset_bytes = 0, Device device = Device::host());

    const TensorInfo& tensor_info() const;
    std::span<const std::byte> data() const;
    const std::vector<std::size_t>& strides_bytes() const;
    bool is_contiguous() const;
    std::size_t byte_size() const;
    const Device& device() const;

  private:
    TensorInfo tensor_info_;
    std::span<const std::byte> data_;
    std::vector<std::size_t> strides_bytes_;
    std::size_t data_offset_bytes_{};
    Device device_;
};

std::string to_string(const TensorView& tensor_view);

// Dense byte strides for a tensor of this metadata.
std::vector<std::size_t> dense_strides_bytes(const TensorInfo& tensor_info);

} // namespace cppinf::tensors
