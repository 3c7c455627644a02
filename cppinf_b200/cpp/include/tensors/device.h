#pragma once

#include <string>

namespace cppinf::tensors {

// Where a tensor's bytes live. Host storage is the reference's std::vector<std::byte>; Cuda storage is stream-ordered
// device memory on GPU `index`. Byte spans of device tensors hold device addresses and are never dereferenced on the
// host.
enum class DeviceKind {
    Host,
    Cuda,
};

struct Device {
    DeviceKind kind = DeviceKind::Host;
    int index = 0;

    static Device host() { return Device{}; }
    static Device cuda(int index = 0) { return Device{DeviceKind::Cuda, index}; }
    bool is_cuda() const { return kind == DeviceKind::Cuda; }

    bool operator==(const Device&) const = default;
};

std::string to_string(const Device& device);

} // namespace cppinf::tensors
