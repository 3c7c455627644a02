#pragma once

#include <cuda_runtime.h>

namespace cppinf::cuda {

// The stream device ops enqueue on, per calling thread. Defaults to cudaStreamPerThread. Ops return without
// synchronising; reading a device result on the host (Tensor::to(Device::host()), operator==) waits for it.
cudaStream_t current_stream();
void set_current_stream(cudaStream_t stream);

// Sets the current stream for a scope.
class StreamGuard {
  public:
    explicit StreamGuard(cudaStream_t stream);
    ~StreamGuard();
    StreamGuard(const StreamGuard&) = delete;
    StreamGuard& operator=(const StreamGuard&) = delete;

  private:
    cudaStream_t previous_;
};

// Throws std::runtime_error with `what` and the CUDA error string when `err` is not cudaSuccess.
void check(cudaError_t err, const char* what);

// Throws the exception type matching a non-zero cppinf C ABI status, with cppinf_last_error() as the message.
void check_status(int status, const char* what);

} // namespace cppinf::cuda
