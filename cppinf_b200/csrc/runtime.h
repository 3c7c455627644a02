// Host-side bookkeeping shared by the C ABI entry points: thread-local error messages, status propagation, launch
// accounting and cached device properties.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>
#include <utility>

#include "cppinf_b200.h"

namespace cppinf::runtime {

// Records `message` as the calling thread's last error and returns `status`.
int fail(int status, const std::string& message);

// Clears the calling thread's last error and returns CPPINF_OK.
int ok();

// Converts a failed CUDA call into CPPINF_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t err, const char* what);

// Checks the launch that was just enqueued and counts it.
int after_launch(const char* kernel_name);

// Number of SMs of the current device (cached per device).
int sm_count();

// Largest number of threads per SM of the current device (cached per device).
int max_threads_per_sm();

// Poll limit for the first wait on each bulk-copy barrier of the kernels launched from now on
// (cppinf_set_wait_poll_limit).
uint32_t wait_poll_limit();

inline bool aligned16(const void* p) {
    return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}

inline cudaStream_t as_stream(void* stream) {
    return static_cast<cudaStream_t>(stream);
}

inline int64_t ceil_div(int64_t a, int64_t b) {
    return (a + b - 1) / b;
}

inline std::size_t dtype_size(cppinf_dtype dtype) {
    return dtype == CPPINF_DTYPE_BF16 ? 2 : 4;
}

inline bool valid_dtype(cppinf_dtype dtype) {
    return dtype == CPPINF_DTYPE_BF16 || dtype == CPPINF_DTYPE_F32;
}

// Launches `kernel` with `smem_bytes` of dynamic shared memory and (see pdl_enabled) programmatic dependent launch
// allowed: the grid
// may be scheduled while the previous kernel in the stream is still finishing. Every kernel of this library executes
// griddepcontrol.wait before it reads memory another kernel writes, which waits for the previous grid to complete
// and its writes to become visible, so results are the same as with plain stream order; only launch latency and the
// previous grid's tail overlap. `cluster_x` > 1 adds a thread-block cluster dimension.
// Programmatic dependent launch is on for every launch of this thread unless a SerialLaunch is alive on it: then the
// grid starts only after the previous kernel of the stream has completed. For a kernel that reads, before its
// dependency wait, data that the kernel before it writes.
bool pdl_enabled();
class SerialLaunch {
public:
    SerialLaunch();
    ~SerialLaunch();
    SerialLaunch(const SerialLaunch&) = delete;
    SerialLaunch& operator=(const SerialLaunch&) = delete;

private:
    bool previous_;
};

template <typename... KernelArgs, typename... Args>
cudaError_t launch_smem(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, std::size_t smem_bytes,
                        cudaStream_t stream, unsigned cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    unsigned n = 0;
    if (pdl_enabled()) {
        attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (cluster_x > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = cluster_x;
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KernelArgs, typename... Args>
cudaError_t launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, cudaStream_t stream, unsigned cluster_x,
                   Args&&... args) {
    return launch_smem(kernel, grid, block, 0, stream, cluster_x, std::forward<Args>(args)...);
}

// Adds `n` (possibly negative) to the launch count: replays of a captured graph, or captured launches that only
// execute when the graph is replayed.
void count_launches(int64_t n);

// Records a failed launch (or checks the one just enqueued) and counts it.
int launched(cudaError_t err, const char* kernel_name);

}  // namespace cppinf::runtime

// Early-return helpers for entry points.
#define CPPINF_REQUIRE(cond, status, msg)                  \
    do {                                                   \
        if (!(cond)) {                                     \
            return ::cppinf::runtime::fail((status), (msg)); \
        }                                                  \
    } while (0)

#define CPPINF_CUDA_TRY(call)                                            \
    do {                                                                 \
        const cudaError_t cppinf_err_ = (call);                          \
        if (cppinf_err_ != cudaSuccess) {                                \
            return ::cppinf::runtime::cuda_fail(cppinf_err_, #call);     \
        }                                                                \
    } while (0)
