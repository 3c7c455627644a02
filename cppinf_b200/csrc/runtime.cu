// Status, error-message and launch bookkeeping behind the C ABI (include/cppinf_b200.h).
#include "runtime.h"

#include <mutex>
#include <string>
#include <vector>

namespace cppinf::runtime {
namespace {

thread_local std::string g_last_error;
thread_local bool g_serial_launch = false;  // a SerialLaunch is alive on this thread
std::atomic<uint64_t> g_launches{0};
std::atomic<uint32_t> g_poll_limit{1u << 24};

struct DeviceProps {
    int sm_count = 0;
    int max_threads_per_sm = 0;
};

std::mutex g_props_mutex;
std::vector<DeviceProps> g_props;

const DeviceProps& props_for_current_device() {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        device = 0;
    }
    std::lock_guard<std::mutex> lock(g_props_mutex);
    if (static_cast<int>(g_props.size()) <= device) {
        g_props.resize(static_cast<std::size_t>(device) + 1);
    }
    auto& p = g_props[static_cast<std::size_t>(device)];
    if (p.sm_count == 0) {
        int sms = 0;
        int threads = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
            sms = 148;
        }
        if (cudaDeviceGetAttribute(&threads, cudaDevAttrMaxThreadsPerMultiProcessor, device) != cudaSuccess ||
            threads <= 0) {
            threads = 2048;
        }
        p.sm_count = sms;
        p.max_threads_per_sm = threads;
    }
    return p;
}

}  // namespace

int fail(int status, const std::string& message) {
    g_last_error = message;
    return status;
}

int ok() {
    g_last_error.clear();
    return CPPINF_OK;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(CPPINF_ERR_CUDA, std::string(what) + " failed: " + cudaGetErrorString(err));
}

int after_launch(const char* kernel_name) {
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        return fail(CPPINF_ERR_CUDA, std::string("launch of ") + kernel_name + " failed: " + cudaGetErrorString(err));
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return ok();
}

void count_launches(int64_t n) {
    g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed);
}

int launched(cudaError_t err, const char* kernel_name) {
    if (err != cudaSuccess) {
        cudaGetLastError();  // clear the launch error so it does not leak into later calls
        return fail(CPPINF_ERR_CUDA, std::string("launch of ") + kernel_name + " failed: " + cudaGetErrorString(err));
    }
    return after_launch(kernel_name);
}

int sm_count() {
    return props_for_current_device().sm_count;
}

int max_threads_per_sm() {
    return props_for_current_device().max_threads_per_sm;
}

bool pdl_enabled() {
    return !g_serial_launch;
}

SerialLaunch::SerialLaunch() : previous_(g_serial_launch) {
    g_serial_launch = true;
}

SerialLaunch::~SerialLaunch() {
    g_serial_launch = previous_;
}

uint32_t wait_poll_limit() {
    return g_poll_limit.load(std::memory_order_relaxed);
}

}  // namespace cppinf::runtime

extern "C" {

int cppinf_abi_version(void) {
    return CPPINF_ABI_VERSION;
}

const char* cppinf_last_error(void) {
    return cppinf::runtime::g_last_error.c_str();
}

const char* cppinf_status_name(int status) {
    switch (status) {
    case CPPINF_OK:
        return "CPPINF_OK";
    case CPPINF_ERR_INVALID_ARGUMENT:
        return "CPPINF_ERR_INVALID_ARGUMENT";
    case CPPINF_ERR_OUT_OF_RANGE:
        return "CPPINF_ERR_OUT_OF_RANGE";
    case CPPINF_ERR_OVERFLOW:
        return "CPPINF_ERR_OVERFLOW";
    case CPPINF_ERR_UNSUPPORTED:
        return "CPPINF_ERR_UNSUPPORTED";
    case CPPINF_ERR_CUDA:
        return "CPPINF_ERR_CUDA";
    default:
        return "CPPINF_ERR_UNKNOWN";
    }
}

uint64_t cppinf_launch_count(void) {
    return cppinf::runtime::g_launches.load(std::memory_order_relaxed);
}

uint32_t cppinf_set_wait_poll_limit(uint32_t polls) {
    return cppinf::runtime::g_poll_limit.exchange(polls, std::memory_order_relaxed);
}

}  // extern "C"
