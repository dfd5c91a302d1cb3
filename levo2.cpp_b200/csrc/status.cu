// Thread-local error reporting and device queries behind the C ABI.
// Mirrors the reference's thread-local last-error pair
// (src/cantor-abi.cpp:55-66): each failing call stores a message that
// levo_ops_last_error() returns on the same thread.
#include <atomic>
#include <string>

#include "common.cuh"

namespace levo {
namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
}  // namespace

int set_error(int code, const std::string &message) {
    g_last_error = message;
    return code;
}

void clear_error() { g_last_error.clear(); }

int check_launch(const char *what) {
    const cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) return LEVO_OPS_OK;
    return set_error(LEVO_OPS_ELAUNCH,
                     std::string(what) + ": kernel launch failed: " + cudaGetErrorString(err));
}

int sm_count() {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return 148;
    int cached = g_sm_count[device].load(std::memory_order_relaxed);
    if (cached > 0) return cached;
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        count <= 0)
        count = 148;
    g_sm_count[device].store(count, std::memory_order_relaxed);
    return count;
}

}  // namespace levo

extern "C" {

LEVO_OPS_API uint32_t levo_ops_abi_version(void) { return LEVO_OPS_ABI; }

LEVO_OPS_API const char *levo_ops_last_error(void) { return levo::g_last_error.c_str(); }

}  // extern "C"
