// Thread-local error reporting and device queries behind the C ABI.
// Mirrors the reference's thread-local last-error pair
// (src/cantor-abi.cpp:55-66): each failing call stores a message that
// levo_ops_last_error() returns on the same thread.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

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

cudaError_t resident_ctas(const void *kernel, int threads, size_t smem_bytes, int *per_sm) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    static std::mutex mu;
    static std::map<std::tuple<const void *, int, int, size_t>, int> occupancy;  // (kernel, device, threads, smem)
    static std::map<std::pair<const void *, int>, size_t> opted;                  // (kernel, device) -> smem
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(kernel, device, threads, smem_bytes);
    const auto hit = occupancy.find(key);
    if (hit != occupancy.end()) {
        *per_sm = hit->second;
        return cudaSuccess;
    }
    if (smem_bytes > 48 * 1024) {
        // the opt-in only ever grows, so an earlier, larger launch of this kernel stays valid
        size_t &limit = opted[std::make_pair(kernel, device)];
        if (limit < smem_bytes) {
            err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem_bytes));
            if (err != cudaSuccess) return err;
            limit = smem_bytes;
        }
    }
    int n = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem_bytes);
    if (err != cudaSuccess) return err;
    n = std::max(n, 1);
    occupancy.emplace(key, n);
    *per_sm = n;
    return cudaSuccess;
}

}  // namespace levo

extern "C" {

LEVO_OPS_API uint32_t levo_ops_abi_version(void) { return LEVO_OPS_ABI; }

LEVO_OPS_API const char *levo_ops_last_error(void) { return levo::g_last_error.c_str(); }

}  // extern "C"
