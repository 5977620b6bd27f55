// Error state, device binding and launch sizing shared by every entry point.
#include "common.cuh"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

namespace ekv {

namespace {
thread_local std::string g_last_error;
std::mutex g_sm_mutex;
std::vector<int> g_sm_counts;
}  // namespace

void set_error(const std::string& message) { g_last_error = message; }
void clear_error() { g_last_error.clear(); }

void bind_device(int device) {
    require(device >= 0, "device ordinal must be non-negative");
    int current = -1;
    cuda_check(cudaGetDevice(&current), "cudaGetDevice");
    if (current != device) cuda_check(cudaSetDevice(device), "cudaSetDevice");
}

int sm_count(int device) {
    std::lock_guard<std::mutex> lock(g_sm_mutex);
    if (device >= static_cast<int>(g_sm_counts.size())) g_sm_counts.resize(device + 1, 0);
    if (!g_sm_counts[device]) {
        int count = 0;
        cuda_check(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device),
                   "query SM count");
        g_sm_counts[device] = count;
    }
    return g_sm_counts[device];
}

int persistent_grid(const void* kernel, int threads, size_t smem, int device) {
    int per_sm = 0;
    cuda_check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem),
               "occupancy query");
    if (per_sm < 1) per_sm = 1;
    return per_sm * sm_count(device);
}

bool dependent_launch_enabled() {
    static const bool enabled = [] {
        const char* value = std::getenv("EKV_B200_PDL");
        return !(value && std::strcmp(value, "0") == 0);
    }();
    return enabled;
}

}  // namespace ekv

extern "C" const char* ekv_error(void) { return ekv::g_last_error.c_str(); }

extern "C" int ekv_abi_version(void) { return EKV_ABI_VERSION; }
