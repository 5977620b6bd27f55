// Shared helpers of libekv_b200.so: error reporting, device binding, launch
// sizing and the small device-side primitives every kernel uses.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

#include "../../../include/ekv_kernels.h"

namespace ekv {

struct Error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void set_error(const std::string& message);
void clear_error();

inline void require(bool ok, const std::string& message) {
    if (!ok) throw Error(message);
}

inline void cuda_check(cudaError_t status, const char* what) {
    if (status != cudaSuccess) {
        throw Error(std::string(what) + ": " + cudaGetErrorString(status));
    }
}

// Run `body`, turning any exception into -1 plus a thread-local message.
template <class Body>
int guarded(Body&& body) {
    try {
        clear_error();
        body();
        return 0;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    } catch (...) {
        set_error("unknown C++ error");
        return -1;
    }
}

// Make `device` current for this thread (in this library's runtime instance).
void bind_device(int device);
// Multiprocessor count of `device`, cached.
int sm_count(int device);
// Persistent grid size for `kernel` with `threads` per block: SMs x resident blocks.
int persistent_grid(const void* kernel, int threads, size_t smem, int device);

inline void check_esize(int esize, const char* name) {
    if (esize != 4 && esize != 8) {
        throw Error(std::string(name) + " element size must be 4 or 8");
    }
}

inline void check_launch(const char* what) {
    cuda_check(cudaGetLastError(), what);
}

// Whether kernels of a decode step are launched as programmatic dependents of
// the work before them in their stream (EKV_B200_PDL=0 turns it off).
bool dependent_launch_enabled();

// Launch `kernel` as a programmatic dependent of the previous work in `stream`:
// its blocks may be scheduled while that work finishes (once every block of a
// preceding kernel has called allow_dependents() or exited), which hides the
// launch latency between the short per-layer kernels of a decode step.  The
// kernel must call grid_dependency_wait() before its first global memory
// access; that wait returns when the preceding grids have completed and their
// writes are visible.
template <typename... Params, typename... Args>
void launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      const char* what, Args&&... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = dependent_launch_enabled() ? 1 : 0;
    cuda_check(cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...), what);
}

// ---------------------------------------------------------------- device side

// Read element i of a signed int32 / int64 array.
__device__ __forceinline__ int64_t load_index(const void* base, int esize, int64_t i) {
    return esize == 8 ? static_cast<const int64_t*>(base)[i]
                      : static_cast<int64_t>(static_cast<const int32_t*>(base)[i]);
}

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// Programmatic dependent launch, device side.  grid_dependency_wait(): block
// until the grids this one was launched behind have completed and their memory
// is visible (immediate for an ordinary launch).  allow_dependents(): let the
// next kernel of the stream start scheduling its blocks; it still waits for
// this grid to complete before reading anything.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Lowest power of two (<= 16) dividing x.
__device__ __forceinline__ int64_t alignment_of(uint64_t x) {
    if (x & 1u) return 1;
    if (x & 2u) return 2;
    if (x & 4u) return 4;
    if (x & 8u) return 8;
    return 16;
}

}  // namespace ekv
