// Demote / promote row movement (R5).
//
// The reference moves a request's committed rows between the device KV planes
// and SGLang's host KV pool with HostKVCache.backup_from_device_all_layer
// (adaptive_sparse/migration.py:109-111: every layer, K and V, rows at
// physical[:len]) and load_to_device_per_layer (migration.py:231-237: one layer,
// host rows -> destination slots).  Both are scattered row copies; here they are
// one kernel over a task list.  Each task copies one row between
//     planes[p] + slot * row_bytes      and      staging + staging_offset
// in either direction.  `staging` is device memory (followed by a copy-engine
// transfer) or pinned host memory mapped into the device address space, in
// which case the kernel's 16-byte stores / loads cross the host link directly
// (posted writes for demotion, so the SMs never wait on the link for it).
// A warp moves one row per step with kUnroll vectors per lane in flight; the
// grid is persistent.
#include "common.cuh"

namespace ekv {
namespace {

struct RowCopyParams {
    const int32_t* plane_index;  // list form when non-null
    const void* slots;
    const void* stage_rows;
    char* staging;
    int64_t stage_plane_stride, row_bytes, n_slots, n_tasks;
    uint64_t addr_or;  // OR of all plane bases and the staging base
    int slots_es, stage_es, n_planes, to_staging;
    char* planes[EKV_MAX_PLANES];
};

constexpr int kCopyThreads = 256;
constexpr int kCopyWarps = kCopyThreads / 32;
constexpr int kUnroll = 4;

template <typename T, int U>
__device__ __forceinline__ void warp_copy(const char* src, char* dst, int64_t n_elems, unsigned lane) {
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    for (int64_t base = 0; base < n_elems; base += 32 * U) {
        T v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t e = base + u * 32 + lane;
            if (e < n_elems) v[u] = s[e];
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t e = base + u * 32 + lane;
            if (e < n_elems) d[e] = v[u];
        }
    }
}

__global__ void __launch_bounds__(kCopyThreads)
row_copy_kernel(const __grid_constant__ RowCopyParams p) {
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kCopyWarps;
    const unsigned lane = lane_id();
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kCopyWarps + (threadIdx.x >> 5); t < p.n_tasks;
         t += warps) {
        int64_t plane, slot, stage_off;
        if (p.plane_index) {
            plane = p.plane_index[t];
            slot = load_index(p.slots, p.slots_es, t);
            const int64_t stage_row = p.stage_rows ? load_index(p.stage_rows, p.stage_es, t) : t;
            stage_off = stage_row * p.row_bytes;
        } else {
            plane = t / p.n_slots;
            const int64_t j = t - plane * p.n_slots;
            slot = load_index(p.slots, p.slots_es, j);
            const int64_t stage_row = p.stage_rows ? load_index(p.stage_rows, p.stage_es, j) : j;
            stage_off = plane * p.stage_plane_stride + stage_row * p.row_bytes;
        }
        if (plane < 0 || plane >= p.n_planes) continue;  // never index past the plane table
        char* device_row = p.planes[plane] + slot * p.row_bytes;
        char* stage_row = p.staging + stage_off;
        const char* src = p.to_staging ? device_row : stage_row;
        char* dst = p.to_staging ? stage_row : device_row;
        const int64_t align = alignment_of(p.addr_or | static_cast<uint64_t>(slot * p.row_bytes) |
                                           static_cast<uint64_t>(stage_off) |
                                           static_cast<uint64_t>(p.row_bytes));
        switch (align) {
            case 16: warp_copy<uint4, kUnroll>(src, dst, p.row_bytes >> 4, lane); break;
            case 8: warp_copy<uint64_t, kUnroll>(src, dst, p.row_bytes >> 3, lane); break;
            case 4: warp_copy<uint32_t, kUnroll>(src, dst, p.row_bytes >> 2, lane); break;
            case 2: warp_copy<uint16_t, kUnroll>(src, dst, p.row_bytes >> 1, lane); break;
            default: warp_copy<uint8_t, kUnroll>(src, dst, p.row_bytes, lane); break;
        }
    }
}

int copy_grid(int device, int64_t n_tasks) {
    static int cached[64] = {0};
    int grid = device < 64 ? cached[device] : 0;
    if (!grid) {
        grid = persistent_grid(reinterpret_cast<const void*>(row_copy_kernel), kCopyThreads, 0, device);
        if (device < 64) cached[device] = grid;
    }
    const int64_t needed = (n_tasks + kCopyWarps - 1) / kCopyWarps;
    return static_cast<int>(needed < grid ? needed : grid);
}

int row_copy_impl(const uint64_t* planes, int n_planes, int64_t row_bytes, const int32_t* plane_index,
                  const void* slots, int slots_esize, int64_t n_slots, const void* stage_rows,
                  int stage_rows_esize, const void* staging, int64_t stage_plane_stride_bytes,
                  int64_t n_tasks, int to_staging, int device, void* stream) {
    return guarded([&] {
        require(n_tasks >= 0 && n_slots >= 0, "sizes must be non-negative");
        require(row_bytes > 0, "row_bytes must be positive");
        require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
        if (!n_tasks) return;
        require(planes && slots && staging, "null pointer argument");
        check_esize(slots_esize, "slots");
        if (stage_rows) check_esize(stage_rows_esize, "stage_rows");
        if (!plane_index) {
            require(n_tasks == static_cast<int64_t>(n_planes) * n_slots,
                    "cross form needs n_tasks == n_planes * n_slots");
        }
        bind_device(device);
        // Staging must be device memory or pinned host memory mapped into the
        // device address space; anything else is refused here rather than
        // faulting in the kernel.
        cudaPointerAttributes attr{};
        cuda_check(cudaPointerGetAttributes(&attr, staging), "query staging pointer");
        void* staging_device = const_cast<void*>(staging);
        if (attr.type == cudaMemoryTypeHost) {
            require(attr.devicePointer != nullptr, "pinned staging is not mapped for device access");
            staging_device = attr.devicePointer;
        } else {
            require(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
                    "staging must be device memory or pinned host memory");
        }
        RowCopyParams p{};
        p.plane_index = plane_index;
        p.slots = slots;
        p.stage_rows = stage_rows;
        p.staging = static_cast<char*>(staging_device);
        p.stage_plane_stride = stage_plane_stride_bytes;
        p.row_bytes = row_bytes;
        p.n_slots = n_slots;
        p.n_tasks = n_tasks;
        p.slots_es = slots_esize;
        p.stage_es = stage_rows ? stage_rows_esize : 8;
        p.n_planes = n_planes;
        p.to_staging = to_staging;
        uint64_t addr_or = reinterpret_cast<uint64_t>(staging_device) |
                           static_cast<uint64_t>(stage_plane_stride_bytes);
        for (int i = 0; i < n_planes; ++i) {
            require(planes[i], "null plane address");
            p.planes[i] = reinterpret_cast<char*>(planes[i]);
            addr_or |= planes[i];
        }
        p.addr_or = addr_or;
        bind_device(device);
        row_copy_kernel<<<copy_grid(device, n_tasks), kCopyThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(p);
        check_launch(to_staging ? "pack_rows launch" : "unpack_rows launch");
    });
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_pack_rows(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const void* stage_rows, int stage_rows_esize,
    void* staging, int64_t stage_plane_stride_bytes, int64_t n_tasks,
    int device, void* stream) {
    return ekv::row_copy_impl(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots,
                              stage_rows, stage_rows_esize, staging, stage_plane_stride_bytes,
                              n_tasks, 1, device, stream);
}

extern "C" int ekv_unpack_rows(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const void* stage_rows, int stage_rows_esize,
    const void* staging, int64_t stage_plane_stride_bytes, int64_t n_tasks,
    int device, void* stream) {
    return ekv::row_copy_impl(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots,
                              stage_rows, stage_rows_esize, staging, stage_plane_stride_bytes,
                              n_tasks, 0, device, stream);
}
