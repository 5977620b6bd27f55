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
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace ekv {
namespace {

struct RowCopyParams {
    const int32_t* plane_index;  // list form when non-null
    const void* slots;
    const void* stage_rows;
    char* staging;
    int64_t stage_plane_stride, row_bytes, n_slots, n_tasks;
    int64_t task_base;  // tasks [task_base, task_base + n_tasks) of the full list
    uint64_t addr_or;   // OR of all plane bases and the staging base
    int slots_es, stage_es, n_planes, to_staging;
    int dense_stage;    // staging row of task t is t - task_base (ring-slot chunks)
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
    for (int64_t local = static_cast<int64_t>(blockIdx.x) * kCopyWarps + (threadIdx.x >> 5);
         local < p.n_tasks; local += warps) {
        const int64_t t = p.task_base + local;
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
        if (p.dense_stage) stage_off = local * p.row_bytes;
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
    static std::atomic<int> cached[64];  // per device; a race computes twice
    int grid = device < 64 ? cached[device].load(std::memory_order_relaxed) : 0;
    if (!grid) {
        grid = persistent_grid(reinterpret_cast<const void*>(row_copy_kernel), kCopyThreads, 0, device);
        if (device < 64) cached[device].store(grid, std::memory_order_relaxed);
    }
    const int64_t needed = (n_tasks + kCopyWarps - 1) / kCopyWarps;
    return static_cast<int>(needed < grid ? needed : grid);
}

// Validated parameters of a task list; the staging side is filled in by the caller.
RowCopyParams task_params(const uint64_t* planes, int n_planes, int64_t row_bytes, const int32_t* plane_index,
                          const void* slots, int slots_esize, int64_t n_slots, int64_t n_tasks,
                          int to_staging) {
    require(planes && slots, "null pointer argument");
    check_esize(slots_esize, "slots");
    if (!plane_index) {
        require(n_tasks == static_cast<int64_t>(n_planes) * n_slots,
                "cross form needs n_tasks == n_planes * n_slots");
    }
    RowCopyParams p{};
    p.plane_index = plane_index;
    p.slots = slots;
    p.row_bytes = row_bytes;
    p.n_slots = n_slots;
    p.n_tasks = n_tasks;
    p.slots_es = slots_esize;
    p.stage_es = 8;
    p.n_planes = n_planes;
    p.to_staging = to_staging;
    uint64_t addr_or = 0;
    for (int i = 0; i < n_planes; ++i) {
        require(planes[i], "null plane address");
        p.planes[i] = reinterpret_cast<char*>(planes[i]);
        addr_or |= planes[i];
    }
    p.addr_or = addr_or;
    return p;
}

void check_sizes(int64_t n_tasks, int64_t n_slots, int64_t row_bytes, int n_planes) {
    require(n_tasks >= 0 && n_slots >= 0, "sizes must be non-negative");
    require(row_bytes > 0, "row_bytes must be positive");
    require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
}

void launch_copy(RowCopyParams& p, int64_t task_base, int64_t count, int device, cudaStream_t stream) {
    p.task_base = task_base;
    p.n_tasks = count;
    row_copy_kernel<<<copy_grid(device, count), kCopyThreads, 0, stream>>>(p);
    check_launch(p.to_staging ? "pack_rows launch" : "unpack_rows launch");
}

cudaMemoryType memory_type(const void* ptr, void** device_view) {
    cudaPointerAttributes attr{};
    cuda_check(cudaPointerGetAttributes(&attr, ptr), "query pointer");
    if (device_view) *device_view = attr.devicePointer;
    return attr.type;
}

int row_copy_impl(const uint64_t* planes, int n_planes, int64_t row_bytes, const int32_t* plane_index,
                  const void* slots, int slots_esize, int64_t n_slots, const void* stage_rows,
                  int stage_rows_esize, const void* staging, int64_t stage_plane_stride_bytes,
                  int64_t n_tasks, int to_staging, int device, void* stream) {
    return guarded([&] {
        check_sizes(n_tasks, n_slots, row_bytes, n_planes);
        if (!n_tasks) return;
        require(staging, "null staging");
        RowCopyParams p = task_params(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots,
                                      n_tasks, to_staging);
        if (stage_rows) check_esize(stage_rows_esize, "stage_rows");
        bind_device(device);
        // Staging must be device memory or pinned host memory mapped into the
        // device address space; anything else is refused here rather than
        // faulting in the kernel.
        void* staging_device = const_cast<void*>(staging);
        void* mapped = nullptr;
        const cudaMemoryType type = memory_type(staging, &mapped);
        if (type == cudaMemoryTypeHost) {
            require(mapped != nullptr, "pinned staging is not mapped for device access");
            staging_device = mapped;
        } else {
            require(type == cudaMemoryTypeDevice || type == cudaMemoryTypeManaged,
                    "staging must be device memory or pinned host memory");
        }
        p.stage_rows = stage_rows;
        p.stage_es = stage_rows ? stage_rows_esize : 8;
        p.staging = static_cast<char*>(staging_device);
        p.stage_plane_stride = stage_plane_stride_bytes;
        p.addr_or |= reinterpret_cast<uint64_t>(staging_device) | static_cast<uint64_t>(stage_plane_stride_bytes);
        launch_copy(p, 0, n_tasks, device, static_cast<cudaStream_t>(stream));
    });
}

// ---------------------------------------------------------------- staged transfers
//
// The copy engines move contiguous ranges between HBM and pinned host memory
// at ~57 / 55 GB/s on this host link, a little more than SM stores / loads
// across the link.  A staged transfer therefore walks the task list in chunks
// through a ring of kRingSlots device slots carved out of the caller's scratch
// buffer: the row-copy kernel packs (or unpacks) one chunk densely into a slot
// on the caller's stream while the copy stream moves another slot across the
// link, one cudaMemcpyAsync per run of rows that are contiguous on the host
// (a "segment").  Events order slot reuse; at the start of a call each stream
// waits for the other's earlier work, and at the end the caller's stream waits
// for the copy stream, so completion of the caller's stream means the transfer
// is complete.  Calls on one device must not overlap (one scheduler thread).

constexpr int kRingSlots = 4;

struct StagedState {
    bool ready = false;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t filled[kRingSlots];
    cudaEvent_t drained[kRingSlots];
    cudaEvent_t caller_mark;
    cudaEvent_t copy_mark;
};

std::mutex g_staged_mutex;
StagedState g_staged[64];

StagedState& staged_state(int device) {
    require(device < 64, "device ordinal too large");
    std::lock_guard<std::mutex> lock(g_staged_mutex);
    StagedState& st = g_staged[device];
    if (!st.ready) {
        cuda_check(cudaStreamCreateWithFlags(&st.copy_stream, cudaStreamNonBlocking), "create copy stream");
        for (int i = 0; i < kRingSlots; ++i) {
            cuda_check(cudaEventCreateWithFlags(&st.filled[i], cudaEventDisableTiming), "create event");
            cuda_check(cudaEventCreateWithFlags(&st.drained[i], cudaEventDisableTiming), "create event");
        }
        cuda_check(cudaEventCreateWithFlags(&st.caller_mark, cudaEventDisableTiming), "create event");
        cuda_check(cudaEventCreateWithFlags(&st.copy_mark, cudaEventDisableTiming), "create event");
        st.ready = true;
    }
    return st;
}

struct Segment {
    int64_t first, count, host_offset;
};

std::vector<Segment> read_segments(const int64_t* segments, int64_t n_segments, int64_t n_tasks) {
    require(segments && n_segments > 0, "staged transfer needs at least one segment");
    std::vector<Segment> out(static_cast<size_t>(n_segments));
    int64_t next = 0;
    for (int64_t i = 0; i < n_segments; ++i) {
        const Segment s{segments[3 * i], segments[3 * i + 1], segments[3 * i + 2]};
        require(s.first == next && s.count > 0 && s.host_offset >= 0,
                "segments must be non-empty, in task order and cover the task list");
        next += s.count;
        out[static_cast<size_t>(i)] = s;
    }
    require(next == n_tasks, "segments must cover exactly n_tasks tasks");
    return out;
}

int staged_impl(const uint64_t* planes, int n_planes, int64_t row_bytes, const int32_t* plane_index,
                const void* slots, int slots_esize, int64_t n_slots, const int64_t* segments,
                int64_t n_segments, const void* host, int64_t n_tasks, void* scratch, int64_t scratch_bytes,
                int to_host, int device, void* stream, void* copy_stream) {
    return guarded([&] {
        check_sizes(n_tasks, n_slots, row_bytes, n_planes);
        if (!n_tasks) return;
        require(host && scratch, "null host staging or scratch");
        const std::vector<Segment> segs = read_segments(segments, n_segments, n_tasks);
        RowCopyParams p = task_params(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots,
                                      n_tasks, to_host);
        bind_device(device);
        require(memory_type(host, nullptr) == cudaMemoryTypeHost,
                "staged transfers need pinned host memory (the copy engine reads / writes it directly)");
        require(memory_type(scratch, nullptr) == cudaMemoryTypeDevice, "scratch must be device memory");
        const int64_t slot_stride = (scratch_bytes / kRingSlots) / 256 * 256;
        const int64_t slot_rows = slot_stride / row_bytes;
        require(slot_rows >= 1, "scratch too small: need room for one row per ring slot");
        StagedState& st = staged_state(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cudaStream_t cs = copy_stream ? static_cast<cudaStream_t>(copy_stream) : st.copy_stream;
        char* ring = static_cast<char*>(scratch);
        char* host_bytes = static_cast<char*>(const_cast<void*>(host));
        p.dense_stage = 1;
        p.addr_or |= reinterpret_cast<uint64_t>(ring) | static_cast<uint64_t>(slot_stride);
        // Each stream first waits for the other's earlier work (slots may still be in use).
        cuda_check(cudaEventRecord(st.caller_mark, s), "record event");
        cuda_check(cudaStreamWaitEvent(cs, st.caller_mark, 0), "wait event");
        cuda_check(cudaEventRecord(st.copy_mark, cs), "record event");
        cuda_check(cudaStreamWaitEvent(s, st.copy_mark, 0), "wait event");
        size_t k = 0;  // first segment that may overlap the current chunk
        int64_t chunk = 0;
        for (int64_t t0 = 0; t0 < n_tasks; t0 += slot_rows, ++chunk) {
            const int64_t t1 = t0 + slot_rows < n_tasks ? t0 + slot_rows : n_tasks;
            const int slot = static_cast<int>(chunk % kRingSlots);
            char* slot_ptr = ring + slot * slot_stride;
            auto move_runs = [&](cudaMemcpyKind kind) {
                while (segs[k].first + segs[k].count <= t0) ++k;
                for (size_t j = k; j < segs.size() && segs[j].first < t1; ++j) {
                    const int64_t a = segs[j].first > t0 ? segs[j].first : t0;
                    const int64_t end = segs[j].first + segs[j].count;
                    const int64_t b = end < t1 ? end : t1;
                    char* h = host_bytes + segs[j].host_offset + (a - segs[j].first) * row_bytes;
                    char* d = slot_ptr + (a - t0) * row_bytes;
                    const size_t bytes = static_cast<size_t>((b - a) * row_bytes);
                    if (kind == cudaMemcpyDeviceToHost) {
                        cuda_check(cudaMemcpyAsync(h, d, bytes, kind, cs), "copy slot to host");
                    } else {
                        cuda_check(cudaMemcpyAsync(d, h, bytes, kind, cs), "copy host to slot");
                    }
                }
            };
            p.staging = slot_ptr;
            if (to_host) {
                if (chunk >= kRingSlots) cuda_check(cudaStreamWaitEvent(s, st.drained[slot], 0), "wait event");
                launch_copy(p, t0, t1 - t0, device, s);
                cuda_check(cudaEventRecord(st.filled[slot], s), "record event");
                cuda_check(cudaStreamWaitEvent(cs, st.filled[slot], 0), "wait event");
                move_runs(cudaMemcpyDeviceToHost);
                cuda_check(cudaEventRecord(st.drained[slot], cs), "record event");
            } else {
                if (chunk >= kRingSlots) cuda_check(cudaStreamWaitEvent(cs, st.drained[slot], 0), "wait event");
                move_runs(cudaMemcpyHostToDevice);
                cuda_check(cudaEventRecord(st.filled[slot], cs), "record event");
                cuda_check(cudaStreamWaitEvent(s, st.filled[slot], 0), "wait event");
                launch_copy(p, t0, t1 - t0, device, s);
                cuda_check(cudaEventRecord(st.drained[slot], s), "record event");
            }
        }
        // The caller's stream completes only after the copy stream's last transfer.
        cuda_check(cudaEventRecord(st.copy_mark, cs), "record event");
        cuda_check(cudaStreamWaitEvent(s, st.copy_mark, 0), "wait event");
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

extern "C" int ekv_pack_rows_staged(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    void* host_staging, int64_t n_tasks,
    void* scratch, int64_t scratch_bytes,
    int device, void* stream, void* copy_stream) {
    return ekv::staged_impl(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots, segments,
                            n_segments, host_staging, n_tasks, scratch, scratch_bytes, 1, device, stream,
                            copy_stream);
}

extern "C" int ekv_unpack_rows_staged(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    const void* host_staging, int64_t n_tasks,
    void* scratch, int64_t scratch_bytes,
    int device, void* stream, void* copy_stream) {
    return ekv::staged_impl(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots, segments,
                            n_segments, host_staging, n_tasks, scratch, scratch_bytes, 0, device, stream,
                            copy_stream);
}

// ---------------------------------------------------------------- staged demotion without allocation
//
// Some callers cannot allocate device memory at the moment they demote: a
// serving engine that reserved all of HBM for its KV pool at start-up (the very
// pressure that triggers a demotion leaves nothing to allocate from), a C / Go
// / Java host that has no device allocator of its own, or code that must not
// touch the allocator in the middle of a step.  ekv_pack_rows_staged_noalloc
// stages through a ring that belongs to the library: a file-scope device array
// of kStaticRingBytes (4 slots of 2 MiB) that every GPU loading the library
// holds until the process exits.  Host code only handles its address, which is
// looked up once per device with that device current (the first call on a
// device does this, so make that first call before any stream capture).  All
// calls share the ring: calls that overlap on the GPU race, and the ring keeps
// the previous call's bytes (nothing in it needs to start at zero, since every
// slot row is written before it is copied out).

namespace {
constexpr int64_t kStaticRingBytes = int64_t{8} << 20;
std::mutex g_static_ring_mutex;
void* g_static_ring_address[64] = {};
}  // namespace

static __device__ __align__(256) unsigned char ekv_static_staging_ring[kStaticRingBytes];

extern "C" int ekv_pack_rows_staged_noalloc(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    void* host_staging, int64_t n_tasks,
    int device, void* stream, void* copy_stream) {
    void* ring = nullptr;
    const int status = ekv::guarded([&] {
        ekv::require(row_bytes > 0 && row_bytes <= kStaticRingBytes / 4,
                     "row_bytes is larger than a slot of the built-in staging ring (2 MiB); "
                     "use ekv_pack_rows_staged with a caller-provided scratch buffer");
        ekv::require(device >= 0 && device < 64, "device ordinal outside [0, 64)");
        std::lock_guard<std::mutex> lock(g_static_ring_mutex);
        if (!g_static_ring_address[device]) {
            ekv::bind_device(device);
            void* address = nullptr;
            ekv::cuda_check(cudaGetSymbolAddress(&address, ekv_static_staging_ring),
                            "look up the built-in staging ring");
            ekv::require(address != nullptr, "built-in staging ring has no device address");
            g_static_ring_address[device] = address;
        }
        ring = g_static_ring_address[device];
    });
    if (status) return status;
    return ekv::staged_impl(planes, n_planes, row_bytes, plane_index, slots, slots_esize, n_slots, segments,
                            n_segments, host_staging, n_tasks, ring, kStaticRingBytes, 1, device, stream,
                            copy_stream);
}
