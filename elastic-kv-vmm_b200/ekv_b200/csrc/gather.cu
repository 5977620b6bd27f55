// Top-K K/V row gather (R3).
//
// Semantics of the Triton `_gather` kernel (experimental/sparse_read.py:11-30):
// row (b, i) of the output is the `width`-element row of `raw` at element offset
//     indirect: slot_offsets[request_table[req, pos]]
//     direct:   sink + req * request_stride + pos * width
// or zeros when pos is outside [0, lengths[b]).  Payload bytes are copied bit
// for bit.
//
// B200 design: the work is pure HBM traffic (a 2 KiB K row + a 2 KiB V row per
// token per layer at the Qwen3-4B-like layout), so one launch covers every
// plane (all layers, K and V): a warp resolves the index chains of 32 rows at
// once (one per lane) and then streams each row out of all planes.  Copies are
// 16-byte vector loads and stores with evict-first hints (each byte is read
// once and written once); each lane keeps kUnroll vectors in flight before
// storing, ~64 KiB of reads outstanding per SM at 16 resident warps, which is
// above the HBM bandwidth-latency product without adding so many concurrent
// random streams that DRAM efficiency drops.  The grid is persistent: SMs x
// resident blocks.  Rows whose addresses are not 16-byte aligned fall back to
// the widest element size that divides every address.  A bulk-copy (TMA
// engine) variant is kept for comparison; see bulk_allowed().
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "bulk.cuh"
#include "common.cuh"

namespace ekv {
namespace {

struct GatherParams {
    const void* positions;
    const void* request_ids;
    const void* lengths;
    const void* request_table;
    const void* slot_offsets;
    int64_t batch, selected, width, itemsize, row_bytes;
    int64_t table_width, request_stride, sink_elements;
    uint64_t plane_or;  // OR of all plane base addresses, for the alignment test
    int pos_es, req_es, len_es, table_es, off_es;
    int indirect;
    int n_planes;
    int vec_shift;  // log2(row_bytes / 16) when that is a power of two, else -1
    const char* src[EKV_MAX_PLANES];
    char* dst[EKV_MAX_PLANES];
};

// Tuning of the register-staged kernel (overridable at build time for sweeps).
// Measured on B200 (config 2, 36 layers): 2 blocks x 8 warps per SM with 8
// vectors per lane (~64 KiB of reads in flight per SM) gives 0.962 of the
// measured copy peak at 2 KiB rows and 0.90 at 256 B rows; 4 blocks per SM
// (more concurrent random streams) drops to 0.91 / 0.85.
#ifndef EKV_GATHER_MIN_BLOCKS
#define EKV_GATHER_MIN_BLOCKS 2  // resident 256-thread blocks per SM the register cap aims for
#endif
#ifndef EKV_GATHER_UNROLL
#define EKV_GATHER_UNROLL 8      // 16-byte vectors in flight per lane
#endif
#ifndef EKV_GATHER_BATCH_RESOLVE
#define EKV_GATHER_BATCH_RESOLVE 1  // resolve 32 rows' index chains at once (one per lane)
#endif

constexpr int kGatherThreads = 256;
constexpr int kGatherWarps = kGatherThreads / 32;
constexpr int kGatherBlocksPerSM = EKV_GATHER_MIN_BLOCKS;
constexpr int kUnroll = EKV_GATHER_UNROLL;

// Rows of at most EKV_GATHER_SMALL_ROW_BYTES per plane (the 256 B rows of a TP8 head
// shard) over more planes than the default instance flattens (all layers' K and V
// in one launch) take a second instance of the kernel: every aligned batch
// flattened and EKV_GATHER_SMALL_UNROLL vectors in flight per lane.  Measured on
// B200 (config 2, 36 layers): 0.916 instead of 0.902 of the copy peak at 256 B rows,
// while at 512 B and 2 KiB rows the same setting was 0.4-0.7 % slower.  A launch
// over few planes (one layer) keeps the default instance: it already flattens
// them, and its 86 registers leave room on each SM for a lookup block beside two
// gather blocks (the small-row instance takes 94).
#ifndef EKV_GATHER_SMALL_ROW_BYTES
#define EKV_GATHER_SMALL_ROW_BYTES 256  // 0 turns the small-row instance off
#endif
#ifndef EKV_GATHER_SMALL_UNROLL
#define EKV_GATHER_SMALL_UNROLL 12
#endif
constexpr int64_t kSmallRowBytes = EKV_GATHER_SMALL_ROW_BYTES;
constexpr int kSmallUnroll = EKV_GATHER_SMALL_UNROLL;

// Byte offset of row r inside every source plane, or valid = false.
__device__ __forceinline__ int64_t resolve_row(const GatherParams& p, int64_t r, bool& valid) {
    const int64_t b = r / p.selected;
    const int64_t pos = load_index(p.positions, p.pos_es, r);
    const int64_t length = load_index(p.lengths, p.len_es, b);
    valid = pos >= 0 && pos < length;
    if (!valid) return 0;
    const int64_t req = load_index(p.request_ids, p.req_es, b);
    int64_t element;
    if (p.indirect == 1) {
        const int64_t logical = load_index(p.request_table, p.table_es, req * p.table_width + pos);
        element = load_index(p.slot_offsets, p.off_es, logical);
    } else if (p.indirect == 2) {
        // Mapped: the table holds the row's slot in the request's fixed region, -1 if
        // absent; a slot past the region reads as absent too (never outside the region).
        const int64_t slot = load_index(p.request_table, p.table_es, req * p.table_width + pos);
        if (slot < 0 || (slot + 1) * p.width > p.request_stride) {
            valid = false;
            return 0;
        }
        element = p.sink_elements + req * p.request_stride + slot * p.width;
    } else {
        element = p.sink_elements + req * p.request_stride + pos * p.width;
    }
    return element * p.itemsize;
}

#ifndef EKV_GATHER_STREAMING
#define EKV_GATHER_STREAMING 1  // evict-first hints on payload loads and stores
#endif

__device__ __forceinline__ uint4 load_vec(const uint4* src) {
#if EKV_GATHER_STREAMING
    return __ldcs(src);
#else
    return __ldg(src);
#endif
}

__device__ __forceinline__ void store_vec(uint4* dst, uint4 value) {
#if EKV_GATHER_STREAMING
    __stcs(dst, value);
#else
    *dst = value;
#endif
}

__device__ __forceinline__ void copy_row_vec16(const GatherParams& p, bool valid, int64_t src_off,
                                               int64_t dst_off, unsigned lane) {
    const int64_t vecs = p.row_bytes >> 4;
    const int64_t total = static_cast<int64_t>(p.n_planes) * vecs;
    for (int64_t base = 0; base < total; base += 32 * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t idx = base + u * 32 + lane;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (valid && idx < total) {
                const int64_t plane = p.vec_shift >= 0 ? (idx >> p.vec_shift) : idx / vecs;
                const int64_t vec = idx - plane * vecs;
                v[u] = load_vec(reinterpret_cast<const uint4*>(p.src[plane] + src_off) + vec);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t idx = base + u * 32 + lane;
            if (idx < total) {
                const int64_t plane = p.vec_shift >= 0 ? (idx >> p.vec_shift) : idx / vecs;
                const int64_t vec = idx - plane * vecs;
                store_vec(reinterpret_cast<uint4*>(p.dst[plane] + dst_off) + vec, v[u]);
            }
        }
    }
}

template <typename T>
__device__ __forceinline__ void copy_row_elems(const GatherParams& p, bool valid, int64_t src_off,
                                               int64_t dst_off, unsigned lane) {
    const int64_t elems = p.row_bytes / static_cast<int64_t>(sizeof(T));
    const int64_t total = static_cast<int64_t>(p.n_planes) * elems;
    for (int64_t idx = lane; idx < total; idx += 32) {
        const int64_t plane = idx / elems;
        const int64_t e = idx - plane * elems;
        T value = T(0);
        if (valid) value = reinterpret_cast<const T*>(p.src[plane] + src_off)[e];
        reinterpret_cast<T*>(p.dst[plane] + dst_off)[e] = value;
    }
}

// Warp-cooperative copy of one row out of every plane, any alignment.
__device__ __forceinline__ void copy_row_any(const GatherParams& p, bool valid, int64_t src_off,
                                             int64_t dst_off, unsigned lane) {
    const int64_t align = alignment_of(p.plane_or | static_cast<uint64_t>(src_off) |
                                       static_cast<uint64_t>(dst_off) | static_cast<uint64_t>(p.row_bytes));
    switch (align) {
        case 16: copy_row_vec16(p, valid, src_off, dst_off, lane); break;
        case 8: copy_row_elems<uint64_t>(p, valid, src_off, dst_off, lane); break;
        case 4: copy_row_elems<uint32_t>(p, valid, src_off, dst_off, lane); break;
        case 2: copy_row_elems<uint16_t>(p, valid, src_off, dst_off, lane); break;
        default: copy_row_elems<uint8_t>(p, valid, src_off, dst_off, lane); break;
    }
}

// Copy of a whole batch of rows (row k of the batch is row0 + k * warps, its
// byte offset in lane k's `mine`) when a row is small: the (row, plane, vector)
// space is flattened so that the kUnroll vectors each lane keeps in flight span
// several rows.  Every address must be 16-byte aligned.
#ifndef EKV_GATHER_FLAT_LIMIT
#define EKV_GATHER_FLAT_LIMIT (32 * kUnroll)
#endif
constexpr uint32_t kFlatRowLimit = EKV_GATHER_FLAT_LIMIT;  // vectors per row (all planes) up to which to flatten

template <int kU>
__device__ __forceinline__ void copy_batch_vec16(const GatherParams& p, int64_t mine, int64_t row0,
                                                 int64_t warps, int nb, unsigned lane) {
    const uint32_t vecs = static_cast<uint32_t>(p.row_bytes >> 4);
    const uint32_t per_row = static_cast<uint32_t>(p.n_planes) * vecs;
    const uint32_t total = static_cast<uint32_t>(nb) * per_row;
    for (uint32_t base = 0; base < total; base += 32 * kU) {
        uint4 v[kU];
        uint32_t row_of[kU];
        uint32_t rem_of[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint32_t idx = base + u * 32 + lane;
            const uint32_t k = idx < total ? idx / per_row : 0;
            const int64_t s = __shfl_sync(0xffffffffu, mine, static_cast<int>(k));
            const uint32_t rem = idx - k * per_row;
            row_of[u] = k;
            rem_of[u] = rem;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (idx < total && s >= 0) {
                const uint32_t plane = p.vec_shift >= 0 ? (rem >> p.vec_shift) : rem / vecs;
                const uint32_t vec = rem - plane * vecs;
                v[u] = load_vec(reinterpret_cast<const uint4*>(p.src[plane] + s) + vec);
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint32_t idx = base + u * 32 + lane;
            if (idx < total) {
                const uint32_t plane = p.vec_shift >= 0 ? (rem_of[u] >> p.vec_shift) : rem_of[u] / vecs;
                const uint32_t vec = rem_of[u] - plane * vecs;
                char* row = p.dst[plane] + (row0 + static_cast<int64_t>(row_of[u]) * warps) * p.row_bytes;
                store_vec(reinterpret_cast<uint4*>(row) + vec, v[u]);
            }
        }
    }
}

// Rows are taken 32 at a time per warp (row0 + k * warps, k < 32): every lane
// resolves one row's index chain, so the three dependent index loads are paid
// once per 32 rows instead of once per row; the warp then streams each row out
// of all planes with the offset broadcast from its lane.
//
// kU: vectors in flight per lane in the flattened batch copy; kFlatAll: flatten
// every 16-byte-aligned batch, whatever its row size (the small-row instance,
// whose rows x planes x vectors stay far below 2^32).
template <int kU, bool kFlatAll>
__global__ void __launch_bounds__(kGatherThreads, kGatherBlocksPerSM)
gather_kernel(const __grid_constant__ GatherParams p) {
    grid_dependency_wait();
    allow_dependents();
    const int64_t n_rows = p.batch * p.selected;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kGatherWarps;
    const unsigned lane = lane_id();
#if !EKV_GATHER_BATCH_RESOLVE
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5); r < n_rows;
         r += warps) {
        bool valid;
        const int64_t src = resolve_row(p, r, valid);
        copy_row_any(p, valid, src, r * p.row_bytes, lane);
    }
#else
    for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5); row0 < n_rows;
         row0 += 32 * warps) {
        const int64_t r = row0 + static_cast<int64_t>(lane) * warps;
        bool valid = false;
        int64_t src = 0;
        if (r < n_rows) src = resolve_row(p, r, valid);
        const int64_t mine = valid ? src : -1;
        const int64_t left = (n_rows - row0 + warps - 1) / warps;
        const int nb = static_cast<int>(left < 32 ? left : 32);
        const bool small_rows = p.row_bytes % 16 == 0 && p.plane_or % 16 == 0 &&
                                (kFlatAll || static_cast<uint64_t>(p.n_planes) * (p.row_bytes >> 4) <= kFlatRowLimit);
        if (small_rows && !__ballot_sync(0xffffffffu, valid && (src & 15))) {
            copy_batch_vec16<kU>(p, mine, row0, warps, nb, lane);
            continue;
        }
        for (int k = 0; k < nb; ++k) {
            const int64_t s = __shfl_sync(0xffffffffu, mine, k);
            copy_row_any(p, s >= 0, s < 0 ? 0 : s, (row0 + k * warps) * p.row_bytes, lane);
        }
    }
#endif
}

// ---------------------------------------------------------------- bulk (TMA engine) variant
//
// Each warp is an independent copy pipeline run by its lane 0: a ring of
// `slots` shared-memory row buffers, one mbarrier per slot.  Rows come in
// batches of 32 (one per lane): all lanes resolve their row's index chain in
// parallel, then lane 0 streams batch-rows x planes items -- bulk load of item
// i + lookahead into its slot, wait for item i, bulk store of item i from its
// slot -- so ~lookahead rows per warp are in flight with no register staging.
// A slot is refilled only after the store that last read it has finished
// reading (bulk wait_group.read), and invalid rows are stored from a shared
// zero row.  Every wait is bounded; an abandoned wait sets g_gather_status.

constexpr int kBulkWarps = 8;
constexpr int kBulkThreads = kBulkWarps * 32;
constexpr int kStoreLag = 8;               // stores allowed to still read their slot when it is refilled: lag - 1
constexpr int kMaxSlots = 32;
constexpr uint32_t kWaitPolls = 1u << 22;  // try_wait polls before a wait is abandoned

__device__ unsigned int g_gather_status;

__global__ void __launch_bounds__(kBulkThreads, 1)
gather_bulk_kernel(const __grid_constant__ GatherParams p, int slots, int slot_bytes) {
    extern __shared__ __align__(128) unsigned char smem[];
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    unsigned char* payload = smem;  // [warps][slots][slot_bytes]
    unsigned char* zero_row = payload + static_cast<size_t>(kBulkWarps) * slots * slot_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(zero_row + slot_bytes);           // [warps][slots]
    int64_t* row_src = reinterpret_cast<int64_t*>(bars + kBulkWarps * slots);      // [warps][32]

    if (lane == 0) {
        for (int s = 0; s < slots; ++s) bulk::mbar_init(bulk::smem_addr(bars + warp * slots + s), 1);
    }
    for (int i = threadIdx.x; i < slot_bytes / 16; i += kBulkThreads) {
        reinterpret_cast<uint4*>(zero_row)[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    bulk::fence_barrier_init();
    bulk::fence_async_shared();
    __syncthreads();

    const uint64_t policy = bulk::policy_evict_first();
    const int64_t n_rows = p.batch * p.selected;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kBulkWarps;
    const uint32_t row_bytes = static_cast<uint32_t>(p.row_bytes);
    const int lookahead = slots - kStoreLag;
    int64_t* my_src = row_src + warp * 32;
    const uint32_t my_payload = bulk::smem_addr(payload + static_cast<size_t>(warp) * slots * slot_bytes);
    const uint32_t my_bars = bulk::smem_addr(bars + warp * slots);
    const uint32_t zero_addr = bulk::smem_addr(zero_row);
    uint64_t done = 0;  // items this warp has pushed through its ring
    bool failed = false;

    for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * kBulkWarps + warp; row0 < n_rows;
         row0 += 32 * warps) {
        const int64_t r = row0 + static_cast<int64_t>(lane) * warps;
        int64_t src = -1;
        bool aligned = true;
        if (r < n_rows) {
            bool valid;
            const int64_t off = resolve_row(p, r, valid);
            if (valid) {
                src = off;
                aligned = (off & 15) == 0;
            }
        }
        const int64_t left = (n_rows - row0 + warps - 1) / warps;
        const int nb = static_cast<int>(left < 32 ? left : 32);
        if (__ballot_sync(0xffffffffu, !aligned)) {
            // A row of this batch is not 16-byte aligned: vector / element copies.
            for (int k = 0; k < nb; ++k) {
                const int64_t s = __shfl_sync(0xffffffffu, src, k);
                copy_row_any(p, s >= 0, s < 0 ? 0 : s, (row0 + k * warps) * p.row_bytes, lane);
            }
            continue;
        }
        my_src[lane] = src;
        __syncwarp();
        if (lane == 0 && !failed) {
            const int64_t items = static_cast<int64_t>(nb) * p.n_planes;
            int64_t issued = 0;
            int issue_row = 0, issue_plane = 0, store_row = 0, store_plane = 0;
            auto issue = [&]() {
                const uint64_t g = done + issued;
                const uint32_t slot = static_cast<uint32_t>(g % slots);
                if (g >= static_cast<uint64_t>(slots)) bulk::wait_read<kStoreLag - 1>();
                const uint32_t bar = my_bars + slot * 8u;
                const int64_t s = my_src[issue_row];
                if (s < 0) {
                    bulk::mbar_arrive(bar);
                } else {
                    bulk::mbar_arrive_expect_tx(bar, row_bytes);
                    bulk::load_async(my_payload + slot * static_cast<uint32_t>(slot_bytes),
                                     p.src[issue_plane] + s, row_bytes, bar, policy);
                }
                ++issued;
                if (++issue_plane == p.n_planes) {
                    issue_plane = 0;
                    ++issue_row;
                }
            };
            while (issued < items && issued < lookahead) issue();
            for (int64_t i = 0; i < items; ++i) {
                if (issued < items) issue();
                const uint64_t g = done + i;
                const uint32_t slot = static_cast<uint32_t>(g % slots);
                if (!bulk::mbar_wait_bounded(my_bars + slot * 8u, static_cast<uint32_t>((g / slots) & 1),
                                             kWaitPolls)) {
                    failed = true;
                    atomicOr(&g_gather_status, 1u);
                    for (int64_t k = i + 1; k < issued; ++k) {  // let in-flight loads land
                        const uint64_t gk = done + k;
                        bulk::mbar_wait_bounded(my_bars + static_cast<uint32_t>(gk % slots) * 8u,
                                                static_cast<uint32_t>((gk / slots) & 1), kWaitPolls);
                    }
                    break;
                }
                const int64_t s = my_src[store_row];
                char* dst = p.dst[store_plane] + (row0 + static_cast<int64_t>(store_row) * warps) * p.row_bytes;
                bulk::store_async(dst, s < 0 ? zero_addr : my_payload + slot * static_cast<uint32_t>(slot_bytes),
                                  row_bytes, policy);
                bulk::commit();
                if (++store_plane == p.n_planes) {
                    store_plane = 0;
                    ++store_row;
                }
            }
            done += items;
        }
        __syncwarp();
    }
    if (lane == 0) bulk::wait_all();
}

struct BulkShape {
    int slots = 0;
    int slot_bytes = 0;
    size_t smem = 0;
};

// Ring geometry for rows of `row_bytes`, or slots == 0 when rows are too big.
BulkShape bulk_shape(int device, int64_t row_bytes) {
    static std::atomic<int> optin[64];  // per device; a race queries twice
    int limit = device < 64 ? optin[device].load(std::memory_order_relaxed) : 0;
    if (!limit) {
        cuda_check(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device),
                   "query shared memory limit");
        if (device < 64) optin[device].store(limit, std::memory_order_relaxed);
    }
    BulkShape shape;
    if (row_bytes <= 0 || row_bytes % 16 || row_bytes > (1 << 20)) return shape;
    shape.slot_bytes = static_cast<int>((row_bytes + 127) / 128 * 128);
    const size_t fixed = static_cast<size_t>(shape.slot_bytes) + 8u * 32u * kBulkWarps;
    const size_t per_slot = static_cast<size_t>(kBulkWarps) * (shape.slot_bytes + 8u);
    if (static_cast<size_t>(limit) <= fixed) return BulkShape{};
    int slots = static_cast<int>((static_cast<size_t>(limit) - fixed) / per_slot);
    slots = slots < kMaxSlots ? slots : kMaxSlots;
    if (slots < kStoreLag + 2) return BulkShape{};
    shape.slots = slots;
    shape.smem = fixed + static_cast<size_t>(slots) * per_slot;
    return shape;
}

// EKV_GATHER_KERNEL=bulk selects the bulk-copy kernel (comparison runs).  It is
// not the default: each bulk copy is one TMA-engine operation, and at about
// 28 M operations/s per SM (two per row) it trails the register-staged kernel
// at 2 KiB rows (0.89 vs 0.96 of the copy peak) and is operation-bound at
// smaller rows (4.5 ms per config-2 launch at any row size).
bool bulk_allowed() {
    const char* mode = std::getenv("EKV_GATHER_KERNEL");
    return mode && std::strcmp(mode, "bulk") == 0;
}

using GatherKernel = void (*)(GatherParams);

// The kernel instance for `n_planes` planes of `row_bytes` rows.
GatherKernel gather_kernel_for(int64_t row_bytes, int n_planes, bool& small) {
    small = kSmallRowBytes > 0 && row_bytes <= kSmallRowBytes &&
            static_cast<uint64_t>(n_planes) * (row_bytes >> 4) > kFlatRowLimit;
    return small ? gather_kernel<kSmallUnroll, true> : gather_kernel<kUnroll, false>;
}

int gather_grid(GatherKernel kernel, bool small, int device, int64_t n_rows) {
    static std::atomic<int> cached[2][64];  // per instance and device; a race computes twice
    int grid = device < 64 ? cached[small][device].load(std::memory_order_relaxed) : 0;
    if (!grid) {
        grid = persistent_grid(reinterpret_cast<const void*>(kernel), kGatherThreads, 0, device);
        if (device < 64) cached[small][device].store(grid, std::memory_order_relaxed);
    }
    const int64_t needed = (n_rows + kGatherWarps - 1) / kGatherWarps;
    return static_cast<int>(needed < grid ? needed : grid);
}

int log2_exact(int64_t x) {
    if (x <= 0 || (x & (x - 1))) return -1;
    int shift = 0;
    while ((int64_t{1} << shift) < x) ++shift;
    return shift;
}

int gather_impl(const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
                const void* positions, int positions_esize, const void* request_ids,
                int request_ids_esize, const void* lengths, int lengths_esize,
                const void* request_table, int table_esize, const void* slot_offsets,
                int offsets_esize, int64_t batch, int64_t selected, int64_t width,
                int64_t table_width, int64_t request_stride, int64_t sink_elements, int indirect,
                int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && selected >= 0 && width >= 0, "sizes must be non-negative");
        require(itemsize > 0, "itemsize must be positive");
        require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
        if (!batch || !selected || !width) return;
        require(src_planes && dst_planes, "null plane array");
        require(positions && request_ids && lengths, "null index argument");
        check_esize(positions_esize, "positions");
        check_esize(request_ids_esize, "request_ids");
        check_esize(lengths_esize, "lengths");
        require(indirect >= 0 && indirect <= 2, "addressing mode must be 0 (direct), 1 (indirect) or 2 (mapped)");
        if (indirect == 1) {
            require(request_table && slot_offsets, "indirect gather needs request_table and slot_offsets");
            check_esize(table_esize, "request_table");
            check_esize(offsets_esize, "slot_offsets");
        } else if (indirect == 2) {
            require(request_table, "mapped gather needs request_table (the residency map)");
            check_esize(table_esize, "request_table");
        }
        GatherParams p{};
        p.positions = positions;
        p.request_ids = request_ids;
        p.lengths = lengths;
        p.request_table = request_table;
        p.slot_offsets = slot_offsets;
        p.batch = batch;
        p.selected = selected;
        p.width = width;
        p.itemsize = itemsize;
        p.row_bytes = width * itemsize;
        p.table_width = table_width;
        p.request_stride = request_stride;
        p.sink_elements = sink_elements;
        p.pos_es = positions_esize;
        p.req_es = request_ids_esize;
        p.len_es = lengths_esize;
        p.table_es = indirect ? table_esize : 8;
        p.off_es = indirect == 1 ? offsets_esize : 8;
        p.indirect = indirect;
        p.n_planes = n_planes;
        p.vec_shift = (p.row_bytes % 16) ? -1 : log2_exact(p.row_bytes / 16);
        uint64_t plane_or = 0;
        for (int i = 0; i < n_planes; ++i) {
            require(src_planes[i] && dst_planes[i], "null plane address");
            p.src[i] = reinterpret_cast<const char*>(src_planes[i]);
            p.dst[i] = reinterpret_cast<char*>(dst_planes[i]);
            plane_or |= src_planes[i] | dst_planes[i];
        }
        p.plane_or = plane_or;
        bind_device(device);
        const int64_t n_rows = batch * selected;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const BulkShape shape = (plane_or % 16 == 0 && bulk_allowed()) ? bulk_shape(device, p.row_bytes)
                                                                        : BulkShape{};
        if (shape.slots) {
            static std::atomic<size_t> configured[64];  // largest opt-in set per device
            if (device >= 64 || configured[device].load(std::memory_order_relaxed) < shape.smem) {
                cuda_check(cudaFuncSetAttribute(gather_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(shape.smem)),
                           "configure bulk gather shared memory");
                if (device < 64) configured[device].store(shape.smem, std::memory_order_relaxed);
            }
            const int64_t needed = (n_rows + kBulkWarps - 1) / kBulkWarps;
            const int64_t sms = sm_count(device);
            const unsigned grid = static_cast<unsigned>(needed < sms ? needed : sms);
            gather_bulk_kernel<<<grid, kBulkThreads, shape.smem, s>>>(p, shape.slots, shape.slot_bytes);
        } else {
            bool small = false;
            const GatherKernel kernel = gather_kernel_for(p.row_bytes, p.n_planes, small);
            launch_dependent(kernel, dim3(gather_grid(kernel, small, device, n_rows)), dim3(kGatherThreads), 0, s,
                             "gather_rows launch", p);
        }
        check_launch("gather_rows launch");
    });
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_gather_rows(
    const void* raw, void* out, int64_t itemsize,
    const void* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* request_table, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream) {
    const uint64_t src = reinterpret_cast<uint64_t>(raw);
    const uint64_t dst = reinterpret_cast<uint64_t>(out);
    return ekv::gather_impl(&src, &dst, 1, itemsize, positions, positions_esize, request_ids,
                            request_ids_esize, lengths, lengths_esize, request_table, table_esize,
                            slot_offsets, offsets_esize, batch, selected, width, table_width,
                            request_stride, sink_elements, indirect, device, stream);
}

extern "C" int ekv_gather_rows_planes(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
    const void* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* request_table, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream) {
    return ekv::gather_impl(src_planes, dst_planes, n_planes, itemsize, positions, positions_esize,
                            request_ids, request_ids_esize, lengths, lengths_esize, request_table,
                            table_esize, slot_offsets, offsets_esize, batch, selected, width,
                            table_width, request_stride, sink_elements, indirect, device, stream);
}

extern "C" int ekv_device_status(int device, unsigned int* status, int clear) {
    return ekv::guarded([&] {
        ekv::require(status != nullptr, "null status pointer");
        ekv::bind_device(device);
        ekv::cuda_check(cudaMemcpyFromSymbol(status, ekv::g_gather_status, sizeof(unsigned int)),
                        "read device status");
        if (clear) {
            const unsigned int zero = 0;
            ekv::cuda_check(cudaMemcpyToSymbol(ekv::g_gather_status, &zero, sizeof(zero)),
                            "clear device status");
        }
    });
}

