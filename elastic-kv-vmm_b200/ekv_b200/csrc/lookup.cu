// Residency lookups.
//
// R1 resolve_resident: Top-K block ids -> token positions -> logical ids
//    (req_to_token) -> physical slots (full_to_hisparse mapping), -1 when the
//    block is padding or the position is past the request length.  Semantics of
//    the Triton `_resolve` kernel, adaptive_sparse/resident_lookup.py:6-26.
// R2 lookup_slots: token ids -> hot slots through a per-request residency map,
//    with a miss mask and a per-request miss list compacted in column order by
//    warp ballots.
//
// Both are latency-bound chains of dependent 4/8-byte gathers (a few hundred KB
// per call), so the kernels keep several independent chains in flight per
// thread rather than chasing bandwidth.
#include "common.cuh"

namespace ekv {
namespace {

struct ResolveParams {
    const void* topk;
    const void* table;
    const void* mapping;
    const void* rows;
    const void* lengths;
    const void* selected;
    int32_t* out;
    int64_t topk_row, topk_col;
    int64_t table_row, table_col;
    int64_t map_stride, rows_stride, len_stride, sel_stride;
    int64_t out_row, out_col;
    int64_t n_selected, width, block_size;
    int topk_es, table_es, map_es, rows_es, len_es, sel_es;
};

constexpr int kResolveThreads = 256;
constexpr int kResolveItems = 4;  // independent lookup chains per thread

// grid.x tiles the width (kResolveThreads * kResolveItems columns per block),
// grid.y walks the selected rows.
__global__ void __launch_bounds__(kResolveThreads)
resolve_kernel(const __grid_constant__ ResolveParams p) {
    grid_dependency_wait();
    allow_dependents();
    for (int64_t s = blockIdx.y; s < p.n_selected; s += gridDim.y) {
        const int64_t row = load_index(p.selected, p.sel_es, s * p.sel_stride);
        const int64_t length = load_index(p.lengths, p.len_es, row * p.len_stride);
        const int64_t req = load_index(p.rows, p.rows_es, row * p.rows_stride);
        const int64_t j0 =
            static_cast<int64_t>(blockIdx.x) * (kResolveThreads * kResolveItems) + threadIdx.x;

        int64_t value[kResolveItems];
        bool valid[kResolveItems];
        // Stage 1: block ids -> positions.
#pragma unroll
        for (int k = 0; k < kResolveItems; ++k) {
            const int64_t j = j0 + k * kResolveThreads;
            valid[k] = false;
            value[k] = 0;
            if (j < p.width) {
                const int64_t block =
                    load_index(p.topk, p.topk_es, row * p.topk_row + (j / p.block_size) * p.topk_col);
                const int64_t position = block * p.block_size + j % p.block_size;
                valid[k] = block >= 0 && position < length;
                value[k] = position;
            }
        }
        // Stage 2: positions -> logical token ids.
#pragma unroll
        for (int k = 0; k < kResolveItems; ++k) {
            if (valid[k]) {
                value[k] = load_index(p.table, p.table_es, req * p.table_row + value[k] * p.table_col);
            }
        }
        // Stage 3: logical ids -> physical slots.
#pragma unroll
        for (int k = 0; k < kResolveItems; ++k) {
            value[k] = valid[k] ? load_index(p.mapping, p.map_es, value[k] * p.map_stride) : -1;
        }
#pragma unroll
        for (int k = 0; k < kResolveItems; ++k) {
            const int64_t j = j0 + k * kResolveThreads;
            if (j < p.width) {
                // int64 slot stored into int32: two's-complement truncation, as
                // the reference's int64 -> int32 store does.
                p.out[row * p.out_row + j * p.out_col] = static_cast<int32_t>(value[k]);
            }
        }
    }
}

struct LookupParams {
    const void* map;
    const void* topk;
    const void* lengths;
    int32_t* slots;
    uint8_t* miss;
    int32_t* miss_list;
    int32_t* miss_count;
    int64_t map_row, map_width, topk_row;
    int64_t batch, k;
    int64_t slots_row, miss_row, list_row;
    int map_es, topk_es, len_es;
};

#ifndef EKV_LOOKUP_THREADS
#define EKV_LOOKUP_THREADS 512
#endif
#ifndef EKV_LOOKUP_MIN_BLOCKS
#define EKV_LOOKUP_MIN_BLOCKS 3
#endif
constexpr int kLookupThreads = EKV_LOOKUP_THREADS;
constexpr int kLookupWarps = kLookupThreads / 32;

// Exclusive prefix of `count` over the block in thread order (warp shuffle scan,
// then a scan of the warp totals in shared memory); `total` receives the block's
// sum.  The caller syncs before `warp_totals` is written again.
__device__ __forceinline__ int block_exclusive_scan(int count, unsigned lane, int warp, int* warp_totals,
                                                    int& total) {
    int inclusive = count;
#pragma unroll
    for (int offset = 1; offset < 32; offset <<= 1) {
        const int other = __shfl_up_sync(0xffffffffu, inclusive, offset);
        if (lane >= static_cast<unsigned>(offset)) inclusive += other;
    }
    if (lane == 31) warp_totals[warp] = inclusive;
    __syncthreads();
    int before = 0;
    total = 0;
#pragma unroll
    for (int w = 0; w < kLookupWarps; ++w) {
        const int warp_count = warp_totals[w];
        before += w < warp ? warp_count : 0;
        total += warp_count;
    }
    return before + inclusive - count;
}

// One block per request row; a pass covers kLookupThreads * kItems Top-K
// columns, each thread kItems consecutive ones, so a row of up to 2048 columns
// is one pass with all its independent map lookups in flight at once (the
// launch picks kItems = 1, 2 or 4; wider rows take several passes).  Misses are
// compacted in column order by a block-wide exclusive scan of the per-thread
// miss counts (warp shuffle scan, then a scan of the warp totals in shared
// memory).  The register cap of 3 blocks per SM (40 registers a thread, no
// spills) lets a 512-thread block fit on an SM beside two blocks of the gather
// kernel, so a layer's lookup can run while the previous layer's gather does
// (swap.py's SwapPipeline); 16 warps per row hide the two dependent loads
// better than 8 (256-thread blocks measured 6 % slower on config 4).
template <int kItems>
__global__ void __launch_bounds__(kLookupThreads, EKV_LOOKUP_MIN_BLOCKS)
lookup_kernel(const __grid_constant__ LookupParams p) {
    grid_dependency_wait();
    allow_dependents();
    constexpr int kLookupItems = kItems;
    constexpr int kLookupTile = kLookupThreads * kItems;
    __shared__ int warp_totals[kLookupWarps];
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    for (int64_t b = blockIdx.x; b < p.batch; b += gridDim.x) {
        int64_t limit = p.map_width;
        if (p.lengths) {
            const int64_t length = load_index(p.lengths, p.len_es, b);
            limit = length < limit ? length : limit;
        }
        int64_t base = 0;
        for (int64_t c0 = 0; c0 < p.k; c0 += kLookupTile) {
            const int64_t first = c0 + static_cast<int64_t>(threadIdx.x) * kLookupItems;
            int64_t token[kLookupItems];
            int64_t slot[kLookupItems];
#pragma unroll
            for (int j = 0; j < kLookupItems; ++j) {
                token[j] = first + j < p.k ? load_index(p.topk, p.topk_es, b * p.topk_row + first + j) : -1;
            }
            int count = 0;
            unsigned miss_bits = 0;
#pragma unroll
            for (int j = 0; j < kLookupItems; ++j) {
                const bool valid = token[j] >= 0 && token[j] < limit;
                slot[j] = valid ? load_index(p.map, p.map_es, b * p.map_row + token[j]) : -1;
                if (valid && slot[j] < 0) {
                    miss_bits |= 1u << j;
                    ++count;
                }
            }
#pragma unroll
            for (int j = 0; j < kLookupItems; ++j) {
                if (first + j < p.k) {
                    p.slots[b * p.slots_row + first + j] = static_cast<int32_t>(slot[j]);
                    if (p.miss) p.miss[b * p.miss_row + first + j] = (miss_bits >> j) & 1u;
                }
            }
            // Exclusive prefix of `count` over the block, in thread (= column) order.
            int total = 0;
            const int before = block_exclusive_scan(count, lane, warp, warp_totals, total);
            if (miss_bits && p.miss_list) {
                int64_t at = base + before;
#pragma unroll
                for (int j = 0; j < kLookupItems; ++j) {
                    if ((miss_bits >> j) & 1u) p.miss_list[b * p.list_row + at++] = static_cast<int32_t>(token[j]);
                }
            }
            base += total;
            __syncthreads();  // warp_totals is rewritten by the next pass
        }
        if (p.miss_list) {
            for (int64_t i = base + threadIdx.x; i < p.k; i += kLookupThreads) {
                p.miss_list[b * p.list_row + i] = -1;
            }
        }
        if (p.miss_count && threadIdx.x == 0) p.miss_count[b] = static_cast<int32_t>(base);
    }
}

// The miss list and count of a lookup whose slots and miss mask are already
// written (by a fused lookup + gather, ekv_lookup_gather_planes): the same
// column-order compaction as lookup_kernel, with the miss bits read from the
// mask instead of recomputed from the residency map.
struct CompactParams {
    const uint8_t* miss;
    const void* topk;
    int32_t* miss_list;
    int32_t* miss_count;
    int64_t batch, k;
    int64_t miss_row, topk_row, list_row;
    int topk_es;
};

template <int kItems>
__global__ void __launch_bounds__(kLookupThreads, EKV_LOOKUP_MIN_BLOCKS)
compact_misses_kernel(const __grid_constant__ CompactParams p) {
    grid_dependency_wait();
    allow_dependents();
    constexpr int kTile = kLookupThreads * kItems;
    __shared__ int warp_totals[kLookupWarps];
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    for (int64_t b = blockIdx.x; b < p.batch; b += gridDim.x) {
        int64_t base = 0;
        for (int64_t c0 = 0; c0 < p.k; c0 += kTile) {
            const int64_t first = c0 + static_cast<int64_t>(threadIdx.x) * kItems;
            unsigned miss_bits = 0;
            int count = 0;
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                if (first + j < p.k && p.miss[b * p.miss_row + first + j]) {
                    miss_bits |= 1u << j;
                    ++count;
                }
            }
            int total = 0;
            const int before = block_exclusive_scan(count, lane, warp, warp_totals, total);
            int64_t at = base + before;
#pragma unroll
            for (int j = 0; j < kItems; ++j) {
                if ((miss_bits >> j) & 1u) {
                    p.miss_list[b * p.list_row + at++] =
                        static_cast<int32_t>(load_index(p.topk, p.topk_es, b * p.topk_row + first + j));
                }
            }
            base += total;
            __syncthreads();  // warp_totals is rewritten by the next pass
        }
        for (int64_t i = base + threadIdx.x; i < p.k; i += kLookupThreads) {
            p.miss_list[b * p.list_row + i] = -1;
        }
        if (p.miss_count && threadIdx.x == 0) p.miss_count[b] = static_cast<int32_t>(base);
    }
}

}  // namespace
}  // namespace ekv

using namespace ekv;

extern "C" int ekv_compact_misses(
    const uint8_t* miss, int64_t miss_row_stride,
    const void* topk, int topk_esize, int64_t topk_row_stride,
    int64_t batch, int64_t k,
    int32_t* miss_list, int64_t miss_list_row_stride,
    int32_t* miss_count,
    int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && k >= 0, "sizes must be non-negative");
        if (!batch) return;
        require(k <= 0x7fffffff, "k must fit in int32");
        if (k) require(miss && topk && miss_list, "null pointer argument");
        check_esize(topk_esize, "topk");
        bind_device(device);
        CompactParams p{};
        p.miss = miss;
        p.topk = topk;
        p.miss_list = miss_list;
        p.miss_count = miss_count;
        p.batch = batch;
        p.k = k;
        p.miss_row = miss_row_stride;
        p.topk_row = topk_row_stride;
        p.list_row = miss_list_row_stride;
        p.topk_es = topk_esize;
        const unsigned grid = static_cast<unsigned>(batch < (1 << 20) ? batch : (1 << 20));
        auto* kernel = k <= kLookupThreads       ? compact_misses_kernel<1>
                       : k <= 2 * kLookupThreads ? compact_misses_kernel<2>
                                                 : compact_misses_kernel<4>;
        launch_dependent(kernel, dim3(grid), dim3(kLookupThreads), 0, static_cast<cudaStream_t>(stream),
                         "compact_misses launch", p);
        check_launch("compact_misses launch");
    });
}

extern "C" int ekv_resolve_resident(
    const void* topk, int topk_esize, int64_t topk_row_stride, int64_t topk_col_stride,
    int64_t topk_width,
    const void* table, int table_esize, int64_t table_row_stride, int64_t table_col_stride,
    const void* mapping, int mapping_esize, int64_t mapping_stride,
    const void* rows, int rows_esize, int64_t rows_stride,
    const void* lengths, int lengths_esize, int64_t lengths_stride,
    const void* selected, int selected_esize, int64_t selected_stride, int64_t n_selected,
    int32_t* out, int64_t out_row_stride, int64_t out_col_stride,
    int64_t block_size, int device, void* stream) {
    return guarded([&] {
        require(topk_width >= 0 && n_selected >= 0, "sizes must be non-negative");
        require(block_size > 0, "block_size must be positive");
        const int64_t width = topk_width * block_size;
        if (!n_selected || !width) return;
        require(topk && table && mapping && rows && lengths && selected && out,
                "null pointer argument");
        check_esize(topk_esize, "topk");
        check_esize(table_esize, "table");
        check_esize(mapping_esize, "mapping");
        check_esize(rows_esize, "rows");
        check_esize(lengths_esize, "lengths");
        check_esize(selected_esize, "selected");
        bind_device(device);
        ResolveParams p{};
        p.topk = topk;
        p.table = table;
        p.mapping = mapping;
        p.rows = rows;
        p.lengths = lengths;
        p.selected = selected;
        p.out = out;
        p.topk_row = topk_row_stride;
        p.topk_col = topk_col_stride;
        p.table_row = table_row_stride;
        p.table_col = table_col_stride;
        p.map_stride = mapping_stride;
        p.rows_stride = rows_stride;
        p.len_stride = lengths_stride;
        p.sel_stride = selected_stride;
        p.out_row = out_row_stride;
        p.out_col = out_col_stride;
        p.n_selected = n_selected;
        p.width = width;
        p.block_size = block_size;
        p.topk_es = topk_esize;
        p.table_es = table_esize;
        p.map_es = mapping_esize;
        p.rows_es = rows_esize;
        p.len_es = lengths_esize;
        p.sel_es = selected_esize;
        const int64_t tile = kResolveThreads * kResolveItems;
        const int64_t gx = (width + tile - 1) / tile;
        require(gx <= 0x7fffffff, "width too large");
        const unsigned gy = static_cast<unsigned>(n_selected < 65535 ? n_selected : 65535);
        launch_dependent(resolve_kernel, dim3(static_cast<unsigned>(gx), gy), dim3(kResolveThreads), 0,
                         static_cast<cudaStream_t>(stream), "resolve_resident launch", p);
        check_launch("resolve_resident launch");
    });
}

extern "C" int ekv_lookup_slots(
    const void* res_map, int map_esize, int64_t map_row_stride, int64_t map_width,
    const void* topk, int topk_esize, int64_t topk_row_stride,
    const void* lengths, int lengths_esize,
    int64_t batch, int64_t k,
    int32_t* slots, int64_t slots_row_stride,
    uint8_t* miss, int64_t miss_row_stride,
    int32_t* miss_list, int64_t miss_list_row_stride,
    int32_t* miss_count,
    int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && k >= 0 && map_width >= 0, "sizes must be non-negative");
        if (!batch) return;
        require(k <= 0x7fffffff, "k must fit in int32");
        // With k == 0 the kernel only writes miss_count (zeros).
        if (k) require(res_map && topk && slots, "null pointer argument");
        check_esize(map_esize, "residency map");
        check_esize(topk_esize, "topk");
        if (lengths) check_esize(lengths_esize, "lengths");
        bind_device(device);
        LookupParams p{};
        p.map = res_map;
        p.topk = topk;
        p.lengths = lengths;
        p.slots = slots;
        p.miss = miss;
        p.miss_list = miss_list;
        p.miss_count = miss_count;
        p.map_row = map_row_stride;
        p.map_width = map_width;
        p.topk_row = topk_row_stride;
        p.batch = batch;
        p.k = k;
        p.slots_row = slots_row_stride;
        p.miss_row = miss_row_stride;
        p.list_row = miss_list_row_stride;
        p.map_es = map_esize;
        p.topk_es = topk_esize;
        p.len_es = lengths ? lengths_esize : 4;
        const unsigned grid = static_cast<unsigned>(batch < (1 << 20) ? batch : (1 << 20));
        const auto cstream = static_cast<cudaStream_t>(stream);
        auto* kernel = k <= kLookupThreads ? lookup_kernel<1> : k <= 2 * kLookupThreads ? lookup_kernel<2>
                                                                                         : lookup_kernel<4>;
        launch_dependent(kernel, dim3(grid), dim3(kLookupThreads), 0, cstream, "lookup_slots launch", p);
        check_launch("lookup_slots launch");
    });
}
