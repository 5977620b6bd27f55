// Hot-buffer swap-in: victim selection and promotion copies for Top-K misses.
//
// The reference hands sparse-attention misses to SGLang's block swap kernel
// (hisparse.cuh, called from adaptive_sparse/request_residency.py:805-809 and
// :829-832): rows missing from a request's fixed hot buffer are loaded from the
// host KV pool into evicted hot slots, least recently used first.  Here the same
// job is split into two device-driven steps so that a decode step needs no host
// round trip (and can be replayed from a CUDA graph):
//
//   swap_select  one block per request.  Hot slots referenced by this step's
//                hits are marked in a shared-memory bitmap; the request's misses
//                (the compacted miss list of the lookup) take the first
//                unreferenced slots in clock order from the request's hand, found
//                with a block-wide ordered scan.  The residency map and the
//                slot -> token table are updated (evicted token -> -1, missed
//                token -> its new slot) and the hand moves past the last victim.
//   promote      a persistent grid copies every miss's row, in every plane of
//                the layer, from host history (pinned memory read through
//                unified addressing, or device memory) into its new hot slot of
//                the fixed-position hot pool (sink chunk, then one region per
//                request), many rows in flight per warp; tasks beyond a
//                request's miss count are skipped.
//
// Victim choice (clock order, hits pinned) is this build's policy; the
// reference's LRU lives in third-party code that is not part of the reference.
#include "common.cuh"

namespace ekv {
namespace {

struct SelectParams {
    int32_t* res_map;
    int32_t* slot_token;
    int32_t* hand;
    const int32_t* slots;
    const int32_t* miss_list;
    const int32_t* miss_count;
    int32_t* promo_slot;
    int64_t map_row, map_width, token_row, hot, slots_row, k, list_row, promo_row, batch;
};

constexpr int kSelectThreads = 512;
constexpr int kSelectWarps = kSelectThreads / 32;
constexpr int kSelectItems = 4;
constexpr int kMaxHot = 1 << 16;  // shared bitmap: 8 KiB

__global__ void __launch_bounds__(kSelectThreads)
swap_select_kernel(const __grid_constant__ SelectParams p) {
    __shared__ uint32_t referenced[kMaxHot / 32];
    __shared__ int warp_totals[kSelectWarps];
    __shared__ int found_total;
    grid_dependency_wait();
    allow_dependents();
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    const int words = static_cast<int>((p.hot + 31) / 32);
    for (int64_t b = blockIdx.x; b < p.batch; b += gridDim.x) {
        for (int w = threadIdx.x; w < words; w += kSelectThreads) referenced[w] = 0u;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < p.k; i += kSelectThreads) {
            const int32_t s = p.slots[b * p.slots_row + i];
            if (s >= 0 && s < p.hot) atomicOr(&referenced[s >> 5], 1u << (s & 31));
        }
        __syncthreads();
        const int64_t misses = p.miss_count[b];
        const int64_t start = ((static_cast<int64_t>(p.hand[b]) % p.hot) + p.hot) % p.hot;
        for (int64_t r = threadIdx.x; r < p.k; r += kSelectThreads) p.promo_slot[b * p.promo_row + r] = -1;
        __syncthreads();
        // Walk the ring from the hand in tiles; rank the free (unreferenced)
        // slots in ring order and give rank r to miss r.
        int64_t taken = 0;
        for (int64_t j0 = 0; j0 < p.hot && taken < misses; j0 += kSelectThreads * kSelectItems) {
            const int64_t first = j0 + static_cast<int64_t>(threadIdx.x) * kSelectItems;
            int64_t slot[kSelectItems];
            unsigned free_bits = 0;
            int count = 0;
#pragma unroll
            for (int j = 0; j < kSelectItems; ++j) {
                slot[j] = -1;
                if (first + j < p.hot) {
                    int64_t s = start + first + j;
                    if (s >= p.hot) s -= p.hot;
                    slot[j] = s;
                    if (!((referenced[s >> 5] >> (s & 31)) & 1u)) {
                        free_bits |= 1u << j;
                        ++count;
                    }
                }
            }
            int inclusive = count;
#pragma unroll
            for (int offset = 1; offset < 32; offset <<= 1) {
                const int other = __shfl_up_sync(0xffffffffu, inclusive, offset);
                if (lane >= static_cast<unsigned>(offset)) inclusive += other;
            }
            if (lane == 31) warp_totals[warp] = inclusive;
            __syncthreads();
            int before = 0, total = 0;
#pragma unroll
            for (int w = 0; w < kSelectWarps; ++w) {
                before += w < warp ? warp_totals[w] : 0;
                total += warp_totals[w];
            }
            int64_t rank = taken + before + inclusive - count;
#pragma unroll
            for (int j = 0; j < kSelectItems; ++j) {
                if ((free_bits >> j) & 1u) {
                    if (rank < misses) {
                        p.promo_slot[b * p.promo_row + rank] = static_cast<int32_t>(slot[j]);
                        if (rank == misses - 1) {
                            const int64_t next = slot[j] + 1;
                            p.hand[b] = static_cast<int32_t>(next == p.hot ? 0 : next);
                        }
                    }
                    ++rank;
                }
            }
            taken += total;
            __syncthreads();  // warp_totals reused; promo_slot visible below
        }
        if (threadIdx.x == 0) found_total = static_cast<int>(taken < misses ? taken : misses);
        __syncthreads();
        const int64_t assigned = found_total;
        // Publish: evicted tokens leave the map, missed tokens enter it.  Every
        // victim holds a distinct resident token and no miss is resident, so the
        // writes never collide.
        for (int64_t r = threadIdx.x; r < assigned; r += kSelectThreads) {
            const int32_t v = p.promo_slot[b * p.promo_row + r];
            const int32_t token = p.miss_list[b * p.list_row + r];
            const int32_t old = p.slot_token[b * p.token_row + v];
            if (old >= 0 && old < p.map_width) p.res_map[b * p.map_row + old] = -1;
            if (token >= 0 && token < p.map_width) p.res_map[b * p.map_row + token] = v;
            p.slot_token[b * p.token_row + v] = token;
        }
        __syncthreads();
    }
}

struct PromoteParams {
    const int32_t* miss_list;
    const int32_t* miss_count;
    const int32_t* promo_slot;
    int64_t list_row, promo_row, batch, k;
    int64_t row_bytes, history_rows_per_request, sink_bytes, request_bytes;
    uint64_t addr_or;
    int n_planes;
    const char* history[EKV_MAX_PLANES];
    char* hot[EKV_MAX_PLANES];
};

#ifndef EKV_PROMOTE_BLOCKS_PER_SM
#define EKV_PROMOTE_BLOCKS_PER_SM 1
#endif
constexpr int kPromoteThreads = 256;
constexpr int kPromoteWarps = kPromoteThreads / 32;
constexpr int kPromoteBlocksPerSm = EKV_PROMOTE_BLOCKS_PER_SM;

template <typename T>
__device__ __forceinline__ void warp_move(const char* src, char* dst, int64_t bytes, unsigned lane) {
    const int64_t n = bytes / static_cast<int64_t>(sizeof(T));
    const T* s = reinterpret_cast<const T*>(src);
    T* d = reinterpret_cast<T*>(dst);
    for (int64_t base = 0; base < n; base += 32 * 4) {
        T v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t e = base + u * 32 + lane;
            if (e < n) v[u] = s[e];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t e = base + u * 32 + lane;
            if (e < n) d[e] = v[u];
        }
    }
}

#ifndef EKV_PROMOTE_UNROLL
#define EKV_PROMOTE_UNROLL 4  // 16-byte vectors in flight per lane
#endif
// Sort each 32-miss batch by history row before loading (config 5 at the TP8 shard:
// 12.60-12.71 against 12.79-13.03 ms per step in paired runs, 40.6 vs 39.8 GB/s; no
// change at 2 KiB rows).
#ifndef EKV_PROMOTE_SORT
#define EKV_PROMOTE_SORT 1
#endif
#ifndef EKV_PROMOTE_MAX_REGISTERS
#define EKV_PROMOTE_MAX_REGISTERS 72  // no spills at 4 in flight
#endif
constexpr int kPromoteUnroll = EKV_PROMOTE_UNROLL;

// Each of a request's warps takes an equal contiguous share of its misses (so no
// time goes to the columns that hit), 32 at a time: one per lane, its history row
// and hot slot resolved once.  The warp then streams the flattened (miss, plane,
// vector) items with kPromoteUnroll 16-byte loads in flight per lane before storing
// them.  The reads cross the host link from pinned memory, so the bytes in flight
// bound the copy: a warp that moved one row at a time kept one 256 B row in flight
// at the TP8 shard (33 GB/s); this keeps up to 32 x 4 x 16 B and measured 40 GB/s
// (config 5 at the TP8 shard, 15.5 -> 12.8 ms per step; equal at 2 KiB rows).  A
// fixed grid of EKV_PROMOTE_BLOCKS_PER_SM blocks per SM (8 warps each) at most
// EKV_PROMOTE_MAX_REGISTERS registers leaves room on every SM for two gather blocks
// of 88 registers, so the swap pipeline runs layer i's gather during layer i+1's
// promotion (6 loads in flight under an 80-register cap spilled and lost that
// overlap: 13.9 ms; a 64-register cap: 14.5 ms).
__global__ void __maxnreg__(EKV_PROMOTE_MAX_REGISTERS)
promote_kernel(const __grid_constant__ PromoteParams p) {
    grid_dependency_wait();
    allow_dependents();
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kPromoteWarps;
    const int64_t w = static_cast<int64_t>(blockIdx.x) * kPromoteWarps + (threadIdx.x >> 5);
    const unsigned lane = lane_id();
    const int64_t per_request = warps >= p.batch ? warps / p.batch : 1;
    const int64_t request_stride = warps / per_request;
    if (w >= per_request * request_stride) return;  // the remainder: every request is covered without it
    const int64_t sub = w % per_request;
    // 16-byte items need aligned addresses and a vector index that fits the item key.
    const bool vec16 = alignment_of(p.addr_or | static_cast<uint64_t>(p.row_bytes)) == 16 &&
                       p.row_bytes <= (int64_t{1} << 20);
    const uint32_t vecs = static_cast<uint32_t>(p.row_bytes >> 4);
    const uint32_t per_miss = static_cast<uint32_t>(p.n_planes) * vecs;
    for (int64_t b = w / per_request; b < p.batch; b += request_stride) {
        const int64_t count = min(static_cast<int64_t>(p.miss_count[b]), p.k);
        const int64_t share = (count + per_request - 1) / per_request;
        const int64_t first = sub * share;
        const int64_t last = min(first + share, count);
        for (int64_t r0 = first; r0 < last; r0 += 32) {
            const int64_t r = r0 + lane;
            int32_t key = 0x7fffffff, hot = -1;  // history row and hot slot of a miss to copy
            if (r < last) {
                const int32_t slot = p.promo_slot[b * p.promo_row + r];
                const int32_t token = p.miss_list[b * p.list_row + r];
                // A slot outside the request's hot region (or a token outside its history)
                // is skipped: the copy never leaves the buffers it was given.
                if (slot >= 0 && token >= 0 && token < p.history_rows_per_request &&
                    (static_cast<int64_t>(slot) + 1) * p.row_bytes <= p.request_bytes) {
                    key = token;
                    hot = slot;
                }
            }
#if EKV_PROMOTE_SORT
            // Order the batch by history row (bitonic sort across the warp; skipped misses
            // last), so one load instruction reads neighbouring host rows.
            for (int k = 2; k <= 32; k <<= 1) {
                for (int j = k >> 1; j > 0; j >>= 1) {
                    const int32_t other_key = __shfl_xor_sync(0xffffffffu, key, j);
                    const int32_t other_hot = __shfl_xor_sync(0xffffffffu, hot, j);
                    const bool ascending = (lane & k) == 0;
                    const bool lower = (lane & j) == 0;
                    if (lower == ascending ? other_key < key : other_key > key) {
                        key = other_key;
                        hot = other_hot;
                    }
                }
            }
#endif
            int64_t src = -1, dst = 0;
            if (hot >= 0) {
                src = (b * p.history_rows_per_request + key) * p.row_bytes;
                dst = p.sink_bytes + b * p.request_bytes + static_cast<int64_t>(hot) * p.row_bytes;
            }
            const int nb = static_cast<int>(last - r0 < 32 ? last - r0 : 32);
            if (vec16) {
                // Item key: miss (5 bits) | plane (8 bits) | vector (16 bits), all ones = no copy.
                const uint32_t total = static_cast<uint32_t>(nb) * per_miss;
                for (uint32_t base = 0; base < total; base += 32 * kPromoteUnroll) {
                    uint4 v[kPromoteUnroll];
                    uint32_t key[kPromoteUnroll];
#pragma unroll
                    for (int u = 0; u < kPromoteUnroll; ++u) {
                        const uint32_t idx = base + u * 32 + lane;
                        const uint32_t m = idx < total ? idx / per_miss : 0;
                        const uint32_t rem = idx - m * per_miss;
                        const uint32_t plane = rem / vecs;
                        const uint32_t vec = rem - plane * vecs;
                        const int64_t s = __shfl_sync(0xffffffffu, src, static_cast<int>(m));
                        key[u] = (idx < total && s >= 0) ? (m << 24) | (plane << 16) | vec : ~0u;
                        if (key[u] != ~0u) {
                            v[u] = *reinterpret_cast<const uint4*>(p.history[plane] + s +
                                                                   (static_cast<int64_t>(vec) << 4));
                        }
                    }
#pragma unroll
                    for (int u = 0; u < kPromoteUnroll; ++u) {
                        const int m = key[u] == ~0u ? 0 : static_cast<int>(key[u] >> 24);
                        const int64_t d = __shfl_sync(0xffffffffu, dst, m);
                        if (key[u] != ~0u) {
                            const uint32_t plane = (key[u] >> 16) & 0xffu;
                            const int64_t vec = key[u] & 0xffffu;
                            *reinterpret_cast<uint4*>(p.hot[plane] + d + (vec << 4)) = v[u];
                        }
                    }
                }
            } else {
                for (int k = 0; k < nb; ++k) {
                    const int64_t s = __shfl_sync(0xffffffffu, src, k);
                    const int64_t d = __shfl_sync(0xffffffffu, dst, k);
                    if (s < 0) continue;
                    for (int plane = 0; plane < p.n_planes; ++plane) {
                        warp_move<uint8_t>(p.history[plane] + s, p.hot[plane] + d, p.row_bytes, lane);
                    }
                }
            }
        }
    }
}

}  // namespace
}  // namespace ekv

using namespace ekv;

extern "C" int ekv_swap_select(
    int32_t* res_map, int64_t map_row_stride, int64_t map_width,
    int32_t* slot_token, int64_t token_row_stride, int64_t hot_capacity,
    int32_t* hand,
    const int32_t* slots, int64_t slots_row_stride, int64_t k,
    const int32_t* miss_list, int64_t list_row_stride, const int32_t* miss_count,
    int32_t* promo_slot, int64_t promo_row_stride,
    int64_t batch, int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && k >= 0 && map_width >= 0, "sizes must be non-negative");
        require(hot_capacity > 0 && hot_capacity <= kMaxHot, "hot capacity outside [1, 65536]");
        if (!batch || !k) return;
        require(res_map && slot_token && hand && slots && miss_list && miss_count && promo_slot,
                "null pointer argument");
        bind_device(device);
        SelectParams p{};
        p.res_map = res_map;
        p.slot_token = slot_token;
        p.hand = hand;
        p.slots = slots;
        p.miss_list = miss_list;
        p.miss_count = miss_count;
        p.promo_slot = promo_slot;
        p.map_row = map_row_stride;
        p.map_width = map_width;
        p.token_row = token_row_stride;
        p.hot = hot_capacity;
        p.slots_row = slots_row_stride;
        p.k = k;
        p.list_row = list_row_stride;
        p.promo_row = promo_row_stride;
        p.batch = batch;
        const unsigned grid = static_cast<unsigned>(batch < (1 << 20) ? batch : (1 << 20));
        launch_dependent(swap_select_kernel, dim3(grid), dim3(kSelectThreads), 0, static_cast<cudaStream_t>(stream),
                         "swap_select launch", p);
        check_launch("swap_select launch");
    });
}

extern "C" int ekv_promote_rows(
    const uint64_t* history_planes, const uint64_t* hot_planes, int n_planes, int64_t row_bytes,
    int64_t history_rows_per_request, int64_t sink_bytes, int64_t request_bytes,
    const int32_t* miss_list, int64_t list_row_stride, const int32_t* miss_count,
    const int32_t* promo_slot, int64_t promo_row_stride,
    int64_t batch, int64_t k, int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && k >= 0, "sizes must be non-negative");
        require(row_bytes > 0 && history_rows_per_request > 0, "row and history sizes must be positive");
        require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
        if (!batch || !k) return;
        require(history_planes && hot_planes && miss_list && miss_count && promo_slot, "null pointer argument");
        bind_device(device);
        PromoteParams p{};
        p.miss_list = miss_list;
        p.miss_count = miss_count;
        p.promo_slot = promo_slot;
        p.list_row = list_row_stride;
        p.promo_row = promo_row_stride;
        p.batch = batch;
        p.k = k;
        p.row_bytes = row_bytes;
        p.history_rows_per_request = history_rows_per_request;
        p.sink_bytes = sink_bytes;
        p.request_bytes = request_bytes;
        p.n_planes = n_planes;
        uint64_t addr_or = static_cast<uint64_t>(sink_bytes) | static_cast<uint64_t>(request_bytes);
        for (int i = 0; i < n_planes; ++i) {
            require(history_planes[i] && hot_planes[i], "null plane address");
            // History may live in pinned host memory: use its device view, refuse anything unmapped.
            cudaPointerAttributes attr{};
            cuda_check(cudaPointerGetAttributes(&attr, reinterpret_cast<const void*>(history_planes[i])),
                       "query history pointer");
            const void* view = reinterpret_cast<const void*>(history_planes[i]);
            if (attr.type == cudaMemoryTypeHost) {
                require(attr.devicePointer != nullptr, "pinned history is not mapped for device access");
                view = attr.devicePointer;
            } else {
                require(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
                        "history must be device memory or pinned host memory");
            }
            p.history[i] = static_cast<const char*>(view);
            p.hot[i] = reinterpret_cast<char*>(hot_planes[i]);
            addr_or |= reinterpret_cast<uint64_t>(view) | hot_planes[i];
        }
        p.addr_or = addr_or;
        const int grid = sm_count(device) * kPromoteBlocksPerSm;
        launch_dependent(promote_kernel, dim3(grid), dim3(kPromoteThreads), 0, static_cast<cudaStream_t>(stream),
                         "promote_rows launch", p);
        check_launch("promote_rows launch");
    });
}
