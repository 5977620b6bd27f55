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
// the widest element size that divides every address.  (A bulk-copy, TMA
// engine, variant measured 0.89 of the copy peak at 2 KiB rows and was bound by
// the bulk-operation rate at smaller rows, so the register-staged kernel is the
// only one.)  When each layer has its own row selection, ekv_gather_layers runs
// every layer's gather in one launch (gather_layers_kernel), so short per-layer
// launches do not each pay a ramp, a tail and a dependency wait.
#include <atomic>

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
    int indirect;       // addressing mode: 0 direct, 1 indirect, 2 mapped
    int indices_ready;  // EKV_GATHER_INDICES_READY was set: see first_batch()
    int disjoint;       // EKV_GATHER_DISJOINT was set: see first_batch() and finish()
    int n_planes;
    int vec_shift;  // log2(row_bytes / 16) when that is a power of two, else -1
    // Fused lookup (ekv_lookup_gather_planes, mapped mode): row r's slot and miss
    // flag, [batch, selected] contiguous; null otherwise.
    int32_t* slots_out;
    uint8_t* miss_out;
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
// Flattened batch copies find an item's row by a division per 16-byte item, or --
// when a row has at least 32 vectors over all planes -- by walking (row, remainder)
// forward 32 items at a time.  At 256 B rows over 36 planes the walk cut 22 % of the
// instructions (ncu: 173 M -> 134 M) yet ran slower (0.881 vs 0.914 of the copy peak
// over 72 planes): that launch is bound by DRAM on random 256 B rows, not by issue.
// EKV_GATHER_WALK applies to the default instance (one layer's K and V at 2 KiB
// rows flattens 256 vectors per row), EKV_GATHER_SMALL_WALK to the many-plane
// small-row instance.
#ifndef EKV_GATHER_WALK
#define EKV_GATHER_WALK 1
#endif
#ifndef EKV_GATHER_SMALL_WALK
#define EKV_GATHER_SMALL_WALK 0
#endif
constexpr int64_t kSmallRowBytes = EKV_GATHER_SMALL_ROW_BYTES;
constexpr int kSmallUnroll = EKV_GATHER_SMALL_UNROLL;

// What a residency lookup reports for a row: its slot (-1 for a position outside
// the valid range) and whether a valid position had no slot (a miss).
struct RowLookup {
    int32_t slot = -1;
    bool miss = false;
};

// Byte offset of row r inside every source plane, or valid = false.  `positions`
// and `table` stand in for p.positions and p.request_table (one layer's of a
// multi-layer launch).  In mapped mode `found` receives the lookup's view of the
// row.
__device__ __forceinline__ int64_t resolve_row_at(const GatherParams& p, const void* positions,
                                                  const void* table, int64_t r, bool& valid, RowLookup& found) {
    const int64_t b = r / p.selected;
    const int64_t pos = load_index(positions, p.pos_es, r);
    const int64_t length = load_index(p.lengths, p.len_es, b);
    // A residency map row has table_width entries: later positions have no slot.
    valid = pos >= 0 && pos < length && (p.indirect != 2 || pos < p.table_width);
    if (!valid) return 0;
    const int64_t req = load_index(p.request_ids, p.req_es, b);
    int64_t element;
    if (p.indirect == 1) {
        const int64_t logical = load_index(table, p.table_es, req * p.table_width + pos);
        element = load_index(p.slot_offsets, p.off_es, logical);
    } else if (p.indirect == 2) {
        // Mapped: the table holds the row's slot in the request's fixed region, -1 if
        // absent; a slot past the region reads as absent too (never outside the region).
        const int64_t slot = load_index(table, p.table_es, req * p.table_width + pos);
        found.slot = static_cast<int32_t>(slot);  // int32 truncation, as ekv_lookup_slots stores it
        found.miss = slot < 0;
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

// Per-row copies: planes plane0 .. plane0 + n_planes - 1.
__device__ __forceinline__ void copy_row_vec16(const GatherParams& p, bool valid, int64_t src_off,
                                               int64_t dst_off, unsigned lane, int plane0, int n_planes) {
    const int64_t vecs = p.row_bytes >> 4;
    const int64_t total = static_cast<int64_t>(n_planes) * vecs;
    for (int64_t base = 0; base < total; base += 32 * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t idx = base + u * 32 + lane;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (valid && idx < total) {
                const int64_t plane = p.vec_shift >= 0 ? (idx >> p.vec_shift) : idx / vecs;
                const int64_t vec = idx - plane * vecs;
                v[u] = load_vec(reinterpret_cast<const uint4*>(p.src[plane0 + plane] + src_off) + vec);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t idx = base + u * 32 + lane;
            if (idx < total) {
                const int64_t plane = p.vec_shift >= 0 ? (idx >> p.vec_shift) : idx / vecs;
                const int64_t vec = idx - plane * vecs;
                store_vec(reinterpret_cast<uint4*>(p.dst[plane0 + plane] + dst_off) + vec, v[u]);
            }
        }
    }
}

template <typename T>
__device__ __forceinline__ void copy_row_elems(const GatherParams& p, bool valid, int64_t src_off,
                                               int64_t dst_off, unsigned lane, int plane0, int n_planes) {
    const int64_t elems = p.row_bytes / static_cast<int64_t>(sizeof(T));
    const int64_t total = static_cast<int64_t>(n_planes) * elems;
    for (int64_t idx = lane; idx < total; idx += 32) {
        const int64_t plane = idx / elems;
        const int64_t e = idx - plane * elems;
        T value = T(0);
        if (valid) value = reinterpret_cast<const T*>(p.src[plane0 + plane] + src_off)[e];
        reinterpret_cast<T*>(p.dst[plane0 + plane] + dst_off)[e] = value;
    }
}

// Warp-cooperative copy of one row out of every plane, any alignment.
__device__ __forceinline__ void copy_row_any(const GatherParams& p, bool valid, int64_t src_off,
                                             int64_t dst_off, unsigned lane, int plane0, int n_planes) {
    const int64_t align = alignment_of(p.plane_or | static_cast<uint64_t>(src_off) |
                                       static_cast<uint64_t>(dst_off) | static_cast<uint64_t>(p.row_bytes));
    switch (align) {
        case 16: copy_row_vec16(p, valid, src_off, dst_off, lane, plane0, n_planes); break;
        case 8: copy_row_elems<uint64_t>(p, valid, src_off, dst_off, lane, plane0, n_planes); break;
        case 4: copy_row_elems<uint32_t>(p, valid, src_off, dst_off, lane, plane0, n_planes); break;
        case 2: copy_row_elems<uint16_t>(p, valid, src_off, dst_off, lane, plane0, n_planes); break;
        default: copy_row_elems<uint8_t>(p, valid, src_off, dst_off, lane, plane0, n_planes); break;
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

// kWalk: rows of at least 32 vectors (all planes).  Item idx = base + u * 32 + lane
// belongs to row idx / per_row of the batch; with kWalk a lane's next item is 32
// further on, so (row, remainder) advance with one compare instead of a division
// per item.
// Planes plane0 .. plane0 + n_planes - 1 of p.src / p.dst are copied.
template <int kU, bool kWalk>
__device__ __forceinline__ void copy_batch_vec16(const GatherParams& p, int64_t mine, int64_t row0,
                                                 int64_t warps, int nb, unsigned lane, int plane0,
                                                 int n_planes) {
    const uint32_t vecs = static_cast<uint32_t>(p.row_bytes >> 4);
    const uint32_t per_row = static_cast<uint32_t>(n_planes) * vecs;
    const uint32_t total = static_cast<uint32_t>(nb) * per_row;
    uint32_t k = 0, rem = lane;
    for (uint32_t base = 0; base < total; base += 32 * kU) {
        uint4 v[kU];
        uint32_t row_of[kU];
        uint32_t rem_of[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint32_t idx = base + u * 32 + lane;
            if (!kWalk) {
                k = idx < total ? idx / per_row : 0;
                rem = idx - k * per_row;
            }
            const bool live = idx < total;
            const int64_t s = __shfl_sync(0xffffffffu, mine, static_cast<int>(live ? k : 0));
            row_of[u] = k;
            rem_of[u] = rem;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (live && s >= 0) {
                const uint32_t plane = p.vec_shift >= 0 ? (rem >> p.vec_shift) : rem / vecs;
                const uint32_t vec = rem - plane * vecs;
                v[u] = load_vec(reinterpret_cast<const uint4*>(p.src[plane0 + plane] + s) + vec);
            }
            if (kWalk) {
                rem += 32;
                if (rem >= per_row) {
                    rem -= per_row;
                    ++k;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const uint32_t idx = base + u * 32 + lane;
            if (idx < total) {
                const uint32_t plane = p.vec_shift >= 0 ? (rem_of[u] >> p.vec_shift) : rem_of[u] / vecs;
                const uint32_t vec = rem_of[u] - plane * vecs;
                char* row = p.dst[plane0 + plane] + (row0 + static_cast<int64_t>(row_of[u]) * warps) * p.row_bytes;
                store_vec(reinterpret_cast<uint4*>(row) + vec, v[u]);
            }
        }
    }
}

// Offset of row row0 + lane * warps in every source plane, or -1 for a zero row
// (invalid position, or a row past the end).  Each lane resolves one row of the
// warp's 32-row batch, so the three dependent index loads are paid once per 32 rows.
__device__ __forceinline__ int64_t resolve_batch_at(const GatherParams& p, const void* positions,
                                                    const void* table, int64_t row0, int64_t warps,
                                                    int64_t n_rows, unsigned lane, RowLookup& found) {
    const int64_t r = row0 + static_cast<int64_t>(lane) * warps;
    bool valid = false;
    int64_t src = 0;
    found = RowLookup{};
    if (r < n_rows) src = resolve_row_at(p, positions, table, r, valid, found);
    return valid ? src : -1;
}

// The fused lookup's outputs for this lane's row of the batch (a no-op unless the
// launch carries them).  Called only after the dependency wait.
__device__ __forceinline__ void emit_lookup(const GatherParams& p, int64_t row0, int64_t warps,
                                            int64_t n_rows, unsigned lane, const RowLookup& found) {
    if (!p.slots_out) return;
    const int64_t r = row0 + static_cast<int64_t>(lane) * warps;
    if (r < n_rows) {
        p.slots_out[r] = found.slot;
        p.miss_out[r] = found.miss ? 1 : 0;
    }
}

__device__ __forceinline__ int64_t resolve_batch(const GatherParams& p, int64_t row0, int64_t warps,
                                                 int64_t n_rows, unsigned lane) {
    RowLookup found;
    const int64_t mine = resolve_batch_at(p, p.positions, p.request_table, row0, warps, n_rows, lane, found);
    emit_lookup(p, row0, warps, n_rows, lane, found);
    return mine;
}

// The first batch's index chain.  With `indices_ready` the caller has promised
// that the kernel launched just before this one in the stream does not write the
// index inputs (positions, request ids, lengths, table, offsets), so the chain is
// walked while that kernel drains and only the payload copy waits for it;
// otherwise everything waits.  Either way no global store happens before the wait.
__device__ __forceinline__ int64_t first_batch(const GatherParams& p, int64_t row0, int64_t warps,
                                               int64_t n_rows, unsigned lane) {
    int64_t mine = -1;
    RowLookup found;
    const bool early = p.indices_ready || p.disjoint;
    if (early) mine = resolve_batch_at(p, p.positions, p.request_table, row0, warps, n_rows, lane, found);
    // Disjoint: the kernels still running touch nothing this one reads or writes, so
    // it copies at once and waits for them only before exiting (finish()), which
    // keeps the stream's order of completion.
    if (!p.disjoint) grid_dependency_wait();
    allow_dependents();
    if (!early) mine = resolve_batch_at(p, p.positions, p.request_table, row0, warps, n_rows, lane, found);
    emit_lookup(p, row0, warps, n_rows, lane, found);
    return mine;
}

// A disjoint launch completes only after the grids before it: its threads wait for
// them before exiting.  The wait holds the exit and orders none of this kernel's own
// accesses, so it carries no memory clobber.
__device__ __forceinline__ void finish(const GatherParams& p) {
    if (p.disjoint) asm volatile("griddepcontrol.wait;");
}

// Rows are taken 32 at a time per warp (row0 + k * warps, k < 32); the warp then
// streams each row out of all planes with the offset broadcast from its lane.
//
// kU: vectors in flight per lane in the flattened batch copy; kFlatAll: flatten
// every 16-byte-aligned batch, whatever its row size (the small-row instance,
// whose rows x planes x vectors stay far below 2^32).
template <int kU, bool kFlatAll, int kWarps = kGatherWarps>
__device__ __forceinline__ void gather_body(const GatherParams& p) {
    const int64_t n_rows = p.batch * p.selected;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarps;
    const unsigned lane = lane_id();
    int64_t row0 = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    int64_t mine = first_batch(p, row0, warps, n_rows, lane);
    const bool small_rows = p.row_bytes % 16 == 0 && p.plane_or % 16 == 0 &&
                            (kFlatAll || static_cast<uint64_t>(p.n_planes) * (p.row_bytes >> 4) <= kFlatRowLimit);
    for (; row0 < n_rows; row0 += 32 * warps) {
        const int64_t left = (n_rows - row0 + warps - 1) / warps;
        const int nb = static_cast<int>(left < 32 ? left : 32);
        if (small_rows && !__ballot_sync(0xffffffffu, mine >= 0 && (mine & 15))) {
            // The division form for the many-plane small-row instance: its walk was
            // slower (see EKV_GATHER_SMALL_WALK).
            if ((kFlatAll ? EKV_GATHER_SMALL_WALK : EKV_GATHER_WALK) && p.n_planes * (p.row_bytes >> 4) >= 32) {
                copy_batch_vec16<kU, true>(p, mine, row0, warps, nb, lane, 0, p.n_planes);
            } else {
                copy_batch_vec16<kU, false>(p, mine, row0, warps, nb, lane, 0, p.n_planes);
            }
        } else {
            for (int k = 0; k < nb; ++k) {
                const int64_t s = __shfl_sync(0xffffffffu, mine, k);
                copy_row_any(p, s >= 0, s < 0 ? 0 : s, (row0 + k * warps) * p.row_bytes, lane, 0, p.n_planes);
            }
        }
        mine = resolve_batch(p, row0 + 32 * warps, warps, n_rows, lane);
    }
}

// The default instance (every launch the grouped copy and the many-plane small-row
// instance do not take) keeps at most 88 registers, so two of its blocks and one
// 512-thread lookup block (40 registers) share an SM in the decode step's
// concurrent form; the many-plane small-row instance runs alone and may use the
// 128 registers of two blocks per SM.
__global__ void __maxnreg__(88) gather_kernel(const __grid_constant__ GatherParams p) {
    gather_body<kUnroll, false>(p);
}

__global__ void __launch_bounds__(kGatherThreads, kGatherBlocksPerSM)
gather_small_rows_kernel(const __grid_constant__ GatherParams p) {
    gather_body<kSmallUnroll, true>(p);
}

// Disjoint launches (EKV_GATHER_DISJOINT) of the default instance and the two-plane
// grouped instance (a layer's K and V): the wait before exiting costs ptxas
// registers (at 88 it spills the copy loops), so these take
// EKV_GATHER_DISJOINT_MAXNREG and leave no room for a lookup block, which the disjoint
// decode step does not run beside them.  Other instances run a disjoint launch as an
// ordinary one (waiting before they copy), which is always correct.
#ifndef EKV_GATHER_DISJOINT_MAXNREG
#define EKV_GATHER_DISJOINT_MAXNREG 96
#endif
// A disjoint launch runs 128-thread blocks, two per SM (8 warps per SM per layer, as the
// ordinary launch), while registers let five such blocks share an SM: two and a half
// layers are resident at once and a layer's blocks are replaced one by one as they
// finish.  Measured on config 4 (48 layers per step, one B200): 256-thread blocks one per
// SM 0.618 / 3.99 ms at the TP8 / TP1 shard, 128-thread blocks two per SM 0.590 / 3.90,
// three per SM 0.619 / 3.86, 64-thread blocks four per SM 0.594 / 3.90, five per SM
// 0.622 / 3.94, 96-thread blocks three per SM 0.616 / 3.97.
#ifndef EKV_GATHER_DISJOINT_THREADS
#define EKV_GATHER_DISJOINT_THREADS 128  // threads per block of a disjoint launch
#endif
constexpr int kDisjointThreads = EKV_GATHER_DISJOINT_THREADS;
constexpr int kDisjointWarps = kDisjointThreads / 32;
__global__ void __maxnreg__(EKV_GATHER_DISJOINT_MAXNREG)
gather_disjoint_kernel(const __grid_constant__ GatherParams p) {
    gather_body<kUnroll, false, kDisjointWarps>(p);
    finish(p);
}

// Rows of G = row_bytes / 16 vectors per plane, G a power of two of at most 32
// (16 to 512 B rows over 16-byte aligned planes; the 256 B rows of a TP8 head
// shard).  Lanes are grouped G per row: lane l copies vector l % G of row l / G
// of an R = 32 / G-row group, so one load instruction moves R whole rows of one
// plane, and a row's offset is broadcast once per row group and reused for every
// plane -- the flattened copy above pays an integer division and a shuffle per
// 16-byte vector, which bound it by instruction issue at these sizes (ncu:
// warp stalls on fixed-latency dependencies and shuffles, DRAM 68 % busy).
// Each pass keeps kRG row groups x kPL planes of loads in flight per lane
// (instances for launches over few planes put the depth into row groups).
template <int kRG, int kPL>
__device__ __forceinline__ void copy_batch_grouped(const GatherParams& p, int64_t mine, int64_t row0,
                                                   int64_t warps, int nb, unsigned lane, int plane0,
                                                   int n_planes) {
    const int gs = p.vec_shift;
    const int rows_per_group = 32 >> gs;
    const int groups = (nb + rows_per_group - 1) / rows_per_group;
    const int sub = static_cast<int>(lane >> gs);
    const int64_t vbyte = static_cast<int64_t>(lane & ((1u << gs) - 1u)) << 4;
    for (int g0 = 0; g0 < groups; g0 += kRG) {
        int64_t src[kRG];
        bool live[kRG];
#pragma unroll
        for (int j = 0; j < kRG; ++j) {
            const int k = (g0 + j) * rows_per_group + sub;  // row of the batch
            const int64_t s = __shfl_sync(0xffffffffu, mine, k < 32 ? k : 31);
            live[j] = k < nb;
            src[j] = s + vbyte;  // < vbyte for a zero row
        }
        for (int pb = 0; pb < n_planes; pb += kPL) {
            uint4 v[kRG][kPL];
#pragma unroll
            for (int j = 0; j < kRG; ++j) {
#pragma unroll
                for (int q = 0; q < kPL; ++q) {
                    v[j][q] = make_uint4(0u, 0u, 0u, 0u);
                    if (live[j] && src[j] >= vbyte && pb + q < n_planes) {
                        v[j][q] = load_vec(reinterpret_cast<const uint4*>(p.src[plane0 + pb + q] + src[j]));
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kRG; ++j) {
                const int64_t k = (g0 + j) * rows_per_group + sub;
                const int64_t dst = (row0 + k * warps) * p.row_bytes + vbyte;
#pragma unroll
                for (int q = 0; q < kPL; ++q) {
                    if (live[j] && pb + q < n_planes) {
                        store_vec(reinterpret_cast<uint4*>(p.dst[plane0 + pb + q] + dst), v[j][q]);
                    }
                }
            }
        }
    }
}

// At most 88 registers: two of these blocks and one 512-thread lookup block
// (40 registers) fill an SM's 64 Ki registers exactly, which the decode step's
// concurrent form (each layer's lookup beside its gather) relies on.
template <int kRG, int kPL, int kWarps = kGatherWarps>
__device__ __forceinline__ void grouped_body(const GatherParams& p) {
    const int64_t n_rows = p.batch * p.selected;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarps;
    const unsigned lane = lane_id();
    int64_t row0 = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    int64_t mine = first_batch(p, row0, warps, n_rows, lane);
    for (; row0 < n_rows; row0 += 32 * warps) {
        const int64_t left = (n_rows - row0 + warps - 1) / warps;
        const int nb = static_cast<int>(left < 32 ? left : 32);
        if (!__ballot_sync(0xffffffffu, mine >= 0 && (mine & 15))) {
            copy_batch_grouped<kRG, kPL>(p, mine, row0, warps, nb, lane, 0, p.n_planes);
        } else {  // a row of this batch starts off a 16-byte boundary
            for (int k = 0; k < nb; ++k) {
                const int64_t s = __shfl_sync(0xffffffffu, mine, k);
                copy_row_any(p, s >= 0, s < 0 ? 0 : s, (row0 + k * warps) * p.row_bytes, lane, 0, p.n_planes);
            }
        }
        mine = resolve_batch(p, row0 + 32 * warps, warps, n_rows, lane);
    }
}

template <int kRG, int kPL>
__global__ void __maxnreg__(88)
gather_grouped_kernel(const __grid_constant__ GatherParams p) {
    grouped_body<kRG, kPL>(p);
}

template <int kRG, int kPL>
__global__ void __maxnreg__(EKV_GATHER_DISJOINT_MAXNREG)
gather_grouped_disjoint_kernel(const __grid_constant__ GatherParams p) {
    grouped_body<kRG, kPL, kDisjointWarps>(p);
    finish(p);
}

// Multi-layer launch (ekv_gather_layers): layer l gathers its rows with its own
// positions and table out of planes l * planes_per_layer ... into the matching
// outputs; request ids, lengths, slot offsets and the row geometry are shared.
struct LayerGatherParams {
    GatherParams p;  // p.src / p.dst hold every layer's planes, layer-major
    const void* positions[EKV_MAX_LAYERS];
    const void* tables[EKV_MAX_LAYERS];
    int n_layers;
    int planes_per_layer;
};

// Every warp walks the layers in order and takes, in each, the rows a per-layer
// launch of the same grid would give it (row0 + k * warps), so a layer's 32-row
// batches are resolved and copied exactly as in the single-layer kernels -- but
// with no launch boundary between layers: while some warps resolve layer l+1's
// index chains, others are still copying layer l, and DRAM sees one continuous
// stream instead of a ramp and a drain per layer.  kRG > 0: grouped copy (rows of
// 16-512 B, at most kPL planes per layer); kRG == 0: flattened copy.  Batches
// with a row off the 16-byte grid take the per-row copy.  At most 88 registers,
// as the single-layer instances, so lookup blocks still fit beside two of these.
#ifndef EKV_GATHER_LAYERS_MAXNREG
#define EKV_GATHER_LAYERS_MAXNREG 88
#endif
#ifndef EKV_GATHER_LAYERS_RG
#define EKV_GATHER_LAYERS_RG 4  // row groups in flight per lane, two planes per layer
#endif
template <int kRG, int kPL>
__global__ void __maxnreg__(EKV_GATHER_LAYERS_MAXNREG)
gather_layers_kernel(const __grid_constant__ LayerGatherParams lp) {
    const GatherParams& p = lp.p;
    const int64_t n_rows = p.batch * p.selected;  // per layer
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kGatherWarps;
    const unsigned lane = lane_id();
    const int64_t first = static_cast<int64_t>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5);
    const int per_layer = lp.planes_per_layer;
    const uint32_t per_row = static_cast<uint32_t>(per_layer) * static_cast<uint32_t>(p.row_bytes >> 4);
    const bool vectors = p.row_bytes % 16 == 0 && p.plane_or % 16 == 0 && (kRG > 0 || per_row <= kFlatRowLimit);
    grid_dependency_wait();
    allow_dependents();
    for (int layer = 0; layer < lp.n_layers; ++layer) {
        const void* positions = lp.positions[layer];
        const void* table = lp.tables[layer];
        const int plane0 = layer * per_layer;
        for (int64_t row0 = first; row0 < n_rows; row0 += 32 * warps) {
            const int64_t left = (n_rows - row0 + warps - 1) / warps;
            const int nb = static_cast<int>(left < 32 ? left : 32);
            RowLookup found;  // no lookup outputs in the multi-layer launch
            const int64_t mine = resolve_batch_at(p, positions, table, row0, warps, n_rows, lane, found);
            if (vectors && !__ballot_sync(0xffffffffu, mine >= 0 && (mine & 15))) {
                if constexpr (kRG > 0) {
                    copy_batch_grouped<kRG, kPL>(p, mine, row0, warps, nb, lane, plane0, per_layer);
                } else if (per_row >= 32) {
                    copy_batch_vec16<kUnroll, true>(p, mine, row0, warps, nb, lane, plane0, per_layer);
                } else {
                    copy_batch_vec16<kUnroll, false>(p, mine, row0, warps, nb, lane, plane0, per_layer);
                }
            } else {
                for (int k = 0; k < nb; ++k) {
                    const int64_t s = __shfl_sync(0xffffffffu, mine, k);
                    copy_row_any(p, s >= 0, s < 0 ? 0 : s, (row0 + k * warps) * p.row_bytes, lane, plane0,
                                 per_layer);
                }
            }
        }
    }
}

// Sweep knobs (build time): launches over at most EKV_GATHER_GROUPED_MAX_PLANES
// planes take the grouped copy (0 = never); the many-plane grouped instance keeps
// EKV_GATHER_MANY_RG row groups x EKV_GATHER_MANY_PL planes in flight; with
// EKV_GATHER_HONOR_READY 0 the indices-ready flag is ignored.
// Measured on B200: the grouped copy takes config 4's per-layer two-plane launches
// at the TP8 shard from 0.660 to 0.527 ms per 48-layer step (one shared output pair),
// but over all 72 planes of a config-2 launch it trails the flattened copy (0.864 vs
// 0.914 of the copy peak at 256 B rows, 0.896 vs 0.930 at 512 B), so only few-plane
// launches take it.
#ifndef EKV_GATHER_GROUPED_MAX_PLANES
#define EKV_GATHER_GROUPED_MAX_PLANES 4
#endif
#ifndef EKV_GATHER_MANY_RG
#define EKV_GATHER_MANY_RG 2
#endif
#ifndef EKV_GATHER_MANY_PL
#define EKV_GATHER_MANY_PL 6
#endif
#ifndef EKV_GATHER_HONOR_READY
#define EKV_GATHER_HONOR_READY 1
#endif

#ifndef EKV_GATHER_DISJOINT_RG
#define EKV_GATHER_DISJOINT_RG 4  // row groups in flight per lane, disjoint two-plane launches
#endif
#ifndef EKV_GATHER_DISJOINT_BLOCKS
#define EKV_GATHER_DISJOINT_BLOCKS 2  // blocks per SM of a disjoint launch's grid
#endif
constexpr int kDisjointSlot = 8, kDisjointGroupedSlot = 9;

using GatherKernel = void (*)(GatherParams);

// The kernel instance for `n_planes` planes of `row_bytes` rows; `slot` names
// it in the per-device grid cache.  A disjoint launch that the chosen instance does
// not serve as such is cleared to an ordinary one.
GatherKernel gather_kernel_for(GatherParams& p, int& slot, size_t& smem) {
    smem = 0;
    if (p.n_planes <= EKV_GATHER_GROUPED_MAX_PLANES && p.plane_or % 16 == 0 && p.vec_shift >= 0 &&
        p.vec_shift <= 5) {
        if (p.n_planes <= 2) {
            slot = p.disjoint ? kDisjointGroupedSlot : 2;
            return p.disjoint ? gather_grouped_disjoint_kernel<EKV_GATHER_DISJOINT_RG, 2>
                              : gather_grouped_kernel<4, 2>;
        }
        p.disjoint = 0;
        if (p.n_planes <= 4) {
            slot = 3;
            return gather_grouped_kernel<3, 4>;
        }
        slot = 4;
        return gather_grouped_kernel<EKV_GATHER_MANY_RG, EKV_GATHER_MANY_PL>;
    }
    const bool small = kSmallRowBytes > 0 && p.row_bytes <= kSmallRowBytes &&
                       static_cast<uint64_t>(p.n_planes) * (p.row_bytes >> 4) > kFlatRowLimit;
    if (small) {
        p.disjoint = 0;
        slot = 1;
        return gather_small_rows_kernel;
    }
    slot = p.disjoint ? kDisjointSlot : 0;
    return p.disjoint ? gather_disjoint_kernel : gather_kernel;
}

int gather_grid(const void* kernel, int slot, size_t smem, int device, int64_t n_rows, int threads) {
    static std::atomic<int> cached[10][64];  // per instance and device; a race computes twice
    int grid = device < 64 ? cached[slot][device].load(std::memory_order_relaxed) : 0;
    if (!grid) {
        if (smem > 48 * 1024) {
            cuda_check(cudaFuncSetAttribute(kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                       "configure gather shared memory");
        }
        grid = persistent_grid(kernel, threads, smem, device);
        if (slot == kDisjointSlot || slot == kDisjointGroupedSlot) {
            // A disjoint launch leaves SM room for the next ones' blocks, which then
            // become resident and start copying while this one runs: no ramp and
            // drain between back-to-back launches.
            const int cap = EKV_GATHER_DISJOINT_BLOCKS * sm_count(device);
            grid = grid < cap ? grid : cap;
        }
        if (device < 64) cached[slot][device].store(grid, std::memory_order_relaxed);
    }
    const int64_t block_warps = threads / 32;
    const int64_t needed = (n_rows + block_warps - 1) / block_warps;
    return static_cast<int>(needed < grid ? needed : grid);
}

int log2_exact(int64_t x) {
    if (x <= 0 || (x & (x - 1))) return -1;
    int shift = 0;
    while ((int64_t{1} << shift) < x) ++shift;
    return shift;
}

// Checks and fields shared by the single- and multi-layer entry points (everything
// but the planes and the per-layer index arrays).  `indirect` carries the mode and
// the flag bits; returns the mode.
int common_params(GatherParams& p, int64_t itemsize, int positions_esize, const void* request_ids,
                  int request_ids_esize, const void* lengths, int lengths_esize, int table_esize,
                  const void* slot_offsets, int offsets_esize, int64_t batch, int64_t selected, int64_t width,
                  int64_t table_width, int64_t request_stride, int64_t sink_elements, int indirect) {
    require(request_ids && lengths, "null index argument");
    check_esize(positions_esize, "positions");
    check_esize(request_ids_esize, "request_ids");
    check_esize(lengths_esize, "lengths");
    const int flags = indirect & ~3;
    require((flags & ~(EKV_GATHER_INDICES_READY | EKV_GATHER_DISJOINT)) == 0, "unknown gather flag bits");
    const int mode = indirect & 3;
    require(mode <= 2, "addressing mode must be 0 (direct), 1 (indirect) or 2 (mapped)");
    if (mode == 1) {
        require(slot_offsets, "indirect gather needs request_table and slot_offsets");
        check_esize(offsets_esize, "slot_offsets");
    }
    if (mode) check_esize(table_esize, "request_table");
    p.request_ids = request_ids;
    p.lengths = lengths;
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
    p.table_es = mode ? table_esize : 8;
    p.off_es = mode == 1 ? offsets_esize : 8;
    p.indirect = mode;
    p.indices_ready = EKV_GATHER_HONOR_READY ? (flags & EKV_GATHER_INDICES_READY) != 0 : 0;
    p.disjoint = (flags & EKV_GATHER_DISJOINT) != 0;
    p.vec_shift = (p.row_bytes % 16) ? -1 : log2_exact(p.row_bytes / 16);
    return mode;
}

void set_planes(GatherParams& p, const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes) {
    require(src_planes && dst_planes, "null plane array");
    uint64_t plane_or = 0;
    for (int i = 0; i < n_planes; ++i) {
        require(src_planes[i] && dst_planes[i], "null plane address");
        p.src[i] = reinterpret_cast<const char*>(src_planes[i]);
        p.dst[i] = reinterpret_cast<char*>(dst_planes[i]);
        plane_or |= src_planes[i] | dst_planes[i];
    }
    p.n_planes = n_planes;
    p.plane_or = plane_or;
}

int gather_impl(const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
                const void* positions, int positions_esize, const void* request_ids,
                int request_ids_esize, const void* lengths, int lengths_esize,
                const void* request_table, int table_esize, const void* slot_offsets,
                int offsets_esize, int64_t batch, int64_t selected, int64_t width,
                int64_t table_width, int64_t request_stride, int64_t sink_elements, int indirect,
                int device, void* stream, int32_t* slots_out = nullptr, uint8_t* miss_out = nullptr) {
    return guarded([&] {
        require(batch >= 0 && selected >= 0 && width >= 0, "sizes must be non-negative");
        require(itemsize > 0, "itemsize must be positive");
        require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
        if (!batch || !selected || !width) return;
        require(src_planes && dst_planes, "null plane array");
        require(positions && request_ids && lengths, "null index argument");
        GatherParams p{};
        const int mode = common_params(p, itemsize, positions_esize, request_ids, request_ids_esize, lengths,
                                       lengths_esize, table_esize, slot_offsets, offsets_esize, batch, selected,
                                       width, table_width, request_stride, sink_elements, indirect);
        if (mode == 1) require(request_table, "indirect gather needs request_table and slot_offsets");
        if (mode == 2) require(request_table, "mapped gather needs request_table (the residency map)");
        if (slots_out || miss_out) {
            require(mode == 2, "lookup outputs come from a mapped gather");
            require(slots_out && miss_out, "a fused lookup writes both slots and miss");
        }
        p.positions = positions;
        p.request_table = request_table;
        p.slots_out = slots_out;
        p.miss_out = miss_out;
        set_planes(p, src_planes, dst_planes, n_planes);
        bind_device(device);
        const int64_t n_rows = batch * selected;
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        int slot = 0;
        size_t smem = 0;
        const GatherKernel kernel = gather_kernel_for(p, slot, smem);
        const int threads = p.disjoint ? kDisjointThreads : kGatherThreads;
        const int grid = gather_grid(reinterpret_cast<const void*>(kernel), slot, smem, device, n_rows, threads);
        launch_dependent(kernel, dim3(grid), dim3(threads), smem, s, "gather_rows launch", p);
        check_launch("gather_rows launch");
    });
}

using LayerGatherKernel = void (*)(LayerGatherParams);

int gather_layers_impl(const uint64_t* src_planes, const uint64_t* dst_planes, int n_layers, int planes_per_layer,
                       int64_t itemsize, const uint64_t* positions, int positions_esize,
                       const void* request_ids, int request_ids_esize, const void* lengths, int lengths_esize,
                       const uint64_t* request_tables, int table_esize, const void* slot_offsets,
                       int offsets_esize, int64_t batch, int64_t selected, int64_t width, int64_t table_width,
                       int64_t request_stride, int64_t sink_elements, int indirect, int device, void* stream) {
    return guarded([&] {
        require(batch >= 0 && selected >= 0 && width >= 0, "sizes must be non-negative");
        require(itemsize > 0, "itemsize must be positive");
        require(n_layers >= 1 && n_layers <= EKV_MAX_LAYERS, "layer count outside [1, EKV_MAX_LAYERS]");
        require(planes_per_layer >= 1 && static_cast<int64_t>(n_layers) * planes_per_layer <= EKV_MAX_PLANES,
                "n_layers * planes_per_layer outside [1, EKV_MAX_PLANES]");
        if (!batch || !selected || !width) return;
        require(src_planes && dst_planes, "null plane array");
        require(positions, "null positions array");
        LayerGatherParams lp{};
        GatherParams& p = lp.p;
        const int mode = common_params(p, itemsize, positions_esize, request_ids, request_ids_esize, lengths,
                                       lengths_esize, table_esize, slot_offsets, offsets_esize, batch, selected,
                                       width, table_width, request_stride, sink_elements, indirect);
        require(!p.indices_ready && !p.disjoint, "gather_layers takes no flag bits");
        if (mode) require(request_tables, "indirect and mapped gathers need one request table per layer");
        for (int l = 0; l < n_layers; ++l) {
            require(positions[l], "null positions address");
            lp.positions[l] = reinterpret_cast<const void*>(positions[l]);
            if (mode) {
                require(request_tables[l], "null request table address");
                lp.tables[l] = reinterpret_cast<const void*>(request_tables[l]);
            }
        }
        lp.n_layers = n_layers;
        lp.planes_per_layer = planes_per_layer;
        set_planes(p, src_planes, dst_planes, n_layers * planes_per_layer);
        bind_device(device);
        // Grouped copy for 16-512 B rows of at most two (or four) planes per layer
        // over 16-byte aligned planes, as the single-layer selection does.
        LayerGatherKernel kernel = gather_layers_kernel<0, 1>;
        int slot = 5;
        if (planes_per_layer <= 4 && p.plane_or % 16 == 0 && p.vec_shift >= 0 && p.vec_shift <= 5) {
            if (planes_per_layer <= 2) {
                kernel = gather_layers_kernel<EKV_GATHER_LAYERS_RG, 2>;
                slot = 6;
            } else {
                kernel = gather_layers_kernel<2, 4>;
                slot = 7;
            }
        }
        const int grid = gather_grid(reinterpret_cast<const void*>(kernel), slot, 0, device, batch * selected,
                                     kGatherThreads);
        launch_dependent(kernel, dim3(grid), dim3(kGatherThreads), 0, static_cast<cudaStream_t>(stream),
                         "gather_layers launch", lp);
        check_launch("gather_layers launch");
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

extern "C" int ekv_lookup_gather_planes(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
    const void* topk, int topk_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* res_map, int map_esize, int64_t map_width,
    int64_t batch, int64_t k, int64_t width,
    int64_t request_stride, int64_t sink_elements,
    int32_t* slots, uint8_t* miss,
    int flags, int device, void* stream) {
    const int rc = ekv::guarded([&] {
        ekv::require((flags & ~(EKV_GATHER_INDICES_READY | EKV_GATHER_DISJOINT)) == 0,
                     "unknown lookup_gather flag bits");
        if (batch > 0 && k > 0) {
            ekv::require(width > 0, "width must be positive");
            ekv::require(slots && miss, "null lookup output");
        }
    });
    if (rc) return rc;
    return ekv::gather_impl(src_planes, dst_planes, n_planes, itemsize, topk, topk_esize, request_ids,
                            request_ids_esize, lengths, lengths_esize, res_map, map_esize, nullptr, 8, batch, k,
                            width, map_width, request_stride, sink_elements, 2 | flags, device, stream, slots, miss);
}

extern "C" int ekv_gather_layers(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_layers, int planes_per_layer,
    int64_t itemsize,
    const uint64_t* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const uint64_t* request_tables, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream) {
    return ekv::gather_layers_impl(src_planes, dst_planes, n_layers, planes_per_layer, itemsize, positions,
                                   positions_esize, request_ids, request_ids_esize, lengths, lengths_esize,
                                   request_tables, table_esize, slot_offsets, offsets_esize, batch, selected,
                                   width, table_width, request_stride, sink_elements, indirect, device, stream);
}
