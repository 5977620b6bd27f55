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
// plane (all layers, K and V): a warp resolves the index chain of its row once
// -- every lane issues the same broadcast loads -- and then streams that row
// out of all planes.  Copies are 16-byte vector loads and stores with
// evict-first hints (each byte is read once and written once), and each lane
// keeps kUnroll vectors in flight before storing, which at 1024 resident
// threads per SM is ~128 KiB of reads outstanding per SM -- several times the
// HBM bandwidth-latency product.  The grid is persistent: SMs x resident blocks.
// Rows whose addresses are not 16-byte aligned fall back to the widest element
// size that divides every address.
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

constexpr int kGatherThreads = 256;
constexpr int kGatherWarps = kGatherThreads / 32;
constexpr int kUnroll = 8;

// Byte offset of row r inside every source plane, or valid = false.
__device__ __forceinline__ int64_t resolve_row(const GatherParams& p, int64_t r, bool& valid) {
    const int64_t b = r / p.selected;
    const int64_t pos = load_index(p.positions, p.pos_es, r);
    const int64_t length = load_index(p.lengths, p.len_es, b);
    valid = pos >= 0 && pos < length;
    if (!valid) return 0;
    const int64_t req = load_index(p.request_ids, p.req_es, b);
    int64_t element;
    if (p.indirect) {
        const int64_t logical = load_index(p.request_table, p.table_es, req * p.table_width + pos);
        element = load_index(p.slot_offsets, p.off_es, logical);
    } else {
        element = p.sink_elements + req * p.request_stride + pos * p.width;
    }
    return element * p.itemsize;
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
                v[u] = __ldcs(reinterpret_cast<const uint4*>(p.src[plane] + src_off) + vec);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t idx = base + u * 32 + lane;
            if (idx < total) {
                const int64_t plane = p.vec_shift >= 0 ? (idx >> p.vec_shift) : idx / vecs;
                const int64_t vec = idx - plane * vecs;
                __stcs(reinterpret_cast<uint4*>(p.dst[plane] + dst_off) + vec, v[u]);
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

__global__ void __launch_bounds__(kGatherThreads)
gather_kernel(const __grid_constant__ GatherParams p) {
    const int64_t n_rows = p.batch * p.selected;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kGatherWarps;
    const unsigned lane = lane_id();
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kGatherWarps + (threadIdx.x >> 5); r < n_rows;
         r += warps) {
        bool valid;
        const int64_t src_off = resolve_row(p, r, valid);
        const int64_t dst_off = r * p.row_bytes;
        const int64_t align = alignment_of(p.plane_or | static_cast<uint64_t>(src_off) |
                                           static_cast<uint64_t>(dst_off) |
                                           static_cast<uint64_t>(p.row_bytes));
        switch (align) {
            case 16: copy_row_vec16(p, valid, src_off, dst_off, lane); break;
            case 8: copy_row_elems<uint64_t>(p, valid, src_off, dst_off, lane); break;
            case 4: copy_row_elems<uint32_t>(p, valid, src_off, dst_off, lane); break;
            case 2: copy_row_elems<uint16_t>(p, valid, src_off, dst_off, lane); break;
            default: copy_row_elems<uint8_t>(p, valid, src_off, dst_off, lane); break;
        }
    }
}

int gather_grid(int device, int64_t n_rows) {
    static int cached[64] = {0};
    int grid = device < 64 ? cached[device] : 0;
    if (!grid) {
        grid = persistent_grid(reinterpret_cast<const void*>(gather_kernel), kGatherThreads, 0, device);
        if (device < 64) cached[device] = grid;
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
        if (indirect) {
            require(request_table && slot_offsets, "indirect gather needs request_table and slot_offsets");
            check_esize(table_esize, "request_table");
            check_esize(offsets_esize, "slot_offsets");
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
        p.off_es = indirect ? offsets_esize : 8;
        p.indirect = indirect ? 1 : 0;
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
        gather_kernel<<<gather_grid(device, n_rows), kGatherThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(p);
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
