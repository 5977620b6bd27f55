// Shared-prefix donor-slot resolution (batched).
//
// For each consumer request r and Top-K block b: the block is shared when it
// lies wholly inside the consumer's shared prefix and sequence, and then its
// block_size positions resolve through the SOURCE request's row of the request
// table to logical slots and through the device mapping to device slots; the
// block is valid only if every position has logical >= 0 and slot > 0.
// Positions and logical ids are clamped before they index, so a device slot is
// written for every block, valid or not.  Semantics of
// resolve_shared_block_locations_batched, adaptive_sparse/shared_prefix.py:188-204;
// `exclude_newest` adds the caller's newest-token rule
// (adaptive_sparse/request_residency.py:220).
//
// Launch shape: a group of G lanes (G = next power of two >= block_size,
// capped at 32) owns one block; its lanes walk the block's positions with
// stride G and agree on "all positions mapped" through one warp ballot.  With
// block_size 1 every lane owns a block, with 64 a warp does.  Like the other
// lookups this is a chain of dependent 4/8-byte loads, bound by latency.
#include "common.cuh"

namespace ekv {
namespace {

struct SharedParams {
    const void* blocks;
    const int64_t* source_rows;    // [requests] or null (then source_row)
    const int64_t* shared_tokens;  // [requests] or null (then shared_count)
    const void* seq_len;
    const void* table;
    const void* mapping;
    uint8_t* valid;
    int32_t* physical;
    void* masked_blocks;
    int64_t source_row, shared_count;
    int64_t block_row, block_col, len_stride;
    int64_t table_rows, table_width, table_row, table_col;
    int64_t map_len, map_stride;
    int64_t requests, per_request, block_size;
    int blocks_es, len_es, table_es, map_es, masked_es;
    int group_log2;
    int exclude_newest;
};

constexpr int kSharedThreads = 256;
constexpr int kSharedInline = EKV_SHARED_INLINE_MAX;

// Launch parameters.  With kInline the per-request source rows and prefix
// lengths travel inside the parameter block (8 KiB at 512 requests; CUDA 12
// allows 32 KiB), so a call with host-side lists needs no copy to the device.
template <int kInline>
struct SharedLaunch {
    SharedParams p;
    int64_t rows[kInline ? kInline : 1];
    int64_t prefixes[kInline ? kInline : 1];
};

__device__ __forceinline__ int64_t wrap_mul(int64_t a, int64_t b) {
    return static_cast<int64_t>(static_cast<uint64_t>(a) * static_cast<uint64_t>(b));
}

__device__ __forceinline__ int64_t wrap_add(int64_t a, int64_t b) {
    return static_cast<int64_t>(static_cast<uint64_t>(a) + static_cast<uint64_t>(b));
}

__device__ __forceinline__ int64_t clamp64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

template <int kInline>
__global__ void __launch_bounds__(kSharedThreads)
shared_blocks_kernel(const __grid_constant__ SharedLaunch<kInline> launch) {
    grid_dependency_wait();
    allow_dependents();
    const SharedParams& p = launch.p;
    const unsigned lane = lane_id();
    const int group = 1 << p.group_log2;
    const int per_warp = 32 >> p.group_log2;
    const unsigned sub = lane & (group - 1);
    const unsigned slot = lane >> p.group_log2;
    const unsigned group_mask =
        (group == 32 ? 0xffffffffu : ((1u << group) - 1u)) << (slot * group);
    const int64_t total = p.requests * p.per_request;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kSharedThreads / 32);
    // Warp-uniform loop: every lane reaches the ballot on every pass.
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (kSharedThreads / 32) + (threadIdx.x >> 5);
         w * per_warp < total; w += warps) {
        const int64_t q = w * per_warp + slot;
        bool lane_ok = true;
        bool shared = false;
        int64_t block = 0;
        int64_t length = 0;
        int64_t r = 0, b = 0;
        if (q < total) {
            r = q / p.per_request;
            b = q - r * p.per_request;
            block = load_index(p.blocks, p.blocks_es, r * p.block_row + b * p.block_col);
            length = load_index(p.seq_len, p.len_es, r * p.len_stride);
            int64_t row, prefix;
            if (kInline) {
                row = launch.rows[r];
                prefix = launch.prefixes[r];
            } else {
                row = p.source_rows ? p.source_rows[r] : p.source_row;
                prefix = p.shared_tokens ? p.shared_tokens[r] : p.shared_count;
            }
            const int64_t start = wrap_mul(block, p.block_size);
            const int64_t end = wrap_add(start, p.block_size);
            shared = block >= 0 && end <= prefix && end <= length;
            // A source row outside the table (rejected by the host API before the
            // launch) resolves nothing: slot 0, block invalid.
            const bool row_ok = row >= 0 && row < p.table_rows;
            for (int64_t j = sub; j < p.block_size; j += group) {
                int64_t slot_value = 0;
                if (row_ok) {
                    const int64_t pos = clamp64(wrap_add(start, j), 0, p.table_width - 1);
                    const int64_t logical = load_index(p.table, p.table_es, row * p.table_row + pos * p.table_col);
                    const int64_t safe = clamp64(logical, 0, p.map_len - 1);
                    slot_value = load_index(p.mapping, p.map_es, safe * p.map_stride);
                    lane_ok = lane_ok && logical >= 0 && slot_value > 0;
                } else {
                    lane_ok = false;
                }
                // int64 -> int32: two's-complement truncation, as the reference's cast.
                p.physical[q * p.block_size + j] = static_cast<int32_t>(slot_value);
            }
        }
        const unsigned ok_bits = __ballot_sync(0xffffffffu, lane_ok);
        if (q < total && sub == 0) {
            bool valid = shared && (ok_bits & group_mask) == group_mask;
            if (p.exclude_newest) valid = valid && wrap_mul(wrap_add(block, 1), p.block_size) < length;
            p.valid[q] = valid ? 1 : 0;
            if (p.masked_blocks) {
                const int64_t value = valid ? -1 : block;
                const int64_t at = r * p.block_row + b * p.block_col;
                if (p.masked_es == 8) {
                    static_cast<int64_t*>(p.masked_blocks)[at] = value;
                } else {
                    static_cast<int32_t*>(p.masked_blocks)[at] = static_cast<int32_t>(value);
                }
            }
        }
    }
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_resolve_shared_blocks(
    const void* block_ids, int block_esize, int64_t requests, int64_t per_request, int64_t block_row,
    int64_t block_col, const int64_t* source_rows, int64_t source_row, const int64_t* shared_tokens,
    int64_t shared_count, const void* seq_len, int len_esize, int64_t len_stride, int64_t block_size,
    const void* request_table, int table_esize, int64_t table_rows, int64_t table_width, int64_t table_row,
    int64_t table_col, const void* device_mapping, int map_esize, int64_t map_len, int64_t map_stride,
    int meta_on_host, uint8_t* valid, int32_t* physical, void* masked_blocks, int exclude_newest, int device,
    void* stream) {
    using namespace ekv;
    return guarded([&] {
        require(requests >= 0 && per_request >= 0, "negative block-id dimensions");
        require(block_size >= 1 && block_size <= (int64_t{1} << 30), "block_size outside [1, 2^30]");
        require(table_rows >= 1 && table_width >= 1 && map_len >= 1, "shared prefix address geometry is empty");
        if (requests == 0 || per_request == 0) return;
        require(block_ids && seq_len && request_table && device_mapping && valid && physical,
                "null pointer argument");
        if (meta_on_host) {
            require(source_rows && shared_tokens, "host metadata needs both source_rows and shared_tokens");
            require(requests <= kSharedInline, "host metadata holds at most EKV_SHARED_INLINE_MAX requests");
        }
        check_esize(block_esize, "block_ids");
        check_esize(len_esize, "seq_len");
        check_esize(table_esize, "request_table");
        check_esize(map_esize, "device_mapping");
        bind_device(device);
        SharedParams p{};
        p.blocks = block_ids;
        p.source_rows = source_rows;
        p.shared_tokens = shared_tokens;
        p.seq_len = seq_len;
        p.table = request_table;
        p.mapping = device_mapping;
        p.valid = valid;
        p.physical = physical;
        p.masked_blocks = masked_blocks;
        p.source_row = source_row;
        p.shared_count = shared_count;
        p.block_row = block_row;
        p.block_col = block_col;
        p.len_stride = len_stride;
        p.table_rows = table_rows;
        p.table_width = table_width;
        p.table_row = table_row;
        p.table_col = table_col;
        p.map_len = map_len;
        p.map_stride = map_stride;
        p.requests = requests;
        p.per_request = per_request;
        p.block_size = block_size;
        p.blocks_es = block_esize;
        p.len_es = len_esize;
        p.table_es = table_esize;
        p.map_es = map_esize;
        p.masked_es = block_esize;
        p.exclude_newest = exclude_newest ? 1 : 0;
        int log2 = 0;
        while ((int64_t{1} << log2) < block_size && log2 < 5) ++log2;
        p.group_log2 = log2;
        const int64_t per_warp = 32 >> log2;
        const int64_t warps = (requests * per_request + per_warp - 1) / per_warp;
        const int64_t wanted = (warps + kSharedThreads / 32 - 1) / (kSharedThreads / 32);
        const int64_t cap = static_cast<int64_t>(sm_count(device)) * 8;
        const int grid = static_cast<int>(wanted < cap ? wanted : cap);
        const auto cstream = static_cast<cudaStream_t>(stream);
        if (meta_on_host) {
            SharedLaunch<kSharedInline> launch{};
            launch.p = p;
            launch.p.source_rows = nullptr;
            launch.p.shared_tokens = nullptr;
            for (int64_t r = 0; r < requests; ++r) {
                launch.rows[r] = source_rows[r];
                launch.prefixes[r] = shared_tokens[r];
            }
            launch_dependent(shared_blocks_kernel<kSharedInline>, dim3(grid), dim3(kSharedThreads), 0, cstream,
                             "shared_blocks launch", launch);
        } else {
            SharedLaunch<0> launch{};
            launch.p = p;
            launch_dependent(shared_blocks_kernel<0>, dim3(grid), dim3(kSharedThreads), 0, cstream,
                             "shared_blocks launch", launch);
        }
        check_launch("shared_blocks launch");
    });
}
