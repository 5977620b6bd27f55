// Logical-shadow checker: bitwise validation of KV rows on the device.
//
// A diagnostic shadow keeps, per layer, a copy of every K/V row a producer
// wrote (indexed by logical slot) plus an "initialized" flag per slot.
//
// shadow_clean_kernel + shadow_tokens_kernel (one decode step of one layer; semantics of
//   LogicalShadow.check, adaptive_sparse/logical_shadow.py:45-86): cleans the
//   Top-K block ids (keeps each row's valid prefix, -1 elsewhere, counts
//   malformed ids), resolves every selected position through the request
//   table to a logical slot, maps it to a physical slot (given, or = logical),
//   and compares the cache's K and V rows at the physical slot with the
//   shadow's at the logical slot, bit for bit.
// shadow_complete_kernel (after a migration; LogicalShadow.check_complete,
//   :88-123): the same comparison for a list of (logical, physical) pairs over
//   every layer of a pool.
// shadow_write_kernel / shadow_reset_kernel: record producer writes
//   (:30-43) and forget reallocated slots (:26-28).
//
// The index chains are resolved one token per lane (32 independent chains per
// warp); the rows of the tokens that need a comparison are then streamed by
// the whole warp with the widest vector that every base, stride and row length
// allows, so a checking run costs one read of each compared row pair and
// finishes at HBM speed.  Counters are reduced per warp and added with one
// atomic per counter per block.
#include <algorithm>
#include <initializer_list>

#include "common.cuh"

namespace ekv {
namespace {

constexpr int kShadowThreads = 256;
constexpr int kShadowWarps = kShadowThreads / 32;
constexpr int kShadowTokensPerBlock = 1024;
constexpr int kShadowMaxLayers = EKV_SHADOW_MAX_LAYERS;

__device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
    const int64_t q = a / b;
    return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

// Warp-cooperative "rows differ" over row_bytes bytes with element type V.
template <class V>
__device__ __forceinline__ bool rows_differ(const char* a, const char* b, int64_t row_bytes, unsigned lane) {
    const int64_t n = row_bytes / static_cast<int64_t>(sizeof(V));
    const V* x = reinterpret_cast<const V*>(a);
    const V* y = reinterpret_cast<const V*>(b);
    bool differ = false;
#pragma unroll 4
    for (int64_t i = lane; i < n; i += 32) {
        const V u = __ldg(x + i);
        const V v = __ldg(y + i);
        if constexpr (sizeof(V) == 16) {
            differ |= (u.x != v.x) | (u.y != v.y) | (u.z != v.z) | (u.w != v.w);
        } else {
            differ |= (u != v);
        }
    }
    return differ;
}

// K and V rows of one token compared in ONE loop, so all of a lane's loads of
// both row pairs are in flight together (one memory round trip per token for
// rows up to 4 vectors per lane).  Requires equal K and V row lengths.
template <class V>
__device__ __forceinline__ bool row_pairs_differ(const char* ka, const char* kb, const char* va, const char* vb,
                                                 int64_t row_bytes, unsigned lane) {
    const int64_t n = row_bytes / static_cast<int64_t>(sizeof(V));
    const V* k0 = reinterpret_cast<const V*>(ka);
    const V* k1 = reinterpret_cast<const V*>(kb);
    const V* v0 = reinterpret_cast<const V*>(va);
    const V* v1 = reinterpret_cast<const V*>(vb);
    bool differ = false;
#pragma unroll 4
    for (int64_t i = lane; i < n; i += 32) {
        const V a = __ldg(k0 + i);
        const V b = __ldg(k1 + i);
        const V c = __ldg(v0 + i);
        const V d = __ldg(v1 + i);
        if constexpr (sizeof(V) == 16) {
            differ |= (a.x != b.x) | (a.y != b.y) | (a.z != b.z) | (a.w != b.w) | (c.x != d.x) | (c.y != d.y) |
                      (c.z != d.z) | (c.w != d.w);
        } else {
            differ |= (a != b) | (c != d);
        }
    }
    return differ;
}

template <class V>
__device__ __forceinline__ bool kv_differ(const char* ka, const char* kb, int64_t k_bytes, const char* va,
                                          const char* vb, int64_t v_bytes, unsigned lane) {
    if (k_bytes == v_bytes) return row_pairs_differ<V>(ka, kb, va, vb, k_bytes, lane);
    return rows_differ<V>(ka, kb, k_bytes, lane) | rows_differ<V>(va, vb, v_bytes, lane);
}

__device__ __forceinline__ void add_counts(unsigned long long* counts, const unsigned (&local)[5],
                                           unsigned (&block_sum)[5], int n) {
    const unsigned lane = lane_id();
    for (int i = 0; i < n; ++i) {
        const unsigned total = __reduce_add_sync(0xffffffffu, local[i]);
        if (lane == 0 && total) atomicAdd(&block_sum[i], total);
    }
}

struct CheckParams {
    const void* blocks;
    const void* lengths;
    const void* rows;
    const void* table;
    const int32_t* physical;
    const uint8_t* live;
    const char* k_cache;
    const char* v_cache;
    const char* k_shadow;
    const char* v_shadow;
    const uint8_t* initialized;
    void* clean_blocks;
    int32_t* physical_out;
    unsigned long long* counts;
    int64_t blocks_row, blocks_col, len_stride, rows_stride;
    int64_t table_width, table_row, table_col;
    int64_t phys_row, phys_col, live_len;
    int64_t cache_rows, k_cache_stride, v_cache_stride;
    int64_t capacity, k_shadow_stride, v_shadow_stride;
    int64_t k_row_bytes, v_row_bytes;
    int64_t batch, n_blocks, block_size, page_size;
    int blocks_es, len_es, rows_es, table_es;
    int vec;
};

// Pass 1, one block per request row: the end of the row's valid prefix (the
// cumulative product of block validity), the cleaned ids (-1 past the prefix)
// and the malformed-id count.  Also counts the call.
__global__ void __launch_bounds__(kShadowThreads)
shadow_clean_kernel(const __grid_constant__ CheckParams p) {
    __shared__ int first_invalid;
    __shared__ unsigned malformed;
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(&p.counts[5], 1ull);  // checked_calls
    for (int64_t b = blockIdx.x; b < p.batch; b += gridDim.x) {
        if (threadIdx.x == 0) {
            first_invalid = static_cast<int>(p.n_blocks);
            malformed = 0;
        }
        __syncthreads();
        const int64_t length = load_index(p.lengths, p.len_es, b * p.len_stride);
        const int64_t limit = floor_div(length + p.block_size - 1, p.block_size);
        for (int64_t k = threadIdx.x; k < p.n_blocks; k += kShadowThreads) {
            const int64_t block = load_index(p.blocks, p.blocks_es, b * p.blocks_row + k * p.blocks_col);
            if (!(block >= 0 && block < limit)) atomicMin(&first_invalid, static_cast<int>(k));
        }
        __syncthreads();
        const int64_t first = first_invalid;
        unsigned local = 0;
        for (int64_t k = threadIdx.x; k < p.n_blocks; k += kShadowThreads) {
            const int64_t block = load_index(p.blocks, p.blocks_es, b * p.blocks_row + k * p.blocks_col);
            const bool valid = block >= 0 && block < limit;
            const bool prefix = k < first;
            local += ((block != -1 && !valid) || (valid && !prefix)) ? 1u : 0u;
            const int64_t c = prefix ? block : -1;
            const int64_t at = b * p.n_blocks + k;
            if (p.blocks_es == 8) {
                static_cast<int64_t*>(p.clean_blocks)[at] = c;
            } else {
                static_cast<int32_t*>(p.clean_blocks)[at] = static_cast<int32_t>(c);
            }
        }
        const unsigned total = __reduce_add_sync(0xffffffffu, local);
        if (lane_id() == 0 && total) atomicAdd(&malformed, total);
        __syncthreads();
        if (threadIdx.x == 0 && malformed) atomicAdd(&p.counts[6], static_cast<unsigned long long>(malformed));
        __syncthreads();  // the shared words are reused by the next row
    }
}

// Pass 2, persistent: every warp takes an equal contiguous slice of all
// (request, token) pairs, so no warp idles while another finishes (ncu showed
// blocks of uneven tiles waiting at their barrier).  Per 32 tokens: one index
// chain per lane, then the warp compares the rows of each checked token.
// 2 blocks per SM leave 128 registers a thread: room for all 16 row vectors a
// lane loads per token (K and V, cache and shadow, 2 KiB rows) to be in flight.
template <class V>
__global__ void __launch_bounds__(kShadowThreads, 2)
shadow_tokens_kernel(const __grid_constant__ CheckParams p) {
    __shared__ unsigned block_sum[5];  // checked, uninitialized, invalid physical, mismatched
    const unsigned lane = lane_id();
    if (threadIdx.x < 5) block_sum[threadIdx.x] = 0;
    __syncthreads();
    const int64_t width = p.n_blocks * p.block_size;
    const int64_t total = p.batch * width;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kShadowWarps;
    const int64_t g = static_cast<int64_t>(blockIdx.x) * kShadowWarps + (threadIdx.x >> 5);
    const int64_t begin = static_cast<int64_t>((static_cast<__int128>(total) * g) / warps);
    const int64_t end = static_cast<int64_t>((static_cast<__int128>(total) * (g + 1)) / warps);
    unsigned local[5] = {0, 0, 0, 0, 0};
    for (int64_t base = begin; base < end; base += 32) {
        const int64_t token = base + lane;
        bool checked = false;
        int64_t safe = 0, logical = 0;
        if (token < end) {
            const int64_t b = token / width;
            const int64_t t = token - b * width;
            const int64_t kk = t / p.block_size;
            const int64_t j = t - kk * p.block_size;
            const int64_t clean = load_index(p.clean_blocks, p.blocks_es, b * p.n_blocks + kk);
            const int64_t length = load_index(p.lengths, p.len_es, b * p.len_stride);
            const int64_t position =
                static_cast<int64_t>(static_cast<uint64_t>(clean) * static_cast<uint64_t>(p.block_size) + j);
            const bool selected = position >= 0 && position < length;
            const bool bounded = selected && position < p.table_width;
            bool logical_valid = false;
            if (bounded) {
                const int64_t req = load_index(p.rows, p.rows_es, b * p.rows_stride);
                logical = load_index(p.table, p.table_es, req * p.table_row + position * p.table_col);
                logical_valid = logical >= p.page_size && logical < p.capacity;
            }
            if (!logical_valid) logical = 0;
            const bool source_valid = logical_valid && p.initialized[logical] != 0;
            const int64_t phys =
                p.physical ? static_cast<int64_t>(p.physical[b * p.phys_row + t * p.phys_col]) : logical;
            const bool in_range = phys >= p.page_size && phys < p.cache_rows;
            safe = in_range ? phys : 0;
            bool backed = in_range;
            if (p.live && backed) {
                const int64_t page = safe / p.page_size;
                backed = page < p.live_len && p.live[page] != 0;
            }
            if (!backed) safe = 0;
            checked = selected && source_valid && backed;
            local[0] += checked ? 1u : 0u;
            local[1] += (selected && !source_valid) ? 1u : 0u;
            local[2] += (selected && !backed) ? 1u : 0u;
            p.physical_out[token] = (selected && !backed) ? 0 : static_cast<int32_t>(phys);
        }
        unsigned pending = __ballot_sync(0xffffffffu, checked);
        while (pending) {
            const int src = __ffs(pending) - 1;
            pending &= pending - 1;
            const int64_t s = __shfl_sync(0xffffffffu, safe, src);
            const int64_t l = __shfl_sync(0xffffffffu, logical, src);
            const bool differ =
                kv_differ<V>(p.k_cache + s * p.k_cache_stride, p.k_shadow + l * p.k_shadow_stride, p.k_row_bytes,
                             p.v_cache + s * p.v_cache_stride, p.v_shadow + l * p.v_shadow_stride, p.v_row_bytes,
                             lane);
            if (__any_sync(0xffffffffu, differ) && lane == static_cast<unsigned>(src)) local[3] += 1u;
        }
    }
    add_counts(p.counts, local, block_sum, 4);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long checked = block_sum[0];
        if (checked) {
            atomicAdd(&p.counts[0], checked);
            atomicAdd(&p.counts[1], checked * static_cast<unsigned long long>(p.k_row_bytes + p.v_row_bytes));
        }
        if (block_sum[1]) atomicAdd(&p.counts[2], static_cast<unsigned long long>(block_sum[1]));
        if (block_sum[2]) atomicAdd(&p.counts[3], static_cast<unsigned long long>(block_sum[2]));
        if (block_sum[3]) atomicAdd(&p.counts[4], static_cast<unsigned long long>(block_sum[3]));
    }
}

struct CompleteParams {
    const void* logical;
    const void* physical;
    const uint8_t* live;
    unsigned long long* counts;
    int64_t n, page_size, pool_size, capacity, live_len, tile;
    int64_t pool_k_stride, pool_v_stride, shadow_k_stride, shadow_v_stride;
    int64_t k_row_bytes, v_row_bytes;
    int logical_es, physical_es, vec, n_layers;
    const char* pool_k[kShadowMaxLayers];
    const char* pool_v[kShadowMaxLayers];
    const char* shadow_k[kShadowMaxLayers];
    const char* shadow_v[kShadowMaxLayers];
    const uint8_t* initialized[kShadowMaxLayers];
};

// grid.x tiles the slot pairs, grid.y walks the layers.
template <class V>
__global__ void __launch_bounds__(kShadowThreads, 2)
shadow_complete_kernel(const __grid_constant__ CompleteParams p) {
    __shared__ unsigned block_sum[5];
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x < 5) block_sum[threadIdx.x] = 0;
    __syncthreads();
    unsigned local[5] = {0, 0, 0, 0, 0};  // checked, invalid, mismatched
    for (int layer = blockIdx.y; layer < p.n_layers; layer += gridDim.y) {
        const int64_t i0 = static_cast<int64_t>(blockIdx.x) * p.tile;
        const int64_t i1 = min(p.n, i0 + p.tile);
        for (int64_t base = i0 + static_cast<int64_t>(warp) * 32; base < i1; base += kShadowThreads) {
            const int64_t i = base + lane;
            bool valid = false;
            int64_t sl = 0, sp = 0;
            if (i < i1) {
                const int64_t logical = load_index(p.logical, p.logical_es, i);
                const int64_t physical = load_index(p.physical, p.physical_es, i);
                const bool logical_valid = logical >= p.page_size && logical < p.capacity;
                bool physical_valid = physical >= p.page_size && physical < p.pool_size + p.page_size;
                sl = logical_valid ? logical : 0;
                sp = physical_valid ? physical : 0;
                const int64_t page = sp / p.page_size;
                physical_valid = physical_valid && page < p.live_len && p.live[page] != 0;
                if (!physical_valid) sp = 0;
                valid = logical_valid && physical_valid && p.initialized[layer][sl] != 0;
                local[0] += valid ? 1u : 0u;
                local[1] += valid ? 0u : 1u;
            }
            unsigned pending = __ballot_sync(0xffffffffu, valid);
            while (pending) {
                const int src = __ffs(pending) - 1;
                pending &= pending - 1;
                const int64_t s = __shfl_sync(0xffffffffu, sp, src);
                const int64_t l = __shfl_sync(0xffffffffu, sl, src);
                const bool differ =
                    kv_differ<V>(p.pool_k[layer] + s * p.pool_k_stride, p.shadow_k[layer] + l * p.shadow_k_stride,
                                 p.k_row_bytes, p.pool_v[layer] + s * p.pool_v_stride,
                                 p.shadow_v[layer] + l * p.shadow_v_stride, p.v_row_bytes, lane);
                if (__any_sync(0xffffffffu, differ) && lane == static_cast<unsigned>(src)) local[2] += 1u;
            }
        }
    }
    add_counts(p.counts, local, block_sum, 3);
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long checked = block_sum[0];
        if (checked) {
            atomicAdd(&p.counts[0], checked);
            atomicAdd(&p.counts[1], checked * static_cast<unsigned long long>(p.k_row_bytes + p.v_row_bytes));
        }
        if (block_sum[1]) atomicAdd(&p.counts[2], static_cast<unsigned long long>(block_sum[1]));
        if (block_sum[2]) atomicAdd(&p.counts[3], static_cast<unsigned long long>(block_sum[2]));
    }
}

struct WriteParams {
    char* k_shadow;
    char* v_shadow;
    uint8_t* initialized;
    const char* key;
    const char* value;
    const void* locations;
    int64_t n, capacity, k_shadow_stride, v_shadow_stride, key_stride, value_stride, k_row_bytes, v_row_bytes;
    int loc_es, vec;
};

template <class V>
__device__ __forceinline__ void copy_row(char* dst, const char* src, int64_t row_bytes, unsigned lane) {
    const int64_t n = row_bytes / static_cast<int64_t>(sizeof(V));
#pragma unroll 4
    for (int64_t i = lane; i < n; i += 32) reinterpret_cast<V*>(dst)[i] = __ldg(reinterpret_cast<const V*>(src) + i);
}

// One warp per written row; slots outside [-capacity, capacity) are skipped,
// negative ones count from the end (Python indexing, as the reference's
// tensor assignment does).
template <class V>
__global__ void __launch_bounds__(kShadowThreads)
shadow_write_kernel(const __grid_constant__ WriteParams p) {
    const unsigned lane = lane_id();
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kShadowWarps;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kShadowWarps + (threadIdx.x >> 5); r < p.n; r += warps) {
        int64_t slot = load_index(p.locations, p.loc_es, r);
        if (slot < 0) slot += p.capacity;
        if (slot < 0 || slot >= p.capacity) continue;
        copy_row<V>(p.k_shadow + slot * p.k_shadow_stride, p.key + r * p.key_stride, p.k_row_bytes, lane);
        copy_row<V>(p.v_shadow + slot * p.v_shadow_stride, p.value + r * p.value_stride, p.v_row_bytes, lane);
        if (lane == 0) p.initialized[slot] = 1;
    }
}

struct ResetParams {
    const void* locations;
    int64_t n, capacity;
    int loc_es, n_layers;
    uint8_t* initialized[kShadowMaxLayers];
};

__global__ void __launch_bounds__(kShadowThreads)
shadow_reset_kernel(const __grid_constant__ ResetParams p) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kShadowThreads;
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * kShadowThreads + threadIdx.x; r < p.n; r += stride) {
        int64_t slot = load_index(p.locations, p.loc_es, r);
        if (slot < 0) slot += p.capacity;
        if (slot < 0 || slot >= p.capacity) continue;
        for (int layer = 0; layer < p.n_layers; ++layer) p.initialized[layer][slot] = 0;
    }
}

// Widest vector (16, 8, 4 or 2 bytes) dividing every value.
int vector_width(std::initializer_list<uint64_t> values) {
    uint64_t bits = 16;
    for (uint64_t v : values) bits |= v;
    for (int w : {16, 8, 4}) {
        if ((bits & static_cast<uint64_t>(w - 1)) == 0) return w;
    }
    return 2;
}

// Call f(V{}) with V the unsigned type of `vec` bytes.
template <class F>
void with_vector(int vec, F&& f) {
    switch (vec) {
        case 16: f(uint4{}); break;
        case 8: f(static_cast<unsigned long long>(0)); break;
        case 4: f(0u); break;
        default: f(static_cast<unsigned short>(0)); break;
    }
}

// Token tile per block so the grid covers every SM a few times over.
int64_t tokens_per_block(int64_t tokens, int device) {
    const int64_t target = static_cast<int64_t>(sm_count(device)) * 2;
    const int64_t per = (tokens + target - 1) / target;
    return std::max<int64_t>(64, std::min<int64_t>(kShadowTokensPerBlock, per));
}

int grid_for(int64_t work, int64_t per_block, int device) {
    const int64_t wanted = (work + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 16;
    return static_cast<int>(std::max<int64_t>(1, std::min(wanted, cap)));
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_shadow_check(
    const void* blocks, int blocks_esize, int64_t batch, int64_t n_blocks, int64_t blocks_row, int64_t blocks_col,
    const void* lengths, int len_esize, int64_t len_stride, const void* rows, int rows_esize, int64_t rows_stride,
    const void* request_table, int table_esize, int64_t table_width, int64_t table_row, int64_t table_col,
    const int32_t* physical, int64_t phys_row, int64_t phys_col, const uint8_t* live_pages, int64_t live_len,
    const void* k_cache, const void* v_cache, int64_t cache_rows, int64_t k_cache_stride, int64_t v_cache_stride,
    const void* k_shadow, const void* v_shadow, const uint8_t* initialized, int64_t capacity,
    int64_t k_shadow_stride, int64_t v_shadow_stride, int64_t k_row_bytes, int64_t v_row_bytes,
    int64_t block_size, int64_t page_size, void* clean_blocks, int32_t* physical_out, uint64_t* counts,
    int device, void* stream) {
    using namespace ekv;
    return guarded([&] {
        require(batch >= 0 && n_blocks >= 0 && batch <= 65535, "batch outside [0, 65535] or negative block count");
        require(block_size >= 1 && page_size >= 1, "block_size and page_size must be positive");
        require(capacity >= 1 && cache_rows >= 1 && table_width >= 1, "empty shadow, cache or request table");
        require(k_row_bytes > 0 && v_row_bytes > 0 && k_row_bytes % 2 == 0 && v_row_bytes % 2 == 0,
                "row sizes must be positive multiples of 2 bytes (bf16 rows)");
        require(n_blocks <= (int64_t{1} << 30), "more than 2^30 Top-K blocks per row");
        require(counts && initialized && k_cache && v_cache && k_shadow && v_shadow, "null pointer argument");
        if (batch > 0 && n_blocks > 0) {
            require(blocks && lengths && rows && request_table && clean_blocks && physical_out,
                    "null pointer argument");
            check_esize(blocks_esize, "blocks");
            check_esize(len_esize, "lengths");
            check_esize(rows_esize, "rows");
            check_esize(table_esize, "request_table");
        }
        bind_device(device);
        CheckParams p{};
        p.blocks = blocks;
        p.lengths = lengths;
        p.rows = rows;
        p.table = request_table;
        p.physical = physical;
        p.live = live_pages;
        p.k_cache = static_cast<const char*>(k_cache);
        p.v_cache = static_cast<const char*>(v_cache);
        p.k_shadow = static_cast<const char*>(k_shadow);
        p.v_shadow = static_cast<const char*>(v_shadow);
        p.initialized = initialized;
        p.clean_blocks = clean_blocks;
        p.physical_out = physical_out;
        p.counts = reinterpret_cast<unsigned long long*>(counts);
        p.blocks_row = blocks_row;
        p.blocks_col = blocks_col;
        p.len_stride = len_stride;
        p.rows_stride = rows_stride;
        p.table_width = table_width;
        p.table_row = table_row;
        p.table_col = table_col;
        p.phys_row = phys_row;
        p.phys_col = phys_col;
        p.live_len = live_len;
        p.cache_rows = cache_rows;
        p.k_cache_stride = k_cache_stride;
        p.v_cache_stride = v_cache_stride;
        p.capacity = capacity;
        p.k_shadow_stride = k_shadow_stride;
        p.v_shadow_stride = v_shadow_stride;
        p.k_row_bytes = k_row_bytes;
        p.v_row_bytes = v_row_bytes;
        p.batch = (n_blocks > 0) ? batch : 0;
        p.n_blocks = n_blocks;
        p.block_size = block_size;
        p.page_size = page_size;
        p.blocks_es = blocks_esize;
        p.len_es = len_esize;
        p.rows_es = rows_esize;
        p.table_es = table_esize;
        p.vec = vector_width({reinterpret_cast<uint64_t>(k_cache), reinterpret_cast<uint64_t>(v_cache),
                              reinterpret_cast<uint64_t>(k_shadow), reinterpret_cast<uint64_t>(v_shadow),
                              static_cast<uint64_t>(k_cache_stride), static_cast<uint64_t>(v_cache_stride),
                              static_cast<uint64_t>(k_shadow_stride), static_cast<uint64_t>(v_shadow_stride),
                              static_cast<uint64_t>(k_row_bytes), static_cast<uint64_t>(v_row_bytes)});
        const auto cstream = static_cast<cudaStream_t>(stream);
        const int rows_grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(p.batch, 65535)));
        shadow_clean_kernel<<<rows_grid, kShadowThreads, 0, cstream>>>(p);
        check_launch("shadow_clean launch");
        const int64_t total = p.batch * n_blocks * block_size;
        if (total > 0) {
            // At least 16 tokens a warp, at most two resident blocks per SM.
            const int64_t wanted = (total + kShadowWarps * 16 - 1) / (kShadowWarps * 16);
            const int grid = static_cast<int>(std::min<int64_t>(wanted, static_cast<int64_t>(sm_count(device)) * 2));
            with_vector(p.vec, [&](auto v) {
                shadow_tokens_kernel<decltype(v)><<<grid, kShadowThreads, 0, cstream>>>(p);
            });
        }
        check_launch("shadow_check launch");
    });
}

extern "C" int ekv_shadow_check_complete(
    const void* logical, int logical_esize, const void* physical, int physical_esize, int64_t n,
    int64_t page_size, int64_t pool_size, int64_t capacity, const uint8_t* live_pages, int64_t live_len,
    const uint64_t* pool_k, const uint64_t* pool_v, const uint64_t* shadow_k, const uint64_t* shadow_v,
    const uint64_t* initialized, int n_layers, int64_t pool_k_stride, int64_t pool_v_stride,
    int64_t shadow_k_stride, int64_t shadow_v_stride, int64_t k_row_bytes, int64_t v_row_bytes, uint64_t* counts,
    int device, void* stream) {
    using namespace ekv;
    return guarded([&] {
        require(n >= 0 && page_size >= 1 && pool_size >= 0 && capacity >= 1, "invalid slot geometry");
        require(n_layers >= 0 && n_layers <= kShadowMaxLayers, "layer count outside [0, EKV_SHADOW_MAX_LAYERS]");
        require(k_row_bytes > 0 && v_row_bytes > 0 && k_row_bytes % 2 == 0 && v_row_bytes % 2 == 0,
                "row sizes must be positive multiples of 2 bytes (bf16 rows)");
        require(counts && live_pages && live_len >= 1, "null pointer argument");
        if (n == 0 || n_layers == 0) return;
        require(logical && physical && pool_k && pool_v && shadow_k && shadow_v && initialized,
                "null pointer argument");
        check_esize(logical_esize, "logical");
        check_esize(physical_esize, "physical");
        bind_device(device);
        CompleteParams p{};
        p.logical = logical;
        p.physical = physical;
        p.live = live_pages;
        p.counts = reinterpret_cast<unsigned long long*>(counts);
        p.n = n;
        p.page_size = page_size;
        p.pool_size = pool_size;
        p.capacity = capacity;
        p.live_len = live_len;
        p.pool_k_stride = pool_k_stride;
        p.pool_v_stride = pool_v_stride;
        p.shadow_k_stride = shadow_k_stride;
        p.shadow_v_stride = shadow_v_stride;
        p.k_row_bytes = k_row_bytes;
        p.v_row_bytes = v_row_bytes;
        p.logical_es = logical_esize;
        p.physical_es = physical_esize;
        p.n_layers = n_layers;
        uint64_t bits = static_cast<uint64_t>(pool_k_stride) | static_cast<uint64_t>(pool_v_stride) |
                        static_cast<uint64_t>(shadow_k_stride) | static_cast<uint64_t>(shadow_v_stride) |
                        static_cast<uint64_t>(k_row_bytes) | static_cast<uint64_t>(v_row_bytes);
        for (int l = 0; l < n_layers; ++l) {
            require(pool_k[l] && pool_v[l] && shadow_k[l] && shadow_v[l] && initialized[l], "null layer pointer");
            p.pool_k[l] = reinterpret_cast<const char*>(pool_k[l]);
            p.pool_v[l] = reinterpret_cast<const char*>(pool_v[l]);
            p.shadow_k[l] = reinterpret_cast<const char*>(shadow_k[l]);
            p.shadow_v[l] = reinterpret_cast<const char*>(shadow_v[l]);
            p.initialized[l] = reinterpret_cast<const uint8_t*>(initialized[l]);
            bits |= pool_k[l] | pool_v[l] | shadow_k[l] | shadow_v[l];
        }
        p.vec = vector_width({bits});
        p.tile = tokens_per_block(n * n_layers, device);
        const int64_t x = (n + p.tile - 1) / p.tile;
        require(x <= 0x7fffffff, "grid too large");
        const dim3 grid(static_cast<unsigned>(x), static_cast<unsigned>(std::min(n_layers, 65535)));
        with_vector(p.vec, [&](auto v) {
            shadow_complete_kernel<decltype(v)><<<grid, kShadowThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
        });
        check_launch("shadow_check_complete launch");
    });
}

extern "C" int ekv_shadow_write(
    void* k_shadow, void* v_shadow, uint8_t* initialized, int64_t capacity, int64_t k_shadow_stride,
    int64_t v_shadow_stride, const void* key, const void* value, int64_t key_stride, int64_t value_stride,
    int64_t k_row_bytes, int64_t v_row_bytes, const void* locations, int loc_esize, int64_t n, int device,
    void* stream) {
    using namespace ekv;
    return guarded([&] {
        require(n >= 0 && capacity >= 1, "invalid shadow geometry");
        require(k_row_bytes > 0 && v_row_bytes > 0 && k_row_bytes % 2 == 0 && v_row_bytes % 2 == 0,
                "row sizes must be positive multiples of 2 bytes (bf16 rows)");
        if (n == 0) return;
        require(k_shadow && v_shadow && initialized && key && value && locations, "null pointer argument");
        check_esize(loc_esize, "locations");
        bind_device(device);
        WriteParams p{};
        p.k_shadow = static_cast<char*>(k_shadow);
        p.v_shadow = static_cast<char*>(v_shadow);
        p.initialized = initialized;
        p.key = static_cast<const char*>(key);
        p.value = static_cast<const char*>(value);
        p.locations = locations;
        p.n = n;
        p.capacity = capacity;
        p.k_shadow_stride = k_shadow_stride;
        p.v_shadow_stride = v_shadow_stride;
        p.key_stride = key_stride;
        p.value_stride = value_stride;
        p.k_row_bytes = k_row_bytes;
        p.v_row_bytes = v_row_bytes;
        p.loc_es = loc_esize;
        p.vec = vector_width({reinterpret_cast<uint64_t>(k_shadow), reinterpret_cast<uint64_t>(v_shadow),
                              reinterpret_cast<uint64_t>(key), reinterpret_cast<uint64_t>(value),
                              static_cast<uint64_t>(k_shadow_stride), static_cast<uint64_t>(v_shadow_stride),
                              static_cast<uint64_t>(key_stride), static_cast<uint64_t>(value_stride),
                              static_cast<uint64_t>(k_row_bytes), static_cast<uint64_t>(v_row_bytes)});
        with_vector(p.vec, [&](auto v) {
            shadow_write_kernel<decltype(v)><<<grid_for(n, kShadowWarps, device), kShadowThreads, 0,
                                               static_cast<cudaStream_t>(stream)>>>(p);
        });
        check_launch("shadow_write launch");
    });
}

extern "C" int ekv_shadow_reset(
    const uint64_t* initialized, int n_layers, int64_t capacity, const void* locations, int loc_esize, int64_t n,
    int device, void* stream) {
    using namespace ekv;
    return guarded([&] {
        require(n_layers >= 0 && n_layers <= kShadowMaxLayers, "layer count outside [0, EKV_SHADOW_MAX_LAYERS]");
        require(n >= 0 && capacity >= 1, "invalid shadow geometry");
        if (n == 0 || n_layers == 0) return;
        require(initialized && locations, "null pointer argument");
        check_esize(loc_esize, "locations");
        bind_device(device);
        ResetParams p{};
        p.locations = locations;
        p.n = n;
        p.capacity = capacity;
        p.loc_es = loc_esize;
        p.n_layers = n_layers;
        for (int l = 0; l < n_layers; ++l) {
            require(initialized[l], "null layer pointer");
            p.initialized[l] = reinterpret_cast<uint8_t*>(initialized[l]);
        }
        shadow_reset_kernel<<<grid_for(n, kShadowThreads, device), kShadowThreads, 0,
                              static_cast<cudaStream_t>(stream)>>>(p);
        check_launch("shadow_reset launch");
    });
}
