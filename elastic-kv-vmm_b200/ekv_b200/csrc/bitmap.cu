// Page -> chunk projection counts and the freeable-chunk bitmap (R4 / R6).
//
// A physical page of `page_size` token slots lives in every K/V plane; plane p
// starts at chunk plane_chunk[p] and holds rows of plane_row_bytes[p] bytes, so
// page g covers the byte range [g*page_size*row, (g+1)*page_size*row) of the
// plane and the chunks under it (PhysicalPages.chunks,
// adaptive_sparse/minimax_vmm.py:40-52).  A set of candidate pages frees chunk
// c iff it holds every reference to c and c is mapped
// (_releasable_counts, adaptive_sparse/scheduler_budget.py:159-162).
//
// chunk_counts is a histogram: tasks run plane-major so that the lanes of a
// warp walk consecutive pages of one plane (usually the same chunk); lanes that
// hit the same chunk are merged with __match_any_sync before one atomic, and
// when the chunk table fits in shared memory each block accumulates a private
// histogram there and flushes its non-zero bins once.  The bitmap is built with
// warp ballots (32 chunks per ballot, two ballots per 64-bit word).
#include <atomic>
#include <vector>

#include "common.cuh"

namespace ekv {
namespace {

struct CountParams {
    const void* pages;
    int32_t* counts;
    int32_t* overflow;
    int64_t n_pages, page_size, chunk_bytes, n_chunks;
    int pages_es, n_planes;
    int64_t plane_chunk[EKV_MAX_PLANES];
    int64_t plane_row_bytes[EKV_MAX_PLANES];
};

constexpr int kCountThreads = 512;
constexpr int64_t kSharedChunkLimit = 48 * 1024;  // 192 KiB of int32 bins

// Add `amount` to bin `chunk`, merging lanes of the warp that target the same
// bin.  All 32 lanes must call it (inactive lanes pass chunk = -1).
template <bool kShared>
__device__ __forceinline__ void add_bin(int32_t* bins, int64_t chunk, unsigned lane) {
    const unsigned peers = __match_any_sync(0xffffffffu, static_cast<unsigned long long>(chunk));
    const unsigned leader = __ffs(peers) - 1;
    if (chunk >= 0 && lane == leader) {
        atomicAdd(bins + chunk, __popc(peers));
    }
}

template <bool kShared>
__global__ void __launch_bounds__(kCountThreads)
chunk_count_kernel(const __grid_constant__ CountParams p) {
    extern __shared__ int32_t shared_bins[];
    int32_t* bins = kShared ? shared_bins : p.counts;
    if (kShared) {
        for (int64_t c = threadIdx.x; c < p.n_chunks; c += kCountThreads) shared_bins[c] = 0;
        __syncthreads();
    }
    const unsigned lane = lane_id();
    const int64_t total = p.n_pages * p.n_planes;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kCountThreads;
    // Round the loop bound up to a whole warp so every lane reaches the match.
    const int64_t bound = (total + 31) & ~int64_t{31};
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kCountThreads + threadIdx.x; t < bound;
         t += stride) {
        int64_t first = -1, last = -2;
        int64_t plane_base = 0;
        if (t < total) {
            const int64_t plane = t / p.n_pages;
            const int64_t page = load_index(p.pages, p.pages_es, t - plane * p.n_pages);
            const int64_t span = p.page_size * p.plane_row_bytes[plane];
            const int64_t begin = page * span;
            plane_base = p.plane_chunk[plane];
            first = plane_base + begin / p.chunk_bytes;
            last = plane_base + (begin + span - 1) / p.chunk_bytes;
        }
        // A page spans one chunk unless it crosses a boundary; walk the span
        // in lock step so the match stays warp-wide.
        int64_t steps = last - first + 1;
        int64_t max_steps = steps;
        for (int offset = 16; offset > 0; offset >>= 1) {
            const int64_t other = __shfl_xor_sync(0xffffffffu, max_steps, offset);
            max_steps = other > max_steps ? other : max_steps;
        }
        for (int64_t s = 0; s < max_steps; ++s) {
            int64_t chunk = -1;
            if (s < steps) {
                chunk = first + s;
                if (chunk < 0 || chunk >= p.n_chunks) {
                    if (p.overflow) atomicAdd(p.overflow, 1);
                    chunk = -1;
                }
            }
            add_bin<kShared>(bins, chunk, lane);
        }
    }
    if (kShared) {
        __syncthreads();
        for (int64_t c = threadIdx.x; c < p.n_chunks; c += kCountThreads) {
            const int32_t v = shared_bins[c];
            if (v) atomicAdd(p.counts + c, v);
        }
    }
}

// Planes with the same row size map page g to the same chunk offsets relative
// to their first chunk, so one histogram of relative chunk offsets over the
// pages serves the whole group: block-private in shared memory (bin n_chunks
// collects offsets past the table, which are past it for every plane), then
// each non-zero bin is added to every plane of the group at that plane's first
// chunk.  Work: n_pages histogram updates + (non-zero bins x planes) atomics,
// instead of n_pages x planes.  Same counts and overflow as the per-plane
// kernel; a negative page (offset < 0) takes the per-plane path inline.
struct GroupParams {
    const void* pages;
    int32_t* counts;
    int32_t* overflow;
    int64_t n_pages, page_size, chunk_bytes, n_chunks, row_bytes;
    int pages_es, n_planes;
    int64_t plane_chunk[EKV_MAX_PLANES];
};

__global__ void __launch_bounds__(kCountThreads)
grouped_count_kernel(const __grid_constant__ GroupParams p) {
    extern __shared__ int32_t bins[];  // n_chunks + 1
    for (int64_t c = threadIdx.x; c <= p.n_chunks; c += kCountThreads) bins[c] = 0;
    __syncthreads();
    const unsigned lane = lane_id();
    const int64_t span = p.page_size * p.row_bytes;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kCountThreads;
    const int64_t bound = (p.n_pages + 31) & ~int64_t{31};
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kCountThreads + threadIdx.x; t < bound; t += stride) {
        int64_t first = 0, last = -1;
        if (t < p.n_pages) {
            const int64_t begin = load_index(p.pages, p.pages_es, t) * span;
            // Truncating division, exactly as the per-plane kernel computes it.
            first = begin / p.chunk_bytes;
            last = (begin + span - 1) / p.chunk_bytes;
        }
        const int64_t steps = last - first + 1;
        int64_t max_steps = steps;
        for (int offset = 16; offset > 0; offset >>= 1) {
            const int64_t other = __shfl_xor_sync(0xffffffffu, max_steps, offset);
            max_steps = other > max_steps ? other : max_steps;
        }
        for (int64_t s = 0; s < max_steps; ++s) {
            int64_t bin = -1;
            if (s < steps) {
                const int64_t rel = first + s;
                if (rel < 0) {
                    // Rare: a negative page.  Resolve it plane by plane, as the per-plane kernel does.
                    for (int q = 0; q < p.n_planes; ++q) {
                        const int64_t chunk = p.plane_chunk[q] + rel;
                        if (chunk >= 0 && chunk < p.n_chunks) {
                            atomicAdd(p.counts + chunk, 1);
                        } else if (p.overflow) {
                            atomicAdd(p.overflow, 1);
                        }
                    }
                } else {
                    bin = rel < p.n_chunks ? rel : p.n_chunks;
                }
            }
            add_bin<true>(bins, bin, lane);
        }
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c <= p.n_chunks; c += kCountThreads) {
        const int32_t v = bins[c];
        if (!v) continue;
        if (c == p.n_chunks) {
            if (p.overflow) atomicAdd(p.overflow, v * p.n_planes);
            continue;
        }
        for (int q = 0; q < p.n_planes; ++q) {
            const int64_t chunk = p.plane_chunk[q] + c;
            if (chunk < p.n_chunks) {
                atomicAdd(p.counts + chunk, v);
            } else if (p.overflow) {
                atomicAdd(p.overflow, v);
            }
        }
    }
}

constexpr int kBitmapThreads = 256;

__global__ void __launch_bounds__(kBitmapThreads)
freeable_kernel(const int32_t* __restrict__ counts, const int32_t* __restrict__ refs,
                const uint64_t* __restrict__ mapped, int64_t n_chunks, uint64_t* __restrict__ out) {
    const unsigned lane = lane_id();
    const int64_t n_words = (n_chunks + 63) / 64;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (kBitmapThreads / 32);
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (kBitmapThreads / 32) + (threadIdx.x >> 5);
         w < n_words; w += warps) {
        unsigned half[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int64_t c = w * 64 + h * 32 + lane;
            bool freeable = false;
            if (c < n_chunks) {
                const int32_t count = counts[c];
                freeable = count > 0 && count == refs[c];
            }
            half[h] = __ballot_sync(0xffffffffu, freeable);
        }
        if (lane == 0) {
            out[w] = ((static_cast<uint64_t>(half[1]) << 32) | half[0]) & mapped[w];
        }
    }
}

__global__ void __launch_bounds__(kBitmapThreads)
and_kernel(const uint64_t* __restrict__ gathered, int n_ranks, int64_t n_words,
           uint64_t* __restrict__ out) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kBitmapThreads;
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * kBitmapThreads + threadIdx.x; w < n_words;
         w += stride) {
        uint64_t acc = ~uint64_t{0};
        for (int r = 0; r < n_ranks; ++r) acc &= gathered[static_cast<int64_t>(r) * n_words + w];
        out[w] = acc;
    }
}

unsigned small_grid(int device, int64_t items, int per_block) {
    const int64_t needed = (items + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(sm_count(device)) * 4;
    return static_cast<unsigned>(needed < cap ? (needed > 0 ? needed : 1) : cap);
}

}  // namespace
}  // namespace ekv

using namespace ekv;

extern "C" int ekv_chunk_counts(
    const void* pages, int pages_esize, int64_t n_pages,
    const int64_t* plane_chunk, const int64_t* plane_row_bytes, int n_planes,
    int64_t page_size, int64_t chunk_bytes,
    int32_t* counts, int64_t n_chunks, int accumulate, int32_t* overflow,
    int device, void* stream) {
    return guarded([&] {
        require(n_pages >= 0 && n_chunks >= 0, "sizes must be non-negative");
        require(page_size > 0 && chunk_bytes > 0, "page_size and chunk_bytes must be positive");
        require(n_planes >= 1 && n_planes <= EKV_MAX_PLANES, "plane count outside [1, EKV_MAX_PLANES]");
        require(plane_chunk && plane_row_bytes, "null plane table");
        if (!n_chunks) return;
        require(counts, "null counts");
        bind_device(device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (!accumulate) {
            cuda_check(cudaMemsetAsync(counts, 0, static_cast<size_t>(n_chunks) * sizeof(int32_t), s),
                       "clear counts");
        }
        if (!n_pages) return;
        require(pages, "null pages");
        check_esize(pages_esize, "pages");
        CountParams p{};
        p.pages = pages;
        p.counts = counts;
        p.overflow = overflow;
        p.n_pages = n_pages;
        p.page_size = page_size;
        p.chunk_bytes = chunk_bytes;
        p.n_chunks = n_chunks;
        p.pages_es = pages_esize;
        p.n_planes = n_planes;
        for (int i = 0; i < n_planes; ++i) {
            require(plane_row_bytes[i] > 0 && plane_chunk[i] >= 0, "invalid plane geometry");
            p.plane_chunk[i] = plane_chunk[i];
            p.plane_row_bytes[i] = plane_row_bytes[i];
        }
        // Planes sharing a row size (usually all K and V planes) go through the
        // grouped histogram when the chunk table fits in shared memory.
        std::vector<char> grouped(n_planes, 0);
        if (n_chunks < kSharedChunkLimit) {
            static std::atomic<bool> grouped_configured[64];  // per device; a race configures twice
            if (device >= 64 || !grouped_configured[device].load(std::memory_order_relaxed)) {
                cuda_check(cudaFuncSetAttribute(grouped_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kSharedChunkLimit * sizeof(int32_t))),
                           "configure grouped histogram");
                if (device < 64) grouped_configured[device].store(true, std::memory_order_relaxed);
            }
            for (int i = 0; i < n_planes; ++i) {
                if (grouped[i]) continue;
                GroupParams g{};
                g.pages = pages;
                g.counts = counts;
                g.overflow = overflow;
                g.n_pages = n_pages;
                g.page_size = page_size;
                g.chunk_bytes = chunk_bytes;
                g.n_chunks = n_chunks;
                g.row_bytes = plane_row_bytes[i];
                g.pages_es = pages_esize;
                for (int j = i; j < n_planes; ++j) {
                    if (plane_row_bytes[j] == plane_row_bytes[i]) g.plane_chunk[g.n_planes++] = plane_chunk[j];
                }
                if (g.n_planes < 2) continue;  // a lone plane: the per-plane kernel below
                for (int j = i; j < n_planes; ++j) {
                    if (plane_row_bytes[j] == plane_row_bytes[i]) grouped[j] = 1;
                }
                const int64_t needed = (n_pages + kCountThreads - 1) / kCountThreads;
                const int64_t cap = sm_count(device);
                const unsigned grid = static_cast<unsigned>(needed < cap ? needed : cap);
                const size_t smem = static_cast<size_t>(n_chunks + 1) * sizeof(int32_t);
                grouped_count_kernel<<<grid, kCountThreads, smem, s>>>(g);
                check_launch("grouped chunk_counts launch");
            }
            int rest = 0;
            for (int i = 0; i < n_planes; ++i) {
                if (!grouped[i]) {
                    p.plane_chunk[rest] = plane_chunk[i];
                    p.plane_row_bytes[rest] = plane_row_bytes[i];
                    ++rest;
                }
            }
            if (!rest) return;
            p.n_planes = rest;
        }
        const int64_t tasks = n_pages * p.n_planes;
        if (n_chunks <= kSharedChunkLimit) {
            const size_t smem = static_cast<size_t>(n_chunks) * sizeof(int32_t);
            static std::atomic<bool> configured[64];  // per device; a race configures twice
            if (device >= 64 || !configured[device].load(std::memory_order_relaxed)) {
                cuda_check(cudaFuncSetAttribute(chunk_count_kernel<true>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(kSharedChunkLimit * sizeof(int32_t))),
                           "configure shared histogram");
                if (device < 64) configured[device].store(true, std::memory_order_relaxed);
            }
            // Few blocks: each one pays a full-table flush.
            const int64_t needed = (tasks + kCountThreads - 1) / kCountThreads;
            const int64_t cap = sm_count(device);
            const unsigned grid = static_cast<unsigned>(needed < cap ? needed : cap);
            chunk_count_kernel<true><<<grid, kCountThreads, smem, s>>>(p);
        } else {
            const unsigned grid = small_grid(device, tasks, kCountThreads);
            chunk_count_kernel<false><<<grid, kCountThreads, 0, s>>>(p);
        }
        check_launch("chunk_counts launch");
    });
}

extern "C" int ekv_freeable_bitmap(
    const int32_t* counts, const int32_t* refs, const uint64_t* mapped_bits,
    int64_t n_chunks, uint64_t* out_bits, int device, void* stream) {
    return guarded([&] {
        require(n_chunks >= 0, "n_chunks must be non-negative");
        if (!n_chunks) return;
        require(counts && refs && mapped_bits && out_bits, "null pointer argument");
        bind_device(device);
        const int64_t words = (n_chunks + 63) / 64;
        freeable_kernel<<<small_grid(device, words, kBitmapThreads / 32), kBitmapThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(counts, refs, mapped_bits, n_chunks,
                                                               out_bits);
        check_launch("freeable_bitmap launch");
    });
}

extern "C" int ekv_bitmap_and(
    const uint64_t* gathered, int n_ranks, int64_t n_words, uint64_t* out,
    int device, void* stream) {
    return guarded([&] {
        require(n_ranks >= 1 && n_words >= 0, "need at least one rank and non-negative words");
        if (!n_words) return;
        require(gathered && out, "null pointer argument");
        bind_device(device);
        and_kernel<<<small_grid(device, n_words, kBitmapThreads), kBitmapThreads, 0,
                     static_cast<cudaStream_t>(stream)>>>(gathered, n_ranks, n_words, out);
        check_launch("bitmap_and launch");
    });
}

// ---------------------------------------------------------------- fused build + cross-rank AND over peer memory
//
// The joint-demotion decision is a compute step (this rank's freeable bitmap)
// followed by a collective (AND over the tensor-parallel ranks).  Instead of an
// NCCL all-gather and a second kernel, one single-block kernel per rank:
//   1. builds its bitmap and writes it into its own peer-visible buffer (slot
//      epoch & 1: a rank can be at most one call ahead of another, so two
//      slots never collide);
//   2. publishes it with a system-scope release store of `epoch` into its flag
//      slot in every peer's buffer;
//   3. waits -- with a poll limit -- until every peer's flag in its own buffer
//      has reached `epoch` (acquire loads);
//   4. ANDs the peers' words, read straight from their memory over NVLink.
// A wait that runs out sets *status and leaves `out` unwritten; the kernel
// never hangs.  Buffer layout per rank: 64 uint32 flags (256 B), then two
// slots of n_words uint64.  Plain peer loads and stores only.

namespace ekv {
namespace {

constexpr int kPeerMaxRanks = 64;
constexpr int kPeerFlagBytes = kPeerMaxRanks * 4;
constexpr int kPeerThreads = 256;

struct PeerParams {
    const int32_t* counts;
    const int32_t* refs;
    const uint64_t* mapped;
    const uint64_t* local_bits;
    uint64_t* out;
    uint64_t* local_out;
    uint32_t* status;
    int64_t n_chunks, n_words;
    int n_ranks, rank;
    uint32_t epoch, max_polls;
    char* buffers[kPeerMaxRanks];
};

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t load_relaxed_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kPeerThreads, 1)
freeable_and_peers_kernel(const __grid_constant__ PeerParams p) {
    __shared__ int failed;
    const unsigned lane = lane_id();
    const int warp = threadIdx.x >> 5;
    const int64_t slot_offset = static_cast<int64_t>(p.epoch & 1u) * p.n_words;
    uint64_t* mine = reinterpret_cast<uint64_t*>(p.buffers[p.rank] + kPeerFlagBytes) + slot_offset;
    if (threadIdx.x == 0) failed = 0;
    // 1. This rank's bitmap.
    if (p.local_bits) {
        for (int64_t w = threadIdx.x; w < p.n_words; w += kPeerThreads) mine[w] = p.local_bits[w];
    } else {
        for (int64_t w = warp; w < p.n_words; w += kPeerThreads / 32) {
            unsigned half[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t c = w * 64 + h * 32 + lane;
                bool freeable = false;
                if (c < p.n_chunks) {
                    const int32_t count = p.counts[c];
                    freeable = count > 0 && count == p.refs[c];
                }
                half[h] = __ballot_sync(0xffffffffu, freeable);
            }
            if (lane == 0) {
                const uint64_t word = ((static_cast<uint64_t>(half[1]) << 32) | half[0]) & p.mapped[w];
                mine[w] = word;
                if (p.local_out) p.local_out[w] = word;
            }
        }
    }
    __syncthreads();
    // 2. Publish (the release is cumulative over the block's writes ordered by the barrier).
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int r = 0; r < p.n_ranks; ++r) {
            if (r != p.rank) store_release_sys(reinterpret_cast<uint32_t*>(p.buffers[r]) + p.rank, p.epoch);
        }
    }
    // 3. Wait for every peer, with a poll limit.
    if (threadIdx.x < p.n_ranks && static_cast<int>(threadIdx.x) != p.rank) {
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(p.buffers[p.rank]) + threadIdx.x;
        bool arrived = false;
        for (uint32_t polls = 0; polls < p.max_polls; ++polls) {
            if (static_cast<int32_t>(load_acquire_sys(flag) - p.epoch) >= 0) {
                arrived = true;
                break;
            }
            __nanosleep(64);
        }
        if (!arrived) atomicExch(&failed, 1);
    }
    __syncthreads();
    if (failed) {
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, 1u);
        return;
    }
    // 4. AND over the ranks.
    for (int64_t w = threadIdx.x; w < p.n_words; w += kPeerThreads) {
        uint64_t acc = mine[w];
        for (int r = 0; r < p.n_ranks; ++r) {
            if (r == p.rank) continue;
            acc &= load_relaxed_sys(reinterpret_cast<const uint64_t*>(p.buffers[r] + kPeerFlagBytes) +
                                    slot_offset + w);
        }
        p.out[w] = acc;
    }
}

}  // namespace
}  // namespace ekv

extern "C" int ekv_freeable_and_peers(
    const int32_t* counts, const int32_t* refs, const uint64_t* mapped_bits, const uint64_t* local_bits,
    int64_t n_chunks, const uint64_t* peer_buffers, int n_ranks, int rank, uint32_t epoch,
    uint32_t max_polls, uint64_t* out, uint64_t* local_out, uint32_t* status, int device, void* stream) {
    return guarded([&] {
        require(n_chunks > 0, "n_chunks must be positive");
        require(n_ranks >= 1 && n_ranks <= kPeerMaxRanks, "rank count outside [1, 64]");
        require(rank >= 0 && rank < n_ranks, "rank outside [0, n_ranks)");
        require(peer_buffers && out, "null pointer argument");
        require(local_bits || (counts && refs && mapped_bits),
                "need either local_bits or counts, refs and mapped_bits");
        require(max_polls > 0, "max_polls must be positive");
        bind_device(device);
        PeerParams p{};
        p.counts = counts;
        p.refs = refs;
        p.mapped = mapped_bits;
        p.local_bits = local_bits;
        p.out = out;
        p.local_out = local_out;
        p.status = status;
        p.n_chunks = n_chunks;
        p.n_words = (n_chunks + 63) / 64;
        p.n_ranks = n_ranks;
        p.rank = rank;
        p.epoch = epoch;
        p.max_polls = max_polls;
        for (int r = 0; r < n_ranks; ++r) {
            require(peer_buffers[r] && peer_buffers[r] % 16 == 0, "peer buffers must be 16-byte aligned");
            p.buffers[r] = reinterpret_cast<char*>(peer_buffers[r]);
        }
        freeable_and_peers_kernel<<<1, kPeerThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
        check_launch("freeable_and_peers launch");
    });
}
