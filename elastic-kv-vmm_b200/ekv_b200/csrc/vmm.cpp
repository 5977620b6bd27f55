// Chunked CUDA virtual-memory backing (the ev_* ABI of include/ekv_vmm.h).
//
// One object owns one VA reservation on one device.  Chunks are committed with
// cuMemCreate + cuMemMap, made accessible with cuMemSetAccess and zero-filled
// before first use; they are returned with cuMemUnmap + cuMemRelease.  The
// entry points keep the reference's ABI (native/elastic_vmm.cpp:316-369) so its
// ctypes loader binds this library unchanged; the code is independent:
//   * driver functions are resolved through cudaGetDriverEntryPointByVersion,
//     so the library loads on hosts without libcuda (the CPU test suite);
//   * chunk state is a dense array indexed by chunk id (a 180 GB HBM pool in
//     2 MiB chunks is ~90k entries), not a tree;
//   * a commit is all-or-nothing: on failure, the chunks this call created are
//     unmapped and released again; if that cleanup (or the wait for the zero
//     fill) fails, the object is marked poisoned and refuses further changes.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <limits>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/ekv_vmm.h"

namespace {

thread_local std::string g_vmm_error;

// Driver entry points used by the backing, resolved once per process.
struct Driver {
    decltype(&::cuGetErrorString) get_error_string = nullptr;
    decltype(&::cuDeviceGet) device_get = nullptr;
    decltype(&::cuDeviceGetAttribute) device_get_attribute = nullptr;
    decltype(&::cuMemGetAllocationGranularity) granularity = nullptr;
    decltype(&::cuDevicePrimaryCtxRetain) primary_retain = nullptr;
    decltype(&::cuDevicePrimaryCtxRelease) primary_release = nullptr;
    decltype(&::cuCtxPushCurrent) ctx_push = nullptr;
    decltype(&::cuCtxPopCurrent) ctx_pop = nullptr;
    decltype(&::cuCtxSynchronize) ctx_synchronize = nullptr;
    decltype(&::cuMemAddressReserve) address_reserve = nullptr;
    decltype(&::cuMemAddressFree) address_free = nullptr;
    decltype(&::cuMemCreate) mem_create = nullptr;
    decltype(&::cuMemRelease) mem_release = nullptr;
    decltype(&::cuMemMap) mem_map = nullptr;
    decltype(&::cuMemUnmap) mem_unmap = nullptr;
    decltype(&::cuMemSetAccess) mem_set_access = nullptr;
    decltype(&::cuMemsetD8Async) memset_async = nullptr;
    decltype(&::cuStreamCreate) stream_create = nullptr;
    decltype(&::cuStreamDestroy) stream_destroy = nullptr;
    decltype(&::cuStreamSynchronize) stream_synchronize = nullptr;
};

template <class Fn>
void resolve(Fn& fn, const char* name) {
    void* address = nullptr;
    cudaDriverEntryPointQueryResult query = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t status =
        cudaGetDriverEntryPointByVersion(name, &address, 12000, cudaEnableDefault, &query);
    if (status != cudaSuccess || query != cudaDriverEntryPointSuccess || !address) {
        throw std::runtime_error(std::string("CUDA driver entry point unavailable: ") + name +
                                 (status != cudaSuccess ? std::string(" (") + cudaGetErrorString(status) + ")"
                                                        : std::string()));
    }
    fn = reinterpret_cast<Fn>(address);
}

const Driver& driver() {
    static std::once_flag once;
    static Driver table;
    static std::string failure;
    std::call_once(once, [] {
        try {
            Driver d;
            resolve(d.get_error_string, "cuGetErrorString");
            resolve(d.device_get, "cuDeviceGet");
            resolve(d.device_get_attribute, "cuDeviceGetAttribute");
            resolve(d.granularity, "cuMemGetAllocationGranularity");
            resolve(d.primary_retain, "cuDevicePrimaryCtxRetain");
            resolve(d.primary_release, "cuDevicePrimaryCtxRelease");
            resolve(d.ctx_push, "cuCtxPushCurrent");
            resolve(d.ctx_pop, "cuCtxPopCurrent");
            resolve(d.ctx_synchronize, "cuCtxSynchronize");
            resolve(d.address_reserve, "cuMemAddressReserve");
            resolve(d.address_free, "cuMemAddressFree");
            resolve(d.mem_create, "cuMemCreate");
            resolve(d.mem_release, "cuMemRelease");
            resolve(d.mem_map, "cuMemMap");
            resolve(d.mem_unmap, "cuMemUnmap");
            resolve(d.mem_set_access, "cuMemSetAccess");
            resolve(d.memset_async, "cuMemsetD8Async");
            resolve(d.stream_create, "cuStreamCreate");
            resolve(d.stream_destroy, "cuStreamDestroy");
            resolve(d.stream_synchronize, "cuStreamSynchronize");
            table = d;
        } catch (const std::exception& e) {
            failure = e.what();
        }
    });
    if (!failure.empty()) throw std::runtime_error(failure);
    return table;
}

void check(CUresult status, const char* what) {
    if (status == CUDA_SUCCESS) return;
    const char* text = nullptr;
    if (driver().get_error_string) driver().get_error_string(status, &text);
    throw std::runtime_error(std::string(what) + ": " + (text ? text : std::to_string(status)));
}

// Pushes a context for the lifetime of the object.
class ContextScope {
public:
    explicit ContextScope(CUcontext ctx) { check(driver().ctx_push(ctx), "push context"); }
    ~ContextScope() {
        CUcontext popped = nullptr;
        driver().ctx_pop(&popped);
    }
    ContextScope(const ContextScope&) = delete;
    ContextScope& operator=(const ContextScope&) = delete;
};

enum : uint8_t { kOwned = 1, kMapped = 2 };

constexpr uint64_t kMaxAccessRunBytes = uint64_t{512} << 20;  // see Reservation::commit

class Reservation {
public:
    Reservation(int ordinal, uint64_t capacity_bytes, uint64_t chunk_bytes) {
        if (!capacity_bytes || !chunk_bytes) {
            throw std::invalid_argument("capacity and chunk size must be positive");
        }
        const Driver& d = driver();
        n_chunks_ = capacity_bytes / chunk_bytes + (capacity_bytes % chunk_bytes ? 1 : 0);
        if (n_chunks_ > std::numeric_limits<uint64_t>::max() / chunk_bytes) {
            throw std::invalid_argument("aligned capacity overflows 64 bits");
        }
        chunk_bytes_ = chunk_bytes;
        reserved_ = n_chunks_ * chunk_bytes;
        check(d.device_get(&device_, ordinal), "cuDeviceGet");
        int vmm = 0;
        check(d.device_get_attribute(&vmm, CU_DEVICE_ATTRIBUTE_VIRTUAL_MEMORY_MANAGEMENT_SUPPORTED, device_),
              "query VMM support");
        if (!vmm) throw std::runtime_error("device does not support CUDA virtual memory management");
        prop_.type = CU_MEM_ALLOCATION_TYPE_PINNED;
        prop_.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        prop_.location.id = device_;
        size_t granularity = 0;
        check(d.granularity(&granularity, &prop_, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
              "cuMemGetAllocationGranularity");
        granularity_ = granularity;
        if (chunk_bytes % granularity_) {
            throw std::invalid_argument("chunk_bytes must be a multiple of the VMM granularity " +
                                        std::to_string(granularity_));
        }
        check(d.primary_retain(&context_, device_), "retain primary context");
        try {
            ContextScope scope(context_);
            check(d.address_reserve(&base_, reserved_, granularity_, 0, 0), "reserve virtual range");
            check(d.stream_create(&zero_stream_, CU_STREAM_NON_BLOCKING), "create zero-fill stream");
        } catch (...) {
            close();
            throw;
        }
        state_.assign(n_chunks_, 0);
        handles_.assign(n_chunks_, CUmemGenericAllocationHandle{});
    }

    ~Reservation() { close(); }

    // Map and zero the listed chunks that are not mapped yet.
    void commit(const uint64_t* ids, size_t count, bool wait) {
        const std::vector<uint64_t> fresh = pending(ids, count, false);
        if (fresh.empty()) {
            if (wait) finish_zero_fill();
            return;
        }
        const Driver& d = driver();
        ContextScope scope(context_);
        size_t created = 0;
        try {
            for (const uint64_t id : fresh) {
                ++created;
                if (!spare_.empty()) {
                    // A handle kept by an earlier decommit: no cuMemCreate.
                    handles_[id] = spare_.back();
                    spare_.pop_back();
                } else {
                    check(d.mem_create(&handles_[id], chunk_bytes_, &prop_, 0), "cuMemCreate");
                }
                state_[id] |= kOwned;
                committed_ += 1;
                check(d.mem_map(address(id), chunk_bytes_, 0, handles_[id], 0), "cuMemMap");
                state_[id] |= kMapped;
            }
            CUmemAccessDesc access{};
            access.location = prop_.location;
            access.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
            // Access rights and zero fill go per run of consecutive chunk ids, a run
            // capped at kMaxAccessRunBytes: measured on B200 (driver 580), the first
            // cuMemUnmap / cuMemRelease of chunks inside one 36 GiB access range cost
            // 3.5x their later price (82 + 82 ms for 256 chunks against 23 + 23 ms),
            // inside ranges of 512 MiB nothing extra; a call's price scales with the
            // physical allocations it covers, so capping the run costs nothing.
            const size_t max_run = kMaxAccessRunBytes / chunk_bytes_ > 0 ? kMaxAccessRunBytes / chunk_bytes_ : 1;
            size_t run = 0;
            while (run < fresh.size()) {
                size_t end = run + 1;
                while (end < fresh.size() && fresh[end] == fresh[end - 1] + 1 && end - run < max_run) ++end;
                const size_t bytes = (end - run) * chunk_bytes_;
                check(d.mem_set_access(address(fresh[run]), bytes, &access, 1), "cuMemSetAccess");
                check(d.memset_async(address(fresh[run]), 0, bytes, zero_stream_), "zero new chunks");
                zero_pending_ = true;
                run = end;
            }
            if (wait) finish_zero_fill();
        } catch (...) {
            // The zero fill may still be writing into these chunks: only undo
            // them once it is known to be finished.
            if (zero_pending_ && d.stream_synchronize(zero_stream_) != CUDA_SUCCESS) {
                poisoned_ = true;
                throw;
            }
            zero_pending_ = false;
            for (size_t i = 0; i < created; ++i) {
                if (release(fresh[i]) != CUDA_SUCCESS) poisoned_ = true;
            }
            throw;
        }
    }

    // Unmap and release the listed chunks that are mapped.  Each run of
    // consecutive chunk ids is unmapped with one call (measured on B200: ~90 us
    // per 2 MiB chunk instead of ~200 us chunk by chunk), then every handle is
    // released -- or, while fewer than spare_limit_ handles are kept, kept for
    // the next commit (cuMemRelease + cuMemCreate cost ~300 us per chunk).
    void decommit(const uint64_t* ids, size_t count) {
        const std::vector<uint64_t> mapped = pending(ids, count, true);
        if (mapped.empty()) return;
        const Driver& d = driver();
        ContextScope scope(context_);
        finish_zero_fill();
        size_t run = 0;
        while (run < mapped.size()) {
            size_t end = run + 1;
            while (end < mapped.size() && mapped[end] == mapped[end - 1] + 1) ++end;
            const CUresult status = d.mem_unmap(address(mapped[run]), (end - run) * chunk_bytes_);
            if (status != CUDA_SUCCESS) {
                poisoned_ = true;  // which mappings of the run are gone is unknown
                check(status, "unmap chunks");
            }
            for (size_t i = run; i < end; ++i) state_[mapped[i]] &= static_cast<uint8_t>(~kMapped);
            run = end;
        }
        for (const uint64_t id : mapped) {
            if (spare_.size() < spare_limit_ && (state_[id] & kOwned)) {
                spare_.push_back(handles_[id]);
                state_[id] &= static_cast<uint8_t>(~kOwned);
                committed_ -= 1;
                continue;
            }
            const CUresult status = release(id);
            if (status != CUDA_SUCCESS) {
                poisoned_ = true;  // earlier chunks of this call are already gone
                check(status, "release chunk");
            }
        }
    }

    // Keep at most `limit` unmapped physical handles for reuse; release the rest.
    void set_spare_limit(uint64_t limit) {
        if (poisoned_) throw std::runtime_error("backing is poisoned after a partial CUDA failure");
        spare_limit_ = limit;
        if (spare_.size() <= limit) return;
        const Driver& d = driver();
        ContextScope scope(context_);
        while (spare_.size() > limit) {
            const CUresult status = d.mem_release(spare_.back());
            if (status != CUDA_SUCCESS) {
                poisoned_ = true;
                check(status, "release spare chunk");
            }
            spare_.pop_back();
        }
    }

    uint64_t spare() const { return static_cast<uint64_t>(spare_.size()) * chunk_bytes_; }

    CUresult close() noexcept {
        if (!context_) return CUDA_SUCCESS;
        const Driver& d = driver();
        CUresult first = d.ctx_push(context_);
        auto keep = [&first](CUresult status) {
            if (first == CUDA_SUCCESS && status != CUDA_SUCCESS) first = status;
        };
        if (first == CUDA_SUCCESS) {
            keep(d.ctx_synchronize());
            for (uint64_t id = 0; id < state_.size(); ++id) {
                if (state_[id]) keep(release(id));
            }
            for (const CUmemGenericAllocationHandle spare : spare_) keep(d.mem_release(spare));
            spare_.clear();
            if (base_) {
                keep(d.address_free(base_, reserved_));
                base_ = 0;
            }
            if (zero_stream_) {
                keep(d.stream_destroy(zero_stream_));
                zero_stream_ = nullptr;
            }
            CUcontext popped = nullptr;
            keep(d.ctx_pop(&popped));
        }
        keep(d.primary_release(device_));
        context_ = nullptr;
        return first;
    }

    uint64_t base() const { return base_; }
    uint64_t reserved() const { return reserved_; }
    uint64_t granularity() const { return granularity_; }
    uint64_t backed() const { return committed_ * chunk_bytes_; }
    bool poisoned() const { return poisoned_; }

private:
    CUdeviceptr address(uint64_t id) const { return base_ + id * chunk_bytes_; }

    void finish_zero_fill() {
        if (!zero_pending_) return;
        check(driver().stream_synchronize(zero_stream_), "wait for chunk zero fill");
        zero_pending_ = false;
    }

    // Sorted, de-duplicated ids whose mapped state equals `mapped`.
    std::vector<uint64_t> pending(const uint64_t* ids, size_t count, bool mapped) const {
        if (poisoned_) throw std::runtime_error("backing is poisoned after a partial CUDA failure");
        if (count && !ids) throw std::invalid_argument("chunk index array is null");
        std::vector<uint64_t> out;
        out.reserve(count);
        for (size_t i = 0; i < count; ++i) {
            if (ids[i] >= n_chunks_) throw std::out_of_range("chunk index outside reserved range");
            if (((state_[ids[i]] & kMapped) != 0) == mapped) out.push_back(ids[i]);
        }
        std::sort(out.begin(), out.end());
        out.erase(std::unique(out.begin(), out.end()), out.end());
        return out;
    }

    // Undo whatever of (create, map) happened for chunk `id`.
    CUresult release(uint64_t id) noexcept {
        const Driver& d = driver();
        if (state_[id] & kMapped) {
            const CUresult status = d.mem_unmap(address(id), chunk_bytes_);
            if (status != CUDA_SUCCESS) return status;
            state_[id] &= static_cast<uint8_t>(~kMapped);
        }
        if (state_[id] & kOwned) {
            const CUresult status = d.mem_release(handles_[id]);
            if (status != CUDA_SUCCESS) return status;
            state_[id] &= static_cast<uint8_t>(~kOwned);
            committed_ -= 1;
        }
        return CUDA_SUCCESS;
    }

    CUcontext context_ = nullptr;
    CUdevice device_ = 0;
    CUdeviceptr base_ = 0;
    CUstream zero_stream_ = nullptr;
    CUmemAllocationProp prop_{};
    uint64_t n_chunks_ = 0;
    uint64_t chunk_bytes_ = 0;
    uint64_t reserved_ = 0;
    uint64_t granularity_ = 0;
    uint64_t committed_ = 0;
    bool zero_pending_ = false;
    bool poisoned_ = false;
    std::vector<uint8_t> state_;
    std::vector<CUmemGenericAllocationHandle> handles_;
    std::vector<CUmemGenericAllocationHandle> spare_;  // unmapped handles kept for reuse
    uint64_t spare_limit_ = 0;
};

Reservation& handle_of(void* handle) {
    if (!handle) throw std::invalid_argument("null backing handle");
    return *static_cast<Reservation*>(handle);
}

template <class Result, class Body>
Result run(Result on_error, Body&& body) {
    try {
        g_vmm_error.clear();
        return body();
    } catch (const std::exception& e) {
        g_vmm_error = e.what();
    } catch (...) {
        g_vmm_error = "unknown C++ error";
    }
    return on_error;
}

constexpr uint64_t kInvalid = std::numeric_limits<uint64_t>::max();

}  // namespace

extern "C" {

void* ev_create(int device, uint64_t capacity_bytes, uint64_t chunk_bytes) {
    return run<void*>(nullptr, [&] {
        auto owner = std::make_unique<Reservation>(device, capacity_bytes, chunk_bytes);
        return static_cast<void*>(owner.release());
    });
}

int ev_ensure(void* handle, const uint64_t* indices, size_t count) {
    return run(-1, [&] {
        handle_of(handle).commit(indices, count, true);
        return 0;
    });
}

int ev_precommit(void* handle, const uint64_t* indices, size_t count) {
    return run(-1, [&] {
        handle_of(handle).commit(indices, count, false);
        return 0;
    });
}

int ev_drop(void* handle, const uint64_t* indices, size_t count) {
    return run(-1, [&] {
        handle_of(handle).decommit(indices, count);
        return 0;
    });
}

uint64_t ev_base(void* handle) { return run(kInvalid, [&] { return handle_of(handle).base(); }); }
uint64_t ev_backed(void* handle) { return run(kInvalid, [&] { return handle_of(handle).backed(); }); }
uint64_t ev_reserved(void* handle) { return run(kInvalid, [&] { return handle_of(handle).reserved(); }); }
uint64_t ev_granularity(void* handle) {
    return run(kInvalid, [&] { return handle_of(handle).granularity(); });
}

int ev_set_spare(void* handle, uint64_t chunks) {
    return run(-1, [&] {
        handle_of(handle).set_spare_limit(chunks);
        return 0;
    });
}

uint64_t ev_spare(void* handle) { return run(kInvalid, [&] { return handle_of(handle).spare(); }); }

int ev_poisoned(void* handle) {
    return run(-1, [&] { return handle_of(handle).poisoned() ? 1 : 0; });
}

const char* ev_error(void) { return g_vmm_error.c_str(); }

int ev_close(void* handle) {
    return run(-1, [&] {
        std::unique_ptr<Reservation> owner(static_cast<Reservation*>(handle));
        if (owner) check(owner->close(), "close backing");
        return 0;
    });
}

}  // extern "C"
