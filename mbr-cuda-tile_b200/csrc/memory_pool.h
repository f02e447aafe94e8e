// memory_pool.h — caching device allocator behind the Tensor API.
//
// Mirrors the reference interface of src/memory_pool.h:21-190
// (CudaMemoryPool::instance / allocate / deallocate / trim_cached_memory /
// release_all / get_stats / print_stats): size-bucketed free lists, requests
// rounded up (512 B below 1 MB, 2 MB below 10 MB, 20 MB above), a cached block
// is reused for requests up to half its size, and a failed cudaMalloc retries
// once after releasing the cache.  Per-device free lists (the reference keeps
// one device); thread-safe.
#pragma once

#include <stddef.h>

#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace cudasep {

class __attribute__((visibility("default"))) CudaMemoryPool {
public:
    static CudaMemoryPool& instance();

    void* allocate(size_t requested_bytes);
    void deallocate(void* ptr);
    void trim_cached_memory();
    void release_all();

    struct Stats {
        size_t allocations = 0;
        size_t deallocations = 0;
        size_t cache_hits = 0;
        size_t total_allocated = 0;
        size_t total_freed = 0;
        size_t active_bytes = 0;
        size_t peak_bytes = 0;
    };
    Stats get_stats() const;
    size_t cached_bytes() const;
    void print_stats() const;

    static size_t round_up(size_t bytes);

private:
    CudaMemoryPool() = default;
    ~CudaMemoryPool();
    void release_cached_locked();

    struct Block {
        size_t size;
        int device;
    };
    mutable std::mutex mutex_;
    // (device, size) -> cached pointers
    std::map<std::pair<int, size_t>, std::vector<void*>> free_;
    std::unordered_map<void*, Block> live_;
    Stats stats_;
};

}  // namespace cudasep
