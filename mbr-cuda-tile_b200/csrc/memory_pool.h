// memory_pool.h — stream-ordered caching device allocator behind the Tensor API.
//
// Mirrors the reference interface of src/memory_pool.h:21-190
// (CudaMemoryPool::instance / allocate / deallocate / trim_cached_memory /
// release_all / get_stats / print_stats): size-bucketed free lists, requests
// rounded up (512 B below 1 MB, 2 MB below 10 MB, 20 MB above), a cached block
// is reused for requests up to half its size, and a failed cudaMalloc retries
// once after releasing the cache.  Per-device free lists (the reference keeps
// one device); thread-safe.
//
// Stream order (the reference's pool has none: its tensors all run on the
// legacy default stream): a block freed with deallocate(p, stream) is tagged
// with that stream and an event recorded on it.  allocate(bytes, stream)
// prefers a block freed on the same stream, which is reusable at once since
// every later use on that stream runs after the free; a block freed on another
// stream is handed out after `stream` is made to wait on its event
// (cudaStreamWaitEvent), so no call waits on the host.  The stream-less
// overloads use the legacy default stream (stream 0), as the reference does.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include <cstddef>
#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace cudasep {

class __attribute__((visibility("default"))) CudaMemoryPool {
public:
    static CudaMemoryPool& instance();

    void* allocate(size_t requested_bytes) { return allocate(requested_bytes, nullptr); }
    void deallocate(void* ptr) { deallocate(ptr, nullptr); }
    // Stream-ordered forms: the block may be used on `stream` at once; it is
    // released for reuse in `stream`'s order.
    void* allocate(size_t requested_bytes, cudaStream_t stream);
    void deallocate(void* ptr, cudaStream_t stream);
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
        size_t cross_stream_reuses = 0;  // reuses ordered by an event wait
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
    struct Cached {
        void* ptr;
        cudaStream_t stream;  // stream of the free
        cudaEvent_t event;    // recorded on it at the free (null for the legacy stream)
    };
    cudaEvent_t take_event_locked(int device);  // an idle event of `device` (current)
    mutable std::mutex mutex_;
    // (device, size) -> cached blocks
    std::map<std::pair<int, size_t>, std::vector<Cached>> free_;
    std::unordered_map<void*, Block> live_;
    std::map<int, std::vector<cudaEvent_t>> spare_events_;  // per device
    Stats stats_;
};

}  // namespace cudasep
