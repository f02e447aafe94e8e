// memory_pool.cpp — caching device allocator (reference: src/memory_pool.h:21-190).
#include "memory_pool.h"

#include <cuda_runtime.h>

#include <iostream>
#include <string>

#include "common.h"

namespace cudasep {

CudaMemoryPool& CudaMemoryPool::instance() {
    static CudaMemoryPool* pool = new CudaMemoryPool();  // never destroyed: outlives every Tensor
    return *pool;
}

CudaMemoryPool::~CudaMemoryPool() { release_all(); }

size_t CudaMemoryPool::round_up(size_t b) {
    const size_t kSmall = 512, kMid = 2u << 20, kLarge = 20u << 20;
    if (b < (1u << 20)) return (b + kSmall - 1) / kSmall * kSmall;
    if (b < (10u << 20)) return (b + kMid - 1) / kMid * kMid;
    return (b + kLarge - 1) / kLarge * kLarge;
}

cudaEvent_t CudaMemoryPool::take_event_locked(int device) {
    std::vector<cudaEvent_t>& spare = spare_events_[device];
    if (!spare.empty()) {
        cudaEvent_t e = spare.back();
        spare.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    MBR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    return e;
}

void* CudaMemoryPool::allocate(size_t requested, cudaStream_t stream) {
    if (requested == 0) return nullptr;
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    const size_t size = round_up(requested);
    std::lock_guard<std::mutex> lock(mutex_);
    // smallest cached block of at least `size` that wastes at most half of itself
    auto it = free_.lower_bound({dev, size});
    if (it != free_.end() && it->first.first == dev && it->first.second <= 2 * size && !it->second.empty()) {
        std::vector<Cached>& v = it->second;
        // a block freed on this stream needs no ordering; else the most recent
        size_t pick = v.size() - 1;
        for (size_t i = v.size(); i-- > 0;)
            if (v[i].stream == stream) {
                pick = i;
                break;
            }
        const Cached c = v[pick];
        v.erase(v.begin() + (std::ptrdiff_t)pick);
        if (c.stream != stream && c.event) {
            // the free's stream order carries over to this stream
            MBR_CUDA(cudaStreamWaitEvent(stream, c.event, 0));
            stats_.cross_stream_reuses++;
        }
        if (c.event) spare_events_[dev].push_back(c.event);
        void* p = c.ptr;
        live_[p] = {it->first.second, dev};
        stats_.allocations++;
        stats_.cache_hits++;
        stats_.active_bytes += it->first.second;
        if (stats_.active_bytes > stats_.peak_bytes) stats_.peak_bytes = stats_.active_bytes;
        return p;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, size);
    if (e != cudaSuccess) {
        cudaGetLastError();
        release_cached_locked();
        e = cudaMalloc(&p, size);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw mbr::Error(mbr::ERR_OOM, "CudaMemoryPool: cudaMalloc failed for " + std::to_string(size) +
                                               " bytes: " + cudaGetErrorString(e));
        }
    }
    live_[p] = {size, dev};
    stats_.allocations++;
    stats_.total_allocated += size;
    stats_.active_bytes += size;
    if (stats_.active_bytes > stats_.peak_bytes) stats_.peak_bytes = stats_.active_bytes;
    return p;
}

void CudaMemoryPool::deallocate(void* p, cudaStream_t stream) {
    if (!p) return;
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = live_.find(p);
    if (it == live_.end()) {
        cudaFree(p);  // not ours: hand back to the runtime
        return;
    }
    // the legacy default stream orders itself with every blocking stream, so a
    // block freed there needs no event
    cudaEvent_t ev = nullptr;
    if (stream != nullptr) {
        int cur = 0;
        cudaGetDevice(&cur);
        if (cur != it->second.device) cudaSetDevice(it->second.device);
        ev = take_event_locked(it->second.device);
        MBR_CUDA(cudaEventRecord(ev, stream));
        if (cur != it->second.device) cudaSetDevice(cur);
    }
    free_[{it->second.device, it->second.size}].push_back({p, stream, ev});
    stats_.deallocations++;
    stats_.active_bytes -= it->second.size;
    live_.erase(it);
}

void CudaMemoryPool::release_cached_locked() {
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto& kv : free_) {
        for (const Cached& c : kv.second) {
            cudaSetDevice(kv.first.first);
            cudaFree(c.ptr);  // cudaFree waits for the device, so pending uses are done
            if (c.event) cudaEventDestroy(c.event);
            stats_.total_freed += kv.first.second;
        }
        kv.second.clear();
    }
    free_.clear();
    cudaSetDevice(cur);
}

void CudaMemoryPool::trim_cached_memory() {
    std::lock_guard<std::mutex> lock(mutex_);
    release_cached_locked();
}

void CudaMemoryPool::release_all() {
    std::lock_guard<std::mutex> lock(mutex_);
    release_cached_locked();
    for (auto& kv : live_) {
        cudaFree(kv.first);
        stats_.total_freed += kv.second.size;
    }
    live_.clear();
    stats_.active_bytes = 0;
}

CudaMemoryPool::Stats CudaMemoryPool::get_stats() const {
    std::lock_guard<std::mutex> lock(mutex_);
    return stats_;
}

size_t CudaMemoryPool::cached_bytes() const {
    std::lock_guard<std::mutex> lock(mutex_);
    size_t n = 0;
    for (auto& kv : free_) n += kv.first.second * kv.second.size();
    return n;
}

void CudaMemoryPool::print_stats() const {
    Stats s = get_stats();
    std::cout << "[MemPool] allocs=" << s.allocations << " frees=" << s.deallocations << " hits=" << s.cache_hits
              << " cross-stream=" << s.cross_stream_reuses
              << " active=" << (s.active_bytes >> 20) << "MB peak=" << (s.peak_bytes >> 20)
              << "MB cached=" << (cached_bytes() >> 20) << "MB" << std::endl;
}

}  // namespace cudasep
