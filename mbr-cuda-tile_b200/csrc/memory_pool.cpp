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

void* CudaMemoryPool::allocate(size_t requested) {
    if (requested == 0) return nullptr;
    int dev = 0;
    MBR_CUDA(cudaGetDevice(&dev));
    const size_t size = round_up(requested);
    std::lock_guard<std::mutex> lock(mutex_);
    // smallest cached block of at least `size` that wastes at most half of itself
    auto it = free_.lower_bound({dev, size});
    if (it != free_.end() && it->first.first == dev && it->first.second <= 2 * size && !it->second.empty()) {
        void* p = it->second.back();
        it->second.pop_back();
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

void CudaMemoryPool::deallocate(void* p) {
    if (!p) return;
    std::lock_guard<std::mutex> lock(mutex_);
    auto it = live_.find(p);
    if (it == live_.end()) {
        cudaFree(p);  // not ours: hand back to the runtime
        return;
    }
    free_[{it->second.device, it->second.size}].push_back(p);
    stats_.deallocations++;
    stats_.active_bytes -= it->second.size;
    live_.erase(it);
}

void CudaMemoryPool::release_cached_locked() {
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto& kv : free_) {
        for (void* p : kv.second) {
            cudaSetDevice(kv.first.first);
            cudaFree(p);
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
              << " active=" << (s.active_bytes >> 20) << "MB peak=" << (s.peak_bytes >> 20)
              << "MB cached=" << (cached_bytes() >> 20) << "MB" << std::endl;
}

}  // namespace cudasep
