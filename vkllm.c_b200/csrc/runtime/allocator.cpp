// Size-class caching allocator for device memory and pinned, device-mapped host memory.
#include "internal.h"

namespace vkb
{

CachingAllocator::~CachingAllocator()
{
    trim();
    for (auto &kv : live_)
        raw_free(kv.first);
    live_.clear();
}

size_t CachingAllocator::size_class(size_t bytes)
{
    if (bytes == 0)
        bytes = 1;
    if (bytes <= (1u << 20))
    {
        // Powers of two from 512 B to 1 MiB.
        size_t c = 512;
        while (c < bytes)
            c <<= 1;
        return c;
    }
    // 2 MiB granules above 1 MiB.
    const size_t g = 2u << 20;
    return (bytes + g - 1) / g * g;
}

void *CachingAllocator::raw_alloc(size_t bytes)
{
    void *p = nullptr;
    cudaError_t e;
    if (host_mapped_)
        e = cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
    else
        e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
    {
        (void)cudaGetLastError();
        return nullptr;
    }
    return p;
}

void CachingAllocator::raw_free(void *p)
{
    if (host_mapped_)
        cudaFreeHost(p);
    else
        cudaFree(p);
}

void *CachingAllocator::alloc(size_t bytes, size_t *capacity)
{
    size_t c = size_class(bytes);
    std::lock_guard<std::mutex> lk(mu_);
    auto it = free_.find(c);
    void *p = nullptr;
    if (it != free_.end() && !it->second.empty())
    {
        p = it->second.back();
        it->second.pop_back();
        cached_ -= c;
    }
    else
    {
        p = raw_alloc(c);
        if (!p && cached_ > 0)
        {
            // Out of memory: return every cached block to CUDA and retry once.
            for (auto &kv : free_)
                for (void *q : kv.second)
                    raw_free(q);
            free_.clear();
            cached_ = 0;
            p = raw_alloc(c);
        }
        if (!p)
            return nullptr;
    }
    live_[p] = c;
    in_use_ += c;
    if (capacity)
        *capacity = c;
    return p;
}

void CachingAllocator::release(void *p)
{
    if (!p)
        return;
    std::lock_guard<std::mutex> lk(mu_);
    auto it = live_.find(p);
    if (it == live_.end())
        return;
    size_t c = it->second;
    live_.erase(it);
    in_use_ -= c;
    free_[c].push_back(p);
    cached_ += c;
}

void CachingAllocator::trim()
{
    std::lock_guard<std::mutex> lk(mu_);
    for (auto &kv : free_)
        for (void *q : kv.second)
            raw_free(q);
    free_.clear();
    cached_ = 0;
}

vkllm_err_t cuda_check(cudaError_t e, const char *what, const char *file, int line)
{
    vkllm_log(VKLLM_LOG_ERROR, file, line, "%s failed: %s (%d)", what, cudaGetErrorString(e), (int)e);
    return VKLLM_ERR_VULKAN;
}

} // namespace vkb
