// Internal runtime definitions shared by the C-ABI layer, the ops and the engine.
// Not installed; the public surface is include/*.h.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "vkllm_commands.h"
#include "vkllm_common.h"
#include "vkllm_context.h"
#include "vkllm_dtypes.h"
#include "vkllm_graph.h"
#include "vkllm_pipeline.h"
#include "vkllm_tensor.h"

// CUDA device record behind the opaque struct vkllm_gpu_device of the public headers.
struct vkllm_gpu_device
{
    int ordinal;
    int sm_count;
    int cc_major, cc_minor;
    size_t smem_optin;
    char name[256];
};

namespace vkb
{

// Node set of a graph built by vkllm_models_llama2_build_graph, kept between vkllm_graph_free and the
// next build for the same model and shapes (models/graph_cache.cpp).
struct GraphCacheEntry;

// Caching allocator: device memory and pinned, device-mapped host memory are recycled through
// size-class free lists so that the reference's allocate-every-node-every-step pattern costs no
// cudaMalloc/cudaFree (which would synchronise the device) after warm-up.
class CachingAllocator
{
  public:
    explicit CachingAllocator(bool host_mapped) : host_mapped_(host_mapped)
    {
    }
    ~CachingAllocator();
    // Returns nullptr on failure. `*capacity` receives the block size actually reserved.
    void *alloc(size_t bytes, size_t *capacity);
    void release(void *p);
    void trim(); // give every cached block back to CUDA
    size_t bytes_in_use() const
    {
        return in_use_;
    }
    size_t bytes_cached() const
    {
        return cached_;
    }

  private:
    static size_t size_class(size_t bytes);
    void *raw_alloc(size_t bytes);
    void raw_free(void *p);
    bool host_mapped_;
    std::mutex mu_;
    std::map<size_t, std::vector<void *>> free_;
    std::map<void *, size_t> live_;
    size_t in_use_ = 0, cached_ = 0;
};

} // namespace vkb

enum vkllm_exec_mode
{
    VKLLM_EXEC_FUSED = 0,  // graphs built by the llama2 builder run the fused engine
    VKLLM_EXEC_STRICT = 1, // every graph runs one kernel per node, like the reference
};

struct vkllm_b200_runtime
{
    cudaStream_t stream = nullptr; // the context's single in-order queue (the reference uses queue 0 for all commands)
    vkb::CachingAllocator *dev_alloc = nullptr;
    vkb::CachingAllocator *host_alloc = nullptr;
    std::map<std::string, vkllm_pipeline *> pipelines; // kernel table, one entry per variant name
    int exec_mode = VKLLM_EXEC_FUSED;
    bool node_timing = false;
    int* dev_error_word = nullptr; // device-side error flag written by kernels with bounded waits
    std::vector<void *> tensor_pool; // freed tensor structs of the pooled size (tensor.cpp)
    std::vector<void *> event_pool;  // completion events of freed commands objects (commands.cpp)
    bool graph_cache_on = true;      // VKLLM_B200_GRAPH_CACHE=0 turns the structural graph cache off
    std::vector<vkb::GraphCacheEntry *> graph_cache;
};

namespace vkb
{

// Logs and converts a CUDA error into VKLLM_ERR_VULKAN (the reference's "device error" code).
vkllm_err_t cuda_check(cudaError_t e, const char *what, const char *file, int line);

#define VKB_CUDA(call)                                                                                                 \
    do                                                                                                                 \
    {                                                                                                                  \
        cudaError_t e__ = (call);                                                                                      \
        if (e__ != cudaSuccess)                                                                                        \
            return ::vkb::cuda_check(e__, #call, __FILE__, __LINE__);                                                  \
    } while (0)

// Size in bytes of one element.
uint32_t dtype_bytes(vkllm_dtype_t dt);

// The tensor that owns the bytes of `t` (follows copy_ref / slice0 views).
vkllm_tensor *storage_owner(vkllm_tensor *t);

// Device address of element [0,0,0,0] of `t`, allocating the owner's storage on first use.
// Returns nullptr (and logs) when the allocation fails.
void *dev_ptr(vkllm_context *ctx, vkllm_tensor *t);

// Element strides (bytes / element size).
struct Strides4
{
    uint32_t s[4];
};
Strides4 elem_strides(const vkllm_tensor *t);

// Looks up (or creates) the named kernel-table entry.
vkllm_pipeline *get_pipeline(vkllm_context *ctx, const char *name, vkllm_op_t op, int variant);

cudaStream_t stream_of(vkllm_context *ctx, vkllm_commands *cmd);

// Brackets a launch with the pipeline's timing events when node timing is on.
void timing_begin(vkllm_context *ctx, vkllm_pipeline *p, cudaStream_t s);
void timing_end(vkllm_context *ctx, vkllm_pipeline *p, cudaStream_t s);

// Maximum grid.x for 1-D launches, and the usual 1-D launch helper.
inline unsigned grid_1d(uint64_t n, unsigned block)
{
    uint64_t g = (n + block - 1) / block;
    if (g > 0x7fffffffull)
        g = 0x7fffffffull;
    return (unsigned)(g == 0 ? 1 : g);
}

} // namespace vkb
