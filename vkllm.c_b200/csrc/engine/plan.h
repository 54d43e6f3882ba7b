// Fused-execution plan attached by vkllm_models_llama2_build_graph to the graphs it builds.
#pragma once

#include <cstdint>

struct vkllm_models_llama2;
struct vkllm_tensor;

namespace vkb
{

struct GraphCacheEntry;

struct Plan
{
    vkllm_models_llama2 *model;
    vkllm_tensor *input_toks; // u32 [1,1,1,S]
    vkllm_tensor *output;     // u32 [1,1,S,1], mapped
    uint32_t offsets;         // position of the first token
    uint32_t seq_len;         // S
    size_t n_nodes;           // node count when built; a later edit disables the plan
    GraphCacheEntry *cache_entry; // structural-cache entry whose nodes this graph holds (models/graph_cache.cpp)
};

} // namespace vkb
