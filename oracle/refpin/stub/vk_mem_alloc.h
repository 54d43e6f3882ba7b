/* TEST INFRASTRUCTURE (oracle pin). The allocator names the reference's src/core/vkllm_tensor.h and
 * vkllm_gpu_device.h mention, declared only so those headers parse (see vulkan/vulkan.h here). */
#ifndef REFPIN_STUB_VK_MEM_ALLOC_H
#define REFPIN_STUB_VK_MEM_ALLOC_H
#include <vulkan/vulkan.h>
typedef struct VmaAllocator_opaque *VmaAllocator;
typedef struct VmaAllocation_opaque *VmaAllocation;
typedef struct { void *pMappedData; uint64_t size; } VmaAllocationInfo;
#endif
