/* TEST INFRASTRUCTURE (oracle pin). Declares just enough Vulkan names for the reference's own
 * headers (src/core/vkllm_tensor.h, vkllm_commands.h, vkllm_pipeline.h, vkllm_gpu_device.h,
 * vkllm_common.h) to parse, so that the CPU reference functions of its tests can be compiled
 * here from the files where they lie. Nothing declared here is ever called: the build keeps
 * only the CPU functions and drops the GPU test bodies. No Vulkan library exists on this
 * machine or the GPU box. */
#ifndef REFPIN_STUB_VULKAN_H
#define REFPIN_STUB_VULKAN_H
#include <stdint.h>

#define REFPIN_HANDLE(n) typedef struct n##_opaque *n
REFPIN_HANDLE(VkInstance);
REFPIN_HANDLE(VkPhysicalDevice);
REFPIN_HANDLE(VkDevice);
REFPIN_HANDLE(VkQueue);
REFPIN_HANDLE(VkCommandBuffer);
REFPIN_HANDLE(VkCommandPool);
REFPIN_HANDLE(VkFence);
REFPIN_HANDLE(VkBuffer);
REFPIN_HANDLE(VkDescriptorSet);
REFPIN_HANDLE(VkDescriptorSetLayout);
REFPIN_HANDLE(VkDescriptorPool);
REFPIN_HANDLE(VkPipeline);
REFPIN_HANDLE(VkPipelineLayout);
REFPIN_HANDLE(VkShaderModule);
REFPIN_HANDLE(VkQueryPool);
REFPIN_HANDLE(VkDebugUtilsMessengerEXT);
#undef REFPIN_HANDLE

typedef enum { VK_SUCCESS = 0 } VkResult;
typedef uint32_t VkAccessFlagBits;
typedef uint32_t VkPipelineStageFlagBits;
typedef uint32_t VkQueueFlagBits;

#define REFPIN_STRUCT(n) typedef struct { uint64_t refpin_unused; } n
REFPIN_STRUCT(VkPhysicalDeviceFeatures);
REFPIN_STRUCT(VkPhysicalDeviceProperties);
REFPIN_STRUCT(VkExtensionProperties);
REFPIN_STRUCT(VkPhysicalDeviceMemoryProperties);
REFPIN_STRUCT(VkQueueFamilyProperties);
REFPIN_STRUCT(VkPhysicalDeviceSubgroupProperties);
REFPIN_STRUCT(VkPhysicalDeviceShaderFloat16Int8Features);
REFPIN_STRUCT(VkPhysicalDevice16BitStorageFeatures);
REFPIN_STRUCT(VkPhysicalDevice8BitStorageFeatures);
REFPIN_STRUCT(VkPhysicalDeviceShaderSubgroupExtendedTypesFeatures);
REFPIN_STRUCT(VkPhysicalDeviceProperties2);
REFPIN_STRUCT(VkPhysicalDeviceFeatures2);
#undef REFPIN_STRUCT

#endif
