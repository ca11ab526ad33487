/*
 * Type names used by vk-compute's public headers (include/session.h,
 * buffer.h, device.h, ...), so that the reference's host program
 * (src/compute.c, src/main.c) compiles unchanged against libvkcompute.
 *
 * Only handle and struct TYPE NAMES are declared.  No API function is
 * declared here and none exists in libvkcompute: its handles carry CUDA
 * objects (a context record, a stream, device pointers), as documented in
 * session.h and buffer.h.
 */
#ifndef VKC_SHIM_VULKAN_H
#define VKC_SHIM_VULKAN_H

#include <stdint.h>

typedef uint64_t VkDeviceSize;

typedef struct VkInstance_T* VkInstance;
typedef struct VkPhysicalDevice_T* VkPhysicalDevice;
typedef struct VkDevice_T* VkDevice;
typedef struct VkQueue_T* VkQueue;
typedef struct VkBuffer_T* VkBuffer;
typedef struct VkDeviceMemory_T* VkDeviceMemory;
typedef struct VkCommandPool_T* VkCommandPool;
typedef struct VkCommandBuffer_T* VkCommandBuffer;
typedef struct VkFence_T* VkFence;
typedef struct VkQueryPool_T* VkQueryPool;
typedef struct VkDescriptorSetLayout_T* VkDescriptorSetLayout;
typedef struct VkDescriptorPool_T* VkDescriptorPool;
typedef struct VkDescriptorSet_T* VkDescriptorSet;
typedef struct VkPipelineLayout_T* VkPipelineLayout;
typedef struct VkPipeline_T* VkPipeline;

typedef struct VkMemoryRequirements {
    VkDeviceSize size;
    VkDeviceSize alignment;
    uint32_t memoryTypeBits;
} VkMemoryRequirements;

#define VK_NULL_HANDLE 0

#endif
