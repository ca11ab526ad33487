/*
 * Drop-in replacement for vk-compute include/descriptor.h.  Kept for header
 * compatibility: binding i of an operation is simply buffers[i]
 * (src/descriptor.c:12-18), so no descriptor object is needed.  The
 * functions exist and return an empty record.
 */
#ifndef descriptor_h
#define descriptor_h
#include <vulkan/vulkan.h>
#include "buffer.h"

typedef struct descriptor {
    VkDescriptorSetLayout layout;
    VkDescriptorPool pool;
    VkDescriptorSet set;
} descriptor;

descriptor createDescriptor(VkDevice device, int bufferCount, buffer buffers[]);
void destroyDescriptor(VkDevice device, descriptor desc);

#endif
