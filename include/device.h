/*
 * Drop-in replacement for vk-compute include/device.h:5-13.
 * In libvkcompute a device is one CUDA device: `device` holds the context
 * record (instance and device both point at it), the session stream (queue)
 * and the CUDA ordinal plus one (physicalDevice).
 */
#ifndef device_h
#define device_h
#include <vulkan/vulkan.h>

typedef struct device {
    VkInstance instance;
    VkDevice device;
    VkQueue queue;
    VkPhysicalDevice physicalDevice;
} device;

/* include/device.h:12 -- opens CUDA device 0 (or $VKC_DEVICE). */
device createDevice();
/* include/device.h:13 */
void destroyDevice(device dev);

#endif
