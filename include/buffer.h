/*
 * Drop-in replacement for vk-compute include/buffer.h:5-22.
 *
 * Every buffer lives in device memory (HBM); `buffer` and `memory` hold the
 * device address, `memReqs.size` the allocated bytes.  createBuffer copies the
 * caller's host data at creation, as the reference does (src/buffer.c:49-54),
 * whichever memoryType is asked for.  mappedMemory stays NULL: host reads go
 * through readBuffer and host writes through writeBuffer.
 */
#ifndef buffer_h
#define buffer_h
#include <vulkan/vulkan.h>

#define MEMORY_RAM 0
#define MEMORY_VRAM 1

typedef struct buffer {
    VkBuffer buffer;
    VkMemoryRequirements memReqs;
    VkDeviceMemory memory;
    VkBuffer stagingBuffer;
    VkDeviceMemory stagingMemory;
    void* mappedMemory;
    int64_t size;
    int memoryType;
} buffer;

/* include/buffer.h:19 -- allocate `size` bytes of HBM and copy `data` (may be
 * NULL: the buffer is then zero-filled). */
buffer createBuffer(VkDevice device, VkPhysicalDevice physicalDevice, void* data, int64_t size, int memoryType);
/* include/buffer.h:20 -- the copies already happened in createBuffer; this
 * waits for them, as the reference's queue wait does (src/buffer.c:110-111). */
void createTransferAndCopy(VkDevice device, VkQueue queue, buffer* buffers, int bufferCount);
/* include/buffer.h:21 -- copy the whole buffer to `output`. */
void readBuffer(VkDevice device, VkPhysicalDevice physicalDevice, VkQueue queue, buffer buf, void* output);
/* include/buffer.h:22 */
void destroyBuffer(VkDevice device, buffer buf);

/* No counterpart in the reference, which writes host-visible memory through
 * mappedMemory.  Copies buf.size bytes from `data` into the buffer and waits. */
void writeBuffer(VkDevice device, VkQueue queue, buffer buf, const void* data);

#endif
