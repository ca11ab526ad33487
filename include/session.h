/*
 * Drop-in replacement for vk-compute include/session.h:8-20.
 * A session is one CUDA device with one stream (dev.queue) and a pair of
 * timing events (held behind qpool); pool, buffer and fence are unused.
 */
#ifndef session_h
#define session_h

#include <vulkan/vulkan.h>
#include "device.h"
#include "buffer.h"

#define TIMESTAMP_QUERY_COUNT 2

typedef struct session {
    device dev;
    VkCommandPool pool;
    VkCommandBuffer buffer;
    VkFence fence;
    VkQueryPool qpool;
} session;

/* include/session.h:18 */
session createSession();
/* include/session.h:19 */
void destroySession(session s);

#endif
