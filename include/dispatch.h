/*
 * Drop-in replacement for vk-compute include/dispatch.h:11-26.
 *
 * `operation.shader` names the operator by the reference's SPIR-V file name
 * ("GEMV-INT4.spv", "RmsNorm-swiglu-ffn-FP16.spv", ...; any directory prefix
 * and the extension are ignored, case-insensitive).  buffers[i] is the
 * shader's binding i and pushConstants its push-constant block, exactly as in
 * the reference (src/descriptor.c:12-18, src/dispatch.c:30-33).
 * dispatchX/Y/Z are accepted and ignored: each operator picks its own grid.
 */
#ifndef dispatch_h
#define dispatch_h

#include <vulkan/vulkan.h>
#include "buffer.h"
#include "device.h"
#include "descriptor.h"
#include "pipeline.h"
#include "session.h"

#define MAX_OP_BUFFERS 16
#define MAX_PUSH_CONSTANTS 8

typedef struct operation {
    char shader[128];
    buffer buffers[MAX_OP_BUFFERS];
    int bufferCount;
    int pushConstants[MAX_PUSH_CONSTANTS];
    int pushConstantCount;
    int dispatchX;
    int dispatchY;
    int dispatchZ;
} operation;

/* include/dispatch.h:25 -- launch ops[0..opCount) in order on the session
 * stream (src/dispatch.c:8-61).  Returns once the work is enqueued: results
 * reach the host only through readBuffer / getExecutionTime, which wait for
 * the stream, so a caller sees what the reference's wait-on-fence execute
 * gives.  Unknown operator names, missing bindings and undersized buffers
 * print to stderr and exit, as the reference does on its fatal paths. */
void execute(session s, operation ops[], int opCount);
/* include/dispatch.h:26 -- device time of the last execute, in ms (0 when
 * timing is off: vkc_set_timing in vk_compute_b200.h). */
double getExecutionTime(session s);

#endif
