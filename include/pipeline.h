/*
 * Drop-in replacement for vk-compute include/pipeline.h.  Kept for header
 * compatibility: operators are compiled CUDA kernels selected by name in
 * execute(), so createPipeline only checks that the name is a known operator
 * (fatal otherwise, like a missing .spv file, src/pipeline.c:9-11).
 */
#ifndef pipeline_h
#define pipeline_h
#include <vulkan/vulkan.h>

#define MAX_PUSH_CONSTANT_SIZE 128

typedef struct pipeline {
    VkPipelineLayout layout;
    VkPipeline pipeline;
} pipeline;

pipeline createPipeline(VkDevice device, VkDescriptorSetLayout descriptorLayout, const char shaderPath[], uint32_t pushConstantSize);
void destroyPipeline(VkDevice device, pipeline pipe);

#endif
