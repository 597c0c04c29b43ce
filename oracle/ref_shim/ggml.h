/* Minimal stand-in for ggml.h so the reference's CUDA kernel file compiles on
 * its own: the kernels only use the fp16 storage type and opaque pointers. */
#pragma once
#include <stdint.h>
typedef uint16_t ggml_fp16_t;
struct ggml_tensor;
struct ggml_context;
struct ggml_cgraph;
