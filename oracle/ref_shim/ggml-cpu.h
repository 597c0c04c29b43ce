/* Stand-in for ggml-cpu.h: nothing from it is used by the CUDA kernels. */
#pragma once
