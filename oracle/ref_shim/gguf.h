/* Stand-in for gguf.h: the reference headers only hold gguf_context pointers. */
#pragma once
struct gguf_context;
