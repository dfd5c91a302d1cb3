/*
 * Minimal stand-in for ggml.h, used ONLY to compile the reference's
 * GGML-free renderer sources (src/levo-flow-renderer.cpp,
 * src/levo-renderer-pattern.cpp) into oracle/_ref/.  Those files use GGML
 * types only as opaque pointers in headers they include; nothing here is
 * GGML functionality.  Test infrastructure, not product code.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
struct ggml_tensor;
struct ggml_context;
struct ggml_cgraph;
