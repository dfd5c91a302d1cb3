/* Minimal stand-in for ggml-backend.h (opaque handle types only); see ggml.h here. */
#pragma once
#include "ggml.h"
typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
