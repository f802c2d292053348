/* Declaration-only stand-in (see ggml.h in this directory). */
#pragma once
#include "ggml.h"
typedef struct ggml_backend* ggml_backend_t;
typedef struct ggml_backend_buffer* ggml_backend_buffer_t;
