/* Declaration-only stand-in (see ggml.h in this directory). */
#pragma once
#include "ggml.h"
struct gguf_context;
