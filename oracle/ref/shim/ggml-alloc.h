/* Declaration-only stand-in (see ggml.h in this directory). */
#pragma once
#include "ggml-backend.h"
typedef struct ggml_gallocr* ggml_gallocr_t;
