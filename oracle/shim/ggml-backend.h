// Test-infrastructure shim (oracle only): opaque backend handles and the one tensor read-back the
// reference planner performs (src/hjepa-plan.cpp:67). Weights live in host memory here.
#pragma once
#include "ggml.h"
typedef struct ggml_backend * ggml_backend_t;
typedef struct ggml_backend_device * ggml_backend_dev_t;
typedef struct ggml_backend_buffer * ggml_backend_buffer_t;
void ggml_backend_tensor_get(const struct ggml_tensor * t, void * data, size_t offset, size_t size);
