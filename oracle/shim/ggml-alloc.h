// Test-infrastructure shim (oracle only): the graph allocator handle named by jepa-internal.h.
#pragma once
typedef struct ggml_gallocr * ggml_gallocr_t;
