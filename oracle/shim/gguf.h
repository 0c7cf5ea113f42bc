// Test-infrastructure shim (oracle only): the GGUF context handle named by jepa-internal.h. The
// shim loader parses files with the project's own reader instead.
#pragma once
struct gguf_context;
