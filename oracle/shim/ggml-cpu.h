// Test-infrastructure shim (oracle only): included by jepa-internal.h; nothing is used from it.
#pragma once
