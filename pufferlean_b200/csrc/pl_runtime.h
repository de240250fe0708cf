// Library-wide runtime state shared by the translation units: launch counter, device checks and a
// per-device cache of grow-only scratch buffers for the host-buffer entry points.
#pragma once
#include <stddef.h>
#include <stdint.h>

namespace pl {
// Records the message pl_last_error returns on this thread and returns code.
int set_error(int code, const char* fmt, ...);
void count_launch(uint64_t n = 1);
int require_device();
// Grow-only device buffer `slot` (0..63) of at least `bytes` on the current device; NULL on failure
// (pl_last_error says why). Buffers live until process exit, like the reference's ts_buf cache.
void* scratch(int slot, size_t bytes);
}  // namespace pl
