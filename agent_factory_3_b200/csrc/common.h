// Per-device error word shared by all kernels of the extension.
#pragma once
#include <cstdint>

namespace af3 {
// Device pointer to this device's error word (allocated on first use).
int* device_error_ptr();
// Reads and clears the error word of the current device (synchronises the current stream).
int64_t device_error_take();
}  // namespace af3
