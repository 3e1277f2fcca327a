// slx_attr.h -- per-device launch settings shared by the kernel launchers.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace slx {

// Raises `func`'s dynamic shared memory limit to at least `bytes` on the current device.
// cudaFuncSetAttribute acts on one device only, so the setting is recorded per (kernel, device):
// a process that drives several GPUs (one context per device) sets it once on each. Thread-safe.
// Requests up to the 48 KiB default need no attribute and return at once.
cudaError_t ensure_smem(const void* func, size_t bytes);

// Streaming multiprocessors of the current device (cached per device).
int device_sm_count();

}  // namespace slx
