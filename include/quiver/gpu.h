// GPU build additions to the Quiver C++ API (no counterpart in the reference). Indexes live on one
// CUDA device chosen when they are constructed or loaded: the device set here, else the
// QUIVER_DEVICE environment variable, else device 0.
#pragma once

namespace quiver::gpu {

/// Device that FlatIndex / IvfPqIndex objects created afterwards (on any thread) are placed on.
void set_device(int device);
int device();

/// Number of CUDA devices visible to the process (0 when there is none).
int device_count() noexcept;

}  // namespace quiver::gpu
