// Per-device status word shared by every kernel of the extension.  Kernels
// record the first error code (bounded-wait timeout, capacity overflow, ...)
// with atomicCAS and return; the host reads and clears it.
#pragma once
namespace mb {
int* status_ptr(int device);
int read_and_clear_status(int device);
}  // namespace mb
