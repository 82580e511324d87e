// runtime.h -- host-side helpers shared by the entry points.
#pragma once
#include <cstddef>

namespace ampb {

// Returns a device buffer of at least `bytes` for staging slot `slot` on the
// current device (grow-only, kept until process exit).  Slots let one call
// hold several live buffers.  Not re-entrant across threads for one slot.
int staging_get(int slot, size_t bytes, void** out);

// Per-device status word written by kernels whose bounded waits expired
// (AMP_DEV_ERR_TIMEOUT); allocated and zeroed on first use.
int device_status(int** out);

}  // namespace ampb
