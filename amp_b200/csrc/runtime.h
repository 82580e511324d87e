// runtime.h -- host-side helpers shared by the entry points.
#pragma once
#include <cstddef>

namespace ampb {

// Returns a device buffer of at least `bytes` for staging slot `slot` on the
// current device (grow-only, kept until process exit).  Slots let one call
// hold several live buffers.  Not re-entrant across threads for one slot.
int staging_get(int slot, size_t bytes, void** out);

}  // namespace ampb
