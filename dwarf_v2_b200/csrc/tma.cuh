// Host side of the TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

namespace dwarf {

// The driver's cuTensorMapEncodeTiled, or nullptr when unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensormap_encoder();

}  // namespace dwarf
