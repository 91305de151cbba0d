// Tensor-map encoding entry point shared by the kernels that copy with TMA.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

namespace spectra {

// cuTensorMapEncodeTiled from the driver, resolved once (nullptr if the
// driver does not provide it).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace spectra
