// tma.cuh - tensor-map (TMA) helpers shared by the kernels: the driver's
// cuTensorMapEncodeTiled looked up at run time (no link-time libcuda
// dependency).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace cnnue {

// cuTensorMapEncodeTiled from the driver, or nullptr when it is unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn();

}  // namespace cnnue
