// Host access to the driver's tensor-map encoder, shared by the kernels that
// copy tiles with TMA.
#pragma once
#include <cuda.h>

namespace aicas {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled obtained through the runtime's driver entry point
// (null when the driver does not provide it).
EncodeTiledFn tensor_map_encoder();

}  // namespace aicas
