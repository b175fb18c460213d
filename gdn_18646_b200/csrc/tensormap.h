// tensormap.h -- host helpers to build TMA descriptors without linking libcuda
// (the driver entry point is fetched through the runtime).
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace gdn {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled tensor_map_encoder();

// bf16 tiled map; dims/strides innermost first (strides for dims 1..rank-1, bytes).
int make_map_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);

}  // namespace gdn
