// Host helper that builds 2-D TMA descriptors (cuTensorMapEncodeTiled).
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace tdb_host {
// inner = contiguous extent (elements), outer = row count, row_stride_elems =
// distance between rows in elements.  Checks the 16-byte rules for the base
// and the stride before calling the driver.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle);
}  // namespace tdb_host
