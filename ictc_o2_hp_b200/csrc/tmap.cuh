// Tiled TMA (cp.async.bulk.tensor) loads of channel tiles of flat TensorProduct
// rows, for sm_100a.
//
// A flat row is [0e: C][0o: C (full)][frequency m = 1..M: copies x C x 2].  The
// channels [c0, c0 + Ct) of one row form two boxes of two 3-D views of the operand:
//   scalar view    (channel C, scalar segment S0, row N), box (Ct, S0, 1);
//   frequency view (2C interleaved (channel, component), M x copies, row N),
//                  box (2 Ct, M x copies, 1)   -- channel-major blocks, or
//                  (channel C, M x copies x 2 components, row N),
//                  box (Ct, 2 M x copies, 1)   -- component-major blocks.
// Landing back to back in shared memory, the two boxes are exactly a row of a
// Ct-channel product in the same layout, so the per-row arithmetic reads a tile
// row as if the product had Ct channels.  No multicast is used.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace ictc {

// The six tensor maps of one backward launch: (x, y, g) x (scalar, frequency).
struct alignas(64) RowTileMaps {
  CUtensorMap m[6];
};

// Host: encodes the scalar and frequency views of one operand (`maps[0]`,
// `maps[1]`).  Returns 0, or -1 when the driver entry point is unavailable or
// the encoding is rejected.
int encode_row_tile_maps(const float* base, int64_t rows, int C, int M, bool full, bool cm,
                         int64_t width, int Ct, CUtensorMap* maps);

// 3-D tile load of box coordinates (x, y, z) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
        "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

}  // namespace ictc
