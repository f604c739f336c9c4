// attn_common.cuh — pieces shared by the attention forward and backward
// kernels: the on-device tile scheduler (a cost-sorted list of work tiles built
// without any host synchronisation) and TMA tensor-map creation for the packed
// (T, H, D) layout.
#pragma once
#include <cuda.h>
#include "common.cuh"
#include "sm100.cuh"

namespace scree {

// A work tile: sequence index and tile index along the outer loop dimension
// (query tiles in the forward, key tiles in the backward).
struct TileRef {
  int32_t seq;
  int32_t tile;
};

// Upper bound on the number of tiles of size `rows` over a batch of B
// sequences with T tokens in total: sum_b ceil(L_b / rows) <= T / rows + B.
inline int64_t max_tiles(int64_t B, int64_t T, int rows) { return (T + rows - 1) / rows + B; }

// Schedule workspace: [count (int32, padded to 16 B)] [TileRef x max_tiles].
inline size_t schedule_bytes(int64_t B, int64_t T, int rows) {
  return 16 + sizeof(TileRef) * (size_t)max_tiles(B, T, rows);
}

// Enqueues the schedule build: writes the tile count and the list of TileRef
// sorted by descending cost into `ws` (schedule_bytes() bytes).
//   forward  (outer = query tiles of `outer` rows, inner = key tiles of `inner`)
//   backward (outer = key tiles, inner = query tiles; bwd = 1)
int launch_build_schedule(const void* offs, int is64, int64_t B, int outer, int inner, int causal,
                          int bwd, void* ws, cudaStream_t stream);

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode_tiled();

// Tensor map over a packed (T, H, D) 16-bit tensor, viewed as dims
// {D, H, T} (innermost first), with a box of {box_d, 1, box_rows}.
// Strides are in elements; they must be multiples of 8 (16 bytes).
int make_thd_map(CUtensorMap* map, const void* base, int64_t T, int64_t H, int D,
                 int64_t row_stride, int64_t head_stride, int box_d, int box_rows, int swizzle_bytes,
                 bool bf16);

}  // namespace scree
