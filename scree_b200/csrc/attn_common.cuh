// attn_common.cuh — pieces shared by the attention forward and backward
// kernels: the on-device tile scheduler (a cost-sorted list of work tiles built
// without any host synchronisation) and TMA tensor-map creation for the packed
// (T, H, D) layout.
#pragma once
#include <cuda.h>
#include "common.cuh"
#include "sm100.cuh"

namespace scree {

// Work schedule.  Work items are (sequence, head, tile) triples enumerated so
// that the CTAs resident at any moment share data in L2:
//   sequences in descending length (cost ~ L^2; longest first = LPT order),
//   then head-major within a sequence, then the sequence's tiles, heaviest first
//   (forward causal: the last query tile; backward causal: the first key tile).
// An item index maps to its item by a binary search over SeqRef::item_start.
struct SeqRef {
  int32_t seq;         // index into offsets
  int32_t ntiles;      // tiles of `outer` rows in this sequence
  int64_t item_start;  // first work item of this sequence (items = ntiles * H)
};

// Upper bound on the number of tiles of size `rows` over a batch of B
// sequences with T tokens in total: sum_b ceil(L_b / rows) <= T / rows + B.
inline int64_t max_tiles(int64_t B, int64_t T, int rows) { return (T + rows - 1) / rows + B; }

// Schedule workspace: [total items (int64)] [item counter (uint64)] [SeqRef x B].
inline size_t schedule_bytes(int64_t B) { return 16 + sizeof(SeqRef) * (size_t)B; }

// Sequences sorted by length on the device (one CTA) when B <= kSortMax;
// larger batches keep their natural order (head-major grouping still applies).
constexpr int kSortMax = 4096;

// Status-word site of rejected offsets (attention schedule and softmax).
constexpr int kSiteBadOffsets = 40;

// Validates the offsets against T and builds the schedule into `ws`
// (schedule_bytes(B)); invalid offsets give a zero-item schedule and a
// SCREE_DEVERR_BAD_INPUT status.
int launch_build_schedule(const void* offs, int is64, int64_t B, int64_t T, int outer, int H,
                          void* ws, cudaStream_t stream);
// The offsets check alone (same status on failure); kernels that later read the
// status word at CTA start then do no work.
int launch_validate_offsets(const void* offs, int is64, int64_t B, int64_t T, cudaStream_t stream);

// Device side: item -> (seq, head, j) with j the rank of the tile within its
// (seq, head) group (0 = first scheduled).
struct WorkItem {
  int32_t seq, head, j, ntiles;
};
__device__ __forceinline__ WorkItem decode_item(const void* ws, int64_t B, int H, int64_t item) {
  const SeqRef* refs = reinterpret_cast<const SeqRef*>(reinterpret_cast<const char*>(ws) + 16);
  int64_t lo = 0, hi = B - 1;
  while (lo < hi) {  // last entry with item_start <= item
    const int64_t mid = (lo + hi + 1) >> 1;
    if (refs[mid].item_start <= item) lo = mid; else hi = mid - 1;
  }
  // Skip empty sequences that share item_start with the owner.
  while (lo < B - 1 && refs[lo].ntiles == 0) ++lo;
  const SeqRef r = refs[lo];
  const int64_t i = item - r.item_start;
  WorkItem w;
  w.seq = r.seq;
  w.ntiles = r.ntiles;
  w.head = (int32_t)(i / r.ntiles);
  w.j = (int32_t)(i % r.ntiles);
  (void)H;
  return w;
}
__device__ __forceinline__ int64_t total_items(const void* ws) {
  return *reinterpret_cast<const int64_t*>(ws);
}
// Items handed out so far to persistent CTAs (bytes [8, 16) of the schedule,
// zeroed by the schedule build that precedes every launch).
__device__ __forceinline__ unsigned long long* item_counter(const void* ws) {
  return reinterpret_cast<unsigned long long*>(const_cast<char*>(reinterpret_cast<const char*>(ws)) + 8);
}

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

// Tensor map over a packed (T, H, D) fp32 tensor (row-major, contiguous), box
// {D, 1, box_rows}, no swizzle; used as the target of TMA reduce-adds.
int make_thd_map_f32(CUtensorMap* map, const void* base, int64_t T, int64_t H, int D,
                     int box_rows);

// fp32 attention (attn_f32.cu): CUDA-core kernels for fp32 inputs.
int attn_fwd_f32(const void* q, const void* k, const void* v, int64_t q_rs, int64_t q_hs,
                 int64_t k_rs, int64_t k_hs, int64_t v_rs, int64_t v_hs, const void* offsets,
                 int is64, int64_t B, int64_t T, int64_t H, int64_t H_kv, int D, int causal,
                 float scale, void* o, int64_t o_rs, int64_t o_hs, float* lse, cudaStream_t s);
int attn_bwd_f32(const void* dout, const void* q, const void* k, const void* v, const void* o,
                 const float* lse, const void* offsets, int is64, int64_t B, int64_t T, int64_t H,
                 int64_t H_kv, int D, int causal, float scale, void* dq, void* dk, void* dv,
                 float* delta, cudaStream_t s);

}  // namespace scree
