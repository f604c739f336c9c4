// attn_common.cu — host side of the attention helpers (tensor-map creation).
#include "attn_common.cuh"

namespace scree {

constexpr int kCostBuckets = 4096;

// Per-tile cost in units of inner tiles.
//   forward  (outer = query tile of `outer` rows, inner = key tiles of `inner`):
//     causal: key tiles up to the diagonal; non-causal: all key tiles.
//   backward (outer = key tile, inner = query tiles):
//     causal: query tiles from the diagonal on; non-causal: all query tiles.
__device__ __forceinline__ int tile_cost(int64_t L, int t, int outer, int inner, int causal,
                                         int bwd) {
  const int64_t n_inner = (L + inner - 1) / inner;
  if (!causal) return (int)n_inner;
  if (!bwd) {
    int64_t last = ((int64_t)(t + 1) * outer - 1) / inner + 1;
    return (int)(last < n_inner ? last : n_inner);
  }
  int64_t first = ((int64_t)t * outer) / inner;
  return (int)(n_inner - first);
}

// Builds the tile list sorted by descending cost (counting sort over cost
// buckets; ties in any order).  One CTA of 1024 threads.  Heavy tiles first
// lets the hardware block scheduler approximate longest-processing-time-first.
__global__ void build_schedule_kernel(const void* offs, int is64, int64_t B, int outer, int inner,
                                      int causal, int bwd, int32_t* count_out,
                                      TileRef* list) {
  __shared__ int hist[kCostBuckets];
  for (int i = threadIdx.x; i < kCostBuckets; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) {
    const int64_t L = load_offset(offs, is64, b + 1) - load_offset(offs, is64, b);
    const int64_t nt = (L + outer - 1) / outer;
    for (int64_t t = 0; t < nt; ++t) {
      int c = tile_cost(L, (int)t, outer, inner, causal, bwd);
      c = c < kCostBuckets - 1 ? c : kCostBuckets - 1;
      atomicAdd(&hist[c], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Exclusive scan from the most expensive bucket down.
    int acc = 0;
    for (int c = kCostBuckets - 1; c >= 0; --c) {
      int n = hist[c];
      hist[c] = acc;
      acc += n;
    }
    *count_out = acc;
  }
  __syncthreads();
  for (int64_t b = threadIdx.x; b < B; b += blockDim.x) {
    const int64_t L = load_offset(offs, is64, b + 1) - load_offset(offs, is64, b);
    const int64_t nt = (L + outer - 1) / outer;
    for (int64_t t = 0; t < nt; ++t) {
      int c = tile_cost(L, (int)t, outer, inner, causal, bwd);
      c = c < kCostBuckets - 1 ? c : kCostBuckets - 1;
      int pos = atomicAdd(&hist[c], 1);
      list[pos] = TileRef{(int32_t)b, (int32_t)t};
    }
  }
}

int launch_build_schedule(const void* offs, int is64, int64_t B, int outer, int inner, int causal,
                          int bwd, void* ws, cudaStream_t stream) {
  build_schedule_kernel<<<1, 1024, 0, stream>>>(offs, is64, B, outer, inner, causal, bwd,
                                                reinterpret_cast<int32_t*>(ws),
                                                reinterpret_cast<TileRef*>((char*)ws + 16));
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}


EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_thd_map(CUtensorMap* map, const void* base, int64_t T, int64_t H, int D,
                 int64_t row_stride, int64_t head_stride, int box_d, int box_rows,
                 int swizzle_bytes, bool bf16) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return SCREE_ERR_CUDA;
  }
  SCREE_CHECK_ARG(((uintptr_t)base % 16) == 0, "attention: tensor base must be 16-byte aligned");
  SCREE_CHECK_ARG((row_stride * 2) % 16 == 0 && (head_stride * 2) % 16 == 0,
                  "attention: row/head strides must be multiples of 8 elements");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)(head_stride * 2), (cuuint64_t)(row_stride * 2)};
  cuuint32_t box[3] = {(cuuint32_t)box_d, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                          : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (CUresult %d): T=%lld H=%lld D=%d strides=%lld,%lld",
                   (int)r, (long long)T, (long long)H, D, (long long)row_stride,
                   (long long)head_stride);
    return SCREE_ERR_CUDA;
  }
  return SCREE_OK;
}

}  // namespace scree
