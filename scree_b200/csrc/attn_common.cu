// attn_common.cu — the attention work scheduler and tensor-map creation.
#include "attn_common.cuh"

namespace scree {

// Whole-block check of an offsets array: offs[0] == 0, non-decreasing,
// offs[B] == T.  Every thread of the block must call it (it ends in a barrier).
__device__ bool offsets_valid_block(const void* offs, int is64, int64_t B, int64_t T) {
  int bad = 0;
  for (int64_t i = threadIdx.x; i < B; i += blockDim.x)
    if (load_offset(offs, is64, i + 1) < load_offset(offs, is64, i)) bad = 1;
  if (threadIdx.x == 0 && (load_offset(offs, is64, 0) != 0 || load_offset(offs, is64, B) != T))
    bad = 1;
  return __syncthreads_or(bad) == 0;
}

__global__ void validate_offsets_kernel(const void* offs, int is64, int64_t B, int64_t T,
                                        int* status) {
  if (!offsets_valid_block(offs, is64, B, T) && threadIdx.x == 0)
    record_device_error(status, SCREE_DEVERR_BAD_INPUT, kSiteBadOffsets);
}

// One CTA of 1024 threads.  First validates the offsets (offs[0] == 0,
// non-decreasing, offs[B] == T); invalid offsets record SCREE_DEVERR_BAD_INPUT
// in the device status word and publish a schedule of zero items, so every
// attention CTA exits before its first load or store.  Then sorts (length,
// index) keys descending with a shared-memory bitonic sort (B <= kSortMax), and
// an exclusive scan of ntiles * H gives each sequence's first work item.
__global__ void build_schedule_kernel(const void* offs, int is64, int64_t B, int64_t T, int outer,
                                      int H, int64_t* total_out, SeqRef* refs, int* status) {
  __shared__ unsigned long long keys[kSortMax];
  __shared__ long long warp_tot[32];
  __shared__ long long carry;
  if (threadIdx.x == 0) total_out[1] = 0;  // the persistent kernels' item counter
  if (!offsets_valid_block(offs, is64, B, T)) {
    if (threadIdx.x == 0) {
      *total_out = 0;
      record_device_error(status, SCREE_DEVERR_BAD_INPUT, kSiteBadOffsets);
    }
    return;
  }
  const bool sorted = B <= kSortMax;
  int n2 = 1;
  while (n2 < B) n2 <<= 1;
  if (sorted) {
    for (int i = threadIdx.x; i < n2; i += blockDim.x) {
      unsigned long long key = 0;  // padding sorts last (length 0, index max)
      if (i < B) {
        const int64_t L = load_offset(offs, is64, i + 1) - load_offset(offs, is64, i);
        // descending length, ties by ascending index: key = (L << 32) | ~index
        key = ((unsigned long long)(L & 0xFFFFFFFF) << 32) | (0xFFFFFFFFu - (unsigned)i);
      }
      keys[i] = key;
    }
    __syncthreads();
    for (int k = 2; k <= n2; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < n2; i += blockDim.x) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const bool desc = (i & k) == 0;  // overall descending
            const unsigned long long a = keys[i], b = keys[ixj];
            if (desc ? (a < b) : (a > b)) {
              keys[i] = b;
              keys[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
    }
  }
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t base = 0; base < B; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    long long items = 0;
    int32_t seq = 0, nt = 0;
    if (i < B) {
      seq = sorted ? (int32_t)(0xFFFFFFFFu - (unsigned)(keys[i] & 0xFFFFFFFFull)) : (int32_t)i;
      const int64_t L = load_offset(offs, is64, seq + 1) - load_offset(offs, is64, seq);
      nt = (int32_t)((L + outer - 1) / outer);
      items = (long long)nt * H;
    }
    long long v = items;  // inclusive warp scan
    for (int o = 1; o < 32; o <<= 1) {
      const long long n = __shfl_up_sync(0xffffffff, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) warp_tot[wid] = v;
    __syncthreads();
    if (wid == 0) {
      long long w = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        const long long n = __shfl_up_sync(0xffffffff, w, o);
        if (lane >= o) w += n;
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    const long long incl = carry + (wid > 0 ? warp_tot[wid - 1] : 0) + v;
    if (i < B) refs[i] = SeqRef{seq, nt, (int64_t)(incl - items)};
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total_out = carry;
}

int launch_build_schedule(const void* offs, int is64, int64_t B, int64_t T, int outer, int H,
                          void* ws, cudaStream_t stream) {
  build_schedule_kernel<<<1, 1024, 0, stream>>>(offs, is64, B, T, outer, H,
                                                reinterpret_cast<int64_t*>(ws),
                                                reinterpret_cast<SeqRef*>((char*)ws + 16),
                                                device_status_ptr());
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

}  // namespace scree

extern "C" int scree_validate_offsets(const void* offsets, int offs_is_i64, int64_t B, int64_t T,
                                      void* stream) {
  using namespace scree;
  SCREE_CHECK_ARG(B >= 1 && T >= 0, "validate_offsets: bad sizes B=%lld T=%lld", (long long)B,
                  (long long)T);
  SCREE_CHECK_ARG(offsets != nullptr, "validate_offsets: null offsets");
  SCREE_BIND_DEVICE(stream, offsets);
  return launch_validate_offsets(offsets, offs_is_i64, B, T, (cudaStream_t)stream);
}

namespace scree {

int launch_validate_offsets(const void* offs, int is64, int64_t B, int64_t T, cudaStream_t stream) {
  validate_offsets_kernel<<<1, 1024, 0, stream>>>(offs, is64, B, T, device_status_ptr());
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

int make_thd_map_f32(CUtensorMap* map, const void* base, int64_t T, int64_t H, int D,
                     int box_rows) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return SCREE_ERR_CUDA;
  }
  SCREE_CHECK_ARG(((uintptr_t)base % 16) == 0, "fp32 map: base must be 16-byte aligned");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)D * 4, (cuuint64_t)(H * D * 4)};
  cuuint32_t box[3] = {(cuuint32_t)D, 1u, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled (fp32) failed (CUresult %d)", (int)r);
    return SCREE_ERR_CUDA;
  }
  return SCREE_OK;
}

}  // namespace scree
