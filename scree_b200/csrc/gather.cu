// gather.cu — the offset gathers of scree._core on the GPU: pack, to_padded,
// from_padded.  All are byte copies (bit-exact for every dtype) and HBM-bound:
// each moves its rows once with 16-byte vector accesses when every row start
// is 16-byte aligned, else falls back to element-width accesses.  Grids are a
// multiple of the SM count and grid-stride over the output.
#include <algorithm>
#include "common.cuh"

namespace scree {
namespace {

constexpr int kThreads = 256;

// Largest power-of-two access width (<= 16 bytes) that divides every address
// the kernel touches.
int pick_width(int64_t row_bytes, std::initializer_list<uintptr_t> ptrs) {
  int w = 16;
  while (w > 1 && (row_bytes % w) != 0) w >>= 1;
  for (uintptr_t p : ptrs)
    while (w > 1 && (p % w) != 0) w >>= 1;
  return w;
}

template <int W> struct Vec;
template <> struct Vec<16> { using T = uint4; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<2> { using T = uint16_t; };
template <> struct Vec<1> { using T = uint8_t; };

// All three gathers use a 2-D grid: blockIdx.y walks sequences (padded rows),
// blockIdx.x a chunk of `rows_per_cta` rows of that sequence; threads stride
// over the W-byte vectors of those rows.  No per-element search and no 64-bit
// division: one 32-bit division by the vectors-per-row count per element.

// ---------------------------------------------------------------- pack
template <int W>
__global__ void __launch_bounds__(kThreads) pack_kernel(
    const void* const* __restrict__ src, const void* offs, int is64, int64_t B, int64_t T,
    int64_t row_bytes, int rows_per_cta, void* __restrict__ dst, int* status) {
  using V = typename Vec<W>::T;
  const uint32_t vpr = (uint32_t)(row_bytes / W);
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
    const int64_t s = load_offset(offs, is64, b);
    const int64_t len = load_offset(offs, is64, b + 1) - s;
    if (s < 0 || len < 0 || s + len > T) {  // malformed offsets: no store, report
      if (threadIdx.x == 0) record_device_error(status, SCREE_DEVERR_BAD_INPUT, 42);
      continue;
    }
    const int64_t j0 = (int64_t)blockIdx.x * rows_per_cta;
    if (j0 >= len) continue;
    const uint32_t nrows = (uint32_t)(rows_per_cta < len - j0 ? rows_per_cta : len - j0);
    const V* __restrict__ sp = reinterpret_cast<const V*>(src[b]) + j0 * vpr;
    V* __restrict__ dp = reinterpret_cast<V*>(dst) + (s + j0) * vpr;
    const uint32_t n = nrows * vpr;
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) dp[v] = sp[v];
  }
}

// ---------------------------------------------------------------- to_padded
template <int W>
__global__ void __launch_bounds__(kThreads) to_padded_kernel(
    const void* __restrict__ values, const void* offs, int is64, int64_t B, int64_t max_len,
    int64_t row_bytes, int rows_per_cta, uint4 fill16, int side_left, void* __restrict__ padded,
    void* __restrict__ mask, int mask_bytes, int* status) {
  using V = typename Vec<W>::T;
  V fill;
  memcpy(&fill, &fill16, sizeof(V));
  const uint32_t vpr = (uint32_t)(row_bytes / W);
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
    const int64_t s = load_offset(offs, is64, b);
    const int64_t len = load_offset(offs, is64, b + 1) - s;
    if (s < 0 || len < 0 || len > max_len) {  // malformed offsets: no access, report
      if (threadIdx.x == 0) record_device_error(status, SCREE_DEVERR_BAD_INPUT, 43);
      continue;
    }
    const int64_t j0 = (int64_t)blockIdx.x * rows_per_cta;
    if (j0 >= max_len) continue;
    const uint32_t nrows = (uint32_t)(rows_per_cta < max_len - j0 ? rows_per_cta : max_len - j0);
    const int64_t shift = side_left ? (max_len - len) : 0;  // padded row j <- source row j - shift
    V* __restrict__ dp = reinterpret_cast<V*>(padded) + (b * max_len + j0) * vpr;
    const V* __restrict__ vp = reinterpret_cast<const V*>(values);
    const uint32_t n = nrows * vpr;
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) {
      const uint32_t r = v / vpr;
      const int64_t src_row = j0 + r - shift;
      V out = fill;
      if (src_row >= 0 && src_row < len) out = vp[(s + src_row) * vpr + (v - r * vpr)];
      dp[v] = out;
    }
    if (mask != nullptr)
      for (uint32_t r = threadIdx.x; r < nrows; r += blockDim.x) {
        const int64_t src_row = j0 + r - shift;
        const int on = (src_row >= 0 && src_row < len) ? 1 : 0;
        const int64_t mi = b * max_len + j0 + r;
        switch (mask_bytes) {  // bool / uint8, int16, int32 or int64 (HF) masks
          case 8: reinterpret_cast<int64_t*>(mask)[mi] = on; break;
          case 4: reinterpret_cast<int32_t*>(mask)[mi] = on; break;
          case 2: reinterpret_cast<int16_t*>(mask)[mi] = (int16_t)on; break;
          default: reinterpret_cast<uint8_t*>(mask)[mi] = (uint8_t)on; break;
        }
      }
  }
}

// ---------------------------------------------------------------- kv append
// out sequence b = cache rows of b, then new rows of b; out_offs[b] =
// cache_offs[b] + new_offs[b] (prefix sums of the summed lengths), written by
// the CTAs of chunk 0.  Sequences whose rows fall outside their buffers are
// skipped and reported.
template <int W>
__global__ void __launch_bounds__(kThreads) kv_append_kernel(
    const void* __restrict__ cache, const void* coffs, const void* __restrict__ fresh,
    const void* noffs, int is64, int64_t B, int64_t Tc, int64_t Tn, int64_t row_bytes,
    int rows_per_cta, void* __restrict__ out, int64_t* __restrict__ out_offs, int* status) {
  using V = typename Vec<W>::T;
  const uint32_t vpr = (uint32_t)(row_bytes / W);
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
    const int64_t cs = load_offset(coffs, is64, b), ce = load_offset(coffs, is64, b + 1);
    const int64_t ns = load_offset(noffs, is64, b), ne = load_offset(noffs, is64, b + 1);
    if (cs < 0 || ce < cs || ce > Tc || ns < 0 || ne < ns || ne > Tn) {
      if (threadIdx.x == 0) record_device_error(status, SCREE_DEVERR_BAD_INPUT, 47);
      continue;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      out_offs[b + 1] = ce + ne;
      if (b == 0) out_offs[0] = 0;
    }
    const int64_t lc = ce - cs, len = lc + (ne - ns);
    const int64_t j0 = (int64_t)blockIdx.x * rows_per_cta;
    if (j0 >= len) continue;
    const uint32_t nrows = (uint32_t)(rows_per_cta < len - j0 ? rows_per_cta : len - j0);
    V* __restrict__ dp = reinterpret_cast<V*>(out) + (cs + ns + j0) * vpr;
    const V* __restrict__ cp = reinterpret_cast<const V*>(cache) + cs * vpr;
    const V* __restrict__ np = reinterpret_cast<const V*>(fresh) + (ns - lc) * vpr;
    const uint32_t n = nrows * vpr;
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) {
      const int64_t j = j0 + v / vpr;
      const int64_t e = j * vpr + (v % vpr);
      dp[v] = j < lc ? cp[e] : np[e];
    }
  }
}

// ---------------------------------------------------------------- from_padded
// Step 1a: one CTA per padded row writes its mask count into offsets[b+1].
template <typename MT>
__global__ void padded_count_kernel(const MT* __restrict__ mask, int64_t max_len,
                                    int32_t* __restrict__ offsets) {
  __shared__ int red[32];
  const int64_t b = blockIdx.x;
  int cnt = 0;
  for (int64_t j = threadIdx.x; j < max_len; j += blockDim.x) cnt += mask[b * max_len + j] != 0;
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffff, cnt, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    offsets[b + 1] = s;
    if (b == 0) offsets[0] = 0;
  }
}

// Step 1b: single-CTA in-place inclusive scan of offsets[1..B], 1024 at a time.
__global__ void inplace_scan_kernel(int32_t* __restrict__ offsets, int64_t B) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t base = 0; base < B; base += blockDim.x) {
    int64_t i = base + threadIdx.x;
    int32_t v = i < B ? offsets[i + 1] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int32_t n = __shfl_up_sync(0xffffffff, v, o);
      if (lane >= o) v += n;
    }
    if (lane == 31) warp_sums[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int32_t ws = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        int32_t n = __shfl_up_sync(0xffffffff, ws, o);
        if (lane >= o) ws += n;
      }
      warp_sums[lane] = ws;
    }
    __syncthreads();
    int32_t add = carry + (wid > 0 ? warp_sums[wid - 1] : 0);
    if (i < B) offsets[i + 1] = v + add;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = v + add;
    __syncthreads();
  }
}

template <int W>
__global__ void __launch_bounds__(kThreads) from_padded_kernel(
    const void* __restrict__ padded, const int32_t* __restrict__ offs, int64_t B,
    int64_t max_len, int64_t row_bytes, int rows_per_cta, void* __restrict__ values) {
  using V = typename Vec<W>::T;
  const uint32_t vpr = (uint32_t)(row_bytes / W);
  for (int64_t b = blockIdx.y; b < B; b += gridDim.y) {
    const int64_t s = offs[b];
    const int64_t len = offs[b + 1] - s;
    const int64_t j0 = (int64_t)blockIdx.x * rows_per_cta;
    if (j0 >= len) continue;
    const uint32_t nrows = (uint32_t)(rows_per_cta < len - j0 ? rows_per_cta : len - j0);
    const V* __restrict__ sp = reinterpret_cast<const V*>(padded) + (b * max_len + j0) * vpr;
    V* __restrict__ dp = reinterpret_cast<V*>(values) + (s + j0) * vpr;
    const uint32_t n = nrows * vpr;
    for (uint32_t v = threadIdx.x; v < n; v += blockDim.x) dp[v] = sp[v];
  }
}

// Rows per CTA so that one CTA moves about 32 KB; grid.x covers `rows` rows,
// grid.y the batch (capped at 65535, the kernels loop over the rest).
dim3 gather_grid(int64_t rows, int64_t B, int64_t row_bytes, int* rows_per_cta) {
  int64_t r = row_bytes > 0 ? (32768 + row_bytes - 1) / row_bytes : 1;
  r = std::max<int64_t>(1, std::min<int64_t>(r, 4096));
  *rows_per_cta = (int)r;
  const int64_t gx = std::max<int64_t>(1, (rows + r - 1) / r);
  return dim3((unsigned)std::min<int64_t>(gx, 2147483647), (unsigned)std::min<int64_t>(B, 65535), 1);
}

}  // namespace
}  // namespace scree

using namespace scree;

#define DISPATCH_WIDTH(w, KERNEL, GRID, STREAM, ...)                                      \
  ProfScope prof_(PROF_GATHER, STREAM);                                                   \
  switch (w) {                                                                            \
    case 16: KERNEL<16><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;                \
    case 8: KERNEL<8><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;                  \
    case 4: KERNEL<4><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;                  \
    case 2: KERNEL<2><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;                  \
    default: KERNEL<1><<<GRID, kThreads, 0, STREAM>>>(__VA_ARGS__); break;                 \
  }

extern "C" int scree_pack(const void* const* src_ptrs, const void* offsets, int offs_is_i64,
                          int64_t B, int64_t T, int64_t max_rows, int64_t row_bytes,
                          int64_t src_align, void* dst, void* stream) {
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && row_bytes >= 0, "scree_pack: bad sizes");
  if (T == 0 || row_bytes == 0) return SCREE_OK;
  SCREE_CHECK_ARG(src_ptrs && offsets && dst, "scree_pack: null pointer");
  SCREE_CHECK_ARG(src_align >= 1, "scree_pack: src_align must be >= 1");
  // The source pointers live in device memory, so the caller states their
  // common alignment; the access width divides it, row_bytes and dst.
  SCREE_CHECK_ARG(row_bytes < (1ll << 31), "scree_pack: rows larger than 2 GB");
  int w = pick_width(row_bytes, {(uintptr_t)dst, (uintptr_t)src_align});
  SCREE_BIND_DEVICE(stream, dst);
  cudaStream_t s = (cudaStream_t)stream;
  int rpc = 1;
  // CTAs past a sequence's end exit at once; without a bound, T rows.
  const dim3 grid = gather_grid(max_rows > 0 ? std::min(max_rows, T) : T, B, row_bytes, &rpc);
  DISPATCH_WIDTH(w, pack_kernel, grid, s, src_ptrs, offsets, offs_is_i64, B, T, row_bytes, rpc, dst,
                 device_status_ptr());
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

extern "C" int scree_to_padded(const void* values, const void* offsets, int offs_is_i64,
                               int64_t B, int64_t max_len, int64_t row_bytes, int64_t elem_bytes,
                               const void* fill_pattern_host, int side_left, void* padded,
                               uint8_t* mask, void* stream) {
  return scree_to_padded_ex(values, offsets, offs_is_i64, B, max_len, row_bytes, elem_bytes,
                            fill_pattern_host, side_left, padded, mask, 1, stream);
}

extern "C" int scree_to_padded_ex(const void* values, const void* offsets, int offs_is_i64,
                                  int64_t B, int64_t max_len, int64_t row_bytes,
                                  int64_t elem_bytes, const void* fill_pattern_host,
                                  int side_left, void* padded, void* mask, int mask_elem_bytes,
                                  void* stream) {
  SCREE_CHECK_ARG(mask_elem_bytes == 1 || mask_elem_bytes == 2 || mask_elem_bytes == 4 ||
                      mask_elem_bytes == 8,
                  "scree_to_padded: mask elements must be 1, 2, 4 or 8 bytes");
  SCREE_CHECK_ARG(B >= 0 && max_len >= 0 && row_bytes >= 0, "scree_to_padded: bad sizes");
  SCREE_CHECK_ARG(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8,
                  "scree_to_padded: elem_bytes must be 1, 2, 4 or 8");
  SCREE_CHECK_ARG(fill_pattern_host != nullptr, "scree_to_padded: null fill pattern");
  if (B == 0 || max_len == 0) return SCREE_OK;
  // Build a 16-byte fill vector by repeating the element pattern.
  uint8_t fill[16];
  for (int i = 0; i < 16; ++i) fill[i] = ((const uint8_t*)fill_pattern_host)[i % elem_bytes];
  uint4 fill16;
  memcpy(&fill16, fill, 16);
  int w = row_bytes == 0 ? 1 : pick_width(row_bytes, {(uintptr_t)values, (uintptr_t)padded});
  if (w < elem_bytes && row_bytes > 0) {
    // The fill vector repeats whole elements only when w is a multiple of elem_bytes.
    SCREE_CHECK_ARG(false, "scree_to_padded: misaligned buffers for element size %lld",
                    (long long)elem_bytes);
  }
  SCREE_CHECK_ARG(row_bytes < (1ll << 31), "scree_to_padded: rows larger than 2 GB");
  SCREE_BIND_DEVICE(stream, mask ? (const void*)mask : padded);
  cudaStream_t s = (cudaStream_t)stream;
  int rpc = 1;
  const dim3 grid = gather_grid(max_len, B, row_bytes == 0 ? w : row_bytes, &rpc);
  // row_bytes == 0 (empty feature dims): only the mask is written; rows of one
  // W-byte "vector" are walked over a null padded pointer with no stores.
  if (row_bytes == 0) {
    to_padded_kernel<1><<<grid, kThreads, 0, s>>>(values, offsets, offs_is_i64, B, max_len, 0,
                                                   rpc, fill16, side_left, nullptr, mask,
                                                   mask_elem_bytes, device_status_ptr());
  } else {
    DISPATCH_WIDTH(w, to_padded_kernel, grid, s, values, offsets, offs_is_i64, B, max_len,
                   row_bytes, rpc, fill16, side_left, padded, mask, mask_elem_bytes,
                   device_status_ptr());
  }
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

extern "C" int scree_padded_lengths(const uint8_t* mask, int64_t B, int64_t max_len,
                                    int32_t* offsets_out, void* stream) {
  return scree_padded_lengths_ex(mask, 1, B, max_len, offsets_out, stream);
}

extern "C" int scree_padded_lengths_ex(const void* mask, int mask_elem_bytes, int64_t B,
                                       int64_t max_len, int32_t* offsets_out, void* stream) {
  SCREE_CHECK_ARG(mask_elem_bytes == 1 || mask_elem_bytes == 2 || mask_elem_bytes == 4 ||
                      mask_elem_bytes == 8,
                  "scree_padded_lengths: mask elements must be 1, 2, 4 or 8 bytes");
  SCREE_CHECK_ARG(B >= 1 && max_len >= 0, "scree_padded_lengths: bad sizes");
  SCREE_CHECK_ARG(offsets_out != nullptr, "scree_padded_lengths: null offsets");
  SCREE_CHECK_ARG(B < (1ll << 31), "scree_padded_lengths: batch too large");
  SCREE_BIND_DEVICE(stream, offsets_out);
  cudaStream_t s = (cudaStream_t)stream;
  if (max_len == 0) {
    SCREE_CUDA_TRY(cudaMemsetAsync(offsets_out, 0, (B + 1) * sizeof(int32_t), s));
    return SCREE_OK;
  }
  SCREE_CHECK_ARG(mask != nullptr, "scree_padded_lengths: null mask");
  switch (mask_elem_bytes) {  // a nonzero element marks a valid position
    case 8:
      padded_count_kernel<<<(unsigned)B, 256, 0, s>>>((const uint64_t*)mask, max_len, offsets_out);
      break;
    case 4:
      padded_count_kernel<<<(unsigned)B, 256, 0, s>>>((const uint32_t*)mask, max_len, offsets_out);
      break;
    case 2:
      padded_count_kernel<<<(unsigned)B, 256, 0, s>>>((const uint16_t*)mask, max_len, offsets_out);
      break;
    default:
      padded_count_kernel<<<(unsigned)B, 256, 0, s>>>((const uint8_t*)mask, max_len, offsets_out);
      break;
  }
  SCREE_LAUNCH_CHECK();
  inplace_scan_kernel<<<1, 1024, 0, s>>>(offsets_out, B);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

extern "C" int scree_from_padded(const void* padded, const int32_t* offsets, int64_t B,
                                 int64_t max_len, int64_t T, int64_t row_bytes, void* values,
                                 void* stream) {
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && max_len >= 0 && row_bytes >= 0,
                  "scree_from_padded: bad sizes");
  if (T == 0 || row_bytes == 0) return SCREE_OK;
  SCREE_CHECK_ARG(row_bytes < (1ll << 31), "scree_from_padded: rows larger than 2 GB");
  int w = pick_width(row_bytes, {(uintptr_t)padded, (uintptr_t)values});
  SCREE_BIND_DEVICE(stream, values);
  cudaStream_t s = (cudaStream_t)stream;
  int rpc = 1;
  const dim3 grid = gather_grid(max_len, B, row_bytes, &rpc);
  DISPATCH_WIDTH(w, from_padded_kernel, grid, s, padded, offsets, B, max_len, row_bytes, rpc,
                 values);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

extern "C" int scree_kv_append(const void* cache, const void* cache_offsets, const void* fresh,
                               const void* fresh_offsets, int offs_is_i64, int64_t B, int64_t Tc,
                               int64_t Tn, int64_t max_rows, int64_t row_bytes, void* out,
                               int64_t* out_offsets, void* stream) {
  SCREE_CHECK_ARG(B >= 1 && Tc >= 0 && Tn >= 0 && row_bytes >= 0, "scree_kv_append: bad sizes");
  SCREE_CHECK_ARG(cache_offsets && fresh_offsets && out_offsets, "scree_kv_append: null offsets");
  SCREE_CHECK_ARG(row_bytes < (1ll << 31), "scree_kv_append: rows larger than 2 GB");
  SCREE_CHECK_ARG(Tc + Tn == 0 || (out && (Tc == 0 || cache) && (Tn == 0 || fresh)),
                  "scree_kv_append: null buffer");
  const int w = row_bytes == 0 ? 1
                               : pick_width(row_bytes, {(uintptr_t)out, (uintptr_t)cache,
                                                        (uintptr_t)fresh});
  SCREE_BIND_DEVICE(stream, out_offsets);
  cudaStream_t s = (cudaStream_t)stream;
  int rpc = 1;
  const int64_t rows = max_rows > 0 ? std::min(max_rows, Tc + Tn) : Tc + Tn;
  const dim3 grid = gather_grid(std::max<int64_t>(rows, 1), B, row_bytes == 0 ? w : row_bytes, &rpc);
  DISPATCH_WIDTH(w, kv_append_kernel, grid, s, cache, cache_offsets, fresh, fresh_offsets,
                 offs_is_i64, B, Tc, Tn, row_bytes, rpc, out, out_offsets, device_status_ptr());
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}
