// softmax.cu — varlen softmax along the ragged dimension, forward and backward.
//
// For every sequence b and every feature column f independently
// (reference/varlen_softmax.py:55-61):
//   y[t, f] = exp(x[t, f] - max_t x[t, f]) / sum_t exp(x[t, f] - max_t x[t, f])
// over the rows t of sequence b.  Backward: dx = y * (dy - sum_t dy * y).
//
// A CTA owns one sequence and a block of 32 * VW feature columns: thread lane
// l of every warp holds VW consecutive columns (16-byte vectors when the row
// allows), and the 8 warps stride over the sequence's rows.  Pass 1 keeps a
// running (max, sum) per column (online rescaling), merged across warps in
// shared memory; pass 2 re-reads the rows (mostly from L2: the CTA touched them
// just before) and writes the result.  fp32 statistics for every dtype.
#include <algorithm>
#include "common.cuh"

namespace scree {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <typename T, int VW> struct alignas(sizeof(T) * VW) SPack { T v[VW]; };

template <typename T, int VW>
__device__ __forceinline__ void sload(const T* p, float (&o)[VW]) {
  const SPack<T, VW> pk = *reinterpret_cast<const SPack<T, VW>*>(p);
#pragma unroll
  for (int i = 0; i < VW; ++i) o[i] = Cvt<T>::to_f(pk.v[i]);
}
template <typename T, int VW>
__device__ __forceinline__ void sstore(T* p, const float (&v)[VW]) {
  SPack<T, VW> pk;
#pragma unroll
  for (int i = 0; i < VW; ++i) pk.v[i] = Cvt<T>::from_f(v[i]);
  *reinterpret_cast<SPack<T, VW>*>(p) = pk;
}

template <typename T, int VW>
__global__ void __launch_bounds__(kThreads) softmax_fwd_kernel(const T* __restrict__ x,
                                                                const void* offs, int is64,
                                                                int64_t F, T* __restrict__ y) {
  __shared__ float sm_m[kWarps][32 * VW], sm_s[kWarps][32 * VW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t r0 = load_offset(offs, is64, b), r1 = load_offset(offs, is64, b + 1);
  const int64_t c0 = (int64_t)blockIdx.x * 32 * VW + lane * VW;
  const bool col_ok = c0 < F;  // F is a multiple of VW
  float m[VW], s[VW];
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    m[i] = -INFINITY;
    s[i] = 0.f;
  }
  if (col_ok) {
    // Rows in groups of 4 per warp: one max update and one rescale per group
    // (no divergent per-element branch), loads of the group issued together.
    constexpr int G = 4;
    int64_t r = r0 + warp;
    for (; r + (G - 1) * kWarps < r1; r += G * kWarps) {
      float v[G][VW];
#pragma unroll
      for (int g = 0; g < G; ++g) sload<T, VW>(x + (r + g * kWarps) * F + c0, v[g]);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float mn = fmaxf(fmaxf(m[i], fmaxf(v[0][i], v[1][i])), fmaxf(v[2][i], v[3][i]));
        float acc = (m[i] == -INFINITY) ? 0.f : s[i] * __expf(m[i] - mn);
#pragma unroll
        for (int g = 0; g < G; ++g) acc += __expf(v[g][i] - mn);
        s[i] = acc;
        m[i] = mn;
      }
    }
    for (; r < r1; r += kWarps) {  // remaining rows one at a time
      float v[VW];
      sload<T, VW>(x + r * F + c0, v);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float mn = fmaxf(m[i], v[i]);
        s[i] = ((m[i] == -INFINITY) ? 0.f : s[i] * __expf(m[i] - mn)) + __expf(v[i] - mn);
        m[i] = mn;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    sm_m[warp][lane * VW + i] = m[i];
    sm_s[warp][lane * VW + i] = s[i];
  }
  __syncthreads();
  // Every warp merges the 8 partial (max, sum) pairs in the same order.
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm_m[w][lane * VW + i]);
    float ss = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm_m[w][lane * VW + i];
      if (mw != -INFINITY) ss += sm_s[w][lane * VW + i] * __expf(mw - mm);
    }
    m[i] = mm;
    s[i] = 1.f / ss;
  }
  if (!col_ok) return;
  for (int64_t r = r0 + warp; r < r1; r += kWarps) {
    float v[VW];
    sload<T, VW>(x + r * F + c0, v);
#pragma unroll
    for (int i = 0; i < VW; ++i) v[i] = __expf(v[i] - m[i]) * s[i];
    sstore<T, VW>(y + r * F + c0, v);
  }
}

template <typename T, int VW>
__global__ void __launch_bounds__(kThreads) softmax_bwd_kernel(const T* __restrict__ dy,
                                                                const T* __restrict__ y,
                                                                const void* offs, int is64,
                                                                int64_t F, T* __restrict__ dx) {
  __shared__ float sm_d[kWarps][32 * VW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t r0 = load_offset(offs, is64, b), r1 = load_offset(offs, is64, b + 1);
  const int64_t c0 = (int64_t)blockIdx.x * 32 * VW + lane * VW;
  const bool col_ok = c0 < F;
  float d[VW];
#pragma unroll
  for (int i = 0; i < VW; ++i) d[i] = 0.f;
  if (col_ok)
    for (int64_t r = r0 + warp; r < r1; r += kWarps) {
      float g[VW], p[VW];
      sload<T, VW>(dy + r * F + c0, g);
      sload<T, VW>(y + r * F + c0, p);
#pragma unroll
      for (int i = 0; i < VW; ++i) d[i] = fmaf(g[i], p[i], d[i]);
    }
#pragma unroll
  for (int i = 0; i < VW; ++i) sm_d[warp][lane * VW + i] = d[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    float t = 0.f;
    for (int w = 0; w < kWarps; ++w) t += sm_d[w][lane * VW + i];
    d[i] = t;
  }
  if (!col_ok) return;
  for (int64_t r = r0 + warp; r < r1; r += kWarps) {
    float g[VW], p[VW];
    sload<T, VW>(dy + r * F + c0, g);
    sload<T, VW>(y + r * F + c0, p);
#pragma unroll
    for (int i = 0; i < VW; ++i) g[i] = p[i] * (g[i] - d[i]);
    sstore<T, VW>(dx + r * F + c0, g);
  }
}

template <typename T>
int launch(bool bwd, const void* a, const void* bb, const void* offs, int is64, int64_t B,
           int64_t F, void* out, cudaStream_t s) {
  const bool vec = (F * (int64_t)sizeof(T)) % 16 == 0 && ((uintptr_t)a % 16) == 0 &&
                   ((uintptr_t)out % 16) == 0 && (!bwd || ((uintptr_t)bb % 16) == 0);
  constexpr int VWV = 16 / sizeof(T);
  const int vw = vec ? VWV : 1;
  const int64_t cols_per_cta = 32 * vw;
  const dim3 grid((unsigned)((F + cols_per_cta - 1) / cols_per_cta),
                  (unsigned)std::min<int64_t>(B, 65535), 1);
  ProfScope prof(bwd ? PROF_NORM_BWD : PROF_NORM_FWD, s);
  for (int64_t b0 = 0; b0 < B; b0 += 65535) {
    // grid.y covers at most 65535 sequences per launch; later chunks shift offs.
    const int64_t nb = std::min<int64_t>(B - b0, 65535);
    const void* o = is64 ? (const void*)((const int64_t*)offs + b0)
                         : (const void*)((const int32_t*)offs + b0);
    const dim3 g(grid.x, (unsigned)nb, 1);
    if (!bwd) {
      if (vec) softmax_fwd_kernel<T, VWV><<<g, kThreads, 0, s>>>((const T*)a, o, is64, F, (T*)out);
      else softmax_fwd_kernel<T, 1><<<g, kThreads, 0, s>>>((const T*)a, o, is64, F, (T*)out);
    } else {
      if (vec)
        softmax_bwd_kernel<T, VWV><<<g, kThreads, 0, s>>>((const T*)a, (const T*)bb, o, is64, F, (T*)out);
      else
        softmax_bwd_kernel<T, 1><<<g, kThreads, 0, s>>>((const T*)a, (const T*)bb, o, is64, F, (T*)out);
    }
    SCREE_LAUNCH_CHECK();
  }
  return SCREE_OK;
}

int dispatch(bool bwd, const void* a, const void* bb, const void* offs, int is64, int64_t B,
             int64_t T, int64_t F, int dtype, void* out, void* stream) {
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && F >= 0, "varlen softmax: bad sizes");
  if (T == 0 || F == 0) return SCREE_OK;
  SCREE_CHECK_ARG(a && out && offs && (!bwd || bb), "varlen softmax: null pointer");
  SCREE_BIND_DEVICE(stream, a);
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case SCREE_F16: return launch<__half>(bwd, a, bb, offs, is64, B, F, out, s);
    case SCREE_BF16: return launch<__nv_bfloat16>(bwd, a, bb, offs, is64, B, F, out, s);
    case SCREE_F32: return launch<float>(bwd, a, bb, offs, is64, B, F, out, s);
    default: break;
  }
  set_last_error("varlen softmax: unsupported dtype %d", dtype);
  return SCREE_ERR_INVALID;
}

}  // namespace
}  // namespace scree

extern "C" int scree_softmax_fwd(const void* x, const void* offsets, int offs_is_i64, int64_t B,
                                 int64_t T, int64_t F, int dtype, void* y, void* stream) {
  return scree::dispatch(false, x, nullptr, offsets, offs_is_i64, B, T, F, dtype, y, stream);
}

extern "C" int scree_softmax_bwd(const void* dy, const void* y, const void* offsets,
                                 int offs_is_i64, int64_t B, int64_t T, int64_t F, int dtype,
                                 void* dx, void* stream) {
  return scree::dispatch(true, dy, y, offsets, offs_is_i64, B, T, F, dtype, dx, stream);
}
