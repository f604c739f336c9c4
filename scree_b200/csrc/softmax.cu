// softmax.cu — varlen softmax along the ragged dimension, forward and backward.
//
// For every sequence b and every feature column f independently
// (reference/varlen_softmax.py:55-61):
//   y[t, f] = exp(x[t, f] - max_t x[t, f]) / sum_t exp(x[t, f] - max_t x[t, f])
// over the rows t of sequence b.  Backward: dx = y * (dy - sum_t dy * y).
//
// A CTA owns one sequence and a block of 8 * VW feature columns: 8 lanes cover
// one row's block (16-byte vectors when the row allows), a warp 4 rows and the
// CTA 32 rows per step, so long sequences are spread over many CTAs (64
// columns each in 16-bit) instead of a few wide ones.  Pass 1 keeps a running
// (max, sum) per column (online rescaling), merged across lanes and warps;
// pass 2 re-reads the rows (from L2: a CTA's block is small and short-lived)
// and writes the result.  fp32 statistics for every dtype.
#include <algorithm>
#include "common.cuh"
#include "sm100.cuh"

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
  cvt_from_f<T, VW>(v, pk.v);
  *reinterpret_cast<SPack<T, VW>*>(p) = pk;
}

// Lane l of a warp covers row (l / kLPR) of the warp's 4-row slab and the VW
// columns (l % kLPR) * VW: a CTA handles kLPR * VW columns, 32 rows per step.
constexpr int kLPR = 8;                 // lanes per row
constexpr int kRPW = 32 / kLPR;         // rows per warp per step
constexpr int kRPC = kWarps * kRPW;     // rows per CTA per step
constexpr float kLog2e = 1.4426950408889634f;

template <typename T, int VW>
__global__ void __launch_bounds__(kThreads, 4) softmax_fwd_kernel(const T* __restrict__ x,
                                                                const void* offs, int is64,
                                                                int64_t T_, int64_t F,
                                                                T* __restrict__ y, int* status) {
  __shared__ float sm_m[kRPC][kLPR * VW], sm_s[kRPC][kLPR * VW];
  __shared__ float fin_m[kLPR * VW], fin_s[kLPR * VW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rsub = lane / kLPR, cv = lane % kLPR;
  const int64_t b = blockIdx.y;
  const int64_t r0 = load_offset(offs, is64, b), r1 = load_offset(offs, is64, b + 1);
  if (r0 < 0 || r1 < r0 || r1 > T_) {  // malformed offsets: no access, report
    if (threadIdx.x == 0) record_device_error(status, SCREE_DEVERR_BAD_INPUT, 41);
    return;
  }
  const int64_t c0 = (int64_t)blockIdx.x * kLPR * VW + cv * VW;
  const bool col_ok = c0 < F;  // F is a multiple of VW
  float m[VW], s[VW];
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    m[i] = -INFINITY;
    s[i] = 0.f;
  }
  const int64_t first = r0 + warp * kRPW + rsub;
  if (col_ok) {
    // Groups of G steps: one max update and one rescale per group, the group's
    // loads issued together (G = 4 rows of loads in flight per thread).
    constexpr int G = 4;
    int64_t r = first;
#pragma unroll 1
    for (; r + (G - 1) * kRPC < r1; r += G * kRPC) {
      SPack<T, VW> pk[G];  // the group stays in its storage type until used
#pragma unroll
      for (int g = 0; g < G; ++g) pk[g] = *reinterpret_cast<const SPack<T, VW>*>(x + (r + g * kRPC) * F + c0);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        float v[G];
#pragma unroll
        for (int g = 0; g < G; ++g) v[g] = Cvt<T>::to_f(pk[g].v[i]);
        float mn = m[i];
#pragma unroll
        for (int g = 0; g < G; ++g) mn = fmaxf(mn, v[g]);
        const float nml = -mn * kLog2e;  // exp(a - mn) = 2^(a log2e - mn log2e)
        float acc = (m[i] == -INFINITY) ? 0.f : s[i] * ex2_approx(fmaf(m[i], kLog2e, nml));
#pragma unroll
        for (int g = 0; g < G; ++g) acc += ex2_approx(fmaf(v[g], kLog2e, nml));
        s[i] = acc;
        m[i] = mn;
      }
    }
#pragma unroll 1
    for (; r < r1; r += kRPC) {  // remaining rows one step at a time
      float v[VW];
      sload<T, VW>(x + r * F + c0, v);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float mn = fmaxf(m[i], v[i]);
        const float nml = -mn * kLog2e;
        s[i] = ((m[i] == -INFINITY) ? 0.f : s[i] * ex2_approx(fmaf(m[i], kLog2e, nml))) +
               ex2_approx(fmaf(v[i], kLog2e, nml));
        m[i] = mn;
      }
    }
  }
  // Every thread's (max, sum) is one of kRPC partials of its columns; one thread
  // per column merges the CTA's partials in a fixed order and publishes
  // (-max * log2e, 1 / sum) for pass 2.
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    sm_m[warp * kRPW + rsub][cv * VW + i] = m[i];
    sm_s[warp * kRPW + rsub][cv * VW + i] = s[i];
  }
  __syncthreads();
  if (threadIdx.x < kLPR * VW) {
    const int col = threadIdx.x;
    float mm = -INFINITY;
#pragma unroll 8
    for (int p = 0; p < kRPC; ++p) mm = fmaxf(mm, sm_m[p][col]);
    float ss = 0.f;
    const float nml = -mm * kLog2e;
#pragma unroll 8
    for (int p = 0; p < kRPC; ++p) {
      const float mp = sm_m[p][col];
      if (mp != -INFINITY) ss += sm_s[p][col] * ex2_approx(fmaf(mp, kLog2e, nml));
    }
    fin_m[col] = nml;
    fin_s[col] = 1.f / ss;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    m[i] = fin_m[cv * VW + i];  // from here on: -max * log2e
    s[i] = fin_s[cv * VW + i];
  }
  if (!col_ok) return;
#pragma unroll 2
  for (int64_t r = first; r < r1; r += kRPC) {
    float v[VW];
    sload<T, VW>(x + r * F + c0, v);
#pragma unroll
    for (int i = 0; i < VW; ++i) v[i] = ex2_approx(fmaf(v[i], kLog2e, m[i])) * s[i];
    sstore<T, VW>(y + r * F + c0, v);
  }
}

template <typename T, int VW>
__global__ void __launch_bounds__(kThreads, 4) softmax_bwd_kernel(const T* __restrict__ dy,
                                                                const T* __restrict__ y,
                                                                const void* offs, int is64,
                                                                int64_t T_, int64_t F,
                                                                T* __restrict__ dx, int* status) {
  __shared__ float sm_d[kWarps][kLPR * VW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rsub = lane / kLPR, cv = lane % kLPR;
  const int64_t b = blockIdx.y;
  const int64_t r0 = load_offset(offs, is64, b), r1 = load_offset(offs, is64, b + 1);
  if (r0 < 0 || r1 < r0 || r1 > T_) {  // malformed offsets: no access, report
    if (threadIdx.x == 0) record_device_error(status, SCREE_DEVERR_BAD_INPUT, 41);
    return;
  }
  const int64_t c0 = (int64_t)blockIdx.x * kLPR * VW + cv * VW;
  const bool col_ok = c0 < F;
  const int64_t first = r0 + warp * kRPW + rsub;
  float d[VW];
#pragma unroll
  for (int i = 0; i < VW; ++i) d[i] = 0.f;
  if (col_ok) {
    constexpr int G = 4;  // 4 rows of dy and y in flight per thread
    int64_t r = first;
    for (; r + (G - 1) * kRPC < r1; r += G * kRPC) {
      float g[G][VW], p[G][VW];
#pragma unroll
      for (int k = 0; k < G; ++k) {
        sload<T, VW>(dy + (r + k * kRPC) * F + c0, g[k]);
        sload<T, VW>(y + (r + k * kRPC) * F + c0, p[k]);
      }
#pragma unroll
      for (int k = 0; k < G; ++k)
#pragma unroll
        for (int i = 0; i < VW; ++i) d[i] = fmaf(g[k][i], p[k][i], d[i]);
    }
    for (; r < r1; r += kRPC) {
      float g[VW], p[VW];
      sload<T, VW>(dy + r * F + c0, g);
      sload<T, VW>(y + r * F + c0, p);
#pragma unroll
      for (int i = 0; i < VW; ++i) d[i] = fmaf(g[i], p[i], d[i]);
    }
  }
#pragma unroll
  for (int o = kLPR; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < VW; ++i) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
  if (rsub == 0)
#pragma unroll
    for (int i = 0; i < VW; ++i) sm_d[warp][cv * VW + i] = d[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < VW; ++i) {
    float t = 0.f;
    for (int w = 0; w < kWarps; ++w) t += sm_d[w][cv * VW + i];
    d[i] = t;
  }
  if (!col_ok) return;
  // Pass 2 walks the rows backwards: the rows pass 1 read last are re-read
  // first, while they are still in L2 (measured: 0.67 -> 0.68 of HBM; the
  // forward, whose pass 2 reads one tensor, did not gain).
  const int64_t last = first < r1 ? first + (r1 - 1 - first) / kRPC * kRPC : first - kRPC;
#pragma unroll 2
  for (int64_t r = last; r >= first; r -= kRPC) {
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
           int64_t Tn, int64_t F, void* out, cudaStream_t s) {
  int* st = device_status_ptr();
  const bool vec = (F * (int64_t)sizeof(T)) % 16 == 0 && ((uintptr_t)a % 16) == 0 &&
                   ((uintptr_t)out % 16) == 0 && (!bwd || ((uintptr_t)bb % 16) == 0);
  constexpr int VWV = 16 / sizeof(T);
  const int vw = vec ? VWV : 1;
  const int64_t cols_per_cta = kLPR * vw;
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
      if (vec) softmax_fwd_kernel<T, VWV><<<g, kThreads, 0, s>>>((const T*)a, o, is64, Tn, F, (T*)out, st);
      else softmax_fwd_kernel<T, 1><<<g, kThreads, 0, s>>>((const T*)a, o, is64, Tn, F, (T*)out, st);
    } else {
      if (vec)
        softmax_bwd_kernel<T, VWV><<<g, kThreads, 0, s>>>((const T*)a, (const T*)bb, o, is64, Tn, F, (T*)out, st);
      else
        softmax_bwd_kernel<T, 1><<<g, kThreads, 0, s>>>((const T*)a, (const T*)bb, o, is64, Tn, F, (T*)out, st);
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
    case SCREE_F16: return launch<__half>(bwd, a, bb, offs, is64, B, T, F, out, s);
    case SCREE_BF16: return launch<__nv_bfloat16>(bwd, a, bb, offs, is64, B, T, F, out, s);
    case SCREE_F32: return launch<float>(bwd, a, bb, offs, is64, B, T, F, out, s);
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
