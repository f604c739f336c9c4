// norms.cu — varlen RMSNorm / LayerNorm forward and backward.
//
// Norms are per-token, so the packed (T, C) buffer is processed row by row; the
// offsets are never needed (scree/kernels/triton/varlen_rmsnorm.py:7-8 makes
// the same observation).  Numerics follow the reference oracle:
//   rmsnorm   y = x / sqrt(mean(x^2) + eps) * w          reference/varlen_rmsnorm.py:58-65
//   layernorm y = (x - mu) / sqrt(var + eps) * w + b      reference/varlen_layernorm.py:64-74
// with biased variance, fp32 statistics and the weight used in its own dtype.
//
// Layout: a row is split over TPR threads (a "row group", TPR a power of two
// >= 32), each thread holding VPT vectors of VW elements in registers, so x is
// read exactly once.  Vectors are 16 bytes whenever C and the row strides allow.
// Backward: dx per row, and dweight/dbias as per-thread fp32 partial sums over
// the rows a thread visits, written to a workspace and reduced column-wise by a
// second kernel in a fixed order (deterministic, no atomics).
#include <algorithm>
#include "common.cuh"

namespace scree {
namespace {

constexpr int kBlock = 256;

template <typename T, int VW> struct alignas(sizeof(T) * VW) Pack { T v[VW]; };

template <typename T, int VW>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[VW]) {
  Pack<T, VW> pk = *reinterpret_cast<const Pack<T, VW>*>(p);
#pragma unroll
  for (int i = 0; i < VW; ++i) out[i] = Cvt<T>::to_f(pk.v[i]);
}
template <typename T, int VW>
__device__ __forceinline__ void store_vec(T* p, const float (&in)[VW]) {
  Pack<T, VW> pk;
#pragma unroll
  for (int i = 0; i < VW; ++i) pk.v[i] = Cvt<T>::from_f(in[i]);
  *reinterpret_cast<Pack<T, VW>*>(p) = pk;
}

// Sum `v` over the TPR threads of this row group.  TPR >= 32; groups of more
// than one warp combine through shared memory (`red` holds one slot per warp).
template <int NV>
__device__ __forceinline__ void group_sum(float (&v)[NV], int tpr, float* red) {
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[k] += __shfl_xor_sync(0xffffffff, v[k], o);
  if (tpr > 32) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpg = tpr >> 5, g0 = (warp / wpg) * wpg;
    __syncthreads();
    if (lane == 0)
#pragma unroll
      for (int k = 0; k < NV; ++k) red[k * (kBlock / 32) + warp] = v[k];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      float s = 0.f;
      for (int w = 0; w < wpg; ++w) s += red[k * (kBlock / 32) + g0 + w];
      v[k] = s;
    }
  }
}

template <typename WT>
__device__ __forceinline__ float ldw(const void* w, int64_t c) {
  return Cvt<WT>::to_f(reinterpret_cast<const WT*>(w)[c]);
}

// ------------------------------------------------------------------ forward
template <typename T, typename WT, int VW, int VPT, bool LAYER>
__global__ void __launch_bounds__(kBlock) norm_fwd_kernel(
    const T* __restrict__ x, int64_t xs, const void* __restrict__ w,
    const void* __restrict__ bias, T* __restrict__ y, int64_t ys, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t rows, int C, int tpr, float eps) {
  __shared__ float red[2 * (kBlock / 32)];
  const int rpc = kBlock / tpr;
  const int g = threadIdx.x / tpr, lt = threadIdx.x % tpr;
  const int nv = C / VW;
  const float invC = 1.0f / (float)C;
  // Uniform trip count across the CTA (group_sum has __syncthreads).
  const int64_t iters = (rows + (int64_t)gridDim.x * rpc - 1) / ((int64_t)gridDim.x * rpc);
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t row = (it * gridDim.x + blockIdx.x) * rpc + g;
    const bool live = row < rows;
    float xv[VPT][VW];
    float s[1] = {0.f};
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lt + i * tpr;
      if (live && vi < nv) {
        load_vec<T, VW>(x + row * xs + (int64_t)vi * VW, xv[i]);
      } else {
#pragma unroll
        for (int e = 0; e < VW; ++e) xv[i][e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < VW; ++e) s[0] += LAYER ? xv[i][e] : xv[i][e] * xv[i][e];
    }
    group_sum<1>(s, tpr, red);
    float mu = 0.f, r;
    if (LAYER) {
      mu = s[0] * invC;
      float q[1] = {0.f};
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lt + i * tpr;
        if (vi < nv)
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            float d = xv[i][e] - mu;
            q[0] += d * d;
          }
      }
      group_sum<1>(q, tpr, red + (kBlock / 32));
      r = 1.0f / sqrtf(q[0] * invC + eps);
    } else {
      r = 1.0f / sqrtf(s[0] * invC + eps);
    }
    if (live) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lt + i * tpr;
        if (vi < nv) {
          float out[VW];
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            const int64_t c = (int64_t)vi * VW + e;
            float t = (xv[i][e] - mu) * r;
            if (w) t *= ldw<WT>(w, c);
            if (LAYER && bias) t += ldw<WT>(bias, c);
            out[e] = t;
          }
          store_vec<T, VW>(y + row * ys + (int64_t)vi * VW, out);
        }
      }
      if (lt == 0) {
        if (rstd_out) rstd_out[row] = r;
        if (LAYER && mean_out) mean_out[row] = mu;
      }
    }
  }
}

// ------------------------------------------------------------------ backward
// g = dy * w, xhat = (x - mu) * r
//   rmsnorm:   dx = r * (g - xhat * mean(g * xhat))
//   layernorm: dx = r * (g - mean(g) - xhat * mean(g * xhat))
//   dweight = sum_rows dy * xhat,  dbias = sum_rows dy
template <typename T, typename WT, int VW, int VPT, bool LAYER>
__global__ void __launch_bounds__(kBlock) norm_bwd_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const void* __restrict__ w,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, T* __restrict__ dx,
    float* __restrict__ part_w, float* __restrict__ part_b, int64_t rows, int C, int tpr) {
  __shared__ float red[2 * (kBlock / 32)];
  const int rpc = kBlock / tpr;
  const int g = threadIdx.x / tpr, lt = threadIdx.x % tpr;
  const int nv = C / VW;
  const float invC = 1.0f / (float)C;
  float accw[VPT][VW], accb[VPT][VW];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int e = 0; e < VW; ++e) accw[i][e] = accb[i][e] = 0.f;
  const int64_t iters = (rows + (int64_t)gridDim.x * rpc - 1) / ((int64_t)gridDim.x * rpc);
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t row = (it * gridDim.x + blockIdx.x) * rpc + g;
    const bool live = row < rows;
    const float r = live ? rstd_in[row] : 0.f;
    const float mu = (LAYER && live) ? mean_in[row] : 0.f;
    float xh[VPT][VW], gv[VPT][VW];
    float s[2] = {0.f, 0.f};  // sum(g), sum(g * xhat)
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lt + i * tpr;
      if (live && vi < nv) {
        float xx[VW], dd[VW];
        load_vec<T, VW>(x + row * (int64_t)C + (int64_t)vi * VW, xx);
        load_vec<T, VW>(dy + row * (int64_t)C + (int64_t)vi * VW, dd);
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          const int64_t c = (int64_t)vi * VW + e;
          xh[i][e] = (xx[e] - mu) * r;
          gv[i][e] = w ? dd[e] * ldw<WT>(w, c) : dd[e];
          accw[i][e] += dd[e] * xh[i][e];
          if (LAYER) accb[i][e] += dd[e];
          s[0] += gv[i][e];
          s[1] += gv[i][e] * xh[i][e];
        }
      } else {
#pragma unroll
        for (int e = 0; e < VW; ++e) xh[i][e] = gv[i][e] = 0.f;
      }
    }
    group_sum<2>(s, tpr, red);
    const float mg = LAYER ? s[0] * invC : 0.f;
    const float mgx = s[1] * invC;
    if (live) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lt + i * tpr;
        if (vi < nv) {
          float out[VW];
#pragma unroll
          for (int e = 0; e < VW; ++e) out[e] = r * (gv[i][e] - mg - xh[i][e] * mgx);
          store_vec<T, VW>(dx + row * (int64_t)C + (int64_t)vi * VW, out);
        }
      }
    }
  }
  if (part_w) {
    const int64_t prow = (int64_t)blockIdx.x * rpc + g;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lt + i * tpr;
      if (vi < nv)
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          part_w[prow * C + (int64_t)vi * VW + e] = accw[i][e];
          if (LAYER && part_b) part_b[prow * C + (int64_t)vi * VW + e] = accb[i][e];
        }
    }
  }
}

// Column sums of a (P, C) fp32 partial matrix: 32 columns x 8 row lanes per
// CTA, fixed summation order.
__global__ void __launch_bounds__(256) column_sum_kernel(const float* __restrict__ part,
                                                         int64_t P, int C,
                                                         float* __restrict__ out) {
  __shared__ float sm[8][33];
  const int cx = threadIdx.x & 31, ry = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + cx;
  float s = 0.f;
  if (c < C)
    for (int64_t p = ry; p < P; p += 8) s += part[p * C + c];
  sm[ry][cx] = s;
  __syncthreads();
  if (ry == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sm[k][cx];
    out[c] = t;
  }
}

struct Plan {
  int vw;   // elements per access
  int tpr;  // threads per row
  int vpt;  // vectors per thread
  int grid;
  bool ok;
};

Plan plan_for(int64_t rows, int64_t C, int esize, bool aligned16, int max_vpt, bool bwd) {
  Plan p{};
  p.vw = (aligned16 && (C * esize) % 16 == 0) ? 16 / esize : 1;
  const int64_t nv = C / p.vw;
  int tpr = 32;
  while (tpr < 1024 && (nv + tpr - 1) / tpr > max_vpt) tpr <<= 1;
  int64_t vpt = (nv + tpr - 1) / tpr;
  int v = 1;
  while (v < vpt) v <<= 1;
  p.ok = v <= max_vpt && tpr <= kBlock * 4;
  // Rows are handled by one CTA of kBlock threads; wider rows are rejected.
  if (tpr > kBlock) p.ok = false;
  p.tpr = tpr;
  p.vpt = v;
  const int rpc = kBlock / tpr;
  const int64_t need = (rows + rpc - 1) / rpc;
  const int64_t cap = (int64_t)num_sms() * (bwd ? 2 : 8);
  p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, cap));
  return p;
}

template <typename T, typename WT, int VW, bool LAYER>
int launch_fwd_vpt(const Plan& p, cudaStream_t s, const void* x, int64_t xs, const void* w,
                   const void* b, void* y, int64_t ys, float* mean, float* rstd, int64_t rows,
                   int C, float eps) {
#define SCREE_FWD(V)                                                                        \
  norm_fwd_kernel<T, WT, VW, V, LAYER><<<p.grid, kBlock, 0, s>>>(                           \
      (const T*)x, xs, w, b, (T*)y, ys, mean, rstd, rows, C, p.tpr, eps)
  ProfScope prof(PROF_NORM_FWD, s);
  switch (p.vpt) {
    case 1: SCREE_FWD(1); break;
    case 2: SCREE_FWD(2); break;
    case 4: SCREE_FWD(4); break;
    case 8: SCREE_FWD(8); break;
    default: SCREE_FWD(16); break;
  }
#undef SCREE_FWD
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

template <typename T, typename WT, bool LAYER>
int launch_fwd(const Plan& p, cudaStream_t s, const void* x, int64_t xs, const void* w,
               const void* b, void* y, int64_t ys, float* mean, float* rstd, int64_t rows, int C,
               float eps) {
  if (p.vw == 1) return launch_fwd_vpt<T, WT, 1, LAYER>(p, s, x, xs, w, b, y, ys, mean, rstd, rows, C, eps);
  return launch_fwd_vpt<T, WT, 16 / sizeof(T), LAYER>(p, s, x, xs, w, b, y, ys, mean, rstd, rows, C, eps);
}

template <typename T, typename WT, int VW, bool LAYER>
int launch_bwd_vpt(const Plan& p, cudaStream_t s, const void* dy, const void* x, const void* w,
                   const float* mean, const float* rstd, void* dx, float* pw, float* pb,
                   int64_t rows, int C) {
#define SCREE_BWD(V)                                                                       \
  norm_bwd_kernel<T, WT, VW, V, LAYER><<<p.grid, kBlock, 0, s>>>(                          \
      (const T*)dy, (const T*)x, w, mean, rstd, (T*)dx, pw, pb, rows, C, p.tpr)
  ProfScope prof(PROF_NORM_BWD, s);
  switch (p.vpt) {
    case 1: SCREE_BWD(1); break;
    case 2: SCREE_BWD(2); break;
    default: SCREE_BWD(4); break;
  }
#undef SCREE_BWD
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

template <typename T, typename WT, bool LAYER>
int launch_bwd(const Plan& p, cudaStream_t s, const void* dy, const void* x, const void* w,
               const float* mean, const float* rstd, void* dx, float* pw, float* pb,
               int64_t rows, int C) {
  if (p.vw == 1) return launch_bwd_vpt<T, WT, 1, LAYER>(p, s, dy, x, w, mean, rstd, dx, pw, pb, rows, C);
  return launch_bwd_vpt<T, WT, 16 / sizeof(T), LAYER>(p, s, dy, x, w, mean, rstd, dx, pw, pb, rows, C);
}

// Dispatch over (x dtype, weight dtype).
template <bool LAYER, typename F>
int dispatch_types(int dtype, int w_dtype, F&& f) {
#define SCREE_W(T)                                                             \
  switch (w_dtype) {                                                           \
    case SCREE_F16: return f((T*)nullptr, (__half*)nullptr);                   \
    case SCREE_BF16: return f((T*)nullptr, (__nv_bfloat16*)nullptr);           \
    case SCREE_F32: return f((T*)nullptr, (float*)nullptr);                    \
    default: break;                                                            \
  }
  switch (dtype) {
    case SCREE_F16: SCREE_W(__half); break;
    case SCREE_BF16: SCREE_W(__nv_bfloat16); break;
    case SCREE_F32: SCREE_W(float); break;
    default: break;
  }
#undef SCREE_W
  set_last_error("unsupported dtype combination (x %d, weight %d)", dtype, w_dtype);
  return SCREE_ERR_INVALID;
}

template <bool LAYER>
int norm_fwd(const void* x, int64_t xs, const void* w, const void* b, int w_dtype, void* y,
             int64_t ys, float* mean, float* rstd, int64_t rows, int64_t C, int dtype, float eps,
             void* stream) {
  SCREE_CHECK_ARG(rows >= 0 && C >= 1 && C < (1ll << 31), "norm: bad sizes rows=%lld C=%lld",
                  (long long)rows, (long long)C);
  if (rows == 0) return SCREE_OK;
  SCREE_CHECK_ARG(x && y, "norm: null x or y");
  const int es = (int)dtype_size(dtype);
  SCREE_CHECK_ARG(es > 0, "norm: bad dtype %d", dtype);
  const bool a16 = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) &&
                   ((xs * es) % 16 == 0) && ((ys * es) % 16 == 0);
  Plan p = plan_for(rows, C, es, a16, 16, false);
  if (!p.ok) {
    set_last_error("norm: feature dim %lld too large", (long long)C);
    return SCREE_ERR_UNSUPPORTED;
  }
  if (!w) w_dtype = dtype;
  SCREE_BIND_DEVICE(stream, x);
  cudaStream_t s = (cudaStream_t)stream;
  return dispatch_types<LAYER>(dtype, w_dtype, [&](auto* tp, auto* wp) {
    using T = std::remove_pointer_t<decltype(tp)>;
    using WT = std::remove_pointer_t<decltype(wp)>;
    return launch_fwd<T, WT, LAYER>(p, s, x, xs, w, b, y, ys, mean, rstd, rows, (int)C, eps);
  });
}

int64_t bwd_partials(int64_t rows, int64_t C) {
  // Upper bound over dtypes: grid <= 2 * SMs, rows per CTA <= kBlock / 32.
  (void)rows;
  return (int64_t)num_sms() * 2 * (kBlock / 32);
}

template <bool LAYER>
int norm_bwd(const void* dy, const void* x, const void* w, int w_dtype, const float* mean,
             const float* rstd, void* dx, float* dw, float* db, int64_t rows, int64_t C,
             int dtype, void* ws, size_t ws_bytes, void* stream) {
  SCREE_CHECK_ARG(rows >= 0 && C >= 1 && C < (1ll << 31), "norm bwd: bad sizes");
  SCREE_CHECK_ARG(dy && x && rstd && dx, "norm bwd: null pointer");
  SCREE_CHECK_ARG(!LAYER || mean, "layernorm bwd: mean required");
  const int es = (int)dtype_size(dtype);
  SCREE_CHECK_ARG(es > 0, "norm bwd: bad dtype %d", dtype);
  SCREE_BIND_DEVICE(stream, x);
  cudaStream_t s = (cudaStream_t)stream;
  const bool want_w = dw != nullptr, want_b = LAYER && db != nullptr;
  if (rows == 0) {
    if (want_w) SCREE_CUDA_TRY(cudaMemsetAsync(dw, 0, C * sizeof(float), s));
    if (want_b) SCREE_CUDA_TRY(cudaMemsetAsync(db, 0, C * sizeof(float), s));
    return SCREE_OK;
  }
  const bool a16 = ((uintptr_t)x % 16 == 0) && ((uintptr_t)dy % 16 == 0) &&
                   ((uintptr_t)dx % 16 == 0);
  Plan p = plan_for(rows, C, es, a16, 4, true);
  if (!p.ok) {
    set_last_error("norm bwd: feature dim %lld too large", (long long)C);
    return SCREE_ERR_UNSUPPORTED;
  }
  const int64_t P = (int64_t)p.grid * (kBlock / p.tpr);
  float* pw = nullptr;
  float* pb = nullptr;
  if (want_w || want_b) {
    const size_t need = (size_t)P * C * sizeof(float) * 2;
    SCREE_CHECK_ARG(ws && ws_bytes >= need, "norm bwd: workspace too small (%zu < %zu)",
                    ws_bytes, need);
    pw = (float*)ws;
    pb = pw + P * C;
  }
  if (!w) w_dtype = dtype;
  int rc = dispatch_types<LAYER>(dtype, w_dtype, [&](auto* tp, auto* wp) {
    using T = std::remove_pointer_t<decltype(tp)>;
    using WT = std::remove_pointer_t<decltype(wp)>;
    return launch_bwd<T, WT, LAYER>(p, s, dy, x, w, mean, rstd, dx, pw, pb, rows, (int)C);
  });
  if (rc != SCREE_OK) return rc;
  const unsigned cgrid = (unsigned)((C + 31) / 32);
  if (want_w) {
    column_sum_kernel<<<cgrid, 256, 0, s>>>(pw, P, (int)C, dw);
    SCREE_LAUNCH_CHECK();
  }
  if (want_b) {
    column_sum_kernel<<<cgrid, 256, 0, s>>>(pb, P, (int)C, db);
    SCREE_LAUNCH_CHECK();
  }
  return SCREE_OK;
}

}  // namespace
}  // namespace scree

using namespace scree;

extern "C" {

size_t scree_norm_bwd_workspace_size(int64_t rows, int64_t C) {
  return (size_t)bwd_partials(rows, C) * (size_t)C * sizeof(float) * 2;
}

int scree_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, int w_dtype,
                      void* y, int64_t y_row_stride, float* rstd, int64_t rows, int64_t C,
                      int dtype, float eps, void* stream) {
  return norm_fwd<false>(x, x_row_stride, weight, nullptr, w_dtype, y, y_row_stride, nullptr,
                         rstd, rows, C, dtype, eps, stream);
}

int scree_layernorm_fwd(const void* x, int64_t x_row_stride, const void* weight,
                        const void* bias, int w_dtype, void* y, int64_t y_row_stride,
                        float* mean, float* rstd, int64_t rows, int64_t C, int dtype, float eps,
                        void* stream) {
  return norm_fwd<true>(x, x_row_stride, weight, bias, w_dtype, y, y_row_stride, mean, rstd,
                        rows, C, dtype, eps, stream);
}

int scree_rmsnorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                      const float* rstd, void* dx, float* dweight, int64_t rows, int64_t C,
                      int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return norm_bwd<false>(dy, x, weight, w_dtype, nullptr, rstd, dx, dweight, nullptr, rows, C,
                         dtype, workspace, workspace_bytes, stream);
}

int scree_layernorm_bwd(const void* dy, const void* x, const void* weight, int w_dtype,
                        const float* mean, const float* rstd, void* dx, float* dweight,
                        float* dbias, int64_t rows, int64_t C, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return norm_bwd<true>(dy, x, weight, w_dtype, mean, rstd, dx, dweight, dbias, rows, C, dtype,
                        workspace, workspace_bytes, stream);
}

}  // extern "C"
