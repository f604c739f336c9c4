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

template <typename T, int VW>
__device__ __forceinline__ void unpack_vec(const Pack<T, VW>& pk, float (&out)[VW]) {
#pragma unroll
  for (int i = 0; i < VW; ++i) out[i] = Cvt<T>::to_f(pk.v[i]);
}

// Weight (and bias) for all C columns staged in shared memory once per CTA.
template <typename WT>
__device__ __forceinline__ void stage_params(float* sm, const void* w, const void* b, int C,
                                             bool layer) {
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    sm[c] = w ? ldw<WT>(w, c) : 1.f;
    if (layer) sm[C + c] = b ? ldw<WT>(b, c) : 0.f;
  }
  __syncthreads();
}

// ------------------------------------------------------------------ forward
// Row group of TPR threads, VPT vectors of VW elements per thread, R rows per
// iteration (kept as packed 16-bit registers until the statistics are known).
//   rmsnorm:   r = 1/sqrt(mean(x^2) + eps),        y = x r w
//   layernorm: mean, biased var from (n, mean, M2), y = (x - mean) r w + b
template <typename T, typename WT, int VW, int VPT, bool LAYER, int R>
__global__ void __launch_bounds__(kBlock) norm_fwd_kernel(
    const T* __restrict__ x, int64_t xs, const void* __restrict__ w,
    const void* __restrict__ bias, T* __restrict__ y, int64_t ys, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t rows, int C, int tpr, float eps) {
  extern __shared__ float params[];  // [C] weight, [C] bias
  __shared__ float red[2 * R * (kBlock / 32)];
  stage_params<WT>(params, w, bias, C, LAYER);
  const int rpc = kBlock / tpr;
  const int g = threadIdx.x / tpr, lt = threadIdx.x % tpr;
  const int nv = C / VW;
  const float invC = 1.0f / (float)C;
  const int64_t step = (int64_t)gridDim.x * rpc;
  const int64_t iters = (rows + R * step - 1) / (R * step);  // uniform across the CTA
  for (int64_t it = 0; it < iters; ++it) {
    int64_t row[R];
    bool live[R];
    Pack<T, VW> xr[R][VPT];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      row[k] = (R * it + k) * step + (int64_t)blockIdx.x * rpc + g;
      live[k] = row[k] < rows;
    }
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lt + i * tpr;
        if (live[k] && vi < nv)
          xr[k][i] = *reinterpret_cast<const Pack<T, VW>*>(x + row[k] * xs + (int64_t)vi * VW);
        else
#pragma unroll
          for (int e = 0; e < VW; ++e) xr[k][i].v[e] = Cvt<T>::from_f(0.f);
      }
    float mu[R], r[R];
    if (LAYER) {
      // Shifted-data variance: with K = the row's first element,
      //   mean = K + S1/C,  var = (S2 - S1^2/C)/C,  S1 = sum(x-K), S2 = sum((x-K)^2),
      // one combined reduction; the shift keeps S2 - S1^2/C free of cancellation
      // for rows whose mean is large against their spread.
      float sv[2 * R], K[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        K[k] = live[k] ? Cvt<T>::to_f(x[row[k] * xs]) : 0.f;
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; ++i)
          if (lt + i * tpr < nv) {
            float xv[VW];
            unpack_vec<T, VW>(xr[k][i], xv);
#pragma unroll
            for (int e = 0; e < VW; ++e) {
              const float d = xv[e] - K[k];
              s1 += d;
              s2 = fmaf(d, d, s2);
            }
          }
        sv[2 * k] = s1;
        sv[2 * k + 1] = s2;
      }
      group_sum<2 * R>(sv, tpr, red);
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const float d1 = sv[2 * k] * invC;
        mu[k] = K[k] + d1;
        const float var = fmaxf(sv[2 * k + 1] * invC - d1 * d1, 0.f);
        r[k] = 1.0f / sqrtf(var + eps);
      }
    } else {
      float ss[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        ss[k] = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          float xv[VW];
          unpack_vec<T, VW>(xr[k][i], xv);
#pragma unroll
          for (int e = 0; e < VW; ++e) ss[k] = fmaf(xv[e], xv[e], ss[k]);
        }
      }
      group_sum<R>(ss, tpr, red);
#pragma unroll
      for (int k = 0; k < R; ++k) {
        mu[k] = 0.f;
        r[k] = 1.0f / sqrtf(ss[k] * invC + eps);
      }
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (!live[k]) continue;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int vi = lt + i * tpr;
        if (vi < nv) {
          float xv[VW], out[VW];
          unpack_vec<T, VW>(xr[k][i], xv);
          const float* wp = params + vi * VW;
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            const float t = (xv[e] - mu[k]) * r[k] * wp[e];
            out[e] = LAYER ? t + wp[C + e] : t;
          }
          store_vec<T, VW>(y + row[k] * ys + (int64_t)vi * VW, out);
        }
      }
      if (lt == 0) {
        if (rstd_out) rstd_out[row[k]] = r[k];
        if (LAYER && mean_out) mean_out[row[k]] = mu[k];
      }
    }
  }
}

// ------------------------------------------------------------------ backward
// g = dy * w, xhat = (x - mu) * r
//   rmsnorm:   dx = r * (g - xhat * mean(g * xhat))
//   layernorm: dx = r * (g - mean(g) - xhat * mean(g * xhat))
//   dweight = sum_rows dy * xhat,  dbias = sum_rows dy
// x and dy stay packed in registers; the weight comes from shared memory; the
// per-thread dweight / dbias partials are written to `part_*` at the end.
template <typename T, typename WT, int VW, int VPT, bool LAYER>
__global__ void __launch_bounds__(kBlock) norm_bwd_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const void* __restrict__ w,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, T* __restrict__ dx,
    float* __restrict__ part_w, float* __restrict__ part_b, int64_t rows, int C, int tpr) {
  extern __shared__ float params[];  // [C] weight
  __shared__ float red[2 * (kBlock / 32)];
  stage_params<WT>(params, w, nullptr, C, false);
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
    Pack<T, VW> xr[VPT], dr[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lt + i * tpr;
      if (live && vi < nv) {
        xr[i] = *reinterpret_cast<const Pack<T, VW>*>(x + row * (int64_t)C + (int64_t)vi * VW);
        dr[i] = *reinterpret_cast<const Pack<T, VW>*>(dy + row * (int64_t)C + (int64_t)vi * VW);
      } else {
#pragma unroll
        for (int e = 0; e < VW; ++e) xr[i].v[e] = dr[i].v[e] = Cvt<T>::from_f(0.f);
      }
    }
    float s[2] = {0.f, 0.f};  // sum(g), sum(g * xhat)
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int vi = lt + i * tpr;
      if (vi < nv) {
        float xx[VW], dd[VW];
        unpack_vec<T, VW>(xr[i], xx);
        unpack_vec<T, VW>(dr[i], dd);
        const float* wp = params + vi * VW;
#pragma unroll
        for (int e = 0; e < VW; ++e) {
          const float xh = (xx[e] - mu) * r;
          const float gv = dd[e] * wp[e];
          accw[i][e] = fmaf(dd[e], xh, accw[i][e]);
          if (LAYER) accb[i][e] += dd[e];
          s[0] += gv;
          s[1] = fmaf(gv, xh, s[1]);
        }
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
          float xx[VW], dd[VW], out[VW];
          unpack_vec<T, VW>(xr[i], xx);
          unpack_vec<T, VW>(dr[i], dd);
          const float* wp = params + vi * VW;
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            const float xh = (xx[e] - mu) * r;
            out[e] = r * (dd[e] * wp[e] - mg - xh * mgx);
          }
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
  int rows_per_iter;  // forward: rows a row group loads before reducing (1 or 2)
  int smem;           // dynamic shared memory: staged weight (and bias)
  bool ok;
};

Plan plan_for(int64_t rows, int64_t C, int esize, bool aligned16, int max_vpt, bool bwd,
              bool layer = false) {
  Plan p{};
  p.vw = (aligned16 && (C * esize) % 16 == 0) ? 16 / esize : 1;
  const int64_t nv = C / p.vw;
  // Prefer few vectors per thread (registers for x and, in the backward, dy and
  // the partial sums); wider rows use more threads.
  const int target_vpt = bwd ? (layer ? 2 : 4) : 4;  // layernorm bwd carries dbias too
  int tpr = 32;
  while (tpr < kBlock && (nv + tpr - 1) / tpr > target_vpt) tpr <<= 1;
  while (tpr < 1024 && (nv + tpr - 1) / tpr > max_vpt) tpr <<= 1;
  int64_t vpt = (nv + tpr - 1) / tpr;
  int v = 1;
  while (v < vpt) v <<= 1;
  p.ok = v <= max_vpt && tpr <= kBlock * 4;
  // Rows are handled by one CTA of kBlock threads; wider rows are rejected.
  if (tpr > kBlock) p.ok = false;
  p.tpr = tpr;
  p.vpt = v;
  if (!p.ok) {  // rows too wide for one CTA: rejected by the caller
    p.grid = 1;
    return p;
  }
  const int rpc = kBlock / tpr;
  const int64_t need = (rows + rpc - 1) / rpc;
  // Grids measured best at cfg3 (hidden 4096): 4 CTAs per SM forward, 2 backward
  // (fewer dweight partial rows); launches also cap at the real occupancy.
  const int64_t cap = (int64_t)num_sms() * (bwd ? 2 : 4);
  p.rows_per_iter = 1;
  // Staged parameters: weight (+ bias in the layernorm forward, sized for both).
  p.smem = (int)(C * sizeof(float) * (bwd ? 1 : 2));
  if (p.smem > 200 * 1024) p.ok = false;
  p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, cap));
  return p;
}

// Launch with the plan's dynamic shared memory (opting in above 48 KB).
template <typename K, typename... Args>
void launch_smem(K kernel, Plan& p, cudaStream_t s, Args... args) {
  if (p.smem > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
  // No more CTAs than fit at once (a second partial wave would idle most SMs):
  // the kernels grid-stride over rows, so any grid is correct.
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kBlock, p.smem) == cudaSuccess &&
      occ > 0)
    p.grid = std::max(1, std::min(p.grid, occ * num_sms()));
  kernel<<<p.grid, kBlock, p.smem, s>>>(args...);
}

template <typename T, typename WT, int VW, bool LAYER>
int launch_fwd_vpt(Plan& p, cudaStream_t s, const void* x, int64_t xs, const void* w,
                   const void* b, void* y, int64_t ys, float* mean, float* rstd, int64_t rows,
                   int C, float eps) {
#define SCREE_FWD(V)                                                                        \
  if (p.rows_per_iter == 1)                                                                 \
    launch_smem(norm_fwd_kernel<T, WT, VW, V, LAYER, 1>, p, s,                              \
        (const T*)x, xs, w, b, (T*)y, ys, mean, rstd, rows, C, p.tpr, eps);                 \
  else                                                                                      \
    launch_smem(norm_fwd_kernel<T, WT, VW, V, LAYER, 2>, p, s,                              \
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
int launch_fwd(Plan& p, cudaStream_t s, const void* x, int64_t xs, const void* w,
               const void* b, void* y, int64_t ys, float* mean, float* rstd, int64_t rows, int C,
               float eps) {
  if (p.vw == 1) return launch_fwd_vpt<T, WT, 1, LAYER>(p, s, x, xs, w, b, y, ys, mean, rstd, rows, C, eps);
  return launch_fwd_vpt<T, WT, 16 / sizeof(T), LAYER>(p, s, x, xs, w, b, y, ys, mean, rstd, rows, C, eps);
}

template <typename T, typename WT, int VW, bool LAYER>
int launch_bwd_vpt(Plan& p, cudaStream_t s, const void* dy, const void* x, const void* w,
                   const float* mean, const float* rstd, void* dx, float* pw, float* pb,
                   int64_t rows, int C) {
#define SCREE_BWD(V)                                                                       \
  launch_smem(norm_bwd_kernel<T, WT, VW, V, LAYER>, p, s,                                   \
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
int launch_bwd(Plan& p, cudaStream_t s, const void* dy, const void* x, const void* w,
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
  // Partial rows = grid x rows per CTA of the backward plan; the maximum over
  // the 16-bit and 32-bit layouts (and over aligned / unaligned access).
  int64_t best = 1;
  for (int es : {2, 4})
    for (bool a16 : {true, false}) {
      Plan p = plan_for(rows, C, es, a16, 4, true, false);  // layernorm plans use fewer rows/CTA
      if (p.ok) best = std::max<int64_t>(best, (int64_t)p.grid * (kBlock / p.tpr));
    }
  return best;
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
  Plan p = plan_for(rows, C, es, a16, 4, true, LAYER);
  if (!p.ok) {
    set_last_error("norm bwd: feature dim %lld too large", (long long)C);
    return SCREE_ERR_UNSUPPORTED;
  }
  // Partial rows: one per row group of the planned grid (the launch may use
  // fewer CTAs, then fewer rows are written and reduced).
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
    column_sum_kernel<<<cgrid, 256, 0, s>>>(pw, (int64_t)p.grid * (kBlock / p.tpr), (int)C, dw);
    SCREE_LAUNCH_CHECK();
  }
  if (want_b) {
    column_sum_kernel<<<cgrid, 256, 0, s>>>(pb, (int64_t)p.grid * (kBlock / p.tpr), (int)C, db);
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
