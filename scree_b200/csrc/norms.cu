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
#include "sm100.cuh"

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
  cvt_from_f<T, VW>(in, pk.v);
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

// Parameters for the streamed kernels, staged as VW/4 planes of float4: plane k
// holds elements 4k..4k+3 of every VW-element vector, so lanes reading
// consecutive vectors read consecutive 16 bytes (no bank conflicts).  The bias
// (layernorm forward) follows at offset C.
template <typename WT, int VW>
__device__ __forceinline__ void stage_params_planar(float* sm, const void* w, const void* b, int C,
                                                    bool layer) {
  const int nv = C / VW;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int v = c / VW, e = c % VW;
    const int idx = ((e >> 2) * nv + v) * 4 + (e & 3);
    sm[idx] = w ? ldw<WT>(w, c) : 1.f;
    if (layer) sm[C + idx] = b ? ldw<WT>(b, c) : 0.f;
  }
  __syncthreads();
}
template <int VW>
__device__ __forceinline__ void load_params(const float* planes, int nv, int v, float (&out)[VW]) {
#pragma unroll
  for (int k = 0; k < VW / 4; ++k) {
    const float4 f = reinterpret_cast<const float4*>(planes)[k * nv + v];
    out[4 * k] = f.x;
    out[4 * k + 1] = f.y;
    out[4 * k + 2] = f.z;
    out[4 * k + 3] = f.w;
  }
}

// Warp sums of N values at once (N a power of two, <= 32) by recursive halving:
// at each step a lane keeps one half of its values and sends the other half to
// its partner, so N values cost N - 1 + log2(32 / N) shuffles instead of
// 5 N.  Returns the warp-wide sum of value (lane >> (5 - log2 N)).
template <int N>
__device__ __forceinline__ float warp_sum_multi(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "N must be a power of two <= 32");
  int off = 16;
#pragma unroll
  for (int cnt = N; cnt > 1; cnt >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < cnt / 2; ++i) {
      const float send = upper ? v[i] : v[i + cnt / 2];
      const float keep = upper ? v[i + cnt / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  float t = v[0];
#pragma unroll
  for (; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  return t;
}

// ------------------------------------------------------- forward, streamed
// Rows of at least 1 KB (C = 4096 in 16-bit is 8 KB): every warp owns whole rows
// (rows warp_id, warp_id + all_warps, ...) and a private ring of `stages` row
// slots in shared memory, filled by 1-D bulk copies (cp.async.bulk) that lane 0
// issues `stages` rows ahead.  Statistics are warp shuffles only, so warps never
// wait on each other and each SM keeps (stages - 1) rows per warp in flight
// while it computes.  Pass 1 reads the slot for the statistics, pass 2 reads it
// again for y, which is stored straight from registers (16-byte vectors).
constexpr int kStreamSite = 92;

__device__ __forceinline__ bool bar_wait_drain(uint64_t* bar, uint32_t parity) {
  // Exit path only: wait (at most the same limit) for a copy still in flight so
  // the CTA never retires with a bulk copy targeting its shared memory.
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_timer_ns() - t0 > SCREE_WAIT_LIMIT_NS) return false;
  return true;
}

template <typename T, typename WT, bool LAYER>
__global__ void __launch_bounds__(2 * kBlock) norm_fwd_stream_kernel(
    const T* __restrict__ x, int64_t xs, const void* __restrict__ w,
    const void* __restrict__ bias, T* __restrict__ y, int64_t ys, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t rows, int C, int stages, float eps, int* status) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int abort_flag;
  constexpr int VW = 16 / sizeof(T);
  const int nwarps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row_bytes = (uint32_t)C * sizeof(T);
  const int nv = C / VW;
  float* params = reinterpret_cast<float*>(smem_raw);
  const size_t poff = ((size_t)C * sizeof(float) * (LAYER ? 2 : 1) + 127) & ~(size_t)127;
  unsigned char* ring = smem_raw + poff + (size_t)warp * stages * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + poff + (size_t)nwarps * stages * row_bytes) +
                   warp * stages;
  if (threadIdx.x == 0) abort_flag = 0;
  if (lane == 0)
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
  fence_mbar_init();
  stage_params_planar<WT, VW>(params, w, bias, C, LAYER);  // ends with __syncthreads

  const int64_t NW = (int64_t)gridDim.x * nwarps;
  const int64_t gw = (int64_t)blockIdx.x * nwarps + warp;
  if (lane == 0)
    for (int s = 0; s < stages; ++s) {
      const int64_t r = gw + s * NW;
      if (r >= rows) break;
      mbar_expect_tx(&bars[s], row_bytes);
      bulk_load_1d(ring + (size_t)s * row_bytes, x + r * xs, row_bytes, &bars[s]);
    }
  const float invC = 1.0f / (float)C;
  int64_t j = 0;
  bool ok = true;
  for (int64_t r = gw; r < rows; r += NW, ++j) {
    const int slot = (int)(j % stages);
    const uint32_t parity = (uint32_t)((j / stages) & 1);
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[slot], parity, &abort_flag, status, kStreamSite));
    if (!ok) break;
    const Pack<T, VW>* src = reinterpret_cast<const Pack<T, VW>*>(ring + (size_t)slot * row_bytes);
    float mu = 0.f, rs;
    if (LAYER) {
      // Shifted-data variance with K = the row's first element (see norm_fwd_kernel).
      const float K = Cvt<T>::to_f(src[0].v[0]);
      const uint64_t K2 = f2_pack(K, K);
      // One accumulator per vector element (short chains), element pairs in
      // packed f32x2 arithmetic.
      uint64_t a1[VW / 2], a2[VW / 2];
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) a1[e] = a2[e] = 0ull;
#pragma unroll 4
      for (int v = lane; v < nv; v += 32) {
        float xv[VW];
        const Pack<T, VW> pk = src[v];  // one 16-byte shared load
        unpack_vec<T, VW>(pk, xv);
#pragma unroll
        for (int e = 0; e < VW / 2; ++e) {
          const uint64_t d = f2_sub(f2_pack(xv[2 * e], xv[2 * e + 1]), K2);
          a1[e] = f2_add(a1[e], d);
          a2[e] = f2_fma(d, d, a2[e]);
        }
      }
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) {
        float p0, p1, q0, q1;
        f2_unpack(a1[e], p0, p1);
        f2_unpack(a2[e], q0, q1);
        s1 += p0;
        s1 += p1;
        s2 += q0;
        s2 += q1;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
        s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      }
      const float d1 = s1 * invC;
      mu = K + d1;
      rs = 1.0f / sqrtf(fmaxf(s2 * invC - d1 * d1, 0.f) + eps);
    } else {
      uint64_t a2[VW / 2];
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) a2[e] = 0ull;
#pragma unroll 4
      for (int v = lane; v < nv; v += 32) {
        float xv[VW];
        const Pack<T, VW> pk = src[v];  // one 16-byte shared load
        unpack_vec<T, VW>(pk, xv);
#pragma unroll
        for (int e = 0; e < VW / 2; ++e) {
          const uint64_t x2 = f2_pack(xv[2 * e], xv[2 * e + 1]);
          a2[e] = f2_fma(x2, x2, a2[e]);
        }
      }
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) {
        float q0, q1;
        f2_unpack(a2[e], q0, q1);
        ss += q0;
        ss += q1;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      rs = 1.0f / sqrtf(ss * invC + eps);
    }
    T* dst = y + r * ys;
    const uint64_t mu2 = f2_pack(mu, mu), rs2 = f2_pack(rs, rs);
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) {
      float xv[VW], out[VW], wv[VW], bv[VW];
      const Pack<T, VW> pk = src[v];
      unpack_vec<T, VW>(pk, xv);
      load_params<VW>(params, nv, v, wv);
      if (LAYER) load_params<VW>(params + C, nv, v, bv);
#pragma unroll
      for (int e = 0; e < VW / 2; ++e) {  // ((x - mu) * rs) * w (+ b), per lane as in scalar code
        uint64_t x2 = f2_pack(xv[2 * e], xv[2 * e + 1]);
        if (LAYER) x2 = f2_sub(x2, mu2);
        uint64_t t = f2_mul(f2_mul(x2, rs2), f2_pack(wv[2 * e], wv[2 * e + 1]));
        if (LAYER) t = f2_add(t, f2_pack(bv[2 * e], bv[2 * e + 1]));
        f2_unpack(t, out[2 * e], out[2 * e + 1]);
      }
      store_vec<T, VW>(dst + (int64_t)v * VW, out);
    }
    if (lane == 0) {
      if (rstd_out) rstd_out[r] = rs;
      if (LAYER && mean_out) mean_out[r] = mu;
    }
    __syncwarp();
    if (lane == 0) {
      const int64_t rn = r + stages * NW;
      if (rn < rows) {
        fence_proxy_async_smem();  // this warp's reads of the slot precede the refill
        mbar_expect_tx(&bars[slot], row_bytes);
        bulk_load_1d(ring + (size_t)slot * row_bytes, x + rn * xs, row_bytes, &bars[slot]);
      }
    }
  }
  if (!ok && lane == 0) {
    // Copies issued for rows j .. j + stages - 1 may still be in flight.
    for (int64_t k = j; k < j + stages; ++k) {
      if (gw + k * NW >= rows) break;
      if (!bar_wait_drain(&bars[k % stages], (uint32_t)((k / stages) & 1))) break;
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

// ------------------------------------------------------ backward, streamed
// Rows of 256..1024 16-byte vectors (C = 2048..8192 in 16-bit): one CTA of NT
// (256, or 512 for rows of at least 512 vectors) threads per SM walks blocks of
// R consecutive rows (blocks blockIdx.x, blockIdx.x + gridDim.x, ...).  x and dy of a block arrive in a shared-memory
// ring slot by two 1-D bulk copies; thread t owns vectors t, t + 256, ... of every
// row, so its dweight / dbias partials stay in registers for the whole kernel.
// One barrier per block: warps publish their 2R row sums into a double-buffered
// slot, and after the barrier every thread of the CTA has finished the previous
// block, so thread 0 refills that block's ring slot.
constexpr int kBwdStreamSite = 93;

template <typename T, typename WT, int NT, int VPT, int R, bool LAYER>
__global__ void __launch_bounds__(NT, 1) norm_bwd_stream_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const void* __restrict__ w,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, T* __restrict__ dx,
    float* __restrict__ part_w, float* __restrict__ part_b, int64_t rows, int C, int stages,
    int* status) {
  constexpr int VW = 16 / sizeof(T);
  constexpr int NWARP = NT / 32;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ float red[2][NWARP][2 * R];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = C / VW;
  const uint32_t row_bytes = (uint32_t)C * sizeof(T);
  const uint32_t slot_bytes = 2u * R * row_bytes;  // [R rows of x][R rows of dy]
  float* params = reinterpret_cast<float*>(smem_raw);
  const size_t poff = ((size_t)C * sizeof(float) + 127) & ~(size_t)127;
  unsigned char* ring = smem_raw + poff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + (size_t)stages * slot_bytes);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  stage_params_planar<WT, VW>(params, w, nullptr, C, false);  // ends with __syncthreads

  const int64_t nblocks = (rows + R - 1) / R;
  auto issue = [&](int64_t blk, int slot) {
    const int64_t r0 = blk * R;
    const uint32_t n = (uint32_t)(rows - r0 < R ? rows - r0 : (int64_t)R) * row_bytes;
    unsigned char* dst = ring + (size_t)slot * slot_bytes;
    mbar_expect_tx(&bars[slot], 2 * n);
    bulk_load_1d(dst, x + r0 * C, n, &bars[slot]);
    bulk_load_1d(dst + (size_t)R * row_bytes, dy + r0 * C, n, &bars[slot]);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < stages; ++s) {
      const int64_t blk = blockIdx.x + (int64_t)s * gridDim.x;
      if (blk >= nblocks) break;
      issue(blk, s);
    }

  const float invC = 1.0f / (float)C;
  // Element pairs in packed f32x2 arithmetic (one instruction per pair, each
  // lane rounded exactly as the scalar operation would be).
  static_assert(VW % 2 == 0, "pairs of elements");
  uint64_t accw[VPT][VW / 2], accb[VPT][VW / 2];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int e = 0; e < VW / 2; ++e) accw[i][e] = accb[i][e] = 0ull;

  // The row statistics of block j + 1 are loaded while block j is processed,
  // so their latency is not exposed when the ring slot is already full.
  float rs_n[R], mu_n[R];
  auto load_stats = [&](int64_t blk) {
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t r = blk * R + k;
      const bool live = blk < nblocks && r < rows;
      rs_n[k] = live ? rstd_in[r] : 0.f;
      mu_n[k] = (LAYER && live) ? mean_in[r] : 0.f;
    }
  };
  load_stats(blockIdx.x);
  int64_t j = 0;
  bool ok = true;
  for (int64_t blk = blockIdx.x; blk < nblocks; blk += gridDim.x, ++j) {
    const int slot = (int)(j % stages);
    const int64_t r0 = blk * R;
    float rs[R], mu[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      rs[k] = rs_n[k];
      mu[k] = mu_n[k];
    }
    load_stats(blk + gridDim.x);
    ok = mbar_wait(&bars[slot], (uint32_t)((j / stages) & 1), &abort_flag, status, kBwdStreamSite);
    ok = __syncthreads_and(ok);
    if (!ok) break;
    const unsigned char* sl = ring + (size_t)slot * slot_bytes;
    float sums[2 * R];  // per row: sum(g), sum(g * xhat)
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const Pack<T, VW>* xr = reinterpret_cast<const Pack<T, VW>*>(sl + (size_t)k * row_bytes);
      const Pack<T, VW>* dr = reinterpret_cast<const Pack<T, VW>*>(sl + (size_t)(R + k) * row_bytes);
      const bool live = r0 + k < rows;
      const uint64_t mu2 = f2_pack(mu[k], mu[k]), rs2 = f2_pack(rs[k], rs[k]);
      uint64_t s0 = 0ull, s1 = 0ull;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int v = threadIdx.x + i * NT;
        if (live && v < nv) {
          float xx[VW], dd[VW], wp[VW];
          const Pack<T, VW> px = xr[v], pd = dr[v];  // 16-byte shared loads
          unpack_vec<T, VW>(px, xx);
          unpack_vec<T, VW>(pd, dd);
          load_params<VW>(params, nv, v, wp);
#pragma unroll
          for (int e = 0; e < VW / 2; ++e) {
            const uint64_t x2 = f2_pack(xx[2 * e], xx[2 * e + 1]);
            const uint64_t d2 = f2_pack(dd[2 * e], dd[2 * e + 1]);
            const uint64_t xh = f2_mul(f2_sub(x2, mu2), rs2);
            const uint64_t gv = f2_mul(d2, f2_pack(wp[2 * e], wp[2 * e + 1]));
            accw[i][e] = f2_fma(d2, xh, accw[i][e]);
            if (LAYER) accb[i][e] = f2_add(accb[i][e], d2);
            s0 = f2_add(s0, gv);
            s1 = f2_fma(gv, xh, s1);
          }
        }
      }
      float a0, a1, b0, b1;
      f2_unpack(s0, a0, a1);
      f2_unpack(s1, b0, b1);
      sums[2 * k] = a0 + a1;
      sums[2 * k + 1] = b0 + b1;
    }
    constexpr int Q2 = 2 * R, LPQ = 32 / Q2;  // lanes per row sum
    const int buf = (int)(j & 1);
    {
      const float t = warp_sum_multi<Q2>(sums, lane);  // sum #(lane / LPQ)
      if (lane % LPQ == 0) red[buf][warp][lane / LPQ] = t;
    }
    __syncthreads();
    // Every thread is past the previous block: its slot can be refilled.
    if (threadIdx.x == 0 && j > 0) {
      const int64_t nb = blk - gridDim.x + (int64_t)stages * gridDim.x;
      if (nb < nblocks) {
        fence_proxy_async_smem();
        issue(nb, (int)((j - 1) % stages));
      }
    }
    {
      // Lanes split the (sum, warp) pairs, reduce, and broadcast the totals.
      const int q = lane / LPQ, g = lane % LPQ;
      float t = 0.f;
#pragma unroll
      for (int wv = g; wv < NWARP; wv += LPQ) t += red[buf][wv][q];
#pragma unroll
      for (int o = LPQ / 2; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
#pragma unroll
      for (int qq = 0; qq < Q2; ++qq) sums[qq] = __shfl_sync(0xffffffffu, t, qq * LPQ);
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (r0 + k >= rows) break;
      const Pack<T, VW>* xr = reinterpret_cast<const Pack<T, VW>*>(sl + (size_t)k * row_bytes);
      const Pack<T, VW>* dr = reinterpret_cast<const Pack<T, VW>*>(sl + (size_t)(R + k) * row_bytes);
      const float mg = LAYER ? sums[2 * k] * invC : 0.f;
      const float mgx = sums[2 * k + 1] * invC;
      const uint64_t mu2 = f2_pack(mu[k], mu[k]), rs2 = f2_pack(rs[k], rs[k]);
      const uint64_t mg2 = f2_pack(mg, mg), nmgx2 = f2_pack(-mgx, -mgx);
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int v = threadIdx.x + i * NT;
        if (v < nv) {
          float xx[VW], dd[VW], out[VW], wp[VW];
          const Pack<T, VW> px = xr[v], pd = dr[v];
          unpack_vec<T, VW>(px, xx);
          unpack_vec<T, VW>(pd, dd);
          load_params<VW>(params, nv, v, wp);
#pragma unroll
          for (int e = 0; e < VW / 2; ++e) {
            const uint64_t xh =
                f2_mul(f2_sub(f2_pack(xx[2 * e], xx[2 * e + 1]), mu2), rs2);
            const uint64_t g =
                f2_sub(f2_mul(f2_pack(dd[2 * e], dd[2 * e + 1]), f2_pack(wp[2 * e], wp[2 * e + 1])), mg2);
            f2_unpack(f2_mul(rs2, f2_fma(xh, nmgx2, g)), out[2 * e], out[2 * e + 1]);
          }
          store_vec<T, VW>(dx + (r0 + k) * (int64_t)C + (int64_t)v * VW, out);
        }
      }
    }
  }
  if (!ok) {
    if (threadIdx.x == 0)  // copies for blocks j .. j + stages - 1 may still be in flight
      for (int64_t k = j; k < j + stages; ++k) {
        if (blockIdx.x + k * gridDim.x >= nblocks) break;
        if (!bar_wait_drain(&bars[k % stages], (uint32_t)((k / stages) & 1))) break;
      }
    return;
  }
  if (part_w) {
    const int64_t prow = blockIdx.x;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int v = threadIdx.x + i * NT;
      if (v < nv)
#pragma unroll
        for (int e = 0; e < VW / 2; ++e) {
          float w0, w1, b0, b1;
          f2_unpack(accw[i][e], w0, w1);
          f2_unpack(accb[i][e], b0, b1);
          part_w[prow * C + (int64_t)v * VW + 2 * e] = w0;
          part_w[prow * C + (int64_t)v * VW + 2 * e + 1] = w1;
          if (LAYER && part_b) {
            part_b[prow * C + (int64_t)v * VW + 2 * e] = b0;
            part_b[prow * C + (int64_t)v * VW + 2 * e + 1] = b1;
          }
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
  launch_smem(norm_fwd_kernel<T, WT, VW, V, LAYER, 1>, p, s,                                \
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

// Streamed forward plan: 12, 8 or 4 warps with 2 or 3 row slots each,
// whatever fits next to the staged parameters; 0 stages = use norm_fwd_kernel.
struct StreamPlan {
  int warps, stages, smem, grid;
};
StreamPlan stream_plan(int64_t rows, int64_t C, int esize, bool aligned16, bool layer) {
  StreamPlan sp{0, 0, 0, 0};
  const int64_t row_bytes = C * esize;
  if (!aligned16 || row_bytes % 16 != 0 || row_bytes < 1024 || row_bytes > 64 * 1024) return sp;
  const int64_t params = ((C * 4 * (layer ? 2 : 1)) + 127) & ~int64_t(127);
  const int64_t limit = 227 * 1024 - 64;  // opt-in maximum minus static shared memory
  // (warps, row slots) in order of preference: 12 x 2 measured faster than 8 x 3
  // for RMSNorm at C = 4096 (more warps, same shared memory), equal for LayerNorm.
  const int cand[5][2] = {{12, 2}, {8, 3}, {8, 2}, {4, 3}, {4, 2}};
  for (const auto& c : cand) {
    const int64_t need = params + (int64_t)c[0] * c[1] * (row_bytes + 8);
    if (need <= limit && sp.stages == 0) {
      sp.warps = c[0];
      sp.stages = c[1];
      sp.smem = (int)need;
    }
  }
  return sp;
}

template <typename T, typename WT, bool LAYER>
int launch_fwd_stream(StreamPlan& sp, cudaStream_t s, const void* x, int64_t xs, const void* w,
                      const void* b, void* y, int64_t ys, float* mean, float* rstd, int64_t rows,
                      int C, float eps) {
  auto kernel = norm_fwd_stream_kernel<T, WT, LAYER>;
  if (sp.smem > 48 * 1024)
    SCREE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sp.smem));
  int occ = 0;
  SCREE_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, sp.warps * 32, sp.smem));
  occ = std::max(occ, 1);
  const int64_t need = (rows + sp.warps - 1) / sp.warps;
  sp.grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)occ * num_sms()));
  ProfScope prof(PROF_NORM_FWD, s);
  kernel<<<sp.grid, sp.warps * 32, sp.smem, s>>>((const T*)x, xs, w, b, (T*)y, ys, mean, rstd,
                                                 rows, C, sp.stages, eps, device_status_ptr());
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

// Streamed backward plan: R rows per block so a ring slot (x and dy) is about
// 64 KB, as many slots (3..8) as fit next to the staged weight; 0 stages = use
// norm_bwd_kernel.
struct BwdStreamPlan {
  int nt, vpt, R, stages, smem, grid;
};
BwdStreamPlan bwd_stream_plan(int64_t rows, int64_t C, int esize, bool aligned16, bool layer) {
  BwdStreamPlan sp{0, 0, 0, 0, 0, 0};
  const int64_t row_bytes = C * esize;
  if (!aligned16 || row_bytes % 16 != 0) return sp;
  const int64_t nv = row_bytes / 16;
  if (nv < 256 || nv > 4 * kBlock) return sp;
  // 512 threads (one vector per thread per row) measured faster at C = 4096
  // for both norms (LayerNorm 0.62 vs 0.58 of HBM, although its dbias partials
  // spill a few registers at 512 threads x 4 rows); wider LayerNorm rows stay
  // at 256 threads, where 4 vectors per thread would not fit.
  sp.nt = (nv >= 2 * kBlock && (!layer || nv == 2 * kBlock)) ? 2 * kBlock : kBlock;
  sp.vpt = (int)((nv + sp.nt - 1) / sp.nt);
  if (sp.vpt == 3) sp.vpt = 4;
  sp.R = row_bytes <= 8192 ? 4 : (row_bytes <= 16384 ? 2 : 1);
  const int64_t slot = 2 * sp.R * row_bytes;
  const int64_t params = (C * 4 + 127) & ~int64_t(127);
  const int64_t limit = 227 * 1024 - 1024;  // opt-in maximum minus static shared memory
  const int64_t st = std::min<int64_t>(8, (limit - params) / (slot + 8));
  if (st < 3) return BwdStreamPlan{0, 0, 0, 0, 0, 0};
  sp.stages = (int)st;
  sp.smem = (int)(params + st * slot + st * 8);
  const int64_t nblocks = (rows + sp.R - 1) / sp.R;
  sp.grid = (int)std::max<int64_t>(1, std::min<int64_t>(nblocks, num_sms()));
  return sp;
}

template <typename T, typename WT, int NT, int VPT, int R, bool LAYER>
int launch_bwd_stream_r(const BwdStreamPlan& sp, cudaStream_t s, const void* dy, const void* x,
                        const void* w, const float* mean, const float* rstd, void* dx, float* pw,
                        float* pb, int64_t rows, int C) {
  auto kernel = norm_bwd_stream_kernel<T, WT, NT, VPT, R, LAYER>;
  SCREE_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sp.smem));
  ProfScope prof(PROF_NORM_BWD, s);
  kernel<<<sp.grid, NT, sp.smem, s>>>((const T*)dy, (const T*)x, w, mean, rstd, (T*)dx, pw, pb,
                                      rows, C, sp.stages, device_status_ptr());
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

template <typename T, typename WT, bool LAYER>
int launch_bwd_stream(const BwdStreamPlan& sp, cudaStream_t s, const void* dy, const void* x,
                      const void* w, const float* mean, const float* rstd, void* dx, float* pw,
                      float* pb, int64_t rows, int C) {
#define SCREE_BS(NTV, V, RR)                                                                  \
  if (sp.nt == NTV && sp.vpt == V && sp.R == RR)                                               \
  return launch_bwd_stream_r<T, WT, NTV, V, RR, LAYER>(sp, s, dy, x, w, mean, rstd, dx, pw, pb, \
                                                        rows, C)
  // The combinations stream_plan can produce (16-byte vectors per row nv,
  // 256..1024): 256 threads with nv <= 256 / 512 / 1024, 512 threads with
  // nv = 512, and for RMSNorm 512 threads with nv up to 1024; R follows from
  // the row size.
  SCREE_BS(kBlock, 1, 4); SCREE_BS(kBlock, 2, 4); SCREE_BS(kBlock, 4, 2);
  SCREE_BS(2 * kBlock, 1, 4);
  if constexpr (!LAYER) {
    SCREE_BS(2 * kBlock, 2, 2);
  }
#undef SCREE_BS
  set_last_error("norm bwd: no streamed variant for nt=%d vpt=%d R=%d", sp.nt, sp.vpt, sp.R);
  return SCREE_ERR_INVALID;
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
  StreamPlan sp = stream_plan(rows, C, es, a16, LAYER);
  SCREE_BIND_DEVICE(stream, x);
  cudaStream_t s = (cudaStream_t)stream;
  return dispatch_types<LAYER>(dtype, w_dtype, [&](auto* tp, auto* wp) {
    using T = std::remove_pointer_t<decltype(tp)>;
    using WT = std::remove_pointer_t<decltype(wp)>;
    if (sp.stages > 0)
      return launch_fwd_stream<T, WT, LAYER>(sp, s, x, xs, w, b, y, ys, mean, rstd, rows, (int)C, eps);
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
  const BwdStreamPlan sp = bwd_stream_plan(rows, C, es, a16, LAYER);
  // Partial rows: one per CTA of the streamed kernel, else one per row group of
  // the planned grid (the launch may use fewer CTAs, then fewer rows are written
  // and reduced).  Both fit the workspace of scree_norm_bwd_workspace_size.
  const int64_t P = sp.stages ? (int64_t)sp.grid : (int64_t)p.grid * (kBlock / p.tpr);
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
    if (sp.stages)
      return launch_bwd_stream<T, WT, LAYER>(sp, s, dy, x, w, mean, rstd, dx, pw, pb, rows, (int)C);
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
