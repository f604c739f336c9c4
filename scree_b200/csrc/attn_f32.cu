// attn_f32.cu — varlen self-attention forward and backward in fp32.
//
// The Array-level entry of the reference, scree.kernels.reference.varlen_attention
// (reference/varlen_attention.py:90-114), computes in the caller's dtype, fp32
// included, on CUDA tensors.  The tensor-core kernels (attn_fwd.cu, attn_bwd.cu)
// take fp16/bf16 operands only, so fp32 inputs run here: fp32 FMA arithmetic and
// expf, giving fp32-grade results (errors of order 1e-6 against the fp64 oracle)
// instead of the 1e-2 / 2e-3 of the 16-bit path.
//
// One warp owns one (row, head) pair.  Lane l holds elements l, l+32, ... of
// every D-vector it touches, so each row read is a coalesced 128-byte access per
// 32 elements, and a dot product is D/32 FMAs per lane plus a warp reduction.
// Keys (or queries) are walked four at a time so four reductions are in flight.
// The eight warps of a CTA take eight consecutive rows of one head, which
// usually share a sequence, so its K/V (or Q/dO) rows are re-read from L1/L2.
//
//   forward   warp = query row t: online softmax over its keys (causal: k <= q),
//             O = P V / l, LSE = m + ln l (natural log, like the 16-bit path)
//   backward  pass 1, warp = query row: Delta = O.dO, dQ = scale * sum_k dS K;
//             pass 2, warp = key row:   dV = sum_q P dO, dK = scale * sum_q dS Q
//             (grouped-query attention: over the queries of every query head
//             that shares the key's K / V head)
//             with P = exp(S - LSE), dS = P (dO.V - Delta); no atomics, so the
//             result is deterministic.
#include "attn_common.cuh"

namespace scree {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

// Sequence containing packed row t: the last b with offs[b] <= t (empty
// sequences before it share its start and are skipped by taking the last).
__device__ __forceinline__ int64_t find_seq(const void* offs, int is64, int64_t B, int64_t t) {
  int64_t lo = 0, hi = B - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (load_offset(offs, is64, mid) <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int D>
struct Row {
  static constexpr int N = D / 32;
  float x[N];
  __device__ __forceinline__ void load(const float* p, int lane) {
#pragma unroll
    for (int i = 0; i < N; ++i) x[i] = p[lane + 32 * i];
  }
  __device__ __forceinline__ float dot(const Row& o) const {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s = fmaf(x[i], o.x[i], s);
    return s;
  }
};

struct F32Params {
  const float *q, *k, *v;
  int64_t q_rs, q_hs, k_rs, k_hs, v_rs, v_hs;
  const void* offs;
  int is64;
  int64_t B, T;
  int H;
  int G;  // query heads per K / V head
  int causal;
  float scale;
  float* o;
  int64_t o_rs, o_hs;
  float* lse;
  int* status;
};

template <int D>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_f32_kernel(const F32Params p) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= p.T * p.H) return;
  const int h = (int)(w / p.T);
  const int64_t t = w % p.T;
  const int64_t b = find_seq(p.offs, p.is64, p.B, t);
  const int64_t s0 = load_offset(p.offs, p.is64, b), s1 = load_offset(p.offs, p.is64, b + 1);
  if (t < s0 || t >= s1 || s0 < 0 || s1 > p.T) {  // offsets inconsistent with T: report, touch nothing
    if (lane == 0) record_device_error(p.status, SCREE_DEVERR_BAD_INPUT, 44);
    return;
  }
  const int64_t kend = p.causal ? t + 1 : s1;
  Row<D> q;
  q.load(p.q + t * p.q_rs + h * p.q_hs, lane);
  Row<D> acc;
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) acc.x[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  for (int64_t j = s0; j < kend; j += 4) {
    float s[4];
    Row<D> vr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u < kend) {
        Row<D> kr;
        kr.load(p.k + (j + u) * p.k_rs + (h / p.G) * p.k_hs, lane);
        vr[u].load(p.v + (j + u) * p.v_rs + (h / p.G) * p.v_hs, lane);
        s[u] = q.dot(kr);
      } else {
        s[u] = 0.f;
#pragma unroll
        for (int i = 0; i < Row<D>::N; ++i) vr[u].x[i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) s[u] = warp_sum(s[u]) * p.scale;
    float mx = m;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (j + u < kend) mx = fmaxf(mx, s[u]);
    const float alpha = expf(m - mx);  // m = -inf on the first chunk: alpha = 0
    l *= alpha;
#pragma unroll
    for (int i = 0; i < Row<D>::N; ++i) acc.x[i] *= alpha;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float pu = (j + u < kend) ? expf(s[u] - mx) : 0.f;
      l += pu;
#pragma unroll
      for (int i = 0; i < Row<D>::N; ++i) acc.x[i] = fmaf(pu, vr[u].x[i], acc.x[i]);
    }
    m = mx;
  }
  const float inv = 1.f / l;
  float* orow = p.o + t * p.o_rs + h * p.o_hs;
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) orow[lane + 32 * i] = acc.x[i] * inv;
  if (p.lse != nullptr && lane == 0) p.lse[t * p.H + h] = m + logf(l);
}

struct F32BwdParams {
  const float *q, *k, *v, *o, *dout, *lse;  // contiguous (T, H, D); lse (T, H)
  const void* offs;
  int is64;
  int64_t B, T;
  int H;    // query heads
  int Hkv;  // K / V heads (H = Hkv * G)
  int G;
  int causal;
  float scale;
  float* delta;  // (T, H) workspace
  float *dq, *dk, *dv;
  int* status;
};

// Pass 1: one warp per query row: Delta = O . dO, dQ = scale * sum_k dS_k K_k.
template <int D>
__global__ void __launch_bounds__(kWarps * 32) attn_bwd_f32_dq_kernel(const F32BwdParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= p.T * p.H) return;
  const int h = (int)(w / p.T);
  const int64_t t = w % p.T;
  const int64_t b = find_seq(p.offs, p.is64, p.B, t);
  const int64_t s0 = load_offset(p.offs, p.is64, b), s1 = load_offset(p.offs, p.is64, b + 1);
  if (t < s0 || t >= s1 || s0 < 0 || s1 > p.T) {
    if (lane == 0) record_device_error(p.status, SCREE_DEVERR_BAD_INPUT, 45);
    return;
  }
  const int64_t row = (t * p.H + h) * D;
  Row<D> q, dO, o;
  q.load(p.q + row, lane);
  dO.load(p.dout + row, lane);
  o.load(p.o + row, lane);
  const float delta = warp_sum(o.dot(dO));
  if (lane == 0) p.delta[t * p.H + h] = delta;
  const float lse = p.lse[t * p.H + h];
  const int64_t kend = p.causal ? t + 1 : s1;
  Row<D> acc;
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) acc.x[i] = 0.f;
  for (int64_t j = s0; j < kend; j += 4) {
    float s[4], dp[4];
    Row<D> kr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (j + u < kend) {
        Row<D> vr;
        kr[u].load(p.k + ((j + u) * p.Hkv + h / p.G) * D, lane);
        vr.load(p.v + ((j + u) * p.Hkv + h / p.G) * D, lane);
        s[u] = q.dot(kr[u]);
        dp[u] = dO.dot(vr);
      } else {
        s[u] = dp[u] = 0.f;
#pragma unroll
        for (int i = 0; i < Row<D>::N; ++i) kr[u].x[i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[u] = warp_sum(s[u]);
      dp[u] = warp_sum(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float pr = (j + u < kend) ? expf(s[u] * p.scale - lse) : 0.f;
      const float ds = pr * (dp[u] - delta);
#pragma unroll
      for (int i = 0; i < Row<D>::N; ++i) acc.x[i] = fmaf(ds, kr[u].x[i], acc.x[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) p.dq[row + lane + 32 * i] = acc.x[i] * p.scale;
}

// Pass 2: one warp per key row: dV = sum_q P dO_q, dK = scale * sum_q dS Q_q.
template <int D>
__global__ void __launch_bounds__(kWarps * 32) attn_bwd_f32_dkv_kernel(const F32BwdParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (w >= p.T * p.Hkv) return;
  const int h = (int)(w / p.T);  // K / V head
  const int64_t t = w % p.T;     // the key row
  const int64_t b = find_seq(p.offs, p.is64, p.B, t);
  const int64_t s0 = load_offset(p.offs, p.is64, b), s1 = load_offset(p.offs, p.is64, b + 1);
  if (t < s0 || t >= s1 || s0 < 0 || s1 > p.T) {
    if (lane == 0) record_device_error(p.status, SCREE_DEVERR_BAD_INPUT, 46);
    return;
  }
  const int64_t row = (t * p.Hkv + h) * D;
  Row<D> kr, vr;
  kr.load(p.k + row, lane);
  vr.load(p.v + row, lane);
  Row<D> dk, dv;
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) dk.x[i] = dv.x[i] = 0.f;
  // Every query of the sequence (causal: from t on) of every query head of the group.
  for (int g = 0; g < p.G; ++g) {
  const int hq = h * p.G + g;
  for (int64_t i0 = p.causal ? t : s0; i0 < s1; i0 += 4) {
    float s[4], dp[4], lse[4], del[4];
    Row<D> qr[4], dor[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t qi = i0 + u;
      if (qi < s1) {
        qr[u].load(p.q + (qi * p.H + hq) * D, lane);
        dor[u].load(p.dout + (qi * p.H + hq) * D, lane);
        s[u] = qr[u].dot(kr);
        dp[u] = dor[u].dot(vr);
        lse[u] = p.lse[qi * p.H + hq];
        del[u] = p.delta[qi * p.H + hq];
      } else {
        s[u] = dp[u] = lse[u] = del[u] = 0.f;
#pragma unroll
        for (int i = 0; i < Row<D>::N; ++i) qr[u].x[i] = dor[u].x[i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      s[u] = warp_sum(s[u]);
      dp[u] = warp_sum(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float pr = (i0 + u < s1) ? expf(s[u] * p.scale - lse[u]) : 0.f;
      const float ds = pr * (dp[u] - del[u]);
#pragma unroll
      for (int i = 0; i < Row<D>::N; ++i) {
        dv.x[i] = fmaf(pr, dor[u].x[i], dv.x[i]);
        dk.x[i] = fmaf(ds, qr[u].x[i], dk.x[i]);
      }
    }
  }
  }
#pragma unroll
  for (int i = 0; i < Row<D>::N; ++i) {
    p.dv[row + lane + 32 * i] = dv.x[i];
    p.dk[row + lane + 32 * i] = dk.x[i] * p.scale;
  }
}

inline unsigned warps_grid(int64_t T, int64_t H) {
  return (unsigned)((T * H + kWarps - 1) / kWarps);
}

}  // namespace

int attn_fwd_f32(const void* q, const void* k, const void* v, int64_t q_rs, int64_t q_hs,
                 int64_t k_rs, int64_t k_hs, int64_t v_rs, int64_t v_hs, const void* offsets,
                 int is64, int64_t B, int64_t T, int64_t H, int64_t H_kv, int D, int causal,
                 float scale, void* o, int64_t o_rs, int64_t o_hs, float* lse, cudaStream_t s) {
  SCREE_CHECK_ARG(T * H / kWarps < (1ll << 31), "attn_fwd (fp32): T x H too large");
  F32Params p{(const float*)q, (const float*)k, (const float*)v, q_rs, q_hs, k_rs, k_hs, v_rs,
              v_hs, offsets, is64, B, T, (int)H, (int)(H / H_kv), causal, scale, (float*)o, o_rs,
              o_hs, lse,
              device_status_ptr()};
  const unsigned grid = warps_grid(T, H);
  ProfScope prof(PROF_ATTN_FWD, s);
  switch (D) {
    case 32: attn_fwd_f32_kernel<32><<<grid, kWarps * 32, 0, s>>>(p); break;
    case 64: attn_fwd_f32_kernel<64><<<grid, kWarps * 32, 0, s>>>(p); break;
    default: attn_fwd_f32_kernel<128><<<grid, kWarps * 32, 0, s>>>(p); break;
  }
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

int attn_bwd_f32(const void* dout, const void* q, const void* k, const void* v, const void* o,
                 const float* lse, const void* offsets, int is64, int64_t B, int64_t T, int64_t H,
                 int64_t H_kv, int D, int causal, float scale, void* dq, void* dk, void* dv,
                 float* delta, cudaStream_t s) {
  SCREE_CHECK_ARG(T * H / kWarps < (1ll << 31), "attn_bwd (fp32): T x H too large");
  F32BwdParams p{(const float*)q, (const float*)k, (const float*)v, (const float*)o,
                 (const float*)dout, lse, offsets, is64, B, T, (int)H, (int)H_kv, (int)(H / H_kv),
                 causal, scale, delta,
                 (float*)dq, (float*)dk, (float*)dv, device_status_ptr()};
  const unsigned grid = warps_grid(T, H), grid_kv = warps_grid(T, H_kv);
  ProfScope prof(PROF_ATTN_BWD, s);
#define SCREE_F32_BWD(DD)                                                   \
  attn_bwd_f32_dq_kernel<DD><<<grid, kWarps * 32, 0, s>>>(p);               \
  SCREE_LAUNCH_CHECK();                                                     \
  attn_bwd_f32_dkv_kernel<DD><<<grid_kv, kWarps * 32, 0, s>>>(p);           \
  SCREE_LAUNCH_CHECK();
  switch (D) {
    case 32: SCREE_F32_BWD(32) break;
    case 64: SCREE_F32_BWD(64) break;
    default: SCREE_F32_BWD(128) break;
  }
#undef SCREE_F32_BWD
  return SCREE_OK;
}

}  // namespace scree
