// prenorm_qkv.cu — RMSNorm fused into the QKV projection on sm_100a tensor cores.
//
// The caller side of the attention path in scree's examples
// (examples/03_train_step.py:26-48, examples/02_no_pad_transformer.py:31-58):
//   h = varlen_rmsnorm(x) * gamma;   qkv = h @ Wqkv   (then viewed as (T, 3, H, D))
// RMSNorm is a per-row scale, so
//   qkv[t, n] = rstd[t] * sum_c x[t, c] * (gamma[c] * Wqkv[c, n]),
//   rstd[t]   = 1 / sqrt(mean_c x[t, c]^2 + eps).
// A row-statistics pass writes rstd (one warp per row), then one GEMM kernel:
// the raw x tiles feed tcgen05.mma straight from the TMA ring and the epilogue
// scales the fp32 accumulator row by rstd before the 16-bit store, so the
// normalised h never exists in memory.  gamma is folded into the weight once
// per call (gamma[c] * Wqkv[c, :], a C x N pass); with gamma = NULL the weight
// is used as is.  (Taking the sums of squares inside the GEMM, from the staged
// x tiles, added 16 KB of shared-memory reads to every 48 KB stage of a kernel
// whose shared-memory port is its limit: 0.58 of the burst GEMM peak against
// the separate pass's x re-read of T x C x 2 bytes.)
//
// N a multiple of 256: CTA pairs (clusters of two) with 256 x 256 pair tiles,
// M = 256 tcgen05 MMAs over both CTAs' shared memory and TMEM, a 6-stage TMA
// ring of 32 KB per CTA (rmsnorm_qkv_pair_kernel).  Otherwise single CTAs with
// 128 x 128 tiles and a 4-stage ring (rmsnorm_qkv_kernel).  K in steps of 64
// (128-byte swizzled rows); persistent CTAs (pairs) walk their tiles with the
// accumulator double-buffered in TMEM.  Warp 0 issues TMA, warp 1 the MMAs,
// warps 2-5 are the epilogue warps (warp w owns TMEM lanes 32 (w % 4) ..).
#include <algorithm>
#include "attn_common.cuh"

namespace scree {
namespace {

constexpr int QM = 128;         // rows per CTA
constexpr int QK = 64;          // K per stage (one 128-byte swizzle row of 16-bit values)
constexpr int QSTAGES = 4;
constexpr int kQThreads = 192;  // TMA warp, MMA warp, 4 epilogue warps

template <int BNT>
struct QCfg {
  static constexpr int A_BYTES = QM * QK * 2;    // 16 KB
  static constexpr int B_BYTES = BNT * QK * 2;   // 32 KB at BNT = 256
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_BAR = QSTAGES * STAGE;
  static constexpr int OFF_END = OFF_BAR + 128;
  static constexpr int SMEM = OFF_END + 1024;
};

struct QParams {
  int64_t T, N, C;
  float eps;
  void* y;           // (T, N) row-major, dtype
  const float* rstd; // (T,), from the statistics pass
  int* status;
};

template <typename T, int BNT>
__global__ void __launch_bounds__(kQThreads, 1)
    rmsnorm_qkv_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w, const QParams p) {
  using Cf = QCfg<BNT>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  // A = x tile (K-major), B = weight tile [K rows][N] (N contiguous: MN-major).
  constexpr uint32_t IDESC = make_idesc_f16(QM, BNT, kBF16, false, true);
  // Persistent: CTA c takes tiles c, c + gridDim.x, ...; tile t covers rows
  // (t / n_tiles_n) * QM and columns (t % n_tiles_n) * BNT.  The accumulator is
  // double-buffered in TMEM (2 x BNT columns), so the epilogue of one tile runs
  // while the tensor core works on the next.
  const int nk = (int)(p.C / QK);
  const int n_tiles_n = (int)(p.N / BNT);
  const int64_t n_tiles = ((p.T + QM - 1) / QM) * n_tiles_n;
  if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) return;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cf::OFF_BAR);
  uint64_t* full = bars;                 // [QSTAGES]
  uint64_t* empty = full + QSTAGES;      // [QSTAGES]
  uint64_t* acc_full = empty + QSTAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // the MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);     // the MMA commit after a tile's last k-step
      mbar_init(&acc_empty[b], 128);  // the epilogue threads after reading it
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc<2 * BNT>(tmem_slot);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (elect_one()) {
      int64_t g = 0;  // k-steps issued by this CTA (ring position)
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const int m0 = (int)(tile / n_tiles_n) * QM, n0 = (int)(tile % n_tiles_n) * BNT;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % QSTAGES);
          if (g >= QSTAGES &&
              !(ok = mbar_wait(&empty[s], (uint32_t)(((g / QSTAGES) - 1) & 1), abort_flag, p.status, 70)))
            break;
          uint8_t* st = smem + s * Cf::STAGE;
          mbar_expect_tx(&full[s], Cf::STAGE);
          tma_load_2d(st, &tm_x, &full[s], kt * QK, m0);
#pragma unroll
          for (int j = 0; j < BNT / 64; ++j)  // 64-column chunks of [QK rows][64 N]
            tma_load_2d(st + Cf::A_BYTES + j * QK * 128, &tm_w, &full[s], n0 + j * 64, kt * QK);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (elect_one()) {
      bool ok = true;
      int64_t g = 0;
      int i = 0;  // tiles done by this CTA
      for (int64_t tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !(ok = mbar_wait(&acc_empty[b], (uint32_t)(((i >> 1) - 1) & 1), abort_flag,
                                       p.status, 74)))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + b * BNT;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % QSTAGES);
          if (!(ok = mbar_wait(&full[s], (uint32_t)((g / QSTAGES) & 1), abort_flag, p.status, 71)))
            break;
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * Cf::STAGE);
          const uint32_t bb = a + Cf::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < QK / 16; ++kk)
            umma_f16_ss(acc, make_sdesc(a + kk * 32, 16, 1024, SW_128B),
                        make_sdesc(bb + kk * 16 * 128, QK * 128, 1024, SW_128B), IDESC,
                        (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int r = q * 32 + lane;       // row within the tile == TMEM lane
    int i = 0;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      bool ok = mbar_wait(&acc_full[b], (uint32_t)((i >> 1) & 1), abort_flag, p.status, 73);
      if (!__all_sync(0xffffffff, ok)) break;
      tc_fence_after();
      const int m0 = (int)(tile / n_tiles_n) * QM, n0 = (int)(tile % n_tiles_n) * BNT;
      const int64_t t = (int64_t)m0 + r;
      const bool row_ok = t < p.T;
      const float rs = row_ok ? p.rstd[t] : 0.f;
      T* yrow = reinterpret_cast<T*>(p.y) + t * p.N + n0;
      const uint32_t lane_base = tmem + b * BNT + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BNT / 32; ++c) {
        float v[32];
        tmem_ld32_sync(lane_base + c * 32, v);
        if (c == BNT / 32 - 1) {  // all of this tile's accumulator is in registers
          tc_fence_before();
          mbar_arrive(&acc_empty[b]);
        }
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = v[u * 8 + e] * rs;
            alignas(16) T pk[8];
            cvt_from_f<T, 8>(o, pk);
            *reinterpret_cast<uint4*>(yrow + c * 32 + u * 8) = *reinterpret_cast<const uint4*>(pk);
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<2 * BNT>(tmem);
  }
}

// ------------------------------------------------------------ CTA-pair GEMM
// Same computation with the tiles of a CTA pair (cluster of two): a pair tile is
// 256 rows x 256 columns; CTA r of the pair stages rows [128 r, 128 r + 128) of
// the x tile and columns [128 r, 128 r + 128) of the weight tile, and the even
// CTA issues M = 256, N = 256 tcgen05 MMAs (.cta_group::2) that read both CTAs'
// shared memory and leave rows 128 r.. of the accumulator in CTA r's TMEM.  Per
// K = 16 step each SM then stages and reads 8 KB instead of 12 KB (one CTA's
// 128 x 256 tile), which is what bounds the single-CTA kernel.
constexpr int PSTAGES = 6;
struct PCfg {
  static constexpr int A_BYTES = 128 * QK * 2;  // this CTA's 128 rows: 16 KB
  static constexpr int B_BYTES = 128 * QK * 2;  // this CTA's 128 columns: 16 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_BAR = PSTAGES * STAGE;
  static constexpr int OFF_END = OFF_BAR + 256;
  static constexpr int SMEM = OFF_END + 1024;
};

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kQThreads, 1)
    rmsnorm_qkv_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                            const __grid_constant__ CUtensorMap tm_w, const QParams p) {
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC = make_idesc_f16(256, 256, kBF16, false, true);
  // Persistent pairs: pair c takes pair tiles c, c + gridDim.x / 2, ...
  const uint32_t rank = cluster_ctarank();
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nk = (int)(p.C / QK);
  const int n_tiles_n = (int)(p.N / 256);
  const int64_t n_tiles = ((p.T + 255) / 256) * n_tiles_n;
  // (No early exit on the status word: both CTAs of a pair must reach the
  // cluster barriers; the bounded waits see it and drain instead.)

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PCfg::OFF_BAR);
  uint64_t* full = bars;                  // [PSTAGES], used in the even CTA: both CTAs' loads
  uint64_t* empty = full + PSTAGES;       // [PSTAGES], both CTAs: the MMA commit
  uint64_t* acc_full = empty + PSTAGES;   // [2], both CTAs: the MMA commit after a tile
  uint64_t* acc_empty = acc_full + 2;     // [2], even CTA: 256 epilogue threads of the pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 256);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair<512>(tmem_slot);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA (both CTAs)
    if (elect_one()) {
      int64_t g = 0;
      bool ok = true;
      for (int64_t tile = pair; ok && tile < n_tiles; tile += npairs) {
        const int m0 = (int)(tile / n_tiles_n) * 256 + (int)rank * 128;
        const int n0 = (int)(tile % n_tiles_n) * 256 + (int)rank * 128;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % PSTAGES);
          if (g >= PSTAGES &&
              !(ok = mbar_wait(&empty[s], (uint32_t)(((g / PSTAGES) - 1) & 1), abort_flag, p.status, 75)))
            break;
          uint8_t* st = smem + s * PCfg::STAGE;
          // The even CTA's barrier counts both CTAs' bytes of the stage.
          if (rank == 0) mbar_expect_tx(&full[s], 2 * PCfg::STAGE);
          const uint32_t fb = smem_peer(smem_u32(&full[s]), 0);
          tma_load_2d_pair(st, &tm_x, fb, kt * QK, m0);
#pragma unroll
          for (int j = 0; j < 2; ++j)  // 64-column chunks of [QK rows][64 N]
            tma_load_2d_pair(st + PCfg::A_BYTES + j * QK * 128, &tm_w, fb, n0 + j * 64, kt * QK);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA (even CTA)
    if (rank == 0 && elect_one()) {
      bool ok = true;
      int64_t g = 0;
      int i = 0;
      for (int64_t tile = pair; ok && tile < n_tiles; tile += npairs, ++i) {
        const int b = i & 1;
        if (i >= 2 && !(ok = mbar_wait(&acc_empty[b], (uint32_t)(((i >> 1) - 1) & 1), abort_flag,
                                       p.status, 76)))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + b * 256;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const int s = (int)(g % PSTAGES);
          if (!(ok = mbar_wait(&full[s], (uint32_t)((g / PSTAGES) & 1), abort_flag, p.status, 77)))
            break;
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * PCfg::STAGE);
          const uint32_t bb = a + PCfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < QK / 16; ++kk)
            umma_f16_ss_pair(acc, make_sdesc(a + kk * 32, 16, 1024, SW_128B),
                             make_sdesc(bb + kk * 16 * 128, QK * 128, 1024, SW_128B), IDESC,
                             (kt > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(smem_peer(smem_u32(&empty[s]), 1));
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&acc_full[b]));
        umma_commit_pair(smem_peer(smem_u32(&acc_full[b]), 1));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row within this CTA's half == TMEM lane
    const uint32_t ae0 = smem_peer(smem_u32(&acc_empty[0]), 0);
    const uint32_t ae1 = smem_peer(smem_u32(&acc_empty[1]), 0);
    int i = 0;
    for (int64_t tile = pair; tile < n_tiles; tile += npairs, ++i) {
      const int b = i & 1;
      bool ok = mbar_wait(&acc_full[b], (uint32_t)((i >> 1) & 1), abort_flag, p.status, 78);
      if (!__all_sync(0xffffffff, ok)) break;
      tc_fence_after();
      const int m0 = (int)(tile / n_tiles_n) * 256 + (int)rank * 128;
      const int n0 = (int)(tile % n_tiles_n) * 256;
      const int64_t t = (int64_t)m0 + r;
      const bool row_ok = t < p.T;
      const float rs = row_ok ? p.rstd[t] : 0.f;
      T* yrow = reinterpret_cast<T*>(p.y) + t * p.N + n0;
      const uint32_t lane_base = tmem + b * 256 + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < 256 / 32; ++c) {
        float v[32];
        tmem_ld32_sync(lane_base + c * 32, v);
        if (c == 256 / 32 - 1) {  // the whole accumulator half is in registers
          tc_fence_before();
          mbar_arrive_cluster(b ? ae1 : ae0);
        }
        if (row_ok) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = v[u * 8 + e] * rs;
            alignas(16) T pk[8];
            cvt_from_f<T, 8>(o, pk);
            *reinterpret_cast<uint4*>(yrow + c * 32 + u * 8) = *reinterpret_cast<const uint4*>(pk);
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();  // no MMA, commit or remote arrival is left for either CTA
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair<512>(tmem);
  }
}

// rstd[t] = 1 / sqrt(mean(x[t]^2) + eps): one warp per row, 16-byte loads.
template <typename T>
__global__ void __launch_bounds__(256) row_rstd_kernel(const T* __restrict__ x, int64_t rs_x,
                                                       int64_t rows, int64_t C, float eps,
                                                       float* __restrict__ rstd) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * rs_x);
  float ss = 0.f;
  for (int64_t v = lane; v < C / 8; v += 32) {
    const uint4 w = xr[v];
    const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float f = Cvt<T>::to_f(e[u]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) rstd[row] = rsqrtf(ss / (float)C + eps);
}

// W'[c][n] = gamma[c] * W[c][n], rounded to the weight's dtype.
template <typename T, typename G>
__global__ void fold_gamma_kernel(const T* __restrict__ w, const G* __restrict__ gamma,
                                  T* __restrict__ out, int64_t C, int64_t N) {
  const int64_t n8 = N / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < C * n8;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c = i / n8;
    const float g = Cvt<G>::to_f(gamma[c]);
    uint4 raw = reinterpret_cast<const uint4*>(w)[i];
    const T* e = reinterpret_cast<const T*>(&raw);
    float f[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) f[u] = Cvt<T>::to_f(e[u]) * g;
    alignas(16) T pk[8];
    cvt_from_f<T, 8>(f, pk);
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<const uint4*>(pk);
  }
}

int make_2d_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer,
                int64_t row_stride_elems, int box_inner, int box_outer, bool bf16) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return SCREE_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled (2-D) failed (CUresult %d)", (int)r);
    return SCREE_ERR_CUDA;
  }
  return SCREE_OK;
}

template <typename T, int BNT>
int launch_qkv(const CUtensorMap& tx, const CUtensorMap& tw, const QParams& p, cudaStream_t s) {
  auto kern = rmsnorm_qkv_kernel<T, BNT>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    SCREE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        QCfg<BNT>::SMEM));
    attr_set[dev & 63] = true;
  }
  const int64_t tiles = ((p.T + QM - 1) / QM) * (p.N / BNT);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, (int64_t)num_sms());  // persistent
  kern<<<grid, kQThreads, QCfg<BNT>::SMEM, s>>>(tx, tw, p);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

template <typename T>
int launch_qkv_pair(const CUtensorMap& tx, const CUtensorMap& tw, const QParams& p, cudaStream_t s) {
  auto kern = rmsnorm_qkv_pair_kernel<T>;
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (max_pairs[dev & 63] == 0) {
    SCREE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg::SMEM));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(2 * num_sms()), 1, 1);
    cfg.blockDim = dim3(kQThreads, 1, 1);
    cfg.dynamicSmemBytes = PCfg::SMEM;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    SCREE_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_pairs[dev & 63] = std::max(n, 1);
  }
  const int64_t tiles = ((p.T + 255) / 256) * (p.N / 256);
  const unsigned grid = 2u * (unsigned)std::min<int64_t>(tiles, (int64_t)max_pairs[dev & 63]);
  kern<<<grid, kQThreads, PCfg::SMEM, s>>>(tx, tw, p);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

}  // namespace
}  // namespace scree

using namespace scree;

// Workspace: [gamma-folded weight, C x N x 2 bytes][rstd scratch, T x 4 bytes].
static size_t qkv_ws_rstd_off(int64_t C, int64_t N) { return ((size_t)C * N * 2 + 255) & ~size_t(255); }

extern "C" size_t scree_rmsnorm_qkv_workspace_size(int64_t T, int64_t C, int64_t N) {
  return qkv_ws_rstd_off(C, N) + (size_t)T * 4;
}

extern "C" int scree_rmsnorm_qkv_fwd(const void* x, int64_t x_row_stride, const void* gamma,
                                     int g_dtype, const void* weight, void* y, float* rstd,
                                     int64_t T, int64_t C, int64_t N, int dtype, float eps,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  SCREE_CHECK_ARG(T >= 0 && C >= 1 && N >= 1, "rmsnorm_qkv: bad sizes");
  SCREE_CHECK_ARG(dtype == SCREE_F16 || dtype == SCREE_BF16, "rmsnorm_qkv: fp16 or bf16 only");
  if (C % QK != 0 || N % 128 != 0) {
    set_last_error("rmsnorm_qkv: C must be a multiple of 64 and N of 128 (C=%lld N=%lld)",
                   (long long)C, (long long)N);
    return SCREE_ERR_UNSUPPORTED;
  }
  SCREE_CHECK_ARG(T < (1ll << 31) && C < (1ll << 31) && N < (1ll << 31), "rmsnorm_qkv: too large");
  if (T == 0) return SCREE_OK;
  SCREE_CHECK_ARG(x && weight && y, "rmsnorm_qkv: null pointer");
  SCREE_CHECK_ARG(((uintptr_t)x % 16) == 0 && (x_row_stride % 8) == 0 && ((uintptr_t)weight % 16) == 0 &&
                      ((uintptr_t)y % 16) == 0,
                  "rmsnorm_qkv: 16-byte aligned tensors and row strides required");
  SCREE_BIND_DEVICE(stream, x);
  cudaStream_t s = (cudaStream_t)stream;
  const bool bf16 = dtype == SCREE_BF16;
  const void* w = weight;
  SCREE_CHECK_ARG(workspace && workspace_bytes >= scree_rmsnorm_qkv_workspace_size(T, C, N),
                  "rmsnorm_qkv: workspace too small");
  if (gamma != nullptr) {  // fold gamma into the weight rows once
    SCREE_CHECK_ARG(g_dtype == SCREE_F16 || g_dtype == SCREE_BF16 || g_dtype == SCREE_F32,
                    "rmsnorm_qkv: gamma dtype");
    const int64_t n = C * N / 8;
    const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8);
#define SCREE_FOLD(TT)                                                                         \
  switch (g_dtype) {                                                                           \
    case SCREE_F32: fold_gamma_kernel<TT, float><<<grid, 256, 0, s>>>((const TT*)weight, (const float*)gamma, (TT*)workspace, C, N); break; \
    case SCREE_BF16: fold_gamma_kernel<TT, __nv_bfloat16><<<grid, 256, 0, s>>>((const TT*)weight, (const __nv_bfloat16*)gamma, (TT*)workspace, C, N); break; \
    default: fold_gamma_kernel<TT, __half><<<grid, 256, 0, s>>>((const TT*)weight, (const __half*)gamma, (TT*)workspace, C, N); break; \
  }
    if (bf16) { SCREE_FOLD(__nv_bfloat16) } else { SCREE_FOLD(__half) }
#undef SCREE_FOLD
    SCREE_LAUNCH_CHECK();
    w = workspace;
  }
  CUtensorMap tx, tw;
  int rc;
  if ((rc = make_2d_map(&tx, x, C, T, x_row_stride, QK, QM, bf16))) return rc;
  const int bnt = (N % 256 == 0) ? 256 : 128;
  if ((rc = make_2d_map(&tw, w, N, C, N, 64, QK, bf16))) return rc;
  float* rs = rstd != nullptr ? rstd
                              : reinterpret_cast<float*>((char*)workspace + qkv_ws_rstd_off(C, N));
  if (bf16)
    row_rstd_kernel<__nv_bfloat16><<<(unsigned)((T + 7) / 8), 256, 0, s>>>(
        (const __nv_bfloat16*)x, x_row_stride, T, C, eps, rs);
  else
    row_rstd_kernel<__half><<<(unsigned)((T + 7) / 8), 256, 0, s>>>((const __half*)x, x_row_stride,
                                                                     T, C, eps, rs);
  SCREE_LAUNCH_CHECK();
  QParams p{T, N, C, eps, y, rs, device_status_ptr()};
  ProfScope prof(PROF_NORM_FWD, s);
#ifndef SCREE_QKV_NO_PAIR
  if (bnt == 256)  // CTA pairs (x boxes of 128 rows per CTA, weight boxes of 64 columns)
    return bf16 ? launch_qkv_pair<__nv_bfloat16>(tx, tw, p, s) : launch_qkv_pair<__half>(tx, tw, p, s);
#endif
  if (bf16)
    return bnt == 256 ? launch_qkv<__nv_bfloat16, 256>(tx, tw, p, s)
                      : launch_qkv<__nv_bfloat16, 128>(tx, tw, p, s);
  return bnt == 256 ? launch_qkv<__half, 256>(tx, tw, p, s) : launch_qkv<__half, 128>(tx, tw, p, s);
}
