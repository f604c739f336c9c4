// attn_bwd.cu — varlen self-attention backward on sm_100a tensor cores.
//
// Gradients of O = softmax(Q K^T * scale) V per sequence and head, recomputing
// P from the saved LSE (the FlashAttention-2 scheme that
// scree/kernels/triton/_backward.py:73-285 also follows):
//   P  = exp(S - LSE),  dV = P^T dO,  dP = dO V^T,
//   dS = P * (dP - Delta),  Delta = rowsum(O * dO)   (_backward.py:37-69)
//   dK = scale * dS^T Q,    dQ = scale * dS K
// Five GEMMs per (key tile, query tile) pair, none recomputed.
//
// A work item is a 128-key tile of one K/V head (K, V resident in shared
// memory); the kernel is persistent (one CTA per SM takes items in schedule
// order from a device counter) and, per item, loops over the sequence's query
// tiles of BQ rows.  Warps, in launch order:
//   4 NP P/dS warps  thread = key row = TMEM lane: P^T, dS^T from S^T, dP^T; the
//                    NP warps of one lane quadrant each take BQ / NP query columns
//                    (NP = 4 at D = 128: 768 threads; NP = 2 below: 512 threads)
//   TMA warp         K, V once; Q_i, dO_i into a ring
//   MMA warp         S^T = K Q_i^T, dP^T = V dO_i^T, dV += P^T dO_i,
//                    dK += dS^T Q_i, dQ_i (see below)
//   two idle warps, then 4 dQ warps: read dQ_i from TMEM and add it into an fp32
//                    accumulator in global memory; a final kernel casts it to q's dtype.
// Two shapes:
//   D = 128: BQ = 64 and dQ_i^T = K^T dS^T (M = D = 128 lanes, N = 64 queries),
//            staged in shared memory and added with one TMA reduce per tile;
//   D <= 64: BQ = 128 and dQ_i = dS K (M = 128 queries, N = D), vector reductions.
// TMEM columns: S^T [0,BQ), dP^T [BQ,2BQ), dV [2BQ,2BQ+D), dK [.., +D), dQ [.., +BQ or D),
// and where the 512 columns allow it (D = 128, D = 32) a second S^T buffer after dQ:
// S^T of tile i + 2 is then issued right after dP^T of tile i + 1.
#include <algorithm>
#ifdef SCREE_TRACE
// Profiling build only: per-site wait cycles (lane 0 of each waiting warp),
// [62] = CTA lifetime cycles.
static __device__ unsigned long long g_bwd_trace[64];
#define SCREE_TRACE_ADD(site, cyc) \
  do { if ((threadIdx.x & 31) == 0 || (site) == 12) atomicAdd(&scree_trace_sm[(site) & 63], (unsigned long long)(cyc)); } while (0)
static __shared__ unsigned long long scree_trace_sm[64];  // per-CTA, flushed at exit
#endif
#include "attn_common.cuh"
#ifdef SCREE_TRACE
#define SW_MARK(site)                          \
  do {                                         \
    const long long t_ = clock64();            \
    SCREE_TRACE_ADD(site, t_ - t_mark);        \
    t_mark = t_;                               \
  } while (0)
#else
#define SW_MARK(site) \
  do {                \
  } while (0)
#endif

namespace scree {
namespace {

constexpr int BN = 128;  // keys per CTA
// Roles: NP P^T / dS^T warpgroups first (the NP warps w % 4 == j share TMEM lanes
// 32j..32j+31, each takes 1/NP of a tile's query columns), then one warpgroup of
// TMA warp, MMA warp and two idle warps, then the four dQ reduction warps.
//   NP = 2 (D <= 64): 512 threads launched at 128 registers; the P/dS warpgroups
//     grow to 152, warpgroup 2 shrinks to 80 and the dQ warps to 120:
//     256 x 152 + 128 x 80 + 128 x 120 = 64,512 <= 65,536.
//   NP = 4 (D = 128, 16 query columns per P/dS thread): 768 threads at the
//     launch's register count (at most 80), no reallocation.
constexpr int kRegsSoftmax = 152, kRegsOther = 80, kRegsDq = 120;
// Item records reach the roles through a ring: the TMA thread takes the next
// item from the schedule's counter and publishes it; the MMA thread, the P/dS
// threads and the 128 dQ threads read it.
constexpr int kItemRing = 4;

template <int D>
struct BwdCfg {
  static constexpr bool DQT = (D == 128);
  static constexpr int BQ = DQT ? 64 : 128;
  // NP P/dS warps per TMEM lane quadrant, each taking BQ / NP query columns.
  static constexpr int NP = D == 128 ? 4 : 2;
  static constexpr int QH = BQ / NP;          // query columns per P/dS thread
  static constexpr int SWT = NP * 128;        // P/dS threads
  static constexpr int THREADS = SWT + 256;
  static constexpr int ITEM_CONSUMERS = 1 + SWT + 128;
  static constexpr int SWB = D >= 64 ? 128 : 64;
  static constexpr int CHUNK = SWB / 2;
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr uint32_t SWZ = SWB == 128 ? SW_128B : SW_64B;
  // S^T double-buffered in TMEM where the columns allow it (D = 128, D = 32): S^T
  // of tile i + 2 is computed while the P/dS warps work on tile i + 1, so they
  // never wait for it; a third Q / dO stage keeps its load ahead of that MMA.
  static constexpr int COL_S1 = 2 * BQ + 2 * D + (DQT ? BQ : D);
#ifdef SCREE_BWD_NO_SDB
  static constexpr bool SDB = false;
#else
  static constexpr bool SDB = COL_S1 + BQ <= 512;
#endif
  static constexpr int STAGES = SDB ? 3 : 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int QT_BYTES = BQ * D * 2;
  static constexpr int PT_BYTES = BN * BQ * 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KV_BYTES;
  static constexpr int OFF_Q = OFF_V + KV_BYTES;
  static constexpr int OFF_DO = OFF_Q + STAGES * QT_BYTES;
  static constexpr int OFF_PT = OFF_DO + STAGES * QT_BYTES;
  static constexpr int OFF_DS = OFF_PT;  // P^T lives in TMEM only (no smem buffer)
  static constexpr int OFF_LD = OFF_DS + PT_BYTES;          // lse2 / delta [2][2][BQ] fp32
  static constexpr int OFF_DQ = OFF_LD + 2 * 2 * BQ * 4;    // DQT: dQ tile [BQ][D] fp32
  static constexpr int DQ_BYTES = DQT ? BQ * D * 4 : 0;
  static constexpr int OFF_BAR = OFF_DQ + DQ_BYTES;
  // At least 120 KB so two CTAs (each holding all 512 TMEM columns) never share an SM.
  static constexpr int OFF_END = OFF_BAR + 512;
  // 1 KB of alignment slack when it fits; the kernel checks the real alignment.
  static constexpr int SMEM_RAW = OFF_END + 1024 <= 232448 ? OFF_END + 1024 : OFF_END;
  static constexpr int SMEM = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
  static constexpr int COL_S = 0, COL_DP = BQ, COL_DV = 2 * BQ, COL_DK = 2 * BQ + D,
                       COL_DQ = 2 * BQ + 2 * D;
  static constexpr int TMEM_COLS = 512;
  static_assert(COL_DQ + (DQT ? BQ : D) <= TMEM_COLS, "TMEM budget");
};

struct BwdParams {
  const void* offs;
  int is64;
  int H;    // query heads
  int Hkv;  // key / value heads (H = Hkv * G)
  int G;
  int T;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  const void* sched;  // schedule (attn_common.cuh)
  int64_t B;
  int* status;  // device status word
  const float* lse2T;   // [H][T], lse * log2(e)
  const float* deltaT;  // [H][T]
  float* dq_acc;        // [T][H][D] fp32
  void* dk;
  void* dv;
};

template <int D>
__device__ __forceinline__ uint64_t kmaj(uint32_t base, int rows, int kk) {
  using C = BwdCfg<D>;
  const int e = kk * 16;
  return make_sdesc(base + (e / C::CHUNK) * rows * C::SWB + (e % C::CHUNK) * 2, 16, 8 * C::SWB,
                    C::SWZ);
}
// MN-major view of a [rows][D] TMA tile, K dimension = rows (16 per k-step).
template <int D>
__device__ __forceinline__ uint64_t mnmaj(uint32_t base, int rows, int kk) {
  using C = BwdCfg<D>;
  return make_sdesc(base + kk * 16 * C::SWB, rows * C::SWB, 8 * C::SWB, C::SWZ);
}
// P^T / dS^T tile [BN keys][BQ queries], 64-query 128B-swizzled column blocks.
// MN-major view with K = keys (16 rows per step), MN = queries:
__device__ __forceinline__ uint64_t pt_mnmaj(uint32_t base, int kk) {
  return make_sdesc(base + kk * 16 * 128, BN * 128, 1024, SW_128B);
}

template <typename T> struct Pk2b;
template <> struct Pk2b<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Pk2b<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// TMEM column of k-step kk (16 queries) of a packed P^T / dS^T tile.  Each of
// the NP parts of the tile's queries is packed into the first half of its own
// fp32 columns: queries [j QH, (j + 1) QH) at columns [j QH, j QH + QH / 2).
template <int BQ, int NP>
__device__ __forceinline__ uint32_t packed_col(int kk) {
  constexpr int KH = BQ / (16 * NP);  // k-steps per part
  return (uint32_t)((kk / KH) * (BQ / NP) + (kk % KH) * 8);
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// Named barriers over the N P/dS threads (the first warps) and the 128 dQ threads.
template <int N>
__device__ __forceinline__ void softmax_group_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void dq_group_sync() {
  asm volatile("bar.sync 2, 128;" ::: "memory");
}

// Row-major [BN][BQ] 16-bit tile in 128B swizzle: write N values of row kr
// starting at column 8 * u0.
template <typename T, int N>
__device__ __forceinline__ void write_row_sw128(uint8_t* base, int kr, const float* v, int u0) {
  const int sw = kr & 7;
#pragma unroll
  for (int i = 0; i < N / 8; ++i) {
    const int u = u0 + i;
    uint4 w;
    w.x = Pk2b<T>::pack(v[i * 8 + 0], v[i * 8 + 1]);
    w.y = Pk2b<T>::pack(v[i * 8 + 2], v[i * 8 + 3]);
    w.z = Pk2b<T>::pack(v[i * 8 + 4], v[i * 8 + 5]);
    w.w = Pk2b<T>::pack(v[i * 8 + 6], v[i * 8 + 7]);
    const int blk = u >> 3, uu = u & 7;
    *reinterpret_cast<uint4*>(base + blk * BN * 128 + kr * 128 + ((uu ^ sw) << 4)) = w;
  }
}

template <int D, typename T, bool CAUSAL, bool GQA>
__global__ void __launch_bounds__(BwdCfg<D>::THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, const BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int BQ = C::BQ;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t ID_S = make_idesc_f16(BN, BQ, kBF16, false, false);
  constexpr uint32_t ID_ACC = make_idesc_f16(BN, D, kBF16, false, true);
  constexpr uint32_t ID_DQ = C::DQT ? make_idesc_f16(D, BQ, kBF16, true, true)
                                    : make_idesc_f16(BQ, D, kBF16, true, true);

  // Persistent: one CTA per SM takes items (128-key tiles of one K / V head)
  // of the longest-first schedule from a device counter as its TMA producer
  // gets to them; the producer publishes each item's record through a ring.
  const int64_t n_items = total_items(p.sched);
  if ((int64_t)blockIdx.x >= n_items) return;
  // A CTA of an earlier failed launch (or of this one) set the status word: skip.
  if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) return;
  struct ItemRec {
    int64_t row0;
    int32_t L, k0, h;  // L < 0: no items left; h: the K / V head
    int32_t pad;
  };
  auto load_rec = [&](int64_t item) {
    ItemRec e;
    e.pad = 0;
    if (item < 0) {
      e.row0 = 0;
      e.L = -1;
      e.k0 = e.h = 0;
      return e;
    }
    const WorkItem wi = decode_item(p.sched, p.B, p.Hkv, item);
    e.h = wi.head;  // K / V head; its G query heads are walked in turn
    e.row0 = load_offset(p.offs, p.is64, wi.seq);
    e.L = (int)(load_offset(p.offs, p.is64, wi.seq + 1) - e.row0);
    e.k0 = wi.j * BN;  // causal: the first key tile has the most query tiles
    return e;
  };
  // Grouped-query attention: an item's K / V tile serves G query heads, so it
  // walks n_it query tiles for each of them (G = 1: plain attention) and
  // accumulates dK, dV over all G * n_it tiles.  Iteration `it` counts those:
  // query tile i_first + it % n_it of query head h * G + it / n_it.
  // (Separate instantiation without grouping: the index arithmetic cost 6% of
  // the backward when it ran for G = 1 too.)
  struct Walk {
    int i_first, n_it, n_all;
  };
  auto walk = [&](const ItemRec& e) {
    Walk w;
    const int nq = (e.L + BQ - 1) / BQ;
    w.i_first = CAUSAL ? e.k0 / BQ : 0;
    w.n_it = nq - w.i_first;  // >= 1 since k0 < L
    w.n_all = GQA ? w.n_it * p.G : w.n_it;
    return w;
  };
  auto q_tile = [&](const Walk& w, int it_) { return GQA ? w.i_first + it_ % w.n_it : w.i_first + it_; };
  auto q_head = [&](const ItemRec& e, const Walk& w, int it_) {
    return GQA ? e.h * p.G + it_ / w.n_it : e.h;
  };

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  {
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if ((uint32_t)(smem - smem_raw) + (uint32_t)C::OFF_END > dyn) {
      if (threadIdx.x == 0) record_device_error(p.status, SCREE_DEVERR_BAD_INPUT, 91);
      return;
    }
  }
  const uint32_t sK = smem_u32(smem + C::OFF_K), sV = smem_u32(smem + C::OFF_V);
  const uint32_t sQ = smem_u32(smem + C::OFF_Q), sDO = smem_u32(smem + C::OFF_DO);
  const uint32_t sPT = smem_u32(smem + C::OFF_PT), sDS = smem_u32(smem + C::OFF_DS);
  float* lds = reinterpret_cast<float*>(smem + C::OFF_LD);  // [buf][0 lse | 1 delta][BQ]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;               // [STAGES]
  uint64_t* q_empty = q_full + C::STAGES;    // [STAGES]
  uint64_t* s_full = q_empty + C::STAGES;  // [2]: one per S^T buffer (SDB)
  uint64_t* dp_full = s_full + 2;
  uint64_t* p_full = dp_full + 1;
  uint64_t* ds_full = p_full + 1;
  uint64_t* p_free = ds_full + 1;
  uint64_t* ds_free = p_free + 1;
  uint64_t* dq_full = ds_free + 1;
  uint64_t* dq_empty = dq_full + 1;
  uint64_t* acc_done = dq_empty + 1;
  uint64_t* acc_empty = acc_done + 1;   // the epilogue has read dV, dK
  uint64_t* kv_empty = acc_empty + 1;   // an item's last MMA is done with K, V
  uint64_t* item_full = kv_empty + 1;   // [kItemRing]
  uint64_t* item_empty = item_full + kItemRing;
  ItemRec* item_ring = reinterpret_cast<ItemRec*>(item_empty + kItemRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_ring + kItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
#ifdef SCREE_TRACE
  const long long t_cta0 = clock64();
#endif

#ifdef SCREE_TRACE
  if (threadIdx.x < 64) scree_trace_sm[threadIdx.x] = 0;
#endif
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(dp_full, 1);
    mbar_init(p_full, C::SWT);
    mbar_init(ds_full, C::SWT);
    mbar_init(p_free, 1);
    mbar_init(ds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(acc_done, 1);
    mbar_init(acc_empty, C::SWT);
    mbar_init(kv_empty, 1);
    for (int k = 0; k < kItemRing; ++k) {
      mbar_init(&item_full[k], 1);
      mbar_init(&item_empty[k], C::ITEM_CONSUMERS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  constexpr int W_TMA = C::SWT / 32, W_MMA = W_TMA + 1, W_DQ = W_TMA + 4;
  if (warp == W_MMA) tmem_alloc<C::TMEM_COLS>(tmem_slot);
  if (warp == W_TMA && (threadIdx.x & 31) == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Record of item k of this CTA from the ring (L < 0: none left); false if the
  // wait gave up.  `release` = false keeps the slot (released by the caller).
  auto take_item = [&](int k, ItemRec& e, bool release) -> bool {
    const int slot = k % kItemRing;
    if (!mbar_wait(&item_full[slot], (uint32_t)((k / kItemRing) & 1), abort_flag, p.status, 34))
      return false;
    e = item_ring[slot];  // ordered after the wait (its asm clobbers memory)
    if (release) mbar_arrive(&item_empty[slot]);
    return true;
  };

  if (warp == W_TMA) {
    // ------------------------------------------------------------ TMA producer
    if constexpr (C::NP == 2) regs_dec<kRegsOther>();
    if (elect_one()) {
      int gq = 0;  // Q / dO tiles loaded so far (ring position)
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k % kItemRing;
        if (k >= kItemRing &&
            !(ok = mbar_wait(&item_empty[slot], ((k / kItemRing) - 1) & 1, abort_flag, p.status, 35)))
          break;
        int64_t item = (int64_t)atomicAdd(item_counter(p.sched), 1ull);
        if (item >= n_items) item = -1;
        const ItemRec e = load_rec(item);
        item_ring[slot] = e;
        mbar_arrive(&item_full[slot]);  // release: the record is visible to the readers
        if (item < 0) break;
        const Walk w = walk(e);
        // K, V are overwritten once the previous item's last MMA has completed.
        if (k > 0 && !(ok = mbar_wait(kv_empty, (k - 1) & 1, abort_flag, p.status, 36))) break;
        mbar_expect_tx(kv_full, 2 * C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCHUNK; ++c) {
          tma_load_3d(smem + C::OFF_K + c * BN * C::SWB, &tm_k, kv_full, c * C::CHUNK, e.h,
                      (int)e.row0 + e.k0);
          tma_load_3d(smem + C::OFF_V + c * BN * C::SWB, &tm_v, kv_full, c * C::CHUNK, e.h,
                      (int)e.row0 + e.k0);
        }
        for (int it = 0; it < w.n_all; ++it, ++gq) {
          const int st = gq % C::STAGES;
          if (gq >= C::STAGES &&
              !(ok = mbar_wait(&q_empty[st], ((gq / C::STAGES) - 1) & 1, abort_flag, p.status, 21)))
            break;
          const int qrow = (int)e.row0 + q_tile(w, it) * BQ;
          const int hq = q_head(e, w, it);
          mbar_expect_tx(&q_full[st], 2 * C::QT_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c) {
            tma_load_3d(smem + C::OFF_Q + st * C::QT_BYTES + c * BQ * C::SWB, &tm_q, &q_full[st],
                        c * C::CHUNK, hq, qrow);
            tma_load_3d(smem + C::OFF_DO + st * C::QT_BYTES + c * BQ * C::SWB, &tm_do,
                        &q_full[st], c * C::CHUNK, hq, qrow);
          }
        }
      }
    }
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if constexpr (C::NP == 2) regs_dec<kRegsOther>();
    if (elect_one()) {
      // S^T or dP^T of the query tile at ring position gpos.
      auto issue_s_dp = [&](int gpos, bool s_part) {
        const int st = gpos % C::STAGES;
        if (s_part) {
          const uint32_t qb = sQ + st * C::QT_BYTES;
          const uint32_t col = (C::SDB && (gpos & 1)) ? C::COL_S1 : C::COL_S;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16_ss(tmem + col, kmaj<D>(sK, BN, kk), kmaj<D>(qb, BQ, kk), ID_S,
                        kk > 0 ? 1u : 0u);
          umma_commit(&s_full[C::SDB ? (gpos & 1) : 0]);
        } else {
          const uint32_t ob = sDO + st * C::QT_BYTES;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_f16_ss(tmem + C::COL_DP, kmaj<D>(sV, BN, kk), kmaj<D>(ob, BQ, kk), ID_S,
                        kk > 0 ? 1u : 0u);
          umma_commit(dp_full);
        }
      };
      int g0 = 0;  // query-tile iterations of earlier items (ring positions, phases)
      bool ok = true;
      if constexpr (C::SDB) {
        // Per tile i: dV_i, dK_i, dP_{i+1}, S_{i+2} (into tile i's S buffer, which
        // dV_i was the last to read), dQ_i.  MMAs of one thread execute in issue
        // order, so an MMA never overwrites TMEM that an earlier one still reads.
        auto wait_q = [&](int gpos) {
          return mbar_wait(&q_full[gpos % C::STAGES], (gpos / C::STAGES) & 1, abort_flag, p.status,
                           25);
        };
        for (int k = 0; ok; ++k) {
          ItemRec e;
          if (!(ok = take_item(k, e, true)) || e.L < 0) break;
          const Walk w = walk(e);
          ok = mbar_wait(kv_full, k & 1, abort_flag, p.status, 22) && wait_q(g0);
          if (!ok) break;
          tc_fence_after();
          issue_s_dp(g0, true);
          issue_s_dp(g0, false);
          if (w.n_all > 1) {
            if (!(ok = wait_q(g0 + 1))) break;
            tc_fence_after();
            issue_s_dp(g0 + 1, true);
          }
          for (int it = 0; ok && it < w.n_all; ++it) {
            const int gi = g0 + it;
            const int st = gi % C::STAGES;
            const uint32_t qb = sQ + st * C::QT_BYTES, ob = sDO + st * C::QT_BYTES;
            const uint32_t col_s = (gi & 1) ? C::COL_S1 : C::COL_S;
            if (!(ok = mbar_wait(p_full, gi & 1, abort_flag, p.status, 24))) break;
            if (it == 0 && k > 0 && !(ok = mbar_wait(acc_empty, (k - 1) & 1, abort_flag, p.status, 37)))
              break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BQ / 16; ++kk)
              umma_f16_ts(tmem + C::COL_DV, tmem + col_s + packed_col<BQ, C::NP>(kk), mnmaj<D>(ob, BQ, kk),
                          ID_ACC, (it > 0 || kk > 0) ? 1u : 0u);  // A = P^T from TMEM
            if (!(ok = mbar_wait(ds_full, gi & 1, abort_flag, p.status, 26))) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BQ / 16; ++kk)
              umma_f16_ts(tmem + C::COL_DK, tmem + C::COL_DP + packed_col<BQ, C::NP>(kk), mnmaj<D>(qb, BQ, kk),
                          ID_ACC, (it > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&q_empty[st]);  // dV_i and dK_i were the last readers of dO_i, Q_i
            if (it + 1 < w.n_all) issue_s_dp(gi + 1, false);
            if (it + 2 < w.n_all) {
              if (!(ok = wait_q(gi + 2))) break;
              tc_fence_after();
              issue_s_dp(gi + 2, true);
            }
            if (gi > 0 && !(ok = mbar_wait(dq_empty, (gi - 1) & 1, abort_flag, p.status, 27))) break;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BN / 16; ++kk) {
              if (C::DQT)
                umma_f16_ss(tmem + C::COL_DQ, mnmaj<D>(sK, BN, kk), pt_mnmaj(sDS, kk), ID_DQ,
                            kk > 0 ? 1u : 0u);
              else
                umma_f16_ss(tmem + C::COL_DQ, pt_mnmaj(sDS, kk), mnmaj<D>(sK, BN, kk), ID_DQ,
                            kk > 0 ? 1u : 0u);
            }
            umma_commit(dq_full);
            umma_commit(ds_free);
          }
          if (!ok) break;
          umma_commit(acc_done);
          umma_commit(kv_empty);
          g0 += w.n_all;
        }
      }
      for (int k = 0; ok && !C::SDB; ++k) {
        ItemRec e;
        if (!(ok = take_item(k, e, true)) || e.L < 0) break;
        const Walk w = walk(e);
        ok = mbar_wait(kv_full, k & 1, abort_flag, p.status, 22) &&
             mbar_wait(&q_full[g0 % C::STAGES], (g0 / C::STAGES) & 1, abort_flag, p.status, 23);
        if (!ok) break;
        tc_fence_after();
        issue_s_dp(g0, true);
        issue_s_dp(g0, false);
        for (int it = 0; ok && it < w.n_all; ++it) {
          const int gi = g0 + it;
          const int st = gi % C::STAGES;
          const uint32_t qb = sQ + st * C::QT_BYTES, ob = sDO + st * C::QT_BYTES;
          // dV += P^T dO_i; the item's first dV / dK overwrite the accumulators
          // once the previous item's epilogue has read them.
          if (!(ok = mbar_wait(p_full, gi & 1, abort_flag, p.status, 24))) break;
          if (it == 0 && k > 0 && !(ok = mbar_wait(acc_empty, (k - 1) & 1, abort_flag, p.status, 37)))
            break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem + C::COL_DV, tmem + C::COL_S + packed_col<BQ, C::NP>(kk), mnmaj<D>(ob, BQ, kk),
                        ID_ACC, (it > 0 || kk > 0) ? 1u : 0u);  // A = P^T from TMEM
          umma_commit(p_free);
          // S^T for the next query tile overlaps the softmax warps' dS work.
          const bool more = it + 1 < w.n_all;
          if (more) {
            const int st1 = (gi + 1) % C::STAGES;
            if (!(ok = mbar_wait(&q_full[st1], ((gi + 1) / C::STAGES) & 1, abort_flag, p.status, 25)))
              break;
            tc_fence_after();
            issue_s_dp(gi + 1, true);
          }
          // dS_i published (in TMEM over dP^T_i's columns and in smem).  dK first:
          // it reads dS^T from those TMEM columns, so dP_{i+1} (which overwrites
          // them) is issued after it; the dQ GEMM follows.
          if (!(ok = mbar_wait(ds_full, gi & 1, abort_flag, p.status, 26))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk)
            umma_f16_ts(tmem + C::COL_DK, tmem + C::COL_DP + packed_col<BQ, C::NP>(kk), mnmaj<D>(qb, BQ, kk),
                        ID_ACC, (it > 0 || kk > 0) ? 1u : 0u);
          if (more) issue_s_dp(gi + 1, false);
          if (gi > 0 && !(ok = mbar_wait(dq_empty, (gi - 1) & 1, abort_flag, p.status, 27))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            if (C::DQT)  // dQ^T = K^T dS^T : A = K (MN-major, M = D), B = dS^T (MN-major, N = q)
              umma_f16_ss(tmem + C::COL_DQ, mnmaj<D>(sK, BN, kk), pt_mnmaj(sDS, kk), ID_DQ,
                          kk > 0 ? 1u : 0u);
            else         // dQ = dS K : A = dS (MN-major, M = q), B = K (MN-major, N = D)
              umma_f16_ss(tmem + C::COL_DQ, pt_mnmaj(sDS, kk), mnmaj<D>(sK, BN, kk), ID_DQ,
                          kk > 0 ? 1u : 0u);
          }
          umma_commit(dq_full);
          umma_commit(ds_free);
          umma_commit(&q_empty[st]);
        }
        if (!ok) break;
        umma_commit(acc_done);
        umma_commit(kv_empty);  // K, V may be replaced by the next item's
        g0 += w.n_all;
      }
    }
  } else if (warp == W_TMA + 2 || warp == W_TMA + 3) {
    // idle: only completes the warpgroup's register release
    if constexpr (C::NP == 2) regs_dec<kRegsOther>();
  } else if (warp < W_TMA) {
    // ------------------------------------------------------------ P^T / dS^T
    if constexpr (C::NP == 2) regs_inc<kRegsSoftmax>();
    constexpr int QH = C::QH;                 // query columns per thread
    const int hf = warp >> 2;                 // which part of the tile's queries
    const int kr = (warp & 3) * 32 + (threadIdx.x & 31);  // key row == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float sl2 = p.scale_log2;
    const int t256 = threadIdx.x;             // 0..SWT-1 over the P/dS warpgroups
    bool ok = true;
    int g0 = 0;  // query-tile iterations of earlier items (barrier phases)
    for (int k = 0; ok; ++k) {
      ItemRec e;
      ok = __all_sync(0xffffffff, take_item(k, e, false));  // released after the epilogue
      if (!ok || e.L < 0) break;
      const Walk w = walk(e);
      const int L = e.L, k0 = e.k0;
      const int kidx = k0 + kr;
      const bool key_ok = kidx < L;
      // LSE / Delta of query tile `it` staged as [BQ lse][BQ delta] (queries past L
      // read as 0; masked below), fetched one tile ahead.
      auto fetch = [&](int it_) -> float {
        if (t256 >= 2 * BQ) return 0.f;
        const int q = q_tile(w, it_) * BQ + (t256 % BQ);
        const int64_t base = (int64_t)q_head(e, w, it_) * p.T + e.row0 + q;
        return q < L ? (t256 < BQ ? p.lse2T[base] : p.deltaT[base]) : 0.f;
      };
      float pre = fetch(0);
      for (int it = 0; it < w.n_all; ++it) {
#ifdef SCREE_TRACE
        long long t_mark = clock64();
#endif
        const int gi = g0 + it;
        const int q0 = q_tile(w, it) * BQ;
        const int qh0 = q0 + hf * QH;           // first query of this part
        float* lse_s = lds + (gi & 1) * 2 * BQ + hf * QH;
        float* del_s = lds + (gi & 1) * 2 * BQ + BQ + hf * QH;
        if (t256 < 2 * BQ) lds[(gi & 1) * 2 * BQ + t256] = pre;
        if (it + 1 < w.n_all) pre = fetch(it + 1);
        softmax_group_sync<C::SWT>();
        SW_MARK(40);
        const bool need_mask = (q0 + BQ > L) || (k0 + BN > L) || (CAUSAL && q0 < k0 + BN - 1);
        // ---- P^T (this half's QH queries) from S^T
        const uint32_t col_s = (C::SDB && (gi & 1)) ? C::COL_S1 : C::COL_S;
        ok = C::SDB ? mbar_wait(&s_full[gi & 1], (gi >> 1) & 1, abort_flag, p.status, 28)
                    : mbar_wait(s_full, gi & 1, abort_flag, p.status, 28);
        if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        SW_MARK(41);
        tc_fence_after();
        float pr[QH];
        tmem_ld_cols<QH>(lane_base + col_s + hf * QH, pr);
        tmem_wait_ld();
        tmem_regs_ready<QH>(pr);
        SW_MARK(42);
        uint32_t pk[QH / 2];
#pragma unroll
        for (int c4 = 0; c4 < QH / 4; ++c4) {
          const float4 l4 = reinterpret_cast<const float4*>(lse_s)[c4];  // one LDS.128
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = c4 * 4 + e;
            float xv = ex2_approx(fmaf(pr[c], sl2, -lv[e]));
            if (need_mask) {
              const int q = qh0 + c;
              const bool valid = key_ok && q < L && (!CAUSAL || q >= kidx);
              xv = valid ? xv : 0.f;
            }
            pr[c] = xv;
          }
          pk[c4 * 2] = Pk2b<T>::pack(pr[c4 * 4], pr[c4 * 4 + 1]);
          pk[c4 * 2 + 1] = Pk2b<T>::pack(pr[c4 * 4 + 2], pr[c4 * 4 + 3]);
        }
        SW_MARK(43);
        if (!C::SDB && gi > 0) {  // dV_{i-1} read P^T_{i-1} from these columns
          ok = mbar_wait(p_free, (gi - 1) & 1, abort_flag, p.status, 29);
          if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        }
        SW_MARK(44);
        // P^T (16-bit, two per column) over the first QH/2 of the QH fp32 columns
        // this half read: never over the other half's columns (warps w and w+4
        // share TMEM lanes and do not wait for each other).
        tmem_st_packed<QH / 2>(lane_base + col_s + hf * QH, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full);
        SW_MARK(45);
        // ---- dS^T = P^T * (dP^T - Delta)
        ok = mbar_wait(dp_full, gi & 1, abort_flag, p.status, 30);
        if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        SW_MARK(46);
        tc_fence_after();
        constexpr int DPC = QH < 32 ? QH : 32;  // dP^T columns per load
#pragma unroll
        for (int c = 0; c < QH / DPC; ++c) {
          float dp[DPC];
          tmem_ld_cols<DPC>(lane_base + C::COL_DP + hf * QH + c * DPC, dp);
          tmem_wait_ld();
          tmem_regs_ready<DPC>(dp);
#pragma unroll
          for (int e4 = 0; e4 < DPC / 4; ++e4) {
            const float4 d4 = reinterpret_cast<const float4*>(del_s)[c * (DPC / 4) + e4];
            pr[c * DPC + e4 * 4 + 0] *= (dp[e4 * 4 + 0] - d4.x);
            pr[c * DPC + e4 * 4 + 1] *= (dp[e4 * 4 + 1] - d4.y);
            pr[c * DPC + e4 * 4 + 2] *= (dp[e4 * 4 + 2] - d4.z);
            pr[c * DPC + e4 * 4 + 3] *= (dp[e4 * 4 + 3] - d4.w);
          }
        }
#pragma unroll
        for (int c = 0; c < QH / 2; ++c) pk[c] = Pk2b<T>::pack(pr[2 * c], pr[2 * c + 1]);
        SW_MARK(47);
        if (gi > 0) {
          ok = mbar_wait(ds_free, (gi - 1) & 1, abort_flag, p.status, 31);
          if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        }
        SW_MARK(48);
        // dS^T: into TMEM over dP^T's first columns (A operand of dK) and into
        // smem (B operand of the dQ GEMM).
        tmem_st_packed<QH / 2>(lane_base + C::COL_DP + hf * QH, pk);
        write_row_sw128<T, QH>(smem + C::OFF_DS, kr, pr, hf * (QH / 8));
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(ds_full);
        SW_MARK(49);
      }
      // ---- dK, dV epilogue: 32-column chunk c belongs to part c % NP
      if (ok) {
        ok = mbar_wait(acc_done, k & 1, abort_flag, p.status, 32);
        ok = __all_sync(0xffffffff, ok);
      }
      if (ok) {
        tc_fence_after();
        // The record is still held in the ring: re-read where the rows go.
        const ItemRec& er = item_ring[k % kItemRing];
        const int64_t row0 = er.row0;
        const int h = er.h;
        T* dvrow = reinterpret_cast<T*>(p.dv) + ((row0 + kidx) * p.Hkv + h) * D;
        T* dkrow = reinterpret_cast<T*>(p.dk) + ((row0 + kidx) * p.Hkv + h) * D;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const int col = pass == 0 ? C::COL_DV : C::COL_DK;
          const float mul = pass == 0 ? 1.f : p.scale;
          T* dst = pass == 0 ? dvrow : dkrow;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            if ((c % C::NP) != hf) continue;
            float v[32];
            tmem_ld32(lane_base + col + c * 32, v);
            tmem_wait_ld();
            if (key_ok) {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                uint4 w;
                w.x = Pk2b<T>::pack(v[u * 8 + 0] * mul, v[u * 8 + 1] * mul);
                w.y = Pk2b<T>::pack(v[u * 8 + 2] * mul, v[u * 8 + 3] * mul);
                w.z = Pk2b<T>::pack(v[u * 8 + 4] * mul, v[u * 8 + 5] * mul);
                w.w = Pk2b<T>::pack(v[u * 8 + 6] * mul, v[u * 8 + 7] * mul);
                *reinterpret_cast<uint4*>(dst + c * 32 + u * 8) = w;
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(acc_empty);  // dV, dK are read: the next item may overwrite them
      }
      if (ok) mbar_arrive(&item_empty[k % kItemRing]);
      g0 += w.n_all;
    }
  } else {
    // ------------------------------------------------------------ dQ reduction warps
    if constexpr (C::NP == 2) regs_dec<kRegsDq>();
    const int ln = threadIdx.x - W_DQ * 32;  // TMEM lane: feature d (DQT) or query row
    const uint32_t lane_base = tmem + ((uint32_t)((warp - W_DQ) * 32) << 16);
    const float sc = p.scale;
    int g0 = 0;  // query-tile iterations of earlier items (barrier phases)
    bool ok = true;
    for (int k = 0; ok; ++k) {
      ItemRec e;
      ok = __all_sync(0xffffffff, take_item(k, e, true));
      if (!ok || e.L < 0) break;
      const Walk w = walk(e);
      const int64_t row0 = e.row0;
      const int L = e.L;
      for (int it = 0; it < w.n_all; ++it) {
        const int gi = g0 + it;
        const int q0 = q_tile(w, it) * BQ;
        const int hq = q_head(e, w, it);
        ok = mbar_wait(dq_full, gi & 1, abort_flag, p.status, 33);
        if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        tc_fence_after();
        if (C::DQT) {
          float v[BQ];
#pragma unroll
          for (int c = 0; c < BQ / 32; ++c)
            tmem_ld32(lane_base + C::COL_DQ + c * 32, *reinterpret_cast<float(*)[32]>(&v[c * 32]));
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(dq_empty);
          {
          // Stage the scaled dQ tile as [BQ][D] fp32 and add it into dq_acc with one
          // TMA reduce.  Queries >= L carry exact zeros (their dS is 0), so adding
          // the whole box is safe even where it overlaps the next sequence.
          if (ln == 0 && gi > 0) bulk_wait_read_all();
          dq_group_sync();
          float* sdq = reinterpret_cast<float*>(smem + C::OFF_DQ);
#pragma unroll
          for (int c = 0; c < BQ; ++c) sdq[c * D + ln] = v[c] * sc;
          fence_proxy_async_smem();
          dq_group_sync();
          if (ln == 0) {
            tma_reduce_add_3d(&tm_dq, sdq, 0, hq, (int)(row0 + q0));
            bulk_commit();
          }
          }
        } else {
          const int q = q0 + ln;
          float* base = p.dq_acc + ((row0 + q) * p.H + hq) * D;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float v[32];
            tmem_ld32(lane_base + C::COL_DQ + c * 32, v);
            tmem_wait_ld();
            if (q < L) {
#pragma unroll
              for (int u = 0; u < 8; ++u)
                red_add_v4(base + c * 32 + u * 4, v[u * 4] * sc, v[u * 4 + 1] * sc,
                           v[u * 4 + 2] * sc, v[u * 4 + 3] * sc);
            }
          }
          tc_fence_before();
          mbar_arrive(dq_empty);
        }
      }
      g0 += w.n_all;
    }
    if (C::DQT && ln == 0) bulk_wait_all();  // smem must outlive the reduces
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
#ifdef SCREE_TRACE
  if (threadIdx.x == 0) {
    scree_trace_sm[62] += (unsigned long long)(clock64() - t_cta0);
  }
  __syncthreads();
  if (threadIdx.x < 64) atomicAdd(&g_bwd_trace[threadIdx.x], scree_trace_sm[threadIdx.x]);
#endif
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc<C::TMEM_COLS>(tmem);
  }
}

// Delta[h][t] = sum_d O[t,h,d] * dO[t,h,d] (fp32) and lse2T[h][t] = lse[t,h] * log2(e).
// 8 threads per (t, h) row, 16-byte loads.
template <typename T, int D>
__global__ void bwd_preprocess_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                      const float* __restrict__ lse, int64_t T_, int H,
                                      float* __restrict__ deltaT, float* __restrict__ lse2T) {
  constexpr int TPR = 8;
  constexpr int EPT = D / TPR;  // elements per thread (4, 8 or 16)
  const int64_t nrows = T_ * H;
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t row = gid / TPR;
  const int sub = (int)(gid % TPR);
  float acc = 0.f;
  if (row < nrows) {
    const T* op = o + row * D + sub * EPT;
    const T* dp = dout + row * D + sub * EPT;
#pragma unroll
    for (int e = 0; e < EPT; e += 4) {
      const uint2 a = *reinterpret_cast<const uint2*>(op + e);
      const uint2 b = *reinterpret_cast<const uint2*>(dp + e);
      const T* ah = reinterpret_cast<const T*>(&a);
      const T* bh = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int k = 0; k < 4; ++k) acc += Cvt<T>::to_f(ah[k]) * Cvt<T>::to_f(bh[k]);
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, off);
  if (row < nrows && sub == 0) {
    const int64_t t = row / H;
    const int hh = (int)(row % H);
    deltaT[(int64_t)hh * T_ + t] = acc;
    lse2T[(int64_t)hh * T_ + t] = lse[row] * 1.4426950408889634f;
  }
}

// dq (dtype) = dq_acc (fp32), 4 elements per thread.
template <typename T>
__global__ void cast_dq_kernel(const float* __restrict__ acc, T* __restrict__ dq, int64_t n4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(acc)[i];
    uint2 w;
    w.x = Pk2b<T>::pack(v.x, v.y);
    w.y = Pk2b<T>::pack(v.z, v.w);
    reinterpret_cast<uint2*>(dq)[i] = w;
  }
}

template <int D, typename T, bool CAUSAL, bool GQA>
int launch_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
               const CUtensorMap& tdo, const CUtensorMap& tdq, const BwdParams& p, int64_t grid,
               cudaStream_t s) {
  auto kern = attn_bwd_kernel<D, T, CAUSAL, GQA>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    SCREE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BwdCfg<D>::SMEM));
    attr_set[dev & 63] = true;
  }
  ProfScope prof(PROF_ATTN_BWD, s);
  kern<<<(unsigned)grid, BwdCfg<D>::THREADS, BwdCfg<D>::SMEM, s>>>(tq, tk, tv, tdo, tdq, p);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

struct BwdWs {
  size_t off_dq, off_delta, off_lse2, off_sched, total;
};
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
BwdWs bwd_ws_layout(int64_t B, int64_t T, int64_t H, int D) {
  BwdWs w;
  w.off_dq = 0;
  w.off_delta = align256(w.off_dq + (size_t)T * H * D * 4);
  w.off_lse2 = align256(w.off_delta + (size_t)T * H * 4);
  w.off_sched = align256(w.off_lse2 + (size_t)T * H * 4);
  w.total = w.off_sched + schedule_bytes(B);
  return w;
}

template <typename T>
int run_bwd_typed(const void* dout, const void* q, const void* k, const void* v, const void* o,
                  const float* lse, const void* offsets, int is64, int64_t B, int64_t Tn, int64_t H,
                  int64_t Hkv, int D, int causal, float scale, void* dq, void* dk, void* dv,
                  char* ws, const BwdWs& L, cudaStream_t s) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const int swb = D >= 64 ? 128 : 64;
  const int bq = D == 128 ? 64 : 128;
  CUtensorMap tq, tk, tv, tdo;
  int rc;
  const int64_t rs = H * D, rs_kv = Hkv * D, hs = D;
  if ((rc = make_thd_map(&tq, q, Tn, H, D, rs, hs, swb / 2, bq, swb, bf16))) return rc;
  if ((rc = make_thd_map(&tdo, dout, Tn, H, D, rs, hs, swb / 2, bq, swb, bf16))) return rc;
  if ((rc = make_thd_map(&tk, k, Tn, Hkv, D, rs_kv, hs, swb / 2, BN, swb, bf16))) return rc;
  if ((rc = make_thd_map(&tv, v, Tn, Hkv, D, rs_kv, hs, swb / 2, BN, swb, bf16))) return rc;

  float* dq_acc = reinterpret_cast<float*>(ws + L.off_dq);
  CUtensorMap tdq;
  if ((rc = make_thd_map_f32(&tdq, dq_acc, Tn, H, D, bq))) return rc;
  float* deltaT = reinterpret_cast<float*>(ws + L.off_delta);
  float* lse2T = reinterpret_cast<float*>(ws + L.off_lse2);
  void* sched = ws + L.off_sched;
  SCREE_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, (size_t)Tn * H * D * 4, s));
  {
    const int64_t threads = Tn * H * 8;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (D == 128) bwd_preprocess_kernel<T, 128><<<blocks, 256, 0, s>>>((const T*)o, (const T*)dout, lse, Tn, (int)H, deltaT, lse2T);
    else if (D == 64) bwd_preprocess_kernel<T, 64><<<blocks, 256, 0, s>>>((const T*)o, (const T*)dout, lse, Tn, (int)H, deltaT, lse2T);
    else bwd_preprocess_kernel<T, 32><<<blocks, 256, 0, s>>>((const T*)o, (const T*)dout, lse, Tn, (int)H, deltaT, lse2T);
    SCREE_LAUNCH_CHECK();
  }
  // One work item per (key tile, K / V head): the CTA walks all G query heads.
  if ((rc = launch_build_schedule(offsets, is64, B, Tn, BN, (int)Hkv, sched, s))) return rc;
  BwdParams p;
  p.offs = offsets;
  p.is64 = is64;
  p.H = (int)H;
  p.Hkv = (int)Hkv;
  p.G = (int)(H / Hkv);
  p.T = (int)Tn;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.sched = sched;
  p.B = B;
  p.status = device_status_ptr();
  p.lse2T = lse2T;
  p.deltaT = deltaT;
  p.dq_acc = dq_acc;
  p.dk = dk;
  p.dv = dv;
  // Persistent CTAs, one per SM (each holds all 512 TMEM columns); the items
  // themselves are counted on the device.
  const int64_t grid = std::min<int64_t>(max_tiles(B, Tn, BN) * Hkv, (int64_t)num_sms());
#define SCREE_BWD_CASE(DD)                                                        \
  if (D == DD) {                                                                  \
    if (p.G > 1)                                                                  \
      rc = causal ? launch_bwd<DD, T, true, true>(tq, tk, tv, tdo, tdq, p, grid, s) \
                  : launch_bwd<DD, T, false, true>(tq, tk, tv, tdo, tdq, p, grid, s); \
    else                                                                          \
      rc = causal ? launch_bwd<DD, T, true, false>(tq, tk, tv, tdo, tdq, p, grid, s) \
                  : launch_bwd<DD, T, false, false>(tq, tk, tv, tdo, tdq, p, grid, s); \
  }
  SCREE_BWD_CASE(128)
  SCREE_BWD_CASE(64)
  SCREE_BWD_CASE(32)
#undef SCREE_BWD_CASE
  if (rc) return rc;
  const int64_t n4 = Tn * H * D / 4;
  const unsigned cgrid = (unsigned)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms() * 16);
  cast_dq_kernel<T><<<cgrid, 256, 0, s>>>(dq_acc, (T*)dq, n4);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

}  // namespace
}  // namespace scree

using namespace scree;

extern "C" size_t scree_attn_bwd_workspace_size(int64_t B, int64_t T, int64_t H, int D) {
  return bwd_ws_layout(B, T, H, D).total;
}

extern "C" int scree_attn_bwd(const void* dout, const void* q, const void* k, const void* v,
                              const void* o, const float* lse, const void* offsets,
                              int offs_is_i64, int64_t B, int64_t T, int64_t H, int D, int dtype,
                              int causal, float scale, int64_t max_seqlen, void* dq, void* dk,
                              void* dv, void* workspace, size_t workspace_bytes, void* stream) {
  return scree_attn_bwd_gqa(dout, q, k, v, o, lse, offsets, offs_is_i64, B, T, H, H, D, dtype,
                            causal, scale, max_seqlen, dq, dk, dv, workspace, workspace_bytes,
                            stream);
}

extern "C" int scree_attn_bwd_gqa(const void* dout, const void* q, const void* k, const void* v,
                                  const void* o, const float* lse, const void* offsets,
                                  int offs_is_i64, int64_t B, int64_t T, int64_t H, int64_t H_kv,
                                  int D, int dtype, int causal, float scale, int64_t max_seqlen,
                                  void* dq, void* dk, void* dv, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  (void)max_seqlen;
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && H >= 1 && H_kv >= 1, "attn_bwd: bad sizes");
  SCREE_CHECK_ARG(H % H_kv == 0, "attn_bwd: query heads (%lld) must be a multiple of K/V heads (%lld)",
                  (long long)H, (long long)H_kv);
  SCREE_CHECK_ARG(T < (1ll << 31) && H < 65536, "attn_bwd: T or H too large");
  if (D != 32 && D != 64 && D != 128) {
    set_last_error("attn_bwd: head_dim %d unsupported (32, 64, 128)", D);
    return SCREE_ERR_UNSUPPORTED;
  }
  SCREE_CHECK_ARG(dtype == SCREE_F16 || dtype == SCREE_BF16 || dtype == SCREE_F32,
                  "attn_bwd: fp16, bf16 or fp32 only");
  if (T == 0) return SCREE_OK;
  SCREE_CHECK_ARG(dout && q && k && v && o && lse && offsets && dq && dk && dv,
                  "attn_bwd: null pointer");
  const BwdWs L = bwd_ws_layout(B, T, H, D);
  SCREE_CHECK_ARG(workspace && workspace_bytes >= L.total,
                  "attn_bwd: workspace too small (%zu < %zu)", workspace_bytes, L.total);
  const void* ptrs[8] = {dout, q, k, v, o, dq, dk, dv};
  for (const void* ptr : ptrs)
    SCREE_CHECK_ARG(((uintptr_t)ptr % 16) == 0, "attn_bwd: tensors must be 16-byte aligned");
  SCREE_BIND_DEVICE(stream, q);
  cudaStream_t s = (cudaStream_t)stream;
  char* ws = reinterpret_cast<char*>(workspace);
  if (dtype == SCREE_F32)
    return attn_bwd_f32(dout, q, k, v, o, lse, offsets, offs_is_i64, B, T, H, H_kv, D, causal,
                        scale, dq, dk, dv, reinterpret_cast<float*>(ws + L.off_delta), s);
  if (dtype == SCREE_BF16)
    return run_bwd_typed<__nv_bfloat16>(dout, q, k, v, o, lse, offsets, offs_is_i64, B, T, H, H_kv,
                                        D, causal, scale, dq, dk, dv, ws, L, s);
  return run_bwd_typed<__half>(dout, q, k, v, o, lse, offsets, offs_is_i64, B, T, H, H_kv, D,
                               causal, scale, dq, dk, dv, ws, L, s);
}

#ifdef SCREE_TRACE
extern "C" int scree_bwd_trace_read(unsigned long long* out64, int reset) {
  SCREE_CUDA_TRY(cudaDeviceSynchronize());
  SCREE_CUDA_TRY(cudaMemcpyFromSymbol(out64, g_bwd_trace, sizeof(unsigned long long) * 64));
  if (reset) {
    unsigned long long z[64] = {0};
    SCREE_CUDA_TRY(cudaMemcpyToSymbol(g_bwd_trace, z, sizeof(z)));
  }
  return SCREE_OK;
}
#endif
