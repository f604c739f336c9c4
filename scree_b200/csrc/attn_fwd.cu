// attn_fwd.cu — varlen self-attention forward on sm_100a tensor cores.
//
// Computes, per sequence b and head h (reference/varlen_attention.py:121-138):
//   S = Q K^T * scale, causal mask k > q -> -inf, P = softmax(S), O = P V,
//   LSE = m + ln(l)  (natural log; triton/varlen_attention.py:160)
//
// A work item is 256 query rows of one head as two 128-row tiles, A and B, that
// share every 128-key K/V tile the sequence streams through shared memory, so
// each K/V byte feeds twice the tensor work of a single-tile item (the L2 -> SM
// feed of K/V is what limits a 128-row tile).  The kernel is persistent: one
// CTA per SM takes items in schedule order from a device counter, and the
// rings and barrier phases below run on across its items.
//
//   warp 8  (TMA)  lane 0: Q_A, Q_B once, then the K ring; lane 1: the V ring
//   warp 9  (MMA)  one thread issues tcgen05.mma: S_X = Q_X K_j^T (X = A, B) and
//                  O_X += P_X V_j, interleaved so the tensor core works on one
//                  tile while the softmax warps of the other tile run
//   warps 0-3      softmax of tile A, warps 4-7 softmax of tile B: thread r owns
//                  query row r (= TMEM lane r), keeps the running max / sum in
//                  registers, writes P (16-bit) back into TMEM, rescales O only
//                  when the max grew by more than 2^8 (exact: P stays <= 256),
//                  and finally stores O / l and the LSE.
//
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [256+D,256+2D).
// P_X is written over the first 64 columns of S_X (two 16-bit values per
// column) and read by O_X += P_X V_j straight from TMEM (A operand in TMEM).
// Reuse is safe because one thread issues all MMAs and they execute in issue
// order: S_X(j+1) is issued after O_X += P_X(j) V_j.
// Softmax works in the exp2 domain with log2(e) folded into the scale.
// Ragged tails: TMA reads whole 128-row boxes, so rows of the next sequence
// arrive in K/V tiles; keys >= L are masked to -inf (P = 0), and query rows
// >= L are computed but never stored.  Rows past T are zero-filled by TMA.
#ifdef SCREE_TRACE
// Profiling build only: per-site wait cycles (lane 0 of each waiting warp),
// [30] = CTA lifetime cycles.
static __device__ unsigned long long g_fwd_trace[32];
#define SCREE_TRACE_ADD(site, cyc) \
  do { if ((threadIdx.x & 31) == 0 || (site) == 12) atomicAdd(&scree_trace_sm[(site) & 31], (unsigned long long)(cyc)); } while (0)
static __shared__ unsigned long long scree_trace_sm[32];  // per-CTA, flushed at exit
#endif
#include <atomic>
#include "attn_common.cuh"

namespace scree {
namespace {

constexpr int BM = 128;      // rows per query tile
constexpr int ROWS = 2 * BM; // query rows per CTA (tiles A and B)
constexpr int BN = 128;      // keys per K/V tile
// 8 softmax warps (warpgroups 0, 1), then warpgroup 2: TMA warp, MMA warp and two
// idle warps.  Launched at 168 registers per thread (65,536 / 384); the
// softmax warpgroups grow to 208 and warpgroup 2 shrinks to 88:
// 256 x 208 + 128 x 88 = 64,512 = 384 x 168.  (224 / 56 left the MMA and TMA
// warps spilling and measured 3% slower.)
constexpr int kThreads = 384;
constexpr int kRegsSoftmax = 208, kRegsOther = 88;
// P_X(j) is handed to the MMA warp in kPParts parts (of BN / kPParts keys);
// 2 parts measured 1.5% faster than 1 and 4% faster than 4 at cfg4.
#ifndef SCREE_P_PARTS
#define SCREE_P_PARTS 2
#endif
constexpr int kPParts = SCREE_P_PARTS;
// Work items reach the CTA's roles through a ring of item ids: the K-loading
// TMA lane takes the next item from the schedule's counter (one atomic per
// item) and publishes it; the V lane, the MMA thread and the 256 softmax
// threads read it.
constexpr int kItemRing = 4;
constexpr int kItemConsumers = 1 + 1 + 256;
static_assert(kPParts == 2 || kPParts == 4, "P parts: 2 or 4");

template <int D>
struct FwdCfg {
  static constexpr int SWB = D >= 64 ? 128 : 64;  // swizzle span in bytes (one smem row)
  static constexpr int CHUNK = SWB / 2;           // elements per swizzle row
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr uint32_t SWZ = SWB == 128 ? SW_128B : SW_64B;
  // K_j frees after both S GEMMs of iteration j-1, V_j only after both PV GEMMs
  // of iteration j; V gets the deeper ring (it has one iteration less slack).
  static constexpr int KSTAGES = D == 128 ? 2 : 3;
  static constexpr int VSTAGES = 3;
  static constexpr int Q_BYTES = BM * D * 2;   // one query tile
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;              // Q_A, Q_B
  static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KSTAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + VSTAGES * KV_BYTES;
  static constexpr int OFF_END = OFF_BAR + 512;  // mbarriers, item ring, TMEM slot, abort flag
  static constexpr int SMEM_RAW = OFF_END + 1024 <= 232448 ? OFF_END + 1024 : OFF_END;
  // At least 120 KB so that two CTAs (each holding all 512 TMEM columns) never
  // share an SM.
  static constexpr int SMEM = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
  static constexpr int COL_S = 0, COL_O = 256;  // S_X at COL_S + X*128, O_X at COL_O + X*D
};

struct FwdParams {
  const void* offs;
  int is64;
  int H;  // query heads
  int G;  // query heads per K / V head (grouped-query attention; 1 = plain)
  int T;
  float scale_log2;
  const void* sched;  // schedule (attn_common.cuh)
  const void* offs_k; // key / value offsets when they differ from the query offsets, else null
  int64_t B;
  int* status;  // device status word
  void* o;
  int64_t o_rs, o_hs;
  float* lse;
};

// K-major operand descriptor for k-step `kk` (16 elements) of a [rows][D] tile
// stored as NCHUNK column blocks of [rows][SWB bytes].
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int rows, int kk) {
  using C = FwdCfg<D>;
  const int e = kk * 16;
  const uint32_t addr = base + (e / C::CHUNK) * rows * C::SWB + (e % C::CHUNK) * 2;
  return make_sdesc(addr, 16, 8 * C::SWB, C::SWZ);
}
// V as the MN-major B operand (N = D, K = keys): k-step kk covers keys
// [16kk, 16kk+16) = 16 smem rows; D-chunks are BN*SWB bytes apart (LBO), groups of
// 8 keys are 8*SWB apart (SBO).
template <int D>
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int kk) {
  using C = FwdCfg<D>;
  return make_sdesc(base + kk * 16 * C::SWB, BN * C::SWB, 8 * C::SWB, C::SWZ);
}

template <typename T> struct Pk2;
template <> struct Pk2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Pk2<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <int D, typename T, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = FwdCfg<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = make_idesc_f16(BM, BN, kBF16, false, false);
  constexpr uint32_t IDESC_O = make_idesc_f16(BM, D, kBF16, false, true);

  // Persistent: one CTA per SM takes items of the longest-first schedule from
  // a device counter, in order, as its K loads get to them (list scheduling);
  // every role decodes the items it reads from the CTA's item ring on its own.
  const int64_t n_items = total_items(p.sched);
  if ((int64_t)blockIdx.x >= n_items) return;
  // A CTA of an earlier failed launch (or of this one) set the status word: skip.
  if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) return;
  // What the producer publishes per item (read from the schedule and the
  // offsets once, by one thread), and what every role derives from it.
  struct ItemRec {
    int64_t seq_start, kv_start;
    int32_t L, Lk, h, q0;  // L < 0: no items left
  };
  struct Geom {
    int nA, nB, n_kv;
    bool hasB;
  };
  auto load_rec = [&](int64_t item) {
    ItemRec e;
    if (item < 0) {
      e.seq_start = e.kv_start = 0;
      e.L = e.Lk = -1;
      e.h = e.q0 = 0;
      return e;
    }
    const WorkItem wi = decode_item(p.sched, p.B, p.H, item);
    e.h = wi.head;
    e.seq_start = load_offset(p.offs, p.is64, wi.seq);
    e.L = (int)(load_offset(p.offs, p.is64, wi.seq + 1) - e.seq_start);  // query rows
    // Keys: the same rows, or (KV-cache attention) a sequence of its own; causal
    // masking is then aligned at the end: query i sees keys <= i + (Lk - L).
    e.kv_start = e.seq_start;
    e.Lk = e.L;
    if (p.offs_k != nullptr) {
      e.kv_start = load_offset(p.offs_k, p.is64, wi.seq);
      e.Lk = (int)(load_offset(p.offs_k, p.is64, wi.seq + 1) - e.kv_start);
    }
    // Causal: heaviest (last) 256-row block first within each (sequence, head).
    e.q0 = (CAUSAL ? (wi.ntiles - 1 - wi.j) : wi.j) * ROWS;
    return e;
  };
  auto derive = [](int L, int Lk, int q0) {
    Geom g;
    const int cdelta = Lk - L;
    const int nk_all = (Lk + BN - 1) / BN;
    // Key tiles each query tile needs (tile B may not exist at a sequence's end).
    auto tiles_upto = [&](int last_q) {
      const int last_k = last_q + cdelta;
      return last_k < 0 ? 0 : min(nk_all, last_k / BN + 1);
    };
    g.nA = CAUSAL ? tiles_upto(q0 + BM - 1) : nk_all;
    g.hasB = q0 + BM < L;
    g.nB = !g.hasB ? 0 : (CAUSAL ? tiles_upto(q0 + 2 * BM - 1) : nk_all);
    g.n_kv = max(g.nA, g.nB);
    return g;
  };

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  {
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if ((uint32_t)(smem - smem_raw) + (uint32_t)C::OFF_END > dyn) {
      if (threadIdx.x == 0) record_device_error(p.status, SCREE_DEVERR_BAD_INPUT, 90);
      return;
    }
  }
  const uint32_t sQ = smem_u32(smem + C::OFF_Q);
  const uint32_t sK = smem_u32(smem + C::OFF_K);
  const uint32_t sV = smem_u32(smem + C::OFF_V);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                  // [KSTAGES]
  uint64_t* k_empty = k_full + C::KSTAGES;      // [KSTAGES]
  uint64_t* v_full = k_empty + C::KSTAGES;      // [VSTAGES]
  uint64_t* v_empty = v_full + C::VSTAGES;      // [VSTAGES]
  uint64_t* s_full = v_empty + C::VSTAGES;      // [2] per tile X
  uint64_t* p_full = s_full + 2;                // [2]
  uint64_t* pv_done = p_full + 2;               // [2]
  uint64_t* p_part = pv_done + 2;               // [2][kPParts - 1] leading parts of P_X
  uint64_t* q_empty = p_part + 2 * (kPParts - 1);  // an item's last S GEMM is done with Q
  uint64_t* o_empty = q_empty + 1;                 // [2] the epilogue has read O_X
  uint64_t* item_full = o_empty + 2;               // [kItemRing] an item id is published
  uint64_t* item_empty = item_full + kItemRing;    // [kItemRing] every role has read it
  ItemRec* item_ring = reinterpret_cast<ItemRec*>(item_empty + kItemRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_ring + kItemRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
#ifdef SCREE_TRACE
  const long long t_cta0 = clock64();
#endif

#ifdef SCREE_TRACE
  if (threadIdx.x < 32) scree_trace_sm[threadIdx.x] = 0;
#endif
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::KSTAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < C::VSTAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 128);
      for (int q = 0; q + 1 < kPParts; ++q) mbar_init(&p_part[x * (kPParts - 1) + q], 128);
      mbar_init(&pv_done[x], 1);
      mbar_init(&o_empty[x], 128);
    }
    mbar_init(q_empty, 1);
    for (int k = 0; k < kItemRing; ++k) {
      mbar_init(&item_full[k], 1);
      mbar_init(&item_empty[k], kItemConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc<512>(tmem_slot);
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Record of item k of this CTA from the ring (L < 0: none left); false if the
  // wait gave up.  `release` = false leaves the slot held (released later by
  // release_item), so that the record can be read again.
  auto take_item = [&](int k, ItemRec& e, bool release) -> bool {
    const int slot = k % kItemRing;
    if (!mbar_wait(&item_full[slot], (uint32_t)((k / kItemRing) & 1), abort_flag, p.status, 16))
      return false;
    e = item_ring[slot];  // ordered after the wait (its asm clobbers memory)
    if (release) mbar_arrive(&item_empty[slot]);
    return true;
  };
  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    regs_dec<kRegsOther>();
    // Ring positions run on across items: kc / vc = K / V tiles loaded so far,
    // qc = items with keys so far (items with n_kv = 0 load and compute nothing).
    if (lane == 0) {
      int kc = 0, qc = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k % kItemRing;
        if (k >= kItemRing &&
            !(ok = mbar_wait(&item_empty[slot], ((k / kItemRing) - 1) & 1, abort_flag, p.status, 15)))
          break;
        int64_t item = (int64_t)atomicAdd(item_counter(p.sched), 1ull);
        if (item >= n_items) item = -1;
        const ItemRec e = load_rec(item);
        item_ring[slot] = e;
        mbar_arrive(&item_full[slot]);  // release: the record is visible to the readers
        if (item < 0) break;
        const Geom g = derive(e.L, e.Lk, e.q0);
        if (g.n_kv == 0) continue;
        const int row0 = (int)e.seq_start, krow0 = (int)e.kv_start, hkv = e.h / p.G;
        // Q is overwritten once the previous item's last S GEMM has completed.
        if (qc > 0 && !(ok = mbar_wait(q_empty, (qc - 1) & 1, abort_flag, p.status, 13))) break;
        mbar_expect_tx(q_full, (g.hasB ? 2 : 1) * C::Q_BYTES);
        for (int x = 0; x < (g.hasB ? 2 : 1); ++x)
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_3d(smem + C::OFF_Q + x * C::Q_BYTES + c * BM * C::SWB, &tm_q, q_full,
                        c * C::CHUNK, e.h, row0 + e.q0 + x * BM);
        for (int j = 0; j < g.n_kv; ++j, ++kc) {
          const int st = kc % C::KSTAGES;
          if (kc >= C::KSTAGES &&
              !(ok = mbar_wait(&k_empty[st], ((kc / C::KSTAGES) - 1) & 1, abort_flag, p.status, 1)))
            break;
          mbar_expect_tx(&k_full[st], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_3d(smem + C::OFF_K + st * C::KV_BYTES + c * BN * C::SWB, &tm_k, &k_full[st],
                        c * C::CHUNK, hkv, krow0 + j * BN);
        }
        ++qc;
      }
    } else if (lane == 1) {
      int vc = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        ItemRec e;
        if (!(ok = take_item(k, e, true)) || e.L < 0) break;
        const Geom g = derive(e.L, e.Lk, e.q0);
        const int krow0 = (int)e.kv_start, hkv = e.h / p.G;
        for (int j = 0; j < g.n_kv; ++j, ++vc) {
          const int st = vc % C::VSTAGES;
          if (vc >= C::VSTAGES &&
              !(ok = mbar_wait(&v_empty[st], ((vc / C::VSTAGES) - 1) & 1, abort_flag, p.status, 12)))
            break;
          mbar_expect_tx(&v_full[st], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_3d(smem + C::OFF_V + st * C::KV_BYTES + c * BN * C::SWB, &tm_v, &v_full[st],
                        c * C::CHUNK, hkv, krow0 + j * BN);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    regs_dec<kRegsOther>();
    if (elect_one()) {
      // Descriptors differ per k-step only in the start address (bits [0,14) =
      // addr >> 4), so they are built once per buffer and advanced by adding
      // the step's byte offset >> 4 (addresses stay below 256 KB: no carry).
      auto kstep_off = [](int kk, int rows) -> uint32_t {
        const int e = kk * 16;
        return (uint32_t)(((e / C::CHUNK) * rows * C::SWB + (e % C::CHUNK) * 2) >> 4);
      };
      // S_X = Q_X K^T with K from ring position kpos.
      auto issue_s = [&](int x, int kpos) {
        const uint32_t kb = sK + (kpos % C::KSTAGES) * C::KV_BYTES;
        const uint32_t qb = sQ + x * C::Q_BYTES;
        const uint64_t dq = kmajor_desc<D>(qb, BM, 0), dk = kmajor_desc<D>(kb, BN, 0);
        const uint32_t dt = tmem + C::COL_S + x * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(dt, dq + kstep_off(kk, BM), dk + kstep_off(kk, BN), IDESC_S,
                      kk > 0 ? 1u : 0u);
        umma_commit(&s_full[x]);
      };
      // O_X += P_X(j) V over keys [16 kk0, 16 kk1) with V from ring position
      // vpos: the first half can run while the softmax warps form the second.
      auto issue_pv = [&](int x, int j, int vpos, int kk0, int kk1) {
        const uint32_t vb = sV + (vpos % C::VSTAGES) * C::KV_BYTES;
        const uint32_t pt = tmem + C::COL_S + x * BN;
        const uint64_t dv = v_desc<D>(vb, 0);
        const uint32_t dt = tmem + C::COL_O + x * D;
#pragma unroll
        for (int kk = kk0; kk < kk1; ++kk)  // 16 keys = 8 packed TMEM columns per step
          umma_f16_ts(dt, pt + kk * 8, dv + (uint32_t)((kk * 16 * C::SWB) >> 4), IDESC_O,
                      (j > 0 || kk > 0) ? 1u : 0u);
      };
      // kc / vc: ring positions of this item's first K / V tile; sc[x]: S_X
      // tiles issued so far (= PVs = softmax rounds of tile X); qc: items with keys.
      int kc = 0, vc = 0, qc = 0;
      int sc[2] = {0, 0};
      bool ok = true;
      for (int k = 0; ok; ++k) {
        ItemRec e;
        if (!(ok = take_item(k, e, true)) || e.L < 0) break;
        const Geom g = derive(e.L, e.Lk, e.q0);
        if (g.n_kv == 0) continue;
        const int nX[2] = {g.nA, g.nB};
        // Prologue: S_A(0), S_B(0).
        ok = mbar_wait(q_full, qc & 1, abort_flag, p.status, 4);
        if (ok) ok = mbar_wait(&k_full[kc % C::KSTAGES], (kc / C::KSTAGES) & 1, abort_flag, p.status, 5);
        if (!ok) break;
        tc_fence_after();
        for (int x = 0; x < 2; ++x)
          if (nX[x] > 0) issue_s(x, kc);
        umma_commit(&k_empty[kc % C::KSTAGES]);
        if (g.n_kv == 1) umma_commit(q_empty);  // the item's last S GEMMs
        for (int j = 0; ok && j < g.n_kv; ++j) {
          const int vpos = vc + j, kn = kc + j + 1;
          const bool next_k = j + 1 < g.n_kv;
          if (!(ok = mbar_wait(&v_full[vpos % C::VSTAGES], (vpos / C::VSTAGES) & 1, abort_flag,
                               p.status, 3)))
            break;
          if (next_k &&
              !(ok = mbar_wait(&k_full[kn % C::KSTAGES], (kn / C::KSTAGES) & 1, abort_flag, p.status, 5)))
            break;
          // Per tile X: O_X += P_X(j) V_j as soon as P_X(j) is ready, then
          // S_X(j+1) into the same TMEM columns (issued after, so executed after).
          for (int x = 0; x < 2; ++x) {
            if (j < nX[x]) {
              const uint32_t ph = (uint32_t)((sc[x] + j) & 1);
              // O_X is overwritten by the first PV once the previous item's
              // epilogue has read it.
              if (j == 0 && qc > 0 &&
                  !(ok = mbar_wait(&o_empty[x], (qc - 1) & 1, abort_flag, p.status, 14)))
                break;
              constexpr int KK = BN / 16 / kPParts;  // PV k-steps per part of P
              for (int q = 0; ok && q + 1 < kPParts; ++q) {
                ok = mbar_wait(&p_part[x * (kPParts - 1) + q], ph, abort_flag, p.status, 10 + x);
                tc_fence_after();
                if (ok) issue_pv(x, j, vpos, q * KK, (q + 1) * KK);
              }
              if (!ok) break;
              if (!(ok = mbar_wait(&p_full[x], ph, abort_flag, p.status, 2 + 4 * x))) break;
              tc_fence_after();
#ifdef SCREE_TRACE
              const long long t_is0 = clock64();
#endif
              issue_pv(x, j, vpos, (kPParts - 1) * KK, BN / 16);
              umma_commit(&pv_done[x]);
              if (j + 1 < nX[x]) issue_s(x, kn);
#ifdef SCREE_TRACE
              SCREE_TRACE_ADD(21, clock64() - t_is0);
#endif
            }
          }
          if (!ok) break;
          if (j + 2 == g.n_kv) umma_commit(q_empty);  // S_X(n_kv - 1) were the last S GEMMs
          umma_commit(&v_empty[vpos % C::VSTAGES]);
          if (next_k) umma_commit(&k_empty[kn % C::KSTAGES]);
        }
        kc += g.n_kv;
        vc += g.n_kv;
        sc[0] += g.nA;
        sc[1] += g.nB;
        ++qc;
      }
    }
  } else if (warp >= 10) {
    regs_dec<kRegsOther>();  // idle: only completes warpgroup 2's register release
  } else {
    // ------------------------------------------------------------ softmax warps
    regs_inc<kRegsSoftmax>();
    const int x = warp >> 2;                  // query tile: 0 = A (warps 0-3), 1 = B (4-7)
    const int r = (warp & 3) * 32 + lane;     // row within the tile == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_s = lane_base + C::COL_S + x * BN;
    const uint32_t col_o = lane_base + C::COL_O + x * D;
    const float sl2 = p.scale_log2;
    int sc = 0;  // softmax rounds of this tile so far (= S_X tiles issued)
    bool ok = true;
    for (int k = 0; ok; ++k) {
      ItemRec e;
      ok = __all_sync(0xffffffff, take_item(k, e, false));  // released after the epilogue
      if (!ok || e.L < 0) break;
      const Geom g = derive(e.L, e.Lk, e.q0);
      const int Lk = e.Lk, cdelta = e.Lk - e.L;
      const int qt0 = e.q0 + x * BM;            // first row of this tile
      const int qi = qt0 + r;                   // query index within the sequence
      const int nmine = x == 0 ? g.nA : g.nB;
      float m_used = -INFINITY;                 // running max, scaled log2 units
      float l = 0.f;
      for (int j = 0; j < nmine; ++j) {
        ok = mbar_wait(&s_full[x], (sc + j) & 1, abort_flag, p.status, 7);
        if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
#ifdef SCREE_TRACE
        const long long t_sm0 = clock64();
#endif
        tc_fence_after();
        // One TMEM load of the whole 128-column row (a single wait::ld).
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32(col_s + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        tmem_wait_ld();
#ifdef SCREE_TRACE
        const long long t_ld = clock64();
        SCREE_TRACE_ADD(22, t_ld - t_sm0);
#endif
        const int k0 = j * BN;
        const bool need_mask = (k0 + BN > Lk) || (CAUSAL && k0 + BN - 1 > qt0 + cdelta);
        if (need_mask) {
          const int lim = CAUSAL ? min(Lk - 1, qi + cdelta) : (Lk - 1);  // last valid key
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (k0 + c > lim) s[c] = -INFINITY;
        }
        // Row max: 8 independent chains of three-input max (two values per step).
        float mx8[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx8[a] = s[a];
#pragma unroll
        for (int c = 8; c < BN; c += 16)
#pragma unroll
          for (int a = 0; a < 8; ++a) mx8[a] = fmax3(mx8[a], s[c + a], s[c + 8 + a < BN ? c + 8 + a : c + a]);
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7]));
        const float m_cand = mx * sl2;
#ifdef SCREE_TRACE
        const long long t_mx = clock64();
        SCREE_TRACE_ADD(23, t_mx - t_ld);
#endif
        float alpha = 1.f;
        bool need = false;
        if (m_used == -INFINITY) {
          need = true;
          alpha = 0.f;
          m_used = m_cand;
        } else if (m_cand > m_used + 8.0f) {
          need = true;
          alpha = ex2_approx(m_used - m_cand);
          m_used = m_cand;
        }
        const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
        // Exponentiate and pack: each pair of S values dies as its packed word appears.
        // Exponentiate and pack, two columns per packed f32x2 FMA / add; each pair of
        // S values dies as its packed 16-bit word appears.
        const uint64_t sl2x2 = f2_pack(sl2, sl2), negm2 = f2_pack(-m_eff, -m_eff);
        uint64_t rs4[4] = {0ull, 0ull, 0ull, 0ull};  // (+0.0f, +0.0f) pairs
        uint32_t pk[BN / 2];
        // Exponentiate and pack columns [c0, c1), two per packed f32x2 FMA / add;
        // each pair of S values dies as its packed 16-bit word appears.
        auto exp_pack = [&](int c0, int c1) {
#pragma unroll
          for (int c = c0; c < c1; c += 2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sl2x2, negm2), x0, x1);
            const float e0 = ex2_approx(x0), e1 = ex2_approx(x1);
            const uint64_t e01 = f2_pack(e0, e1);
            rs4[(c / 2) & 3] = f2_add(rs4[(c / 2) & 3], e01);
            pk[c / 2] = Pk2<T>::pack(e0, e1);
          }
        };
        constexpr int PC = BN / kPParts;  // keys per part of P
        auto store_part = [&](int q) {   // packed columns [q PC / 2, (q + 1) PC / 2)
          if constexpr (PC / 2 == 32)
            tmem_st32u(col_s + q * 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[q * 32]));
          else
            tmem_st16u(col_s + q * 16, &pk[q * 16]);
        };
        exp_pack(0, PC);
        if (j >= 1) {
          // O_X += P_X(j-1) V_{j-1} must be complete before O_X is rescaled and
          // before P_X(j) overwrites the columns it read.  It already is in the
          // common case: S_X(j) was issued after it and s_full covers both.
          ok = mbar_wait(&pv_done[x], (sc + j - 1) & 1, abort_flag, p.status, 8);
          if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
          tc_fence_after();
          if (__any_sync(0xffffffff, need)) {
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              float o[32];
              tmem_ld32(col_o + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] *= alpha;
              tmem_st32(col_o + c * 32, o);
            }
          }
        }
        // P_X(j) is published part by part: the MMA warp starts O_X += P V on
        // the first keys while the later ones are formed.
#pragma unroll
        for (int q = 0; q + 1 < kPParts; ++q) {
          store_part(q);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_part[x * (kPParts - 1) + q]);
          exp_pack((q + 1) * PC, (q + 2) * PC);
        }
        store_part(kPParts - 1);
        float ra, rb;
        f2_unpack(f2_add(f2_add(rs4[0], rs4[1]), f2_add(rs4[2], rs4[3])), ra, rb);
        l = l * alpha + (ra + rb);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[x]);
#ifdef SCREE_TRACE
        SCREE_TRACE_ADD(20, clock64() - t_sm0);
#endif
      }
      // ------------------------------------------------------------ epilogue
      // The item's record is still held in the ring: re-read what the epilogue
      // needs rather than keep it in registers through the key loop.
      const ItemRec& er = item_ring[k % kItemRing];
      const int L = er.L, h = er.h;
      const int64_t seq_start = er.seq_start;
      if (ok && nmine > 0) {
        ok = mbar_wait(&pv_done[x], (sc + nmine - 1) & 1, abort_flag, p.status, 9);
        ok = __all_sync(0xffffffff, ok);
      }
      if (ok && nmine > 0) {
        tc_fence_after();
        const bool row_ok = qi < L;
        // l = 0: a query with no key at all (KV-cache attention with fewer keys
        // than queries, causal) gets O = 0 and LSE = -inf.
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
        T* orow = reinterpret_cast<T*>(p.o) + (seq_start + qi) * p.o_rs + (int64_t)h * p.o_hs;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float o[32];
          tmem_ld32(col_o + c * 32, o);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint4 w;
              w.x = Pk2<T>::pack(o[u * 8 + 0] * inv_l, o[u * 8 + 1] * inv_l);
              w.y = Pk2<T>::pack(o[u * 8 + 2] * inv_l, o[u * 8 + 3] * inv_l);
              w.z = Pk2<T>::pack(o[u * 8 + 4] * inv_l, o[u * 8 + 5] * inv_l);
              w.w = Pk2<T>::pack(o[u * 8 + 6] * inv_l, o[u * 8 + 7] * inv_l);
              *reinterpret_cast<uint4*>(orow + c * 32 + u * 8) = w;
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty[x]);  // O_X is in registers: the next item may overwrite it
        if (row_ok && p.lse != nullptr)
          p.lse[(seq_start + qi) * p.H + h] =
              l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY;
      }
      if (ok && nmine == 0 && qi < L) {  // no key tile at all for this query tile
        T* orow = reinterpret_cast<T*>(p.o) + (seq_start + qi) * p.o_rs + (int64_t)h * p.o_hs;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(0, 0, 0, 0);
        if (p.lse != nullptr) p.lse[(seq_start + qi) * p.H + h] = -INFINITY;
      }
      if (ok && nmine == 0 && g.n_kv > 0) mbar_arrive(&o_empty[x]);
      mbar_arrive(&item_empty[k % kItemRing]);
      sc += nmine;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
#ifdef SCREE_TRACE
  if (threadIdx.x == 0) {
    scree_trace_sm[30] += (unsigned long long)(clock64() - t_cta0);
  }
  __syncthreads();
  if (threadIdx.x < 32) atomicAdd(&g_fwd_trace[threadIdx.x], scree_trace_sm[threadIdx.x]);
#endif
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

template <int D, typename T, bool CAUSAL>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
               const FwdParams& p, int64_t grid, cudaStream_t s) {
  auto kern = attn_fwd_kernel<D, T, CAUSAL>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    SCREE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        FwdCfg<D>::SMEM));
    attr_set[dev & 63] = true;
  }
  ProfScope prof(PROF_ATTN_FWD, s);
  kern<<<(unsigned)grid, kThreads, FwdCfg<D>::SMEM, s>>>(tq, tk, tv, p);
  SCREE_LAUNCH_CHECK();
  return SCREE_OK;
}

}  // namespace
}  // namespace scree

using namespace scree;

extern "C" size_t scree_attn_fwd_workspace_size(int64_t B, int64_t T, int64_t H, int D) {
  (void)H;
  (void)D;
  return schedule_bytes(B);
}

extern "C" int scree_attn_fwd(const void* q, const void* k, const void* v, int64_t q_rs,
                              int64_t q_hs, int64_t k_rs, int64_t k_hs, int64_t v_rs,
                              int64_t v_hs, const void* offsets, int offs_is_i64, int64_t B,
                              int64_t T, int64_t H, int D, int dtype, int causal, float scale,
                              int64_t max_seqlen, void* o, int64_t o_rs, int64_t o_hs, float* lse,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return scree_attn_fwd_gqa(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets, offs_is_i64, B,
                            T, H, H, D, dtype, causal, scale, max_seqlen, o, o_rs, o_hs, lse,
                            workspace, workspace_bytes, stream);
}

namespace scree {
namespace {
int run_fwd(const void* q, const void* k, const void* v, int64_t q_rs, int64_t q_hs, int64_t k_rs,
            int64_t k_hs, int64_t v_rs, int64_t v_hs, const void* offsets,
            const void* offsets_k, int offs_is_i64, int64_t B, int64_t T, int64_t Tk, int64_t H,
            int64_t H_kv, int D, int dtype, int causal, float scale, int64_t max_seqlen, void* o,
            int64_t o_rs, int64_t o_hs, float* lse, void* workspace, size_t workspace_bytes,
            void* stream) {
  (void)max_seqlen;
  SCREE_CHECK_ARG(H_kv >= 1 && H % H_kv == 0,
                  "attn_fwd: query heads (%lld) must be a multiple of K/V heads (%lld)",
                  (long long)H, (long long)H_kv);
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && H >= 1, "attn_fwd: bad sizes B=%lld T=%lld H=%lld",
                  (long long)B, (long long)T, (long long)H);
  SCREE_CHECK_ARG(T < (1ll << 31) && H < 65536, "attn_fwd: T or H too large");
  if (D != 32 && D != 64 && D != 128) {
    set_last_error("attn_fwd: head_dim %d unsupported (32, 64, 128)", D);
    return SCREE_ERR_UNSUPPORTED;
  }
  SCREE_CHECK_ARG(dtype == SCREE_F16 || dtype == SCREE_BF16 || dtype == SCREE_F32,
                  "attn_fwd: fp16, bf16 or fp32 only");
  if (T == 0) return SCREE_OK;
  SCREE_CHECK_ARG(q && k && v && o && offsets, "attn_fwd: null pointer");
  if (dtype == SCREE_F32) {  // CUDA-core fp32 kernels; no workspace needed
    SCREE_BIND_DEVICE(stream, q);
    return attn_fwd_f32(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets, offs_is_i64, B, T,
                        H, H_kv, D, causal, scale, o, o_rs, o_hs, lse, (cudaStream_t)stream);
  }
  SCREE_CHECK_ARG(workspace && workspace_bytes >= schedule_bytes(B),
                  "attn_fwd: workspace too small");
  SCREE_CHECK_ARG(((uintptr_t)o % 16) == 0 && (o_rs % 8) == 0 && (o_hs % 8) == 0,
                  "attn_fwd: output must be 16-byte aligned with strides multiple of 8");
  SCREE_BIND_DEVICE(stream, q);
  cudaStream_t s = (cudaStream_t)stream;
  const bool bf16 = dtype == SCREE_BF16;
  const int swb = D >= 64 ? 128 : 64;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_thd_map(&tq, q, T, H, D, q_rs, q_hs, swb / 2, BM, swb, bf16))) return rc;
  if (Tk == 0) Tk = 1;  // keys all empty: a 1-row map that no tile reads
  if ((rc = make_thd_map(&tk, k, Tk, H_kv, D, k_rs, k_hs, swb / 2, BN, swb, bf16))) return rc;
  if ((rc = make_thd_map(&tv, v, Tk, H_kv, D, v_rs, v_hs, swb / 2, BN, swb, bf16))) return rc;
  if (offsets_k != nullptr && (rc = launch_validate_offsets(offsets_k, offs_is_i64, B, Tk, s)))
    return rc;
  if ((rc = launch_build_schedule(offsets, offs_is_i64, B, T, ROWS, (int)H, workspace, s))) return rc;
  FwdParams p;
  p.offs = offsets;
  p.is64 = offs_is_i64;
  p.H = (int)H;
  p.G = (int)(H / H_kv);
  p.T = (int)T;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.sched = workspace;
  p.offs_k = offsets_k;
  p.B = B;
  p.status = device_status_ptr();
  p.o = o;
  p.o_rs = o_rs;
  p.o_hs = o_hs;
  p.lse = lse;
  // Persistent CTAs, one per SM (each holds all 512 TMEM columns); the items
  // themselves are counted on the device.
  const int64_t grid = std::min<int64_t>(max_tiles(B, T, ROWS) * H, (int64_t)num_sms());
#define SCREE_FWD_CASE(DD)                                                              \
  if (D == DD) {                                                                        \
    if (bf16)                                                                           \
      return causal ? launch_fwd<DD, __nv_bfloat16, true>(tq, tk, tv, p, grid, s)       \
                    : launch_fwd<DD, __nv_bfloat16, false>(tq, tk, tv, p, grid, s);     \
    return causal ? launch_fwd<DD, __half, true>(tq, tk, tv, p, grid, s)                \
                  : launch_fwd<DD, __half, false>(tq, tk, tv, p, grid, s);              \
  }
  SCREE_FWD_CASE(128)
  SCREE_FWD_CASE(64)
  SCREE_FWD_CASE(32)
#undef SCREE_FWD_CASE
  return SCREE_ERR_UNSUPPORTED;
}
}  // namespace
}  // namespace scree

extern "C" int scree_attn_fwd_gqa(const void* q, const void* k, const void* v, int64_t q_rs,
                                  int64_t q_hs, int64_t k_rs, int64_t k_hs, int64_t v_rs,
                                  int64_t v_hs, const void* offsets, int offs_is_i64, int64_t B,
                                  int64_t T, int64_t H, int64_t H_kv, int D, int dtype,
                                  int causal, float scale, int64_t max_seqlen, void* o,
                                  int64_t o_rs, int64_t o_hs, float* lse, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  return run_fwd(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets, nullptr, offs_is_i64, B, T,
                 T, H, H_kv, D, dtype, causal, scale, max_seqlen, o, o_rs, o_hs, lse, workspace,
                 workspace_bytes, stream);
}

extern "C" int scree_attn_fwd_kv(const void* q, const void* k, const void* v, int64_t q_rs,
                                 int64_t q_hs, int64_t k_rs, int64_t k_hs, int64_t v_rs,
                                 int64_t v_hs, const void* offsets_q, const void* offsets_k,
                                 int offs_is_i64, int64_t B, int64_t Tq, int64_t Tk, int64_t H,
                                 int64_t H_kv, int D, int dtype, int causal, float scale, void* o,
                                 int64_t o_rs, int64_t o_hs, float* lse, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  SCREE_CHECK_ARG(offsets_k != nullptr, "attn_fwd_kv: null key offsets");
  SCREE_CHECK_ARG(Tk >= 0 && Tk < (1ll << 31), "attn_fwd_kv: bad key row count");
  if (dtype == SCREE_F32) {
    set_last_error("attn_fwd_kv: fp16 / bf16 only");
    return SCREE_ERR_UNSUPPORTED;
  }
  return run_fwd(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets_q, offsets_k, offs_is_i64, B,
                 Tq, Tk, H, H_kv, D, dtype, causal, scale, 0, o, o_rs, o_hs, lse, workspace,
                 workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of scree_attn_fwd.
//
// Some callers cannot allocate device memory at the point where they run
// attention: an inference engine or plugin host that owns a fixed,
// pre-planned memory arena and forbids allocation after start-up, or code whose
// allocator is not reachable from the C side at all (a foreign-language binding
// that only holds raw pointers to inputs and outputs).  For them this entry
// point takes the forward's only scratch, the work schedule (16 bytes per
// sequence plus a 16-byte header), from a fixed array compiled into the
// library instead of a caller-provided workspace.
//
// Limits and rules:
//  * The array holds kNoAllocScratchBytes = 64 KiB per GPU that loads the
//    library, for as long as the process lives, so at most
//    (64 KiB - 16) / 16 = 4095 sequences per call; larger batches are rejected
//    with SCREE_ERR_INVALID before any work is enqueued.
//  * All calls on a device share the one array.  The schedule kernel rewrites
//    every byte the attention kernel later reads, so nothing has to start at
//    zero, but two calls whose work overlaps on the GPU (different streams
//    without ordering between them) race on the array and give wrong results.
//    Serialise them, e.g. issue them on one stream.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture.  Later calls reuse the cached address, which
//    a cudaDeviceReset of that device makes stale: after a reset, do not call
//    this entry point on that device again in the same process.
// It allocates nothing itself: no cudaMalloc, cudaFree or allocating library
// routine, and it then runs exactly the scree_attn_fwd path.
namespace {
constexpr size_t kNoAllocScratchBytes = 64 * 1024;
static __device__ __align__(256) unsigned char g_fwd_noalloc_scratch[kNoAllocScratchBytes];
}  // namespace

extern "C" int scree_attn_fwd_noalloc(const void* q, const void* k, const void* v, int64_t q_rs,
                                      int64_t q_hs, int64_t k_rs, int64_t k_hs, int64_t v_rs,
                                      int64_t v_hs, const void* offsets, int offs_is_i64,
                                      int64_t B, int64_t T, int64_t H, int D, int dtype,
                                      int causal, float scale, int64_t max_seqlen, void* o,
                                      int64_t o_rs, int64_t o_hs, float* lse, void* stream) {
  SCREE_CHECK_ARG(B >= 1, "attn_fwd_noalloc: bad batch size %lld", (long long)B);
  SCREE_CHECK_ARG(schedule_bytes(B) <= kNoAllocScratchBytes,
                  "attn_fwd_noalloc: %lld sequences exceed the built-in scratch limit of %lld "
                  "(64 KiB); use scree_attn_fwd with a caller workspace",
                  (long long)B, (long long)((kNoAllocScratchBytes - 16) / 16));
  if (T == 0) return SCREE_OK;
  SCREE_CHECK_ARG(q != nullptr, "attn_fwd_noalloc: null q");
  // Make the device that owns the stream (or q) current, then resolve the
  // array's address on that device once.
  SCREE_BIND_DEVICE(stream, q);
  static std::atomic<void*> scratch_ptr[64];
  int dev = 0;
  SCREE_CUDA_TRY(cudaGetDevice(&dev));
  SCREE_CHECK_ARG(dev >= 0 && dev < 64, "attn_fwd_noalloc: device index %d out of range", dev);
  void* scratch = scratch_ptr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // Concurrent first calls on one device resolve the same address; storing
    // it twice is harmless.
    SCREE_CUDA_TRY(cudaGetSymbolAddress(&scratch, g_fwd_noalloc_scratch));
    scratch_ptr[dev].store(scratch, std::memory_order_release);
  }
  return scree_attn_fwd(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets, offs_is_i64, B, T,
                        H, D, dtype, causal, scale, max_seqlen, o, o_rs, o_hs, lse,
                        scratch, kNoAllocScratchBytes, stream);
}

#ifdef SCREE_TRACE
extern "C" int scree_fwd_trace_read(unsigned long long* out32, int reset) {
  SCREE_CUDA_TRY(cudaDeviceSynchronize());
  SCREE_CUDA_TRY(cudaMemcpyFromSymbol(out32, g_fwd_trace, sizeof(unsigned long long) * 32));
  if (reset) {
    unsigned long long z[32] = {0};
    SCREE_CUDA_TRY(cudaMemcpyToSymbol(g_fwd_trace, z, sizeof(z)));
  }
  return SCREE_OK;
}
#endif
