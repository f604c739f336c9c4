// attn_fwd.cu — varlen self-attention forward on sm_100a tensor cores.
//
// Computes, per sequence b and head h (reference/varlen_attention.py:121-138):
//   S = Q K^T * scale, causal mask k > q -> -inf, P = softmax(S), O = P V,
//   LSE = m + ln(l)  (natural log; triton/varlen_attention.py:160)
// One CTA owns one 128-row query tile of one head and streams the sequence's
// 128-key tiles through a TMA -> tcgen05.mma pipeline:
//
//   warp 8  (TMA)      Q once; K_j and V_j into separate rings (mbarrier tx)
//   warp 9  (MMA)      S_j = Q K_j^T into TMEM buffer j%2, then O += P_{j-1} V_{j-1}
//   warps 0-7 (softmax) warps w, w+4 own query rows 32(w%4).. (TMEM lanes), one half of the key columns each: read S_j,
//                      masks, keeps running max/sum in registers, writes P_j
//                      (bf16/fp16, 128B-swizzled K-major) to shared memory,
//                      rescales O in TMEM only when the max grew by more than
//                      2^8 (exact: P stays <= 256), and finally writes O / l, LSE.
//
// TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+D).
// Softmax works in the exp2 domain with log2(e) folded into the scale.
// Ragged tails: TMA reads whole 128-row boxes, so rows of the next sequence
// arrive in K/V tiles; keys >= L are masked to -inf (P = 0), and query rows
// >= L are computed but never stored.  Rows past T are zero-filled by TMA.
#include "attn_common.cuh"

namespace scree {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int kThreads = 320;  // 8 softmax warps, TMA warp, MMA warp

template <int D>
struct FwdCfg {
  static constexpr int SWB = D >= 64 ? 128 : 64;  // swizzle span in bytes (one smem row)
  static constexpr int CHUNK = SWB / 2;           // elements per swizzle row
  static constexpr int NCHUNK = D / CHUNK;
  static constexpr uint32_t SWZ = SWB == 128 ? SW_128B : SW_64B;
  // K is released right after S = Q K^T, V only after O += P V, so they have
  // separate rings; K gets the deeper one because S_{j} is issued first.
  static constexpr int KSTAGES = 3;
  static constexpr int VSTAGES = D == 128 ? 2 : 3;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + KSTAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + VSTAGES * KV_BYTES;
  // One P buffer: the softmax writes P_j only after O += P_{j-1} V_{j-1} completed
  // (it must wait for that anyway before rescaling O).
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  static constexpr int OFF_RED = OFF_BAR + 192;           // [2 parity][2 half][BM] fp32
  static constexpr int OFF_END = OFF_RED + 2 * 2 * BM * 4;
  // 1 KB of alignment slack when it fits; the kernel checks the real alignment.
  static constexpr int SMEM_RAW = OFF_END + 1024 <= 232448 ? OFF_END + 1024 : OFF_END;
  // At least 120 KB so that two CTAs (each holding all 512 TMEM columns) never
  // share an SM.
  static constexpr int SMEM = SMEM_RAW > 120 * 1024 ? SMEM_RAW : 120 * 1024;
};

struct FwdParams {
  const void* offs;
  int is64;
  int H;
  int T;
  float scale_log2;
  const void* sched;  // schedule (attn_common.cuh)
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
// P tile: [BM][BN] with 64-key 128-byte swizzled column blocks.
__device__ __forceinline__ uint64_t p_desc(uint32_t base, int kk) {
  const int e = kk * 16;
  const uint32_t addr = base + (e / 64) * BM * 128 + (e % 64) * 2;
  return make_sdesc(addr, 16, 1024, SW_128B);
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

  const int64_t item = blockIdx.x;
  if (item >= total_items(p.sched)) return;
  // A CTA of an earlier failed launch (or of this one) set the status word: skip.
  if (p.status && *reinterpret_cast<volatile int*>(p.status) != 0) return;
  const WorkItem wi = decode_item(p.sched, p.B, p.H, item);
  const int h = wi.head;
  const int64_t seq_start = load_offset(p.offs, p.is64, wi.seq);
  const int L = (int)(load_offset(p.offs, p.is64, wi.seq + 1) - seq_start);
  // Causal: heaviest (last) query tile first within each (sequence, head).
  const int q0 = (CAUSAL ? (wi.ntiles - 1 - wi.j) : wi.j) * BM;
  const int nk_all = (L + BN - 1) / BN;
  const int n_kv = CAUSAL ? min(nk_all, (q0 + BM - 1) / BN + 1) : nk_all;

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
  const uint32_t sP = smem_u32(smem + C::OFF_P);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                  // [KSTAGES]
  uint64_t* k_empty = k_full + C::KSTAGES;      // [KSTAGES]
  uint64_t* v_full = k_empty + C::KSTAGES;      // [VSTAGES]
  uint64_t* v_empty = v_full + C::VSTAGES;      // [VSTAGES]
  uint64_t* s_full = v_empty + C::VSTAGES;      // [2]
  uint64_t* s_empty = s_full + 2;               // [2]
  uint64_t* p_full = s_empty + 2;               // [2]
  uint64_t* pv_done = p_full + 2;               // [2]
  uint64_t* xch = pv_done + 2;                  // [2] row-max exchange between column halves
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xch + 2);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

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
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 256);
      mbar_init(&p_full[b], 256);
      mbar_init(&pv_done[b], 1);
      mbar_init(&xch[b], 256);
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

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    // Lane 0 streams Q and the K ring, lane 1 the V ring, each at its own pace.
    const int row0 = (int)seq_start;
    if (lane == 0) {
      mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < C::NCHUNK; ++c)
        tma_load_3d(smem + C::OFF_Q + c * BM * C::SWB, &tm_q, q_full, c * C::CHUNK, h, row0 + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::KSTAGES;
        if (j >= C::KSTAGES &&
            !mbar_wait(&k_empty[st], ((j / C::KSTAGES) - 1) & 1, abort_flag, p.status, 1))
          break;
        mbar_expect_tx(&k_full[st], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_3d(smem + C::OFF_K + st * C::KV_BYTES + c * BN * C::SWB, &tm_k, &k_full[st],
                      c * C::CHUNK, h, row0 + j * BN);
      }
    } else if (lane == 1) {
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::VSTAGES;
        if (j >= C::VSTAGES &&
            !mbar_wait(&v_empty[st], ((j / C::VSTAGES) - 1) & 1, abort_flag, p.status, 12))
          break;
        mbar_expect_tx(&v_full[st], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_3d(smem + C::OFF_V + st * C::KV_BYTES + c * BN * C::SWB, &tm_v, &v_full[st],
                      c * C::CHUNK, h, row0 + j * BN);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      auto issue_pv = [&](int i) -> bool {
        const int b2 = i & 1, st = i % C::VSTAGES;
        if (!mbar_wait(&p_full[b2], (i >> 1) & 1, abort_flag, p.status, 2)) return false;
        if (!mbar_wait(&v_full[st], (i / C::VSTAGES) & 1, abort_flag, p.status, 3)) return false;
        tc_fence_after();
        const uint32_t pb = sP;
        const uint32_t vb = sV + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          umma_f16_ss(tmem + 256, p_desc(pb, kk), v_desc<D>(vb, kk), IDESC_O,
                      (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[b2]);
        umma_commit(&v_empty[st]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, 4);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % C::KSTAGES, b2 = j & 1;
        if (!mbar_wait(&k_full[st], (j / C::KSTAGES) & 1, abort_flag, p.status, 5)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&s_empty[b2], ((j - 2) >> 1) & 1, abort_flag, p.status, 6)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sK + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(tmem + b2 * BN, kmajor_desc<D>(sQ, BM, kk), kmajor_desc<D>(kb, BN, kk),
                      IDESC_S, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[b2]);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n_kv > 0) issue_pv(n_kv - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    // Warps w and w+4 share TMEM lanes 32*(w%4)..+31 (query rows); warp w < 4
    // takes key columns [0,64) of each tile, warp w+4 columns [64,128).  The two
    // halves exchange their row maxima once per tile (mbarrier xch, so the wait
    // stays bounded) and their partial sums once at the end.
    const int hf = warp >> 2;                 // column half
    const int r = (warp & 3) * 32 + lane;     // query row within the tile == TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int qi = q0 + r;                    // query index within the sequence
    const float sl2 = p.scale_log2;
    constexpr int HN = BN / 2;                // columns per half
    float m_used = -INFINITY;                 // running max, scaled log2 units
    float l = 0.f;                            // partial sum over this half's columns
    bool ok = true;
    uint8_t* prow_base = smem + C::OFF_P + hf * BM * 128 + r * 128;
    const int sw = r & 7;
    for (int j = 0; j < n_kv; ++j) {
      const int b2 = j & 1;
      ok = mbar_wait(&s_full[b2], (j >> 1) & 1, abort_flag, p.status, 7);
      if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
      tc_fence_after();
      float s[HN];
#pragma unroll
      for (int c = 0; c < HN / 32; ++c)
        tmem_ld32(lane_base + b2 * BN + hf * HN + c * 32,
                  *reinterpret_cast<float(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_empty[b2]);

      const int k0 = j * BN + hf * HN;
      const bool need_mask = (j * BN + BN > L) || (CAUSAL && j * BN + BN - 1 > q0);
      if (need_mask) {
        const int lim = CAUSAL ? min(L - 1, qi) : (L - 1);  // last valid key
#pragma unroll
        for (int c = 0; c < HN; ++c)
          if (k0 + c > lim) s[c] = -INFINITY;
      }
      // Row max: 8 independent chains, then the other half's value.
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = s[a];
#pragma unroll
      for (int c = 8; c < HN; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      red[(b2 * 2 + hf) * BM + r] = mx;
      mbar_arrive(&xch[b2]);
      ok = mbar_wait(&xch[b2], (j >> 1) & 1, abort_flag, p.status, 10);
      if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
      mx = fmaxf(mx, red[(b2 * 2 + (hf ^ 1)) * BM + r]);
      // Both halves now see the same max, so their lazy-rescale decisions agree.
      const float m_cand = mx * sl2;
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
      float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < HN; ++c) {
        s[c] = ex2_approx(fmaf(s[c], sl2, -m_eff));
        rs8[c & 7] += s[c];
      }
      const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      if (j >= 1) {
        ok = mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.status, 8);
        if (!__all_sync(0xffffffff, ok)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffff, need)) {
          // O columns in 32-wide chunks; chunk c belongs to half c % 2.
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            if ((c & 1) != hf) continue;
            float o[32];
            tmem_ld32(lane_base + 256 + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(lane_base + 256 + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      l = l * alpha + rs;
      // This half's 64 keys are one 128-byte swizzled column block of P:
      // 16-byte unit u of row r lives at unit position u ^ (r % 8).
      uint8_t* prow = prow_base;
#pragma unroll
      for (int u = 0; u < HN / 8; ++u) {
        uint4 w;
        w.x = Pk2<T>::pack(s[u * 8 + 0], s[u * 8 + 1]);
        w.y = Pk2<T>::pack(s[u * 8 + 2], s[u * 8 + 3]);
        w.z = Pk2<T>::pack(s[u * 8 + 4], s[u * 8 + 5]);
        w.w = Pk2<T>::pack(s[u * 8 + 6], s[u * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + ((u ^ sw) << 4)) = w;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b2]);
    }
    // ------------------------------------------------------------ epilogue
    if (ok && n_kv > 0) {
      ok = mbar_wait(&pv_done[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, abort_flag, p.status, 9);
      ok = __all_sync(0xffffffff, ok);
    }
    if (ok && n_kv > 0) {
      // Total row sum: exchange the partial sums through the exchange buffer of
      // the parity the last tile did not use (its readers have moved on).
      const int pb = n_kv & 1;
      red[(pb * 2 + hf) * BM + r] = l;
      mbar_arrive(&xch[pb]);
      ok = mbar_wait(&xch[pb], (n_kv >> 1) & 1, abort_flag, p.status, 11);
      ok = __all_sync(0xffffffff, ok);
      if (ok) l += red[(pb * 2 + (hf ^ 1)) * BM + r];
    }
    if (ok && n_kv > 0) {
      tc_fence_after();
      const bool row_ok = qi < L;
      const float inv_l = 1.0f / l;
      T* orow = reinterpret_cast<T*>(p.o) + (seq_start + qi) * p.o_rs + (int64_t)h * p.o_hs;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        if ((c & 1) != hf) continue;
        float o[32];
        tmem_ld32(lane_base + 256 + c * 32, o);
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
      if (hf == 0 && row_ok && p.lse != nullptr)
        p.lse[(seq_start + qi) * p.H + h] = (m_used + log2f(l)) * 0.69314718055994531f;
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
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
  (void)max_seqlen;
  SCREE_CHECK_ARG(B >= 1 && T >= 0 && H >= 1, "attn_fwd: bad sizes B=%lld T=%lld H=%lld",
                  (long long)B, (long long)T, (long long)H);
  SCREE_CHECK_ARG(T < (1ll << 31) && H < 65536, "attn_fwd: T or H too large");
  if (D != 32 && D != 64 && D != 128) {
    set_last_error("attn_fwd: head_dim %d unsupported (32, 64, 128)", D);
    return SCREE_ERR_UNSUPPORTED;
  }
  SCREE_CHECK_ARG(dtype == SCREE_F16 || dtype == SCREE_BF16, "attn_fwd: fp16 or bf16 only");
  if (T == 0) return SCREE_OK;
  SCREE_CHECK_ARG(q && k && v && o && offsets, "attn_fwd: null pointer");
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
  if ((rc = make_thd_map(&tk, k, T, H, D, k_rs, k_hs, swb / 2, BN, swb, bf16))) return rc;
  if ((rc = make_thd_map(&tv, v, T, H, D, v_rs, v_hs, swb / 2, BN, swb, bf16))) return rc;
  if ((rc = launch_build_schedule(offsets, offs_is_i64, B, BM, (int)H, workspace, s))) return rc;
  FwdParams p;
  p.offs = offsets;
  p.is64 = offs_is_i64;
  p.H = (int)H;
  p.T = (int)T;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.sched = workspace;
  p.B = B;
  p.status = device_status_ptr();
  p.o = o;
  p.o_rs = o_rs;
  p.o_hs = o_hs;
  p.lse = lse;
  const int64_t grid = max_tiles(B, T, BM) * H;
  SCREE_CHECK_ARG(grid < (1ll << 31), "attn_fwd: grid too large");
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
//    before any stream capture.  Later calls reuse the cached address.
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
  static void* scratch_ptr[64] = {nullptr};
  int dev = 0;
  SCREE_CUDA_TRY(cudaGetDevice(&dev));
  SCREE_CHECK_ARG(dev >= 0 && dev < 64, "attn_fwd_noalloc: device index %d out of range", dev);
  if (scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    SCREE_CUDA_TRY(cudaGetSymbolAddress(&p, g_fwd_noalloc_scratch));
    scratch_ptr[dev] = p;
  }
  return scree_attn_fwd(q, k, v, q_rs, q_hs, k_rs, k_hs, v_rs, v_hs, offsets, offs_is_i64, B, T,
                        H, D, dtype, causal, scale, max_seqlen, o, o_rs, o_hs, lse,
                        scratch_ptr[dev], kNoAllocScratchBytes, stream);
}
