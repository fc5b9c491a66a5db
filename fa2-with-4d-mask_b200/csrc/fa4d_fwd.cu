// fa4d_fwd.cu — FlashAttention-2 forward for sm_100a with an optional 4D mask/score.
//
// Semantics follow the reference forward kernel (python/fa2.py:22-139) and its
// oracle (benchmark/precision_check.py:133-180): S = Q K^T (+ score) is scaled,
// causal / key-bound / mask-False entries become -inf, the row softmax is taken
// in the exp2 domain and O = P V.  LSE is saved in the log2 domain
// (log2(rowsum) + rowmax of the scaled logits, python/fa2.py:137-139).  Rows whose
// first key tiles are fully masked are handled like the oracle (the running max
// stays -inf and contributes nothing); rows with no valid key at all produce NaN,
// as softmax over an all -inf row does in the oracle.
//
// CTA = 2 query slots x 128 rows of one (batch, query head); 384 threads:
//   warp 0      TMA producer (Q once, then K/V tiles into a 2-stage ring each)
//   warp 1      tcgen05.mma issuer (one thread)
//   warp 2      TMEM allocator
//   warps 4-7   softmax + epilogue for query slot 0 (one thread per row)
//   warps 8-11  softmax + epilogue for query slot 1
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// P (16-bit) overwrites the first 64 columns of S and feeds the PV MMA from TMEM.
#include <cfloat>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"

namespace fa4d {

namespace {

constexpr int kFwdThreads = 384;
// Register split (launch: 384 threads x 168 = 64512): producer/MMA warpgroup 112,
// the two softmax warpgroups 192 -> 128*112 + 256*192 = 63488.
constexpr uint32_t kFwdRegsLaunch = 168, kFwdRegsCtl = 112, kFwdRegsSoftmax = 192;
static_assert(128 * kFwdRegsCtl + 256 * kFwdRegsSoftmax <= kFwdThreads * kFwdRegsLaunch,
              "register split exceeds the launch allocation");
constexpr float kNegInf = -INFINITY;
// O is only rescaled when the running max grows by more than this (log2 units);
// in between, P = exp2(s - stale max) stays <= 2^8, exact after the final 1/l.
constexpr float kRescaleThreshold = 8.0f;

template <int D>
struct FwdLayout {
  static constexpr int kTile = 128 * D * 2;  // one 128-row tile of 16-bit elements
  static constexpr int kQ = 0;               // 2 query slots
  static constexpr int kK = kQ + 2 * kTile;  // 2 stages
  static constexpr int kV = kK + 2 * kTile;  // 2 stages
  static constexpr int kBar = kV + 2 * kTile;
  static constexpr int kNumBars = 16;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

// S[slot] = Q[slot] K^T : M=128, N=128, K=D; both operands K-major, 128-B swizzled.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_qk(uint32_t tS, uint32_t sQ, uint32_t sK) {
  constexpr uint32_t idesc = make_idesc(128, 128, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
    mma_ss(tS, sw128_desc(sQ + off, 16, 1024), sw128_desc(sK + off, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// O[slot] (+)= P[slot] V : M=128, N=D, K=128; P from TMEM, V MN-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_pv(uint32_t tO, uint32_t tP, uint32_t sV, bool accumulate) {
  constexpr uint32_t idesc = make_idesc(128, D, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    mma_ts(tO, tP + kk * 8, sw128_desc(sV + kk * 2048, 16384, 1024), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
  }
}

// Number of 128-key tiles query rows [qs, qe) need.
__device__ __forceinline__ int kv_tiles_for(int qs, int qe, const FwdParams& p) {
  if (qs >= p.Tq) return 0;
  int kv_end = p.Tk;
  if (p.causal) {
    const long long lim = static_cast<long long>(qe) + p.causal_off;  // keys < qe + off
    kv_end = lim < p.Tk ? static_cast<int>(lim) : p.Tk;
  }
  return kv_end > 0 ? (kv_end + 127) / 128 : 0;
}

template <int D, bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kFwdThreads, 1) fwd_kernel(const __grid_constant__ FwdParams p) {
  using L = FwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] per slot
  uint64_t* p_full = bars + 11;  // [2] per slot
  uint64_t* o_full = bars + 13;  // [2] per slot
  uint64_t* mma_drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qblk = p.causal ? static_cast<int>(gridDim.x - 1 - blockIdx.x) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qblk * 256;

  int n_slot[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + 128 * t;
    const int qe = min(qs + 128, p.Tq);
    n_slot[t] = kv_tiles_for(qs, qe, p);
  }
  const int n_max = max(n_slot[0], n_slot[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // Each role starts with its register budget so the compiler allocates that
    // role's code under it.
    regs_dec<kFwdRegsCtl>();
    if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_max > 0) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      uint8_t* sQ = smem + L::kQ;
      uint8_t* sK = smem + L::kK;
      uint8_t* sV = smem + L::kV;
      mbar_arrive_expect_tx(q_full, 2 * L::kTile);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sQ + t * L::kTile + c * 16384, &p.tm_q, q_full, c * 64, q0 + 128 * t, h, b);
      int issued = 0;
      for (int j = 0; j < n_max; ++j) {
        const int s = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], par, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sK + s * L::kTile + c * 16384, &p.tm_k, &k_full[s], c * 64, j * 128, hk, b);
        if (!mbar_wait(&v_empty[s], par, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sV + s * L::kTile + c * 16384, &p.tm_v, &v_full[s], c * 64, j * 128, hk, b);
        issued = j + 1;
      }
      // Abort path only: make sure no copy is still writing shared memory.
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        mbar_wait_short(q_full, 0);
        for (int j = max(0, issued - 2); j < issued; ++j) {
          mbar_wait_short(&k_full[j & 1], (j >> 1) & 1);
          mbar_wait_short(&v_full[j & 1], (j >> 1) & 1);
        }
      }
    }
    __syncwarp();
    } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (waits included); each group of MMAs and its
    // commits is issued by one elected lane, keeping the issue state uniform.
    if (n_max > 0) {
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sK = smem_u32(smem + L::kK);
      const uint32_t sV = smem_u32(smem + L::kV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      bool ok = wait(q_full, 0) && wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (n_slot[t] > 0) {
              issue_qk<D, kBF16>(tmem + 128 * t, sQ + t * L::kTile, sK);
              tc_commit(&s_full[t]);
            }
          }
          tc_commit(&k_empty[0]);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_max; ++j) {
        const int sv = j & 1;
        ok = wait(&v_full[sv], (j >> 1) & 1);
        if (!ok) break;
        const bool has_next = j + 1 < n_max;
        const int sk = (j + 1) & 1;
        if (has_next) {
          ok = wait(&k_full[sk], ((j + 1) >> 1) & 1);
          if (!ok) break;
        }
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j < n_slot[t]) {
            ok = wait(&p_full[t], j & 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_pv<D, kBF16>(tmem + 256 + D * t, tmem + 128 * t, sV + sv * L::kTile, j > 0);
              if (j + 1 < n_slot[t]) {
                issue_qk<D, kBF16>(tmem + 128 * t, sQ + t * L::kTile, sK + sk * L::kTile);
                tc_commit(&s_full[t]);
              } else {
                tc_commit(&o_full[t]);
              }
            }
            __syncwarp();
          }
        }
        if (!ok) break;
        if (elect_one()) {
          tc_commit(&v_empty[sv]);
          if (has_next) tc_commit(&k_empty[sk]);
        }
        __syncwarp();
      }
      // Every MMA must have completed before TMEM is released.
      if (elect_one()) tc_commit(mma_drain);
      __syncwarp();
      wait(mma_drain, 0);
    }
    __syncwarp();
    }
  } else {
    regs_inc<kFwdRegsSoftmax>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int row = (warp & 3) * 32 + lane;
    const int qs = q0 + 128 * t;
    const int q = qs + row;
    const bool q_valid = q < p.Tq;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + 128 * t;
    const uint32_t tO = tmem + lane_base + 256 + D * t;
    const int n = n_slot[t];

    // Rows past Tq read row Tq-1 (always in bounds) and are never stored: the loads
    // below carry no per-lane branch, so the warp stays converged for the TMEM ops.
    const int64_t qc = min(q, p.Tq - 1);
    const float* score_row = nullptr;
    const uint8_t* mask_row = nullptr;
    if (kScore) score_row = p.score + b * p.score_stride[0] + h * p.score_stride[1] + qc * p.score_stride[2];
    if (kMask) mask_row = p.mask + b * p.mask_stride[0] + h * p.mask_stride[1] + qc * p.mask_stride[2];

    float m_run = kNegInf;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      // Warp-uniform outcome: the tcgen05.ld below is warp-collective.
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * c]));
      tmem_wait_ld();

      const int kbase = j * 128;
      const bool need_bounds = kbase + 128 > p.Tk;
      const bool need_causal = p.causal && (kbase + 127 > qs + p.causal_off);
      // Interior tile (warp-uniform): nothing to add or mask, so the row max is taken
      // on raw S and the scale is folded into the exponent's FMA below.
      const bool fast = !kMask && !kScore && !need_bounds && !need_causal && p.scale_log2 > 0.f;
      float m_tile = kNegInf;
      if (fast) {
        float m4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(sr[i]));
        m_tile = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
      } else {
#pragma unroll
      for (int c4 = 0; c4 < 32; ++c4) {
        const int k4 = kbase + 4 * c4;
        float add[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t keep_bits = 0xFu;
        // k4 is the same for every lane, so these branches are warp-uniform.
        if constexpr (kScore) {
          if (p.score_vec && k4 + 3 < p.Tk) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(score_row + k4));
            add[0] = v.x; add[1] = v.y; add[2] = v.z; add[3] = v.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (k4 + e < p.Tk) add[e] = __ldg(score_row + k4 + e);
          }
        }
        if constexpr (kMask) {
          keep_bits = 0u;
          if (p.mask_vec && k4 + 3 < p.Tk) {
            const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(mask_row + k4));
#pragma unroll
            for (int e = 0; e < 4; ++e) keep_bits |= (((w >> (8 * e)) & 0xFFu) != 0u ? 1u : 0u) << e;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (k4 + e < p.Tk) keep_bits |= (__ldg(mask_row + k4 + e) != 0 ? 1u : 0u) << e;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = 4 * c4 + e;
          const int k = k4 + e;
          float x = __uint_as_float(sr[i]);
          if constexpr (kScore) x += add[e];
          x *= p.scale_log2;
          bool keep = (keep_bits >> e) & 1u;
          if (need_bounds) keep = keep && (k < p.Tk);
          if (need_causal) keep = keep && (k <= q + p.causal_off);
          x = keep ? x : kNegInf;
          sr[i] = __float_as_uint(x);
          m_tile = fmaxf(m_tile, x);
        }
      }
      }

      // Online softmax with lazy rescaling of O.
      const float m_new = fmaxf(m_run, m_tile);
      const bool need = m_new > m_run + kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = ex2(m_run - m_new);  // m_run == -inf -> 0
        l_run *= alpha;
        m_run = m_new;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // PV of tile j-1 has completed (S of tile j was issued after it).
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(tO + 16 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(tO + 16 * c, o);
        }
      }
      const float m_use = (m_run == kNegInf) ? 0.f : m_run;
      float rowsum = 0.f;
      if (fast) {
        // exp2(s * scale * log2(e) - m); one element in four on the FMA pipe
        // (ex2_poly) so the MUFU unit is not the limit.
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = fmaf(__uint_as_float(sr[32 * c + 2 * i]), p.scale_log2, -m_use);
            const float a1 = fmaf(__uint_as_float(sr[32 * c + 2 * i + 1]), p.scale_log2, -m_use);
            const float p0 = ex2(a0);
            const float p1 = (i & 1) ? ex2_poly(a1) : ex2(a1);
            rowsum += p0 + p1;
            pk[i] = pack2<kBF16>(p0, p1);
          }
          tmem_st16(tS + 16 * c, pk);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ex2(__uint_as_float(sr[32 * c + 2 * i]) - m_use);
            const float p1 = ex2(__uint_as_float(sr[32 * c + 2 * i + 1]) - m_use);
            rowsum += p0 + p1;
            pk[i] = pack2<kBF16>(p0, p1);
          }
          tmem_st16(tS + 16 * c, pk);
        }
      }
      l_run += rowsum;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }

    // Epilogue: O / l and LSE.
    using Elem = uint16_t;
    Elem* o_row = nullptr;
    if (q_valid)
      o_row = reinterpret_cast<Elem*>(p.o) + b * p.o_stride[0] + static_cast<int64_t>(q) * p.o_stride[1] +
              h * p.o_stride[2];
    if (n > 0 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], 0, abort_flag));
      tc_fence_after();
      const float inv_l = 1.f / l_run;  // l == 0 (no valid key) -> inf -> O = NaN like the oracle
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        if (q_valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack2<kBF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(o_row + 32 * c);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
    } else if (q_valid) {
      const uint32_t nan2 = pack2<kBF16>(NAN, NAN);
      uint4* dst = reinterpret_cast<uint4*>(o_row);
#pragma unroll
      for (int v = 0; v < D / 8; ++v) dst[v] = make_uint4(nan2, nan2, nan2, nan2);
    }
    if (q_valid) {
      const float lse = (l_run > 0.f) ? (__log2f(l_run) + m_run) : kNegInf;
      p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q] = lse;
    }
    tc_fence_before();
  }

  __syncthreads();
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(abort_flag)) atomicOr(p.status, FA4D_DEV_TIMEOUT_FWD);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool kBF16, bool kMask, bool kScore>
cudaError_t launch_fwd_t(const FwdParams& p, cudaStream_t s) {
  using L = FwdLayout<D>;
  auto kern = fwd_kernel<D, kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  dim3 grid((p.Tq + 255) / 256, p.Hq, p.B);
  kern<<<grid, kFwdThreads, L::kAlloc, s>>>(p);
  return cudaGetLastError();
}

template <int D, bool kBF16>
cudaError_t launch_fwd_d(const FwdParams& p, bool m, bool sc, cudaStream_t s) {
  if (m && sc) return launch_fwd_t<D, kBF16, true, true>(p, s);
  if (m) return launch_fwd_t<D, kBF16, true, false>(p, s);
  if (sc) return launch_fwd_t<D, kBF16, false, true>(p, s);
  return launch_fwd_t<D, kBF16, false, false>(p, s);
}

}  // namespace

cudaError_t launch_fwd(const FwdParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s) {
  if (D == 128) return bf16 ? launch_fwd_d<128, true>(p, has_mask, has_score, s)
                            : launch_fwd_d<128, false>(p, has_mask, has_score, s);
  if (D == 64) return bf16 ? launch_fwd_d<64, true>(p, has_mask, has_score, s)
                           : launch_fwd_d<64, false>(p, has_mask, has_score, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa4d

namespace {

// out[i] = ex2_poly(x_i) / exp2f(x_i) - 1 on an even grid x_i over [lo, hi].
__global__ void exp2_check_kernel(float* out, int n, float lo, float hi) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = lo + (hi - lo) * (static_cast<float>(i) / static_cast<float>(n - 1));
  out[i] = fa4d::ex2_poly(x) / exp2f(x) - 1.0f;
}

}  // namespace

namespace fa4d {
cudaError_t launch_exp2_check(float* out, int n, float lo, float hi, cudaStream_t s) {
  exp2_check_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, n, lo, hi);
  return cudaGetLastError();
}
}  // namespace fa4d
