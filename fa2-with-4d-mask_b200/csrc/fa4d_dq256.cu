// fa4d_dq256.cu — deterministic dQ at head dim 256 (use_atomic_backward=False).
//
// As dq_kernel for the other head dims (fa4d_dq.cu): one CTA owns a 128-row query tile
// of one (batch, head), walks its key tiles in order, recomputes S = Q K^T and
// dP = dO V^T, forms dS = P (dP - Delta) with P = exp2(S * scale * log2(e) - LSE)
// (python/fa2.py:242-290) and accumulates dQ = dS K in tensor memory; dQ is written
// once, scaled, in the input dtype, so the result is bit-reproducible.
// At D = 256 the 128-row Q and dO tiles take 128 KB of shared memory, so each 128-key
// tile is walked as two 64-key halves: K in a 2-stage ring of 32 KB halves, V in one
// 32 KB stage (free again as soon as dP of its half is done).
//
// CTA = 128 query rows, 384 threads: warp 0 TMA (Q, dO, LSE, Delta, K halves), warp 1
// MMA issue, warp 2 TMEM allocation, warp 3 TMA (V halves), warps 4-7 and 8-11 one
// thread per query row, warpgroup wg taking keys 32 wg .. 32 wg + 31 of every half
// and dQ columns 128 wg .. 128 wg + 127 in the epilogue.
// TMEM: S x2 [0,128) (dS as 16-bit overwrites the first 16 of each warpgroup's 32 S
// columns), dP x2 [128,256), dQ [256,512).  Per 64-key half u the MMAs go S(u),
// dQ += dS K of half u-1 (A = dS from TMEM, B = K MN-major, N = 256), dP(u): S and dP
// of half u run while the row threads form dS of half u-1, and the K half of u-1 is
// released (for the load of u+1) before dP(u) runs.
#include <cfloat>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kThreads = 384;

struct Layout {
  static constexpr int kQT = 128 * 256 * 2;  // Q or dO tile (128 rows x 256)
  static constexpr int kKT = 64 * 256 * 2;   // K or V half tile (64 keys x 256)
  static constexpr int kQ = 0;
  static constexpr int kDO = kQ + kQT;
  static constexpr int kK = kDO + kQT;  // 2 stages
  static constexpr int kV = kK + 2 * kKT;
  static constexpr int kLSE = kV + kKT;
  static constexpr int kDelta = kLSE + 512;
  static constexpr int kBar = kDelta + 512;
  static constexpr int kNumBars = 13;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 256;  // S, dP: 2 buffers of 64 columns

// D[128 x 64] = A[128 rows x 256] B[64 rows x 256]^T, both K-major (S = Q K^T, dP = dO V^T).
template <bool kBF16>
__device__ __forceinline__ void issue_abt(uint32_t tD, uint32_t sA, uint32_t sB) {
  constexpr uint32_t idesc = make_idesc(128, 64, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < 16; ++kk) {
    const uint32_t offa = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
    const uint32_t offb = static_cast<uint32_t>((kk >> 2) * 8192 + (kk & 3) * 32);
    mma_ss(tD, sw128_desc(sA + offa, 16, 1024), sw128_desc(sB + offb, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// dQ (+)= dS K : M=128 queries, N=256, K=64 keys; dS from TMEM (keys 0-31 in columns
// [0,16), keys 32-63 in [32,48) of the S buffer), K MN-major (4 chunks).
template <bool kBF16>
__device__ __forceinline__ void issue_dsk(uint32_t tDQ, uint32_t tDS, uint32_t sK, bool accumulate) {
  constexpr uint32_t idesc = make_idesc(128, 256, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tDQ, tDS + (kk >> 1) * 32 + (kk & 1) * 8, sw128_desc(sK + kk * 2048, 8192, 1024), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

// Number of 64-key halves of key tile kt that hold keys below kv_end (1 or 2).
__device__ __forceinline__ int halves(int kt, int kv_end) { return kt * 128 + 64 < kv_end ? 2 : 1; }

template <bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kThreads, 1) dq256_kernel(const __grid_constant__ DqParams p) {
  // With a mask or score the row threads take longer per half, and a single issuing
  // thread, which issues dP(u) only after dQ of half u-1 (and so after its dS), stalls
  // behind them: those variants give dP to warp 2 (dQ pass with mask + score at B1 T4096
  // H16: 0.984 -> 0.660 ms).  The dense variants keep one issuer (1% faster there).
  constexpr bool kTwoIssuers = kMask || kScore;
  using L = Layout;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;    // [2] S and dP of the half are in TMEM (one commit per issuer)
  uint64_t* ds_full = bars + 9;   // [2] dS written to TMEM (256 arrivals)
  uint64_t* mma_drain = bars + 11;
  uint64_t* mma_drain_dp = bars + 12;  // the dP issuer's MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qblk = p.causal ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : static_cast<int>(blockIdx.y);
  const int h = blockIdx.x;
  const int b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qblk * 128;

  SlotTiles<kMask> tl;
  tl.n = kv_tile_count(q0, min(q0 + 128, p.Tq), p.Tq, p.Tk, p.causal, p.causal_off);
  tl.map = (kMask && p.mask_blocks && tl.n > 0)
               ? p.mask_blocks + b * p.mb_stride[0] + h * p.mb_stride[1] + static_cast<int64_t>(qblk) * p.nkb
               : nullptr;
  const int kt_first = tl.next(0);
  const bool any_work = kt_first < tl.n;
  // Keys below kv_end can be kept by some row of the tile (key bound and causal limit).
  int kv_end = p.Tk;
  if (p.causal) {
    const long long lim = static_cast<long long>(min(q0 + 128, p.Tq)) + p.causal_off;
    kv_end = lim < p.Tk ? static_cast<int>(lim) : p.Tk;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], kTwoIssuers ? 2 : 1);
      mbar_init(&ds_full[i], 256);
    }
    mbar_init(mma_drain, 1);
    mbar_init(mma_drain_dp, 1);
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

  if ((warp == 0 || warp == 3) && lane == 0 && any_work) {
    // ------------------------------------------------------------ TMA producers
    // Warp 0: Q, dO, LSE, Delta once, then the K half of every half u (2-stage ring,
    // a stage freed by dQ of its half); warp 3: the V half of every half (one stage,
    // freed by dP of its half).
    const bool is_k = warp == 0;
    if (is_k) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_do);
      prefetch_tmap(&p.tm_k);
      mbar_arrive_expect_tx(q_full, 2 * L::kQT + 1024);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(smem + L::kQ + c * 16384, &p.tm_q, q_full, c * 64, q0, h, b);
        tma_load_4d(smem + L::kDO + c * 16384, &p.tm_do, q_full, c * 64, q0, h, b);
      }
      const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0;
      bulk_load(smem + L::kLSE, p.lse + row, 512, q_full);
      bulk_load(smem + L::kDelta, p.delta + row, 512, q_full);
    } else {
      prefetch_tmap(&p.tm_v);
    }
    int u = 0;  // halves whose load was issued
    bool stop = false;
    for (int kt = kt_first; kt < tl.n && !stop; kt = tl.next(kt + 1)) {
      const int nh = halves(kt, kv_end);
      for (int j = 0; j < nh; ++j) {
        const int key0 = kt * 128 + 64 * j;
        if (is_k) {
          const int s = u & 1;
          if (!mbar_wait(&k_empty[s], ((u >> 1) & 1) ^ 1, abort_flag)) {
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&k_full[s], L::kKT);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tma_load_4d(smem + L::kK + s * L::kKT + c * 8192, &p.tm_k, &k_full[s], c * 64, key0, hk, b);
        } else {
          if (!mbar_wait(v_empty, (u & 1) ^ 1, abort_flag)) {
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(v_full, L::kKT);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tma_load_4d(smem + L::kV + c * 8192, &p.tm_v, v_full, c * 64, key0, hk, b);
        }
        ++u;
      }
    }
    if (*reinterpret_cast<volatile int*>(abort_flag)) {
      // Wait (bounded) for this producer's copies still in flight.
      if (is_k) {
        mbar_wait_short(q_full, 0);
        for (int jj = max(0, u - 2); jj < u; ++jj) mbar_wait_short(&k_full[jj & 1], (jj >> 1) & 1);
      } else if (u > 0) {
        mbar_wait_short(v_full, (u - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (S, dQ, dP)
    // Per half u: S(u) into buffer u & 1, then dQ += dS K of half u-1 (its dS sits in
    // the other buffer; issuing it frees that K stage), then dP(u) (from warp 2 in the
    // mask / score variants).  S(u) overwrites the dS of half u-2, which dQ read one half
    // earlier (MMAs of one thread run in issue order).  s_full of a half completes with
    // the commit after dP, or with two issuers with one commit after each of S and dP.
    if (any_work) {
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sDO = smem_u32(smem + L::kDO);
      const uint32_t sK = smem_u32(smem + L::kK);
      const uint32_t sV = smem_u32(smem + L::kV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      // dQ += dS K of half w (dS in S buffer w & 1, K in stage w & 1).
      auto issue_dq = [&](int w) {
        if (!wait(&ds_full[w & 1], (w >> 1) & 1)) return false;
        tc_fence_after();
        if (elect_one()) {
          issue_dsk<kBF16>(tmem + kColDQ, tmem + kColS + 64 * (w & 1), sK + (w & 1) * L::kKT, w > 0);
          tc_commit(&k_empty[w & 1]);
        }
        __syncwarp();
        return true;
      };
      bool ok = wait(q_full, 0);
      int u = 0;
      for (int kt = kt_first; ok && kt < tl.n; kt = tl.next(kt + 1)) {
        const int nh = halves(kt, kv_end);
        for (int j = 0; ok && j < nh; ++j, ++u) {
          const int s = u & 1;
          ok = wait(&k_full[s], (u >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_abt<kBF16>(tmem + kColS + 64 * s, sQ, sK + s * L::kKT);
            if (kTwoIssuers) tc_commit(&s_full[s]);
          }
          __syncwarp();
          if (u > 0) {
            ok = issue_dq(u - 1);
            if (!ok) break;
          }
          if constexpr (!kTwoIssuers) {
            ok = wait(v_full, u & 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_abt<kBF16>(tmem + kColDP + 64 * s, sDO, sV);
              tc_commit(v_empty);
              tc_commit(&s_full[s]);
            }
            __syncwarp();
          }
        }
      }
      if (ok && u > 0) ok = issue_dq(u - 1);
      if (elect_one()) tc_commit(mma_drain);
      __syncwarp();
      wait(mma_drain, 0);
    }
    __syncwarp();
  } else if (kTwoIssuers && warp == 2) {
    // ------------------------------------------------------------ MMA issuer (dP)
    // dP(u) into buffer u & 1 once V(u) has landed and the row threads have read dP of
    // half u-2 out of that buffer (they arrive on ds_full after reading it).
    if (any_work) {
      const uint32_t sDO = smem_u32(smem + L::kDO);
      const uint32_t sV = smem_u32(smem + L::kV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      bool ok = wait(q_full, 0);
      int u = 0;
      for (int kt = kt_first; ok && kt < tl.n; kt = tl.next(kt + 1)) {
        const int nh = halves(kt, kv_end);
        for (int j = 0; ok && j < nh; ++j, ++u) {
          const int s = u & 1;
          if (u >= 2) {
            ok = wait(&ds_full[s], ((u - 2) >> 1) & 1);
            if (!ok) break;
          }
          ok = wait(v_full, u & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_abt<kBF16>(tmem + kColDP + 64 * s, sDO, sV);
            tc_commit(v_empty);
            tc_commit(&s_full[s]);
          }
          __syncwarp();
        }
      }
      if (elect_one()) tc_commit(mma_drain_dp);
      __syncwarp();
      wait(mma_drain_dp, 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dS and epilogue
    const int wg = (warp - 4) >> 2;  // keys 32 wg .. 32 wg + 31 of every half
    const int row = (warp & 3) * 32 + lane;
    const int q = q0 + row;
    const bool q_valid = q < p.Tq;
    const int64_t qc = min(q, p.Tq - 1);
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float* score_row = nullptr;
    const uint8_t* mask_row = nullptr;
    const uint4* bits_row = nullptr;
    if (kScore) score_row = p.score + b * p.score_stride[0] + h * p.score_stride[1] + qc * p.score_stride[2];
    if (kMask) {
      mask_row = p.mask + b * p.mask_stride[0] + h * p.mask_stride[1] + qc * p.mask_stride[2];
      if (p.mask_bits)
        bits_row = reinterpret_cast<const uint4*>(p.mask_bits + b * p.mbits_stride[0] + h * p.mbits_stride[1]) + qc;
    }
    const int key_lim = p.causal ? static_cast<int>(min(static_cast<long long>(q) + p.causal_off + 1,
                                                        static_cast<long long>(p.Tk)))
                                 : p.Tk;
    bool ok = __all_sync(0xffffffffu, !any_work || mbar_wait(q_full, 0, abort_flag));
    const float lse = reinterpret_cast<const float*>(smem + L::kLSE)[row];
    const float delta = reinterpret_cast<const float*>(smem + L::kDelta)[row];
    int u = 0;
    for (int kt = kt_first; ok && kt < tl.n; kt = tl.next(kt + 1)) {
      const int st = tl.state(kt);
      const bool use_mask = kMask && st == 1;
      uint32_t mw[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      if (kMask && use_mask) {
        const uint4 v = bits_row ? __ldg(bits_row + static_cast<int64_t>(kt) * p.Tq)
                                 : mask_words_from_bytes(mask_row, kt * 128, p.Tk, p.mask_vec);
        mw[0] = v.x;
        mw[1] = v.y;
        mw[2] = v.z;
        mw[3] = v.w;
      }
      const int nh = halves(kt, kv_end);
      for (int j = 0; ok && j < nh; ++j, ++u) {
        const int kbase = kt * 128 + 64 * j;
        uint32_t w2[2] = {mw[2 * j], mw[2 * j + 1]};
        if (kbase + 64 > p.Tk || (p.causal && kbase + 63 > q0 + p.causal_off)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) w2[c] &= low_bits(key_lim - (kbase + 32 * c));
        }
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[u & 1], (u >> 1) & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_base + kColS + 64 * (u & 1);
        const uint32_t tDP = tmem + lane_base + kColDP + 64 * (u & 1);
        {
          const int c = wg;
          const uint32_t keep = wg ? w2[1] : w2[0];
          uint32_t sv[32], dpv[32];
          tmem_ld32(tS + 32 * c, sv);
          tmem_ld32(tDP + 32 * c, dpv);
          tmem_wait_ld();
          const int kc = kbase + 32 * c;
          float add[32];
          if constexpr (kScore) {
            if (p.score_vec && kc + 31 < p.Tk) {
#pragma unroll
              for (int e4 = 0; e4 < 8; ++e4) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(score_row + kc) + e4);
                add[4 * e4] = v.x;
                add[4 * e4 + 1] = v.y;
                add[4 * e4 + 2] = v.z;
                add[4 * e4 + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) add[e] = (kc + e < p.Tk) ? __ldg(score_row + kc + e) : 0.f;
            }
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float ds2[2];
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int i = 2 * e + jj;
              float x = __uint_as_float(sv[i]);
              if constexpr (kScore) x += add[i];
              const float pr = ex2(fmaf(x, p.scale_log2, -lse));
              // dS without the softmax scale (applied to dQ at the end).
              ds2[jj] = ((keep >> i) & 1u) ? pr * (__uint_as_float(dpv[i]) - delta) : 0.f;
            }
            pk[e] = pack2<kBF16>(ds2[0], ds2[1]);
          }
          // dS (16-bit) for keys 32c..32c+31 goes to columns 32c..32c+15: S values this
          // warpgroup has already read (the other warpgroup reads only its own 32).
          tmem_st16(tS + 32 * c, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&ds_full[u & 1]);
      }
    }
    // Epilogue: dQ = scale * accumulated dS K, in the input dtype.
    uint16_t* dst = q_valid ? reinterpret_cast<uint16_t*>(p.dq) + b * p.dq_stride[0] +
                                  static_cast<int64_t>(q) * p.dq_stride[1] + h * p.dq_stride[2]
                            : nullptr;
    if (u > 0 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(mma_drain, 0, abort_flag));
      tc_fence_after();
#pragma unroll
      for (int c = 4 * wg; c < 4 * wg + 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + kColDQ + 32 * c, v);
        tmem_wait_ld();
        if (q_valid) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            pk[i] = pack2<kBF16>(__uint_as_float(v[2 * i]) * p.scale, __uint_as_float(v[2 * i + 1]) * p.scale);
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int w = 0; w < 4; ++w) d4[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        }
      }
    } else if (q_valid) {
#pragma unroll
      for (int w = 16 * wg; w < 16 * wg + 16; ++w) reinterpret_cast<uint4*>(dst)[w] = make_uint4(0u, 0u, 0u, 0u);
    }
    tc_fence_before();
  }

  __syncthreads();
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(abort_flag)) atomicOr(p.status, FA4D_DEV_TIMEOUT_BWD);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kBF16, bool kMask, bool kScore>
cudaError_t launch_t(const DqParams& p, cudaStream_t s) {
  auto kern = dq256_kernel<kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::kAlloc);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Hq, (p.Tq + 127) / 128, p.B);
  kern<<<grid, kThreads, Layout::kAlloc, s>>>(p);
  return cudaGetLastError();
}

template <bool kBF16>
cudaError_t launch_d(const DqParams& p, bool m, bool sc, cudaStream_t s) {
  if (m && sc) return launch_t<kBF16, true, true>(p, s);
  if (m) return launch_t<kBF16, true, false>(p, s);
  if (sc) return launch_t<kBF16, false, true>(p, s);
  return launch_t<kBF16, false, false>(p, s);
}

}  // namespace

cudaError_t launch_dq256(const DqParams& p, bool bf16, bool has_mask, bool has_score, cudaStream_t s) {
  return bf16 ? launch_d<true>(p, has_mask, has_score, s) : launch_d<false>(p, has_mask, has_score, s);
}

}  // namespace fa4d
