// fa4d_dq.cu — deterministic dQ for the backward (use_atomic_backward=False).
//
// The main backward kernel owns a key tile and adds each query tile's dQ contribution
// into an fp32 accumulator as it goes, so the order of the additions depends on
// scheduling.  Here one CTA owns a 128-row query tile of one (batch, head) and walks
// its key tiles in order, recomputing S = Q K^T and dP = dO V^T, forming
// dS = P (dP - Delta) with P = exp2(S * scale * log2(e) - LSE) (python/fa2.py:242-290)
// and accumulating dQ = dS K in tensor memory; dQ is written once, scaled, in the
// input dtype.  The result is bit-reproducible.  The main kernel then skips its dQ
// products (BwdParams::skip_dq).
//
// CTA = 128 query rows, 384 threads: warp 0 TMA (Q, dO, LSE, Delta once; K/V rings),
// warp 1 MMA issue, warp 2 TMEM allocation, warps 4-7 and 8-11 two warpgroups that
// share each key tile: one thread per query row, warpgroup w on keys [64w, 64w + 64)
// (P and dS are elementwise once LSE is known, so the halves need no exchange).
// TMEM: S x2 [0,256) (a tile's dS as 16-bit overwrites columns [0,32) and [64,96) of
// its S buffer), dP [256,384), dQ [384,384+D).  Per key tile u the MMA warp waits for
// dS(u), then issues dP(u+1) (the dP buffer is free once dS(u) is formed), dQ += dS(u)
// K(u) (A = dS from TMEM, B = K, MN-major) and S(u+2) into the S buffer dQ(u) has just
// read; S(u+1) was issued a tile earlier, so the warpgroups start P(u+1) at once and
// dQ(u) runs under the next dS.
#include <cfloat>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kDqThreads = 384;

template <int D>
struct DqLayout {
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kDO = kQ + kTile;
  static constexpr int kK = kDO + kTile;     // 2 stages
  static constexpr int kV = kK + 2 * kTile;  // 2 stages
  static constexpr int kLSE = kV + 2 * kTile;
  static constexpr int kDelta = kLSE + 512;
  static constexpr int kBar = kDelta + 512;
  static constexpr int kNumBars = 14;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

// D[128 x 128] = A[128 rows x D] B[128 rows x D]^T, both K-major (S = Q K^T, dP = dO V^T).
template <int D, bool kBF16>
__device__ __forceinline__ void issue_abt(uint32_t tD, uint32_t sA, uint32_t sB) {
  constexpr uint32_t idesc = make_idesc(128, 128, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
    mma_ss(tD, sw128_desc(sA + off, 16, 1024), sw128_desc(sB + off, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// dQ (+)= dS K : M=128 queries, N=D, K=128 keys; dS from TMEM (keys 0-63 at columns
// [0,32) of the S buffer, keys 64-127 at [64,96)), K MN-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_dsk(uint32_t tDQ, uint32_t tDS, uint32_t sK, bool accumulate) {
  constexpr uint32_t idesc = make_idesc(128, D, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    mma_ts(tDQ, tDS + (kk >> 2) * 64 + (kk & 3) * 8, sw128_desc(sK + kk * 2048, 16384, 1024), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

template <int D, bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kDqThreads, 1) dq_kernel(const __grid_constant__ DqParams p) {
  using L = DqLayout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] S of a tile is in S buffer u & 1
  uint64_t* dp_full = bars + 11; // dP of the current tile is in TMEM
  uint64_t* ds_full = bars + 12; // dS written to TMEM, dP read (256 arrivals)
  uint64_t* mma_drain = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (Hq, query tiles, B), heads fastest; causal runs the longest tiles first.
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

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_full, 256);
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
  constexpr uint32_t kColS = 0, kColDP = 256, kColDQ = 384;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && any_work) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_do);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      mbar_arrive_expect_tx(q_full, 2 * L::kTile + 1024);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(smem + L::kQ + c * 16384, &p.tm_q, q_full, c * 64, q0, h, b);
        tma_load_4d(smem + L::kDO + c * 16384, &p.tm_do, q_full, c * 64, q0, h, b);
      }
      const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0;
      bulk_load(smem + L::kLSE, p.lse + row, 512, q_full);
      bulk_load(smem + L::kDelta, p.delta + row, 512, q_full);
      int u = 0;
      bool k_pending = false;
      for (int kt = kt_first; kt < tl.n; kt = tl.next(kt + 1), ++u) {
        const int s = u & 1;
        const uint32_t par = ((u >> 1) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], par, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + L::kK + s * L::kTile + c * 16384, &p.tm_k, &k_full[s], c * 64, kt * 128, hk, b);
        if (!mbar_wait(&v_empty[s], par, abort_flag)) {
          k_pending = true;
          break;
        }
        mbar_arrive_expect_tx(&v_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + L::kV + s * L::kTile + c * 16384, &p.tm_v, &v_full[s], c * 64, kt * 128, hk, b);
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        mbar_wait_short(q_full, 0);
        for (int j = max(0, u - 2); j < u; ++j) {
          mbar_wait_short(&k_full[j & 1], (j >> 1) & 1);
          mbar_wait_short(&v_full[j & 1], (j >> 1) & 1);
        }
        if (k_pending) mbar_wait_short(&k_full[u & 1], (u >> 1) & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (any_work) {
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sDO = smem_u32(smem + L::kDO);
      const uint32_t sK = smem_u32(smem + L::kK);
      const uint32_t sV = smem_u32(smem + L::kV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      // Tiles u = 0, 1, ... are the visited key tiles in order (K/V stage u & 1).
      const int k1 = tl.next(kt_first + 1);
      bool ok = wait(q_full, 0) && wait(&k_full[0], 0) && wait(&v_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
          issue_abt<D, kBF16>(tmem + kColS, sQ, sK);
          tc_commit(&s_full[0]);
          issue_abt<D, kBF16>(tmem + kColDP, sDO, sV);
          tc_commit(dp_full);
          tc_commit(&v_empty[0]);
        }
        __syncwarp();
      }
      if (ok && k1 < tl.n) {
        ok = wait(&k_full[1], 0);
        if (ok) {
          tc_fence_after();
          if (elect_one()) {
            issue_abt<D, kBF16>(tmem + kColS + 128, sQ, sK + L::kTile);
            tc_commit(&s_full[1]);
          }
          __syncwarp();
        }
      }
      int u = 0;
      int kt_a = k1;                  // tile u + 1
      int kt_b = k1 < tl.n ? tl.next(k1 + 1) : tl.n;  // tile u + 2
      for (int kt = kt_first; ok && kt < tl.n; kt = kt_a, kt_a = kt_b, kt_b = kt_b < tl.n ? tl.next(kt_b + 1) : tl.n, ++u) {
        const int s = u & 1;
        ok = wait(ds_full, u & 1);
        if (!ok) break;
        const bool has1 = kt_a < tl.n, has2 = kt_b < tl.n;
        if (has1) {
          ok = wait(&v_full[s ^ 1], ((u + 1) >> 1) & 1);
          if (!ok) break;
        }
        tc_fence_after();
        if (elect_one()) {
          if (has1) {
            // dP of tile u+1: the warpgroups have read dP(u) (ds_full).
            issue_abt<D, kBF16>(tmem + kColDP, sDO, sV + (s ^ 1) * L::kTile);
            tc_commit(dp_full);
            tc_commit(&v_empty[s ^ 1]);
          }
          issue_dsk<D, kBF16>(tmem + kColDQ, tmem + kColS + 128 * s, sK + s * L::kTile, u > 0);
          tc_commit(&k_empty[s]);
        }
        __syncwarp();
        if (has2) {
          // S of tile u+2 into the buffer whose dS the dQ above read (issued in order).
          ok = wait(&k_full[s], ((u + 2) >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_abt<D, kBF16>(tmem + kColS + 128 * s, sQ, sK + s * L::kTile);
            tc_commit(&s_full[s]);
          }
          __syncwarp();
        }
      }
      if (elect_one()) tc_commit(mma_drain);
      __syncwarp();
      wait(mma_drain, 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ dS and epilogue
    const int wg = (warp - 4) >> 2;  // keys [64 wg, 64 wg + 64) of every tile
    const int row = (warp & 3) * 32 + lane;
    const int q = q0 + row;
    const bool q_valid = q < p.Tq;
    const int64_t qc = min(q, p.Tq - 1);
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS0 = tmem + lane_base + kColS + 64 * wg;
    const uint32_t tDP = tmem + lane_base + kColDP + 64 * wg;
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
    for (int kt = kt_first; ok && kt < tl.n; kt = tl.next(kt + 1), ++u) {
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
      const int kbase = kt * 128;
      if (kbase + 128 > p.Tk || (p.causal && kbase + 127 > q0 + p.causal_off)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) mw[c] &= low_bits(key_lim - (kbase + 32 * c));
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[u & 1], (u >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tS0 + 128 * (u & 1);
      // P for this warpgroup's 64 keys (kept in registers), then dS once dP is in.
      float pr[64];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * wg + cc;
        uint32_t sv[32];
        tmem_ld32(tS + 32 * cc, sv);
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
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = __uint_as_float(sv[i]);
          if constexpr (kScore) x += add[i];
          const float e = ex2(fmaf(x, p.scale_log2, -lse));
          pr[32 * cc + i] = ((mw[c] >> i) & 1u) ? e : 0.f;
        }
      }
      ok = __all_sync(0xffffffffu, mbar_wait(dp_full, u & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t dpv[32];
        tmem_ld32(tDP + 32 * cc, dpv);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          // dS without the softmax scale (applied to dQ at the end).
          pk[e] = pack2<kBF16>(pr[32 * cc + 2 * e] * (__uint_as_float(dpv[2 * e]) - delta),
                               pr[32 * cc + 2 * e + 1] * (__uint_as_float(dpv[2 * e + 1]) - delta));
        // dS (16-bit) for this warpgroup's keys 32cc..32cc+31 goes to columns
        // 16cc..16cc+15 of its half of the S buffer, which hold S values already read.
        tmem_st16(tS + 16 * cc, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    // Epilogue: dQ = scale * accumulated dS K, in the input dtype.
    uint16_t* dst = q_valid ? reinterpret_cast<uint16_t*>(p.dq) + b * p.dq_stride[0] +
                                  static_cast<int64_t>(q) * p.dq_stride[1] + h * p.dq_stride[2]
                            : nullptr;
    if (u > 0 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(mma_drain, 0, abort_flag));
      tc_fence_after();
#pragma unroll
      for (int c = wg * (D / 64); c < (wg + 1) * (D / 64); ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + kColDQ + 32 * c, v);
        tmem_wait_ld();
        if (q_valid && 32 * c < p.d_out) {
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
      for (int w = wg * (D / 16); w < (wg + 1) * (D / 16); ++w)
        if (8 * w < p.d_out) reinterpret_cast<uint4*>(dst)[w] = make_uint4(0u, 0u, 0u, 0u);
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

template <int D, bool kBF16, bool kMask, bool kScore>
cudaError_t launch_dq_t(const DqParams& p, cudaStream_t s) {
  using L = DqLayout<D>;
  auto kern = dq_kernel<D, kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Hq, (p.Tq + 127) / 128, p.B);
  kern<<<grid, kDqThreads, L::kAlloc, s>>>(p);
  return cudaGetLastError();
}

template <int D, bool kBF16>
cudaError_t launch_dq_d(const DqParams& p, bool m, bool sc, cudaStream_t s) {
  if (m && sc) return launch_dq_t<D, kBF16, true, true>(p, s);
  if (m) return launch_dq_t<D, kBF16, true, false>(p, s);
  if (sc) return launch_dq_t<D, kBF16, false, true>(p, s);
  return launch_dq_t<D, kBF16, false, false>(p, s);
}

}  // namespace

cudaError_t launch_dq(const DqParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s) {
  if (D == 128) return bf16 ? launch_dq_d<128, true>(p, has_mask, has_score, s)
                            : launch_dq_d<128, false>(p, has_mask, has_score, s);
  if (D == 64) return bf16 ? launch_dq_d<64, true>(p, has_mask, has_score, s)
                           : launch_dq_d<64, false>(p, has_mask, has_score, s);
  if (D == 256) return launch_dq256(p, bf16, has_mask, has_score, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa4d
