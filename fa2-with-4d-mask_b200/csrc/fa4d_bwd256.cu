// fa4d_bwd256.cu — FlashAttention-2 backward at head dim 256 for sm_100a, with an
// optional 4D mask/score.
//
// Same math as the other head dims (python/fa2.py:181-302; dS carried without the
// factor `scale`, applied to dK in its epilogue and to dQ at conversion).  At D = 256
// the dK and dV accumulators of a 128-key tile would take all 512 TMEM columns, so the
// output columns are split: CTA pair (ch = 0, 1) shares one 128-key tile of one
// (batch, KV head) and CTA ch owns columns [128 ch, 128 ch + 128) of dK and dV.
// Both CTAs of a pair compute the full S^T = K Q^T and dP^T = V dO^T (contraction over
// all 256 columns); each then does its half of dV += P^T dO and dK += dS^T Q.
// dQ comes from the ordered pass (dq256_kernel, fa4d_dq256.cu) at this head dim: with
// one S / dP buffer pair, adding dQ^T here (its product and drain between one tile's
// dS and the next tile's dP) ran slower than the separate pass.
//
// CTA = 128 keys x one (batch, KV head) x one column half; 384 threads:
//   warp 0       TMA producer (K once; Q, dO, LSE, Delta per 64-row query tile,
//                2-stage ring)
//   warp 1       tcgen05.mma issuer
//   warp 2       TMEM allocator
//   warps 4-7    queries 0-31 of every tile (one thread per key row), then dV out;
//                at the start they copy V columns 0-127 into TMEM
//   warps 8-11   queries 32-63 of every tile, then dK out; V columns 128-255
// TMEM (512 columns): S^T [0,64) (P^T of queries 0-31 then 32-63 is written over
// columns [0,16) and [32,48)), dP^T [64,128), V [128,256) (16-bit pairs, the A
// operand of dP^T), dV half [256,384), dK half [384,512).
// Shared memory: K 64 KB, Q and dO 2 x 32 KB each, dS^T 16 KB, LSE / Delta: 210 KB.
#include <algorithm>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kThreads = 384;
constexpr int kStages = 2;
// Register split (launch: 384 threads x 168 = 64512): producer/MMA warpgroup 112,
// P/dS warpgroups 192 -> 128*112 + 256*192 = 63488.
constexpr uint32_t kRegsLaunch = 168, kRegsCtl = 112, kRegsSoftmax = 192;
static_assert(128 * kRegsCtl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");

struct Layout {
  static constexpr int kKT = 128 * 256 * 2;  // K tile (128 keys x 256)
  static constexpr int kQT = 64 * 256 * 2;   // Q or dO tile (64 queries x 256)
  static constexpr int kDS = 128 * 64 * 2;   // dS^T tile (128 keys x 64 queries, 16-bit)
  static constexpr int kK = 0;
  static constexpr int kQ = kK + kKT;               // kStages stages
  static constexpr int kDO = kQ + kStages * kQT;    // kStages stages
  static constexpr int kDSb = kDO + kStages * kQT;
  static constexpr int kLSE = kDSb + kDS;             // kStages x 64 floats
  static constexpr int kDelta = kLSE + kStages * 256;  // kStages x 64 floats
  static constexpr int kBar = kDelta + kStages * 256;
  static constexpr int kNumBars = 13;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

constexpr uint32_t kColS = 0, kColDP = 64, kColV = 128, kColDV = 256, kColDK = 384;

// S^T = K Q^T: M=128 keys, N=64 queries, K=256; both K-major (4 chunks of 64 columns).
template <bool kBF16>
__device__ __forceinline__ void issue_s(uint32_t tD, uint32_t sK, uint32_t sQ) {
  constexpr uint32_t idesc = make_idesc(128, 64, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < 16; ++kk) {
    const uint32_t offa = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
    const uint32_t offb = static_cast<uint32_t>((kk >> 2) * 8192 + (kk & 3) * 32);
    mma_ss(tD, sw128_desc(sK + offa, 16, 1024), sw128_desc(sQ + offb, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// dP^T = V dO^T: M=128 keys, N=64 queries, K=256; V from TMEM (columns kk*8 hold the
// 16-bit pairs of row elements 16kk..16kk+15), dO K-major.
template <bool kBF16>
__device__ __forceinline__ void issue_dp(uint32_t tD, uint32_t tV, uint32_t sDO) {
  constexpr uint32_t idesc = make_idesc(128, 64, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < 16; ++kk) {
    const uint32_t offb = static_cast<uint32_t>((kk >> 2) * 8192 + (kk & 3) * 32);
    mma_ts(tD, tV + kk * 8, sw128_desc(sDO + offb, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// dV_half += P^T dO_half: M=128 keys, N=128, K=64 queries.  P^T of queries 0-31 sits in
// S columns [0,16) and of queries 32-63 in [32,48); dO_half MN-major (2 chunks).
template <bool kBF16>
__device__ __forceinline__ void issue_dv(uint32_t tD, uint32_t tS, uint32_t sDOh, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, 128, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tD, tS + (kk >> 1) * 32 + (kk & 1) * 8, sw128_desc(sDOh + kk * 2048, 8192, 1024), idesc,
           (acc || kk > 0) ? 1u : 0u);
}

// dK_half += dS^T Q_half: M=128 keys, N=128, K=64 queries; dS^T K-major, Q_half MN-major.
template <bool kBF16>
__device__ __forceinline__ void issue_dk(uint32_t tD, uint32_t sDS, uint32_t sQh, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, 128, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ss(tD, sw128_desc(sDS + kk * 32, 16, 1024), sw128_desc(sQh + kk * 2048, 8192, 1024), idesc,
           (acc || kk > 0) ? 1u : 0u);
}

template <bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kThreads, 1) bwd256_kernel(const __grid_constant__ BwdParams p) {
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bars + 0;    // K in shared memory (TMA)
  uint64_t* v_full = bars + 1;     // V in TMEM (256 arrivals)
  uint64_t* dkv_full = bars + 2;   // every dV / dK product done
  uint64_t* mma_drain = bars + 3;
  uint64_t* s_full = bars + 4;     // S^T of the tile is in TMEM
  uint64_t* p_full = bars + 5;     // P^T written to TMEM (256 arrivals)
  uint64_t* dp_full = bars + 6;    // dP^T of the tile is in TMEM
  uint64_t* ds_full = bars + 7;    // dS^T written to shared memory (256 arrivals)
  uint64_t* ds_empty = bars + 8;   // dS^T buffer free again
  uint64_t* q_full = bars + 9;     // [kStages]
  uint64_t* q_empty = bars + 11;   // [kStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid as in the other head dims, with the column half innermost in the head index:
  // hx = (KV head x split) * 2 + ch.
  const int kb = p.kb_fastest ? blockIdx.x : blockIdx.y;
  const int hx = p.kb_fastest ? blockIdx.y : blockIdx.x;
  const int ch = hx & 1;
  const int k0 = kb * 128;
  const int hk = (hx >> 1) / p.g_split;
  const int split = (hx >> 1) - hk * p.g_split;
  const int b = blockIdx.z;
  const int G = p.Hq / p.Hk / p.g_split;
  const int h_first = hk * (p.Hq / p.Hk) + split * G;

  int first_qt = 0;
  if (p.causal) {
    const long long qmin = static_cast<long long>(k0) - p.causal_off;  // q >= k - off
    first_qt = qmin <= 0 ? 0 : static_cast<int>(qmin / 64);
  }
  const int num_qt_total = (p.Tq + 63) / 64;
  const int nq = max(0, num_qt_total - first_qt);
  QTiles<kMask> first;
  first.map = (kMask && p.mask_blocks)
                  ? p.mask_blocks + b * p.mb_stride[0] + static_cast<int64_t>(h_first) * p.mb_stride[1] + kb
                  : nullptr;
  first.head_stride = p.mb_stride[1];
  first.row_stride = p.nkb;
  first.nq = max(nq, 1);
  first.first_qt = first_qt;
  first.N = G * nq;
  first.lin = 0;
  first.skip_empty();
  const bool any_work = first.valid();

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(v_full, 256);
    mbar_init(dkv_full, 1);
    mbar_init(mma_drain, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dp_full, 1);
    mbar_init(ds_full, 256);
    mbar_init(ds_empty, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
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
    regs_dec<kRegsCtl>();
    if (warp == 0) {
      // ---------------------------------------------------------- TMA producer
      if (lane == 0 && any_work) {
        prefetch_tmap(&p.tm_q);
        prefetch_tmap(&p.tm_do);
        prefetch_tmap(&p.tm_k);
        if (kScore && p.score_pf) prefetch_tmap(&p.tm_score);
        mbar_arrive_expect_tx(kv_full, L::kKT);
#pragma unroll
        for (int c = 0; c < 4; ++c) tma_load_4d(smem + L::kK + c * 16384, &p.tm_k, kv_full, c * 64, k0, hk, b);
        int issued = 0;
        QTiles<kMask> cur = first;
        for (int it = 0; cur.valid(); ++it, cur.advance()) {
          const int qs = it & 1;
          const int h = h_first + cur.g();
          const int q0 = cur.q0();
          if (!mbar_wait(&q_empty[qs], ((it >> 1) & 1) ^ 1, abort_flag)) break;
          mbar_arrive_expect_tx(&q_full[qs], 2 * L::kQT + 512);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tma_load_4d(smem + L::kQ + qs * L::kQT + c * 8192, &p.tm_q, &q_full[qs], c * 64, q0, h, b);
            tma_load_4d(smem + L::kDO + qs * L::kQT + c * 8192, &p.tm_do, &q_full[qs], c * 64, q0, h, b);
          }
          const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0;
          bulk_load(smem + L::kLSE + qs * 256, p.lse + row, 256, &q_full[qs]);
          bulk_load(smem + L::kDelta + qs * 256, p.delta + row, 256, &q_full[qs]);
          if (kScore && p.score_pf) {
            const int hs = p.score_stride[1] ? h : 0, bs = p.score_stride[0] ? b : 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) tma_prefetch_l2_4d(&p.tm_score, k0 + 32 * c, q0, hs, bs);
          }
          issued = it + 1;
        }
        if (*reinterpret_cast<volatile int*>(abort_flag)) {
          mbar_wait_short(kv_full, 0);
          for (int it = max(0, issued - kStages); it < issued; ++it) mbar_wait_short(&q_full[it & 1], (it >> 1) & 1);
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ---------------------------------------------------------- MMA issuer
      // Per tile: dV after P^T, then S^T of the next tile (its P/dS warps start on it
      // while dS^T of this tile is finished), dK after dS^T, then dP^T of the next tile
      // (the P/dS warps read this tile's dP^T before dS^T was complete).
      if (any_work) {
        const uint32_t sK = smem_u32(smem + L::kK);
        const uint32_t sQ = smem_u32(smem + L::kQ);
        const uint32_t sDO = smem_u32(smem + L::kDO);
        const uint32_t sDS = smem_u32(smem + L::kDSb);
        const uint32_t tS = tmem + kColS, tDP = tmem + kColDP, tV = tmem + kColV;
        auto wait = [&](uint64_t* bar, uint32_t parity) {
          return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
        };
        bool ok = wait(kv_full, 0) && wait(v_full, 0) && wait(&q_full[0], 0);
        if (ok) {
          tc_fence_after();
          if (elect_one()) {
            issue_s<kBF16>(tS, sK, sQ);
            tc_commit(s_full);
            issue_dp<kBF16>(tDP, tV, sDO);
            tc_commit(dp_full);
          }
          __syncwarp();
        }
        QTiles<kMask> cur = first;
        for (int it = 0; ok && cur.valid(); ++it) {
          QTiles<kMask> nxt = cur;
          nxt.advance();
          const int qs = it & 1, qn = (it + 1) & 1;
          const uint32_t par = it & 1;
          ok = wait(p_full, par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) issue_dv<kBF16>(tmem + kColDV, tS, sDO + qs * L::kQT + ch * 16384, it > 0);
          __syncwarp();
          if (nxt.valid()) {
            // S^T of the next tile overwrites P^T after dV has read it (MMAs run in
            // issue order).
            ok = wait(&q_full[qn], ((it + 1) >> 1) & 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_s<kBF16>(tS, sK, sQ + qn * L::kQT);
              tc_commit(s_full);
            }
            __syncwarp();
          }
          ok = wait(ds_full, par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_dk<kBF16>(tmem + kColDK, sDS, sQ + qs * L::kQT + ch * 16384, it > 0);
            tc_commit(&q_empty[qs]);
            tc_commit(ds_empty);
            if (nxt.valid()) {
              issue_dp<kBF16>(tDP, tV, sDO + qn * L::kQT);
              tc_commit(dp_full);
            }
          }
          __syncwarp();
          cur = nxt;
        }
        if (elect_one()) {
          if (ok) tc_commit(dkv_full);
          tc_commit(mma_drain);
        }
        __syncwarp();
        wait(mma_drain, 0);
      }
    }
  } else {
    regs_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ P, dS and dK/dV epilogue
    const int wg = (warp - 4) >> 2;  // queries 32*wg .. 32*wg+31 of every tile
    const int r = (warp & 3) * 32 + lane;
    const int k = k0 + r;
    const bool k_valid = k < p.Tk;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int kc = min(k, p.Tk - 1);
    const float* sLSE = reinterpret_cast<const float*>(smem + L::kLSE);
    const float* sDelta = reinterpret_cast<const float*>(smem + L::kDelta);
    bool ok = true;
    if (any_work) {
      // V columns [128 wg, 128 wg + 128) of this key into TMEM (zeros past Tk).
      const uint4* vrow = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.v) + b * p.v_stride[0] +
                                                         static_cast<int64_t>(kc) * p.v_stride[1] +
                                                         hk * p.v_stride[2] + 128 * wg);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t w[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 x = k_valid ? __ldg(vrow + 4 * j + u) : make_uint4(0u, 0u, 0u, 0u);
          w[4 * u] = x.x;
          w[4 * u + 1] = x.y;
          w[4 * u + 2] = x.z;
          w[4 * u + 3] = x.w;
        }
        tmem_st16(tmem + lane_base + kColV + 64 * wg + 16 * j, w);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(v_full);
    }
    QTiles<kMask> cur = first;
    auto load_bits = [&](const QTiles<kMask>& c) {
      const int hh = h_first + c.g();
      const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(p.mask_bits_t + b * p.mbt_stride[0] + hh * p.mbt_stride[1]) +
                             static_cast<int64_t>(c.q0() >> 6) * p.Tk + kc);
      return wg ? v2.y : v2.x;
    };
    uint32_t bits_next = 0u;
    if (kMask && p.mask_bits_t && cur.valid() && cur.state() == 1) bits_next = load_bits(cur);
    for (int it = 0; cur.valid(); ++it) {
      QTiles<kMask> nxt = cur;
      nxt.advance();
      const uint32_t bits_cur = bits_next;
      if (kMask && p.mask_bits_t && nxt.valid() && nxt.state() == 1) bits_next = load_bits(nxt);
      const uint32_t par = it & 1;
      const int qs = it & 1;
      const int h = h_first + cur.g();
      const int q0 = cur.q0();
      const int qb = q0 + 32 * wg;  // this warpgroup's first query
      const bool use_mask = kMask && cur.state() == 1;
      float scv[kScore ? 32 : 1];
      if constexpr (kScore) {
        const float* sc = p.score + b * p.score_stride[0] + h * p.score_stride[1] + kc;
#pragma unroll
        for (int c = 0; c < 32; ++c) scv[c] = __ldg(sc + min(qb + c, p.Tq - 1) * p.score_stride[2]);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, par, abort_flag) &&
                                       mbar_wait(&q_full[qs], (it >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + kColS + 32 * wg;
      const bool need_causal = p.causal && (k0 + 127 > q0 + p.causal_off);
      const bool need_bounds = (q0 + 64 > p.Tq) || (k0 + 128 > p.Tk);
      const bool fast = !use_mask && !kScore && !need_causal && !need_bounds;
      const float* lse = sLSE + qs * 64 + 32 * wg;
      // Keep flags of this warpgroup's 32 queries for this key (bit c = query qb + c).
      uint32_t kw = 0xffffffffu;
      if (!fast) {
        if (use_mask) {
          if (p.mask_bits_t) {
            kw = bits_cur;
          } else {
            const uint8_t* mask_col = p.mask + b * p.mask_stride[0] + h * p.mask_stride[1] + kc;
#pragma unroll 8
            for (int c = 0; c < 32; ++c) {
              const int64_t qc = min(qb + c, p.Tq - 1);
              if (__ldg(mask_col + qc * p.mask_stride[2]) == 0) kw &= ~(1u << c);
            }
          }
        }
        if (need_bounds || need_causal) {
          uint32_t lim = k_valid ? low_bits(p.Tq - qb) : 0u;
          if (need_causal) lim &= ~low_bits(k - p.causal_off - qb);  // keep q >= k - off
          kw &= lim;
        }
      }
      float pv[32];
      {
        uint32_t sr[32];
        tmem_ld32(tS, sr);
        tmem_wait_ld();
        if (fast) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 l = reinterpret_cast<const float4*>(lse)[i];
            pv[4 * i] = ex2(fmaf(__uint_as_float(sr[4 * i]), p.scale_log2, -l.x));
            pv[4 * i + 1] = ex2(fmaf(__uint_as_float(sr[4 * i + 1]), p.scale_log2, -l.y));
            pv[4 * i + 2] = ex2(fmaf(__uint_as_float(sr[4 * i + 2]), p.scale_log2, -l.z));
            pv[4 * i + 3] = ex2(fmaf(__uint_as_float(sr[4 * i + 3]), p.scale_log2, -l.w));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(sr[i]);
            if constexpr (kScore) x += scv[i];
            const float e = ex2(fmaf(x, p.scale_log2, -lse[i]));
            pv[i] = ((kw >> i) & 1u) ? e : 0.f;
          }
        }
        // P^T (16-bit) of these 32 queries over the first 16 of this warpgroup's 32 S
        // columns (all of which this thread has read).
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<kBF16>(pv[2 * i], pv[2 * i + 1]);
        tmem_st16(tS, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);

      ok = __all_sync(0xffffffffu, mbar_wait(dp_full, par, abort_flag) && mbar_wait(ds_empty, par ^ 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      {
        const float4* d4 = reinterpret_cast<const float4*>(sDelta + qs * 64 + 32 * wg);
        uint8_t* ds_row = smem + L::kDSb + r * 128;
        uint32_t sr[32];
        tmem_ld32(tmem + lane_base + kColDP + 32 * wg, sr);
        tmem_wait_ld();
        uint32_t dsk[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = d4[i];
          dsk[2 * i] = pack2<kBF16>(pv[4 * i] * (__uint_as_float(sr[4 * i]) - t.x),
                                    pv[4 * i + 1] * (__uint_as_float(sr[4 * i + 1]) - t.y));
          dsk[2 * i + 1] = pack2<kBF16>(pv[4 * i + 2] * (__uint_as_float(sr[4 * i + 2]) - t.z),
                                        pv[4 * i + 3] * (__uint_as_float(sr[4 * i + 3]) - t.w));
        }
        // Row r of the dS^T tile: 128 B in 8 chunks of 16 B, 128-B swizzled (chunk ^ (row % 8));
        // this warpgroup's queries are chunks 4 wg .. 4 wg + 3.
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4*>(ds_row + (((4 * wg + cc) ^ (r & 7)) << 4)) =
              make_uint4(dsk[4 * cc], dsk[4 * cc + 1], dsk[4 * cc + 2], dsk[4 * cc + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      cur = nxt;
    }

    // Epilogue: warpgroup 0 writes this CTA's half of dV, warpgroup 1 its half of dK
    // (zeros when no query interacts with this key tile).
    const int col0 = 128 * ch;
    if (p.g_split > 1) {
      float* part = (wg == 0 ? p.dv_part : p.dk_part) + split * p.part_stride +
                    ((static_cast<int64_t>(b) * p.Tk + kc) * p.Hk + hk) * 256 + col0;
      if (any_work && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
        tc_fence_after();
        const uint32_t tA = tmem + lane_base + (wg == 0 ? kColDV : kColDK);
        const float out_scale = wg == 0 ? 1.f : p.scale;  // dK = scale * dS^T Q
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tA + 32 * c, v);
          tmem_wait_ld();
          if (k_valid) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<float4*>(part + 32 * c + 4 * u) =
                  make_float4(__uint_as_float(v[4 * u]) * out_scale, __uint_as_float(v[4 * u + 1]) * out_scale,
                              __uint_as_float(v[4 * u + 2]) * out_scale, __uint_as_float(v[4 * u + 3]) * out_scale);
          }
        }
      } else if (k_valid && !any_work) {
#pragma unroll
        for (int u = 0; u < 32; ++u) reinterpret_cast<float4*>(part)[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      tc_fence_before();
    } else {
      uint16_t* dst_row = nullptr;
      if (k_valid) {
        const int64_t* st3 = wg == 0 ? p.dv_stride : p.dk_stride;
        dst_row = reinterpret_cast<uint16_t*>(wg == 0 ? p.dv : p.dk) + b * st3[0] +
                  static_cast<int64_t>(k) * st3[1] + hk * st3[2] + col0;
      }
      if (any_work && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
        tc_fence_after();
        const uint32_t tA = tmem + lane_base + (wg == 0 ? kColDV : kColDK);
        const float out_scale = wg == 0 ? 1.f : p.scale;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tA + 32 * c, v);
          tmem_wait_ld();
          if (k_valid) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack2<kBF16>(__uint_as_float(v[2 * i]) * out_scale, __uint_as_float(v[2 * i + 1]) * out_scale);
            uint4* dst = reinterpret_cast<uint4*>(dst_row + 32 * c);
#pragma unroll
            for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
          }
        }
      } else if (k_valid && !any_work) {
#pragma unroll
        for (int u = 0; u < 16; ++u) reinterpret_cast<uint4*>(dst_row)[u] = make_uint4(0, 0, 0, 0);
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(abort_flag)) atomicOr(p.status, FA4D_DEV_TIMEOUT_BWD);
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kBF16, bool kMask, bool kScore>
cudaError_t launch_t(const BwdParams& p, cudaStream_t s) {
  auto kern = bwd256_kernel<kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout::kAlloc);
  if (e != cudaSuccess) return e;
  const unsigned nkb = (p.Tk + 127) / 128, nh = 2 * p.Hk * p.g_split;
  const dim3 grid = p.kb_fastest ? dim3(nkb, nh, p.B) : dim3(nh, nkb, p.B);
  kern<<<grid, kThreads, Layout::kAlloc, s>>>(p);
  return cudaGetLastError();
}

template <bool kBF16>
cudaError_t launch_d(const BwdParams& p, bool m, bool sc, cudaStream_t s) {
  if (m && sc) return launch_t<kBF16, true, true>(p, s);
  if (m) return launch_t<kBF16, true, false>(p, s);
  if (sc) return launch_t<kBF16, false, true>(p, s);
  return launch_t<kBF16, false, false>(p, s);
}

}  // namespace

cudaError_t launch_bwd256(const BwdParams& p, bool bf16, bool has_mask, bool has_score, cudaStream_t s) {
  return bf16 ? launch_d<true>(p, has_mask, has_score, s) : launch_d<false>(p, has_mask, has_score, s);
}

}  // namespace fa4d
