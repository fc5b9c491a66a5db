// fa4d_bwd.cu — FlashAttention-2 backward for sm_100a with an optional 4D mask/score.
//
// Math follows the reference backward (python/fa2.py:181-302): P is recomputed from
// the saved log2-domain LSE, dV = P^T dO, dP = dO V^T, dS = P (dP - Delta) scale,
// dK = dS^T Q, dQ = dS K, with Delta = rowsum(O * dO) (python/fa2.py:142-179).
// The kernels carry dS without the factor `scale` and apply it once to the dK
// tile in its epilogue and to dQ when the accumulator is converted.
// Unlike the reference, one CTA owns a 128-key tile of one KV head and loops over
// every query head of its GQA group, so dK/dV are summed in tensor memory and
// stored once in the input dtype (the reference sums the group with fp32 atomics,
// python/fa2.py:299-302, or with a bf16 host-side sum, python/fa2.py:548-549).
// Each 64-query dQ tile is added to an fp32 accumulator straight from registers
// (red.global.add.f32, one contiguous run of D columns per warp and query).
//
// CTA = 128 keys x one (batch, KV head); 512 threads:
//   warp 0       TMA producer (K/V once; Q, dO, LSE, Delta per 64-row query tile,
//                3-stage ring)
//   warps 1, 3   tcgen05.mma issuers, two query tiles ahead of the P/dS warpgroups:
//                warp 1 issues S^T and dV, warp 3 issues dP^T, dK and dQ^T
//   warp 2       TMEM allocator
//   warps 4-7    P / dS of the even query tiles (one thread per key row), then dV out
//   warps 8-11   P / dS of the odd query tiles, then dK out
//   warps 12-15  dQ drain: TMEM -> registers -> reduce-add into the global accumulator
// The two P/dS warpgroups ping-pong, so the hand-off latency of one tile (MMA
// completion -> P -> MMA -> dS -> MMA) overlaps the other tile's work.
// TMEM (512 columns): S^T x2 [0,128), X x2 [128,256) (a tile's dP^T, later its
// dQ^T), dV [256,256+D), dK [256+D,256+2D).  All MMAs are kind::f16, fp32 accumulate.
#include <algorithm>
#include <cfloat>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kBwdThreads = 512;
// Depth of the Q / dO / LSE / Delta ring: the load for query tile it+Q-1 is issued
// while tile it is still being consumed, which hides its L2/HBM latency.  The variants
// without a mask or score take 4 stages (the Sᵀ issuer waited on the third stage's load
// for ~1200 clocks per tile; config 2 backward main -5%, causal -3%), the others 3 (4
// measured 2-3% slower there).  At 4 stages with D = 128 the layout leaves no room for
// the 1 KB alignment slack: the kernel then relies on the dynamic shared memory base
// being 1024-byte aligned (as it is on this hardware) and checks it.
template <bool kMask, bool kScore>
constexpr int kQStagesFor = (kMask || kScore) ? 3 : 4;
// Register split (launch: 512 threads x 128 = 65536): producer/MMA warpgroup 88,
// P/dS warpgroups 160, dQ drain 96 -> 128*88 + 256*160 + 128*96 = 64512 (no variant
// spills; 152 / 112 left the P/dS code 16-32 bytes of spills).
constexpr uint32_t kRegsLaunch = 128, kRegsCtl = 88, kRegsSoftmax = 160, kRegsDrain = 96;
static_assert(128 * kRegsCtl + 256 * kRegsSoftmax + 128 * kRegsDrain <= kBwdThreads * kRegsLaunch,
              "register split exceeds the launch allocation");

template <int D, int kQStages>
struct BwdLayout {
  static constexpr int kKV = 128 * D * 2;   // K or V tile (128 keys)
  static constexpr int kQT = 64 * D * 2;    // Q or dO tile (64 queries)
  static constexpr int kDS = 128 * 64 * 2;  // dS^T tile (128 keys x 64 queries, 16-bit)
  static constexpr int kK = 0;
  static constexpr int kV = kK + kKV;
  static constexpr int kQ = kV + kKV;                 // kQStages stages
  static constexpr int kDO = kQ + kQStages * kQT;     // kQStages stages
  static constexpr int kDSb = kDO + kQStages * kQT;   // 2 buffers
  static constexpr int kLSE = kDSb + 2 * kDS;            // kQStages x 64 floats
  static constexpr int kDelta = kLSE + kQStages * 256;   // kQStages x 64 floats
  static constexpr int kBar = kDelta + kQStages * 256;
  static constexpr int kNumBars = 18 + 2 * kQStages;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  // Slack to align the base to 1024 B when it fits; without it the base must already be.
  static constexpr int kSlack = kBytes + 1024 <= 232448 ? 1024 : 0;
  static constexpr int kAlloc = kBytes + kSlack;
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

// S^T = K Q^T (or dP^T = V dO^T): M=128 keys, N=64 queries, K=D; both K-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_kt(uint32_t tD, uint32_t sA, uint32_t sB) {
  constexpr uint32_t idesc = make_idesc(128, 64, kBF16, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t offa = static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 32);
    const uint32_t offb = static_cast<uint32_t>((kk >> 2) * 8192 + (kk & 3) * 32);
    mma_ss(tD, sw128_desc(sA + offa, 16, 1024), sw128_desc(sB + offb, 16, 1024), idesc, kk > 0 ? 1u : 0u);
  }
}

// dV += P^T dO : M=128 keys, N=D, K=64 queries; P^T from TMEM, dO MN-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_dv(uint32_t tD, uint32_t tP, uint32_t sDO, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, D, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tD, tP + kk * 8, sw128_desc(sDO + kk * 2048, 8192, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
}

// dK += dS^T Q : M=128 keys, N=D, K=64 queries; dS^T from TMEM (16-bit pairs written
// over the tile's dP^T columns), Q MN-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_dk(uint32_t tD, uint32_t tDS, uint32_t sQ, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, D, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tD, tDS + kk * 8, sw128_desc(sQ + kk * 2048, 8192, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
}

// dQ^T = K^T dS^T : M=D, N=64 queries, K=128 keys; K MN-major, dS^T MN-major.
template <int D, bool kBF16>
__device__ __forceinline__ void issue_dq(uint32_t tD, uint32_t sK, uint32_t sDS) {
  constexpr uint32_t idesc = make_idesc(D, 64, kBF16, true, true);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    mma_ss(tD, sw128_desc(sK + kk * 2048, 16384, 1024), sw128_desc(sDS + kk * 2048, 8192, 1024), idesc,
           kk > 0 ? 1u : 0u);
}

template <int D, bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_kernel(const __grid_constant__ BwdParams p) {
  constexpr int kQStages = kQStagesFor<kMask, kScore>;
  using L = BwdLayout<D, kQStages>;
  extern __shared__ uint8_t smem_raw[];
  if (L::kSlack == 0 && (smem_u32(smem_raw) & 1023u) != 0u) {
    // No room to realign: report and leave before touching anything (uniform exit).
    if (threadIdx.x == 0) atomicOr(p.status, FA4D_DEV_SMEM_ALIGN);
    return;
  }
  // 1024-B aligned base, derived by pointer arithmetic on the shared array so the
  // compiler keeps the shared address space (LDS/STS rather than generic loads/stores).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* dkv_full = bars + 1;   // dV and dK complete (one arrival per MMA issuer)
  uint64_t* mma_drain = bars + 2;  // MMAs of issuer warp 1 complete
  uint64_t* mma_drain_b = bars + 3;  // MMAs of issuer warp 3 complete
  // Per tile parity (tile it uses buffer it & 1; each is owned by one P/dS warpgroup).
  uint64_t* s_full = bars + 4;     // [2] S^T of the tile is in TMEM
  uint64_t* p_full = bars + 6;     // [2] P^T written to TMEM (128 arrivals)
  uint64_t* dp_full = bars + 8;    // [2] dP^T of the tile is in TMEM
  uint64_t* ds_full = bars + 10;   // [2] dS^T written to smem (128 arrivals)
  uint64_t* ds_empty = bars + 12;  // [2] dS^T smem buffer free again
  uint64_t* dq_full = bars + 14;   // [2] dQ^T of the tile is in TMEM
  uint64_t* dq_empty = bars + 16;  // [2] drain has read dQ^T (128 arrivals)
  uint64_t* q_full = bars + 18;    // [kQStages]
  uint64_t* q_empty = bars + 18 + kQStages;  // [kQStages] (2 arrivals: the last dV and the last dK reading the stage)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (Hk x group split, key tiles, B), dispatched x-fastest: all heads of one key
  // tile go out together, and under a causal mask the first key tiles (which see the
  // most queries) go first.  KV head x split: the CTA takes query heads
  // [h_first, h_first + G) of its KV head's group (G = Hq / Hk / g_split).
  // With p.kb_fastest the grid is (key tiles, KV head x split, B) instead; with
  // p.kb_order (a prepared block map) it is (KV head x split, key-tile rank x B), the
  // batch fastest in y and the key tile of each rank taken from the prepared order,
  // which lists the key tiles with the most live query blocks first.
  const int hx = p.kb_fastest ? blockIdx.y : blockIdx.x;
  const int hk = hx / p.g_split;
  const int split = hx - hk * p.g_split;
  const int b = p.kb_order ? static_cast<int>(blockIdx.y) % p.B : static_cast<int>(blockIdx.z);
  const int G = p.Hq / p.Hk / p.g_split;
  const int h_first = hk * (p.Hq / p.Hk) + split * G;
  const int kb = p.kb_order ? __ldg(p.kb_order + b * p.ko_stride[0] + static_cast<int64_t>(h_first) * p.ko_stride[1] +
                                    static_cast<int>(blockIdx.y) / p.B)
                            : (p.kb_fastest ? blockIdx.x : blockIdx.y);
  const int k0 = kb * 128;

  // Query tiles this key tile interacts with.
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
    mbar_init(dkv_full, 2);
    mbar_init(mma_drain, 1);
    mbar_init(mma_drain_b, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&dp_full[i], 1);
      mbar_init(&ds_full[i], 128);
      mbar_init(&ds_empty[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 128);
    }
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);
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
  // S^T x2, then X x2 (dP^T of a tile, later overwritten by its dQ^T), dV, dK.
  constexpr uint32_t kColS = 0, kColX = 128, kColDV = 256, kColDK = 256 + D;

  if (warp < 4) {
    // Each role starts with its register budget so the compiler allocates that
    // role's code under it.
    regs_dec<kRegsCtl>();
    if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && any_work) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_do);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      if (kScore && p.score_pf) prefetch_tmap(&p.tm_score);
      mbar_arrive_expect_tx(kv_full, 2 * L::kKV);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(smem + L::kK + c * 16384, &p.tm_k, kv_full, c * 64, k0, hk, b);
        tma_load_4d(smem + L::kV + c * 16384, &p.tm_v, kv_full, c * 64, k0, hk, b);
      }
      int issued = 0;
      QTiles<kMask> cur = first;
      for (int it = 0; cur.valid(); ++it, cur.advance()) {
        const int qs = it % kQStages;
        const int h = h_first + cur.g();
        const int q0 = cur.q0();
        if (!mbar_wait(&q_empty[qs], ((it / kQStages) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qs], 2 * L::kQT + 512);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_4d(smem + L::kQ + qs * L::kQT + c * 8192, &p.tm_q, &q_full[qs], c * 64, q0, h, b);
          tma_load_4d(smem + L::kDO + qs * L::kQT + c * 8192, &p.tm_do, &q_full[qs], c * 64, q0, h, b);
        }
        const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0;
        bulk_load(smem + L::kLSE + qs * 256, p.lse + row, 256, &q_full[qs]);
        bulk_load(smem + L::kDelta + qs * 256, p.delta + row, 256, &q_full[qs]);
        if (kScore && p.score_pf) {
          // The P/dS warpgroups read this tile's score column by column about two
          // tiles from now; have it in L2 by then.
          const int hs = p.score_stride[1] ? h : 0, bs = p.score_stride[0] ? b : 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) tma_prefetch_l2_4d(&p.tm_score, k0 + 32 * c, q0, hs, bs);
        }
        issued = it + 1;
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        mbar_wait_short(kv_full, 0);
        for (int it = max(0, issued - kQStages); it < issued; ++it)
          mbar_wait_short(&q_full[it % kQStages], (it / kQStages) & 1);
      }
    }
    __syncwarp();
    } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------ MMA issuers
    // One tcgen05.mma issue occupies the issuing thread for about 45 SM clocks, longer
    // than an N = 64 product runs, so one issuing thread cannot keep the tensor pipe
    // busy with this tile's 32 instructions; two threads can.  Warp 1 issues S^T and dV
    // (it alone writes the S^T buffers and the dV accumulator), warp 3 issues dP^T, dK
    // and dQ^T (the X buffers, the dK accumulator, the dS^T shared buffers), so every
    // TMEM region is written and later reused by one issuer, whose own issue order
    // keeps its reads before its overwrites.  Each runs two tiles ahead of the P/dS
    // warpgroups; the whole warp runs the loop (waits included) and one elected lane
    // issues each group of MMAs and its commits.
    if (any_work) {
      const bool is_a = warp == 1;
      const uint32_t sK = smem_u32(smem + L::kK);
      const uint32_t sV = smem_u32(smem + L::kV);
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sDO = smem_u32(smem + L::kDO);
      const uint32_t sDS = smem_u32(smem + L::kDSb);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      bool ok = wait(kv_full, 0);
      // `ahead` walks the pair list two entries in front of `it`; n_known counts the
      // pairs whose first product (S^T, or dP^T) has been issued.
      QTiles<kMask> ahead = first;
      int n_known = 0;
      for (int j = 0; ok && j < 2 && ahead.valid(); ++j, ahead.advance(), ++n_known) {
        ok = wait(&q_full[j], 0);
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          if (is_a) {
            issue_kt<D, kBF16>(tmem + kColS + 64 * j, sK, sQ + j * L::kQT);
            tc_commit(&s_full[j]);
          } else {
            issue_kt<D, kBF16>(tmem + kColX + 64 * j, sV, sDO + j * L::kQT);
            tc_commit(&dp_full[j]);
          }
        }
        __syncwarp();
      }
      for (int it = 0; ok && it < n_known; ++it) {
        const int st = it & 1;
        const uint32_t par = (it >> 1) & 1;
        const int qs = it % kQStages;
        if (is_a) {
          ok = wait(&p_full[st], par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_dv<D, kBF16>(tmem + kColDV, tmem + kColS + 64 * st, sDO + qs * L::kQT, it > 0);
            tc_commit(&q_empty[qs]);
          }
          __syncwarp();
        } else {
          ok = wait(&ds_full[st], par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_dk<D, kBF16>(tmem + kColDK, tmem + kColX + 64 * st, sQ + qs * L::kQT, it > 0);
            tc_commit(&q_empty[qs]);
            if (!p.skip_dq) {
              // dQ^T overwrites this tile's dP^T (read before ds_full).
              issue_dq<D, kBF16>(tmem + kColX + 64 * st, sK, sDS + st * L::kDS);
              tc_commit(&dq_full[st]);
            }
            tc_commit(&ds_empty[st]);
          }
          __syncwarp();
        }
        if (ahead.valid()) {
          const int jn = it + 2;
          ahead.advance();
          ++n_known;
          const int qn = jn % kQStages;
          ok = wait(&q_full[qn], (jn / kQStages) & 1);
          if (!ok) break;
          // Warp 3: dP^T of tile it+2 reuses X[st] once the drain has read dQ^T of tile
          // it (at once when dQ is left to the deterministic kernel: ds_full ended the
          // reads).  Warp 1: S^T of tile it+2 reuses S[st], whose P^T the dV above read.
          if (!is_a && !p.skip_dq) ok = wait(&dq_empty[st], par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            if (is_a) {
              issue_kt<D, kBF16>(tmem + kColS + 64 * st, sK, sQ + qn * L::kQT);
              tc_commit(&s_full[st]);
            } else {
              issue_kt<D, kBF16>(tmem + kColX + 64 * st, sV, sDO + qn * L::kQT);
              tc_commit(&dp_full[st]);
            }
          }
          __syncwarp();
        }
      }
      uint64_t* drain_bar = is_a ? mma_drain : mma_drain_b;
      if (elect_one()) {
        if (ok) tc_commit(dkv_full);
        tc_commit(drain_bar);
      }
      __syncwarp();
      wait(drain_bar, 0);
    }
    }
  } else if (warp < 12) {
    regs_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ P, dS and dK/dV epilogue
    const int wg = (warp - 4) >> 2;  // this warpgroup takes tiles it with it % 2 == wg
    const int r = (warp & 3) * 32 + lane;
    const int k = k0 + r;
    const bool k_valid = k < p.Tk;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float* sLSE = reinterpret_cast<const float*>(smem + L::kLSE);
    const float* sDelta = reinterpret_cast<const float*>(smem + L::kDelta);
    // Mask/score are read at clamped (always in-bounds) addresses and applied with
    // selects, so lanes never branch apart before the warp-collective TMEM ops.
    const int kc = min(k, p.Tk - 1);
    bool ok = true;
    QTiles<kMask> cur = first;
    if (wg == 1) cur.advance();
    // Prepared mask bits of this warpgroup's next PARTIAL tile, loaded one tile ahead.
    auto load_bits = [&](const QTiles<kMask>& c) {
      const int hh = h_first + c.g();
      return __ldg(reinterpret_cast<const uint2*>(p.mask_bits_t + b * p.mbt_stride[0] + hh * p.mbt_stride[1]) +
                   static_cast<int64_t>(c.q0() >> 6) * p.Tk + kc);
    };
    uint2 bits_next = make_uint2(0u, 0u);
    if (kMask && p.mask_bits_t && cur.valid() && cur.state() == 1) bits_next = load_bits(cur);
    for (int it = wg; cur.valid(); it += 2) {
      QTiles<kMask> nxt = cur;
      nxt.advance();
      nxt.advance();
      const uint2 bits_cur = bits_next;
      if (kMask && p.mask_bits_t && nxt.valid() && nxt.state() == 1) bits_next = load_bits(nxt);
      const int st = wg;
      const uint32_t par = (it >> 1) & 1;
      const int qs = it % kQStages;
      const int h = h_first + cur.g();
      const int q0 = cur.q0();
      const bool use_mask = kMask && cur.state() == 1;  // warp-uniform
      // This key's score for the tile's 64 queries, requested before the wait for S so
      // the loads (L2 hits: the producer prefetched the tile) overlap it.
      float scv[kScore ? 64 : 1];
      if constexpr (kScore) {
        const float* sc = p.score + b * p.score_stride[0] + h * p.score_stride[1] + kc;
#pragma unroll
        for (int c = 0; c < 64; ++c) scv[c] = __ldg(sc + min(q0 + c, p.Tq - 1) * p.score_stride[2]);
      }
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[st], par, abort_flag) &&
                                       mbar_wait(&q_full[qs], (it / kQStages) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + kColS + 64 * st;
      const bool need_causal = p.causal && (k0 + 127 > q0 + p.causal_off);
      const bool need_bounds = (q0 + 64 > p.Tq) || (k0 + 128 > p.Tk);
      const bool fast = !use_mask && !kScore && !need_causal && !need_bounds;  // warp-uniform
      const float4* l4 = reinterpret_cast<const float4*>(sLSE + qs * 64);
      const uint8_t* mask_col = nullptr;
      if (kMask) mask_col = p.mask + b * p.mask_stride[0] + h * p.mask_stride[1] + kc;
      // Keep flags of the tile's 64 queries for this key (bit c = query q0 + c): mask,
      // query bound, key bound and causal limit, applied as whole-word masks.
      uint32_t kw[2] = {0xffffffffu, 0xffffffffu};
      if (!fast) {
        if (use_mask) {
          if (p.mask_bits_t) {
            kw[0] = bits_cur.x;
            kw[1] = bits_cur.y;
          } else {
#pragma unroll 8
            for (int c = 0; c < 64; ++c) {
              const int64_t qc = min(q0 + c, p.Tq - 1);
              if (__ldg(mask_col + qc * p.mask_stride[2]) == 0) kw[c >> 5] &= ~(1u << (c & 31));
            }
          }
        }
        if (need_bounds || need_causal) {
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int base = q0 + 32 * w;
            uint32_t lim = k_valid ? low_bits(p.Tq - base) : 0u;
            if (need_causal) lim &= ~low_bits(k - p.causal_off - base);  // keep q >= k - off
            kw[w] &= lim;
          }
        }
      }
      float pv[64];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sr[32];
        tmem_ld32(tS + 32 * half, sr);
        tmem_wait_ld();
        if (fast) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 l = l4[8 * half + i];
            const int c = 32 * half + 4 * i;
            pv[c] = ex2(fmaf(__uint_as_float(sr[4 * i]), p.scale_log2, -l.x));
            pv[c + 1] = ex2(fmaf(__uint_as_float(sr[4 * i + 1]), p.scale_log2, -l.y));
            pv[c + 2] = ex2(fmaf(__uint_as_float(sr[4 * i + 2]), p.scale_log2, -l.z));
            pv[c + 3] = ex2(fmaf(__uint_as_float(sr[4 * i + 3]), p.scale_log2, -l.w));
          }
        } else {
          const uint32_t w = kw[half];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = 32 * half + i;
            float x = __uint_as_float(sr[i]);
            if constexpr (kScore) x += scv[c];
            const float e = ex2(fmaf(x, p.scale_log2, -sLSE[qs * 64 + c]));
            pv[c] = ((w >> i) & 1u) ? e : 0.f;
          }
        }
        // P^T (16-bit) for these 32 queries goes to columns 16*half .. 16*half+15,
        // which hold S^T values this thread has already read.
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<kBF16>(pv[32 * half + 2 * i], pv[32 * half + 2 * i + 1]);
        tmem_st16(tS + 16 * half, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[st]);

      ok = __all_sync(0xffffffffu, mbar_wait(&dp_full[st], par, abort_flag) &&
                                       mbar_wait(&ds_empty[st], par ^ 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const float4* d4 = reinterpret_cast<const float4*>(sDelta + qs * 64);
      uint8_t* ds_row = smem + L::kDSb + st * L::kDS + r * 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sr[32];
        tmem_ld32(tmem + lane_base + kColX + 64 * st + 32 * half, sr);
        tmem_wait_ld();
        // dS without the softmax scale: dK and dQ are scaled once at their outputs.
        uint32_t dsk[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = d4[8 * half + i];
          const int c = 32 * half + 4 * i;
          dsk[2 * i] = pack2<kBF16>(pv[c] * (__uint_as_float(sr[4 * i]) - t.x),
                                    pv[c + 1] * (__uint_as_float(sr[4 * i + 1]) - t.y));
          dsk[2 * i + 1] = pack2<kBF16>(pv[c + 2] * (__uint_as_float(sr[4 * i + 2]) - t.z),
                                        pv[c + 3] * (__uint_as_float(sr[4 * i + 3]) - t.w));
        }
        // Row r of the dS^T tile: 128 B in 8 chunks of 16 B, 128-B swizzled (chunk ^ (row % 8)),
        // the B operand of dQ^T; the same 16-bit pairs go to TMEM columns 16*half ..
        // 16*half+15 of X (dP^T values this thread has read), the A operand of dK.
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4*>(ds_row + (((4 * half + cc) ^ (r & 7)) << 4)) =
              make_uint4(dsk[4 * cc], dsk[4 * cc + 1], dsk[4 * cc + 2], dsk[4 * cc + 3]);
        tmem_st16(tmem + lane_base + kColX + 64 * st + 16 * half, dsk);
      }
      tmem_wait_st();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&ds_full[st]);
      cur = nxt;
    }

    // Epilogue: warpgroup 0 writes dV, warpgroup 1 writes dK (zeros when no query
    // interacts with this key tile).  With a split group each CTA writes its partial
    // sums (fp32) into its own slice; dkv_convert_kernel adds the slices in order.
    if (p.g_split > 1) {
      float* part = (wg == 0 ? p.dv_part : p.dk_part) + split * p.part_stride +
                    ((static_cast<int64_t>(b) * p.Tk + kc) * p.Hk + hk) * D;
      if (any_work && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
        tc_fence_after();
        const uint32_t tA = tmem + lane_base + (wg == 0 ? kColDV : kColDK);
        const float out_scale = wg == 0 ? 1.f : p.scale;  // dK = scale * dS^T Q
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
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
        for (int u = 0; u < D / 4; ++u) reinterpret_cast<float4*>(part)[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      tc_fence_before();
    } else {
    uint16_t* dst_row = nullptr;
    if (k_valid) {
      const int64_t* st3 = wg == 0 ? p.dv_stride : p.dk_stride;
      dst_row = reinterpret_cast<uint16_t*>(wg == 0 ? p.dv : p.dk) + b * st3[0] + static_cast<int64_t>(k) * st3[1] +
                hk * st3[2];
    }
    if (any_work && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
      tc_fence_after();
      const uint32_t tA = tmem + lane_base + (wg == 0 ? kColDV : kColDK);
      const float out_scale = wg == 0 ? 1.f : p.scale;  // dK = scale * dS^T Q
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tA + 32 * c, v);
        tmem_wait_ld();
        if (k_valid && 32 * c < p.d_out) {
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
      for (int u = 0; u < D / 8; ++u)
        if (8 * u < p.d_out) reinterpret_cast<uint4*>(dst_row)[u] = make_uint4(0, 0, 0, 0);
    }
    tc_fence_before();
    }
  } else {
    regs_dec<kRegsDrain>();
    // ------------------------------------------------------------ dQ drain
    const int wq = warp & 3;
    // M = D accumulator layout: D=128 uses all 128 lanes; D=64 (M=64) puts rows
    // 16*wq .. 16*wq+15 in lanes 0-15 of each 32-lane quadrant.
    const int d = (D == 128) ? (wq * 32 + lane) : (wq * 16 + lane);
    const bool d_valid = (D == 128) || (lane < 16);
    QTiles<kMask> cur = first;
    for (int it = 0; !p.skip_dq && cur.valid(); ++it, cur.advance()) {
      const int st = it & 1;
      const int h = h_first + cur.g();
      const int q0 = cur.q0();
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&dq_full[st], (it >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tDQ = tmem + (static_cast<uint32_t>(wq * 32) << 16) + kColX + 64 * st;
      uint32_t v[64];
      tmem_ld32(tDQ, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(tDQ + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&dq_empty[st]);
      // Rows q0..q0+63 of head h are contiguous in the [B, Hq, Tq_pad, D] accumulator
      // (rows past Tq land in the padding and are never read); for each query the warp's
      // lanes add one contiguous run of D columns.
      if (d_valid) {
        float* dst = p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0) * D + d;
#pragma unroll
        for (int c = 0; c < 64; ++c) red_add_f32(dst + c * D, __uint_as_float(v[c]));
      }
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

// Delta[b, h, t] = sum over the d_out columns of O * dO (0 for padding rows t >= Tq)
// and zeroing of the dQ accumulator rows (b, h, t < Tq), layout [B, Hq, lse_ld, D]
// with D the compute width.  One block per (b, t); each thread takes 8 columns of one
// head (one 16-byte load of O and of dO) and the D / 8 threads of a head reduce the
// row with shuffles.
template <int D, bool kBF16>
__global__ void __launch_bounds__(1024) bwd_prep_kernel(const PrepParams p) {
  constexpr int kTPR = D / 8;  // threads per head row
  const int b = blockIdx.x / p.lse_ld;
  const int t = blockIdx.x - b * p.lse_ld;
  const int total = p.Hq * kTPR;
  const bool row_live = t < p.Tq;
  // Uniform trip count for the whole block, so every lane reaches the shuffles.
  for (int c0 = 0; c0 < total; c0 += blockDim.x) {
    const int c = c0 + static_cast<int>(threadIdx.x);
    const bool live = c < total;
    const int h = c / kTPR, part = c % kTPR;
    float acc = 0.f;
    if (live && row_live) {
      if (8 * part < p.d_out) {
        const uint4 ov = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.o) + b * p.o_stride[0] +
                                                         static_cast<int64_t>(t) * p.o_stride[1] + h * p.o_stride[2] +
                                                         8 * part);
        const uint4 gv = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const uint16_t*>(p.dout) + b * p.do_stride[0] + static_cast<int64_t>(t) * p.do_stride[1] +
            h * p.do_stride[2] + 8 * part);
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 o2 = unpack2<kBF16>(ow[i]), g2 = unpack2<kBF16>(gw[i]);
          acc += o2.x * g2.x + o2.y * g2.y;
        }
      }
      if (p.dq_acc) {  // null in deterministic mode (dQ is not accumulated)
        float4* dq = reinterpret_cast<float4*>(p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + t) * D +
                                               8 * part);
        dq[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        dq[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int off = kTPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (live && part == 0) p.delta[(static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + t] = acc;
  }
}

// dK, dV (input dtype, caller strides) = sum over the split slices [n_split][B, Tk, Hk,
// D] of the split-group backward's fp32 partials (dK already scaled), added in slice
// order so the result does not depend on scheduling.  One block per (b, t) row and
// tensor (blockIdx.y: 0 dK, 1 dV); each thread sums 8 columns of one head.
template <bool kBF16>
__global__ void __launch_bounds__(1024) dkv_convert_kernel(const DkvConvertParams p) {
  const int per_row = p.d_out / 8;
  const int b = blockIdx.x / p.Tk;
  const int t = blockIdx.x - b * p.Tk;
  const bool is_v = blockIdx.y != 0;
  const float* base = (is_v ? p.dv_part : p.dk_part) + (static_cast<int64_t>(b) * p.Tk + t) * p.Hk * p.D;
  const int64_t* st = is_v ? p.dv_stride : p.dk_stride;
  uint16_t* out = reinterpret_cast<uint16_t*>(is_v ? p.dv : p.dk) + b * st[0] + static_cast<int64_t>(t) * st[1];
  for (int c = static_cast<int>(threadIdx.x); c < p.Hk * per_row; c += blockDim.x) {
    const int h = c / per_row, d8 = c - h * per_row;
    const float* src = base + h * p.D + d8 * 8;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), e = a;
    for (int sidx = 0; sidx < p.n_split; ++sidx) {
      const float4* s4 = reinterpret_cast<const float4*>(src + sidx * p.part_stride);
      const float4 x = s4[0], y = s4[1];
      a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
      e.x += y.x; e.y += y.y; e.z += y.z; e.w += y.w;
    }
    *reinterpret_cast<uint4*>(out + h * st[2] + d8 * 8) =
        make_uint4(pack2<kBF16>(a.x, a.y), pack2<kBF16>(a.z, a.w), pack2<kBF16>(e.x, e.y), pack2<kBF16>(e.z, e.w));
  }
}

// dQ (input dtype, caller strides) = scale * dq_acc [B, Hq, lse_ld, D] over the d_out
// columns.  One block per 32 rows of one (b, h), so each block reads one contiguous
// 32 x D run of the accumulator; each thread converts 8 columns of a row at a time.
template <bool kBF16>
__global__ void __launch_bounds__(256) dq_convert_kernel(const ConvertParams p) {
  const int per_row = p.d_out / 8;
  const int t0 = blockIdx.x * 32;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const float* src = p.dq_acc + ((static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + t0) * p.D;
  uint16_t* dst = reinterpret_cast<uint16_t*>(p.dq) + b * p.dq_stride[0] + h * p.dq_stride[2];
  const float sc = p.scale;  // dQ = scale * dS K (dS is accumulated without the scale)
  for (int c = static_cast<int>(threadIdx.x); c < 32 * per_row; c += blockDim.x) {
    const int r = c / per_row, d8 = c - r * per_row;
    if (t0 + r >= p.Tq) break;  // rows only grow with c
    const float4* s4 = reinterpret_cast<const float4*>(src + static_cast<int64_t>(r) * p.D + d8 * 8);
    const float4 a = s4[0], e = s4[1];
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(t0 + r) * p.dq_stride[1] + d8 * 8) =
        make_uint4(pack2<kBF16>(a.x * sc, a.y * sc), pack2<kBF16>(a.z * sc, a.w * sc),
                   pack2<kBF16>(e.x * sc, e.y * sc), pack2<kBF16>(e.z * sc, e.w * sc));
  }
}

template <int D, bool kBF16, bool kMask, bool kScore>
cudaError_t launch_bwd_t(const BwdParams& p, cudaStream_t s) {
  using L = BwdLayout<D, kQStagesFor<kMask, kScore>>;
  auto kern = bwd_kernel<D, kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  const unsigned nkb = (p.Tk + 127) / 128, nh = p.Hk * p.g_split;
  const dim3 grid = p.kb_order ? dim3(nh, nkb * p.B, 1) : (p.kb_fastest ? dim3(nkb, nh, p.B) : dim3(nh, nkb, p.B));
  kern<<<grid, kBwdThreads, L::kAlloc, s>>>(p);
  return cudaGetLastError();
}

template <int D, bool kBF16>
cudaError_t launch_bwd_d(const BwdParams& p, bool m, bool sc, cudaStream_t s) {
  if (m && sc) return launch_bwd_t<D, kBF16, true, true>(p, s);
  if (m) return launch_bwd_t<D, kBF16, true, false>(p, s);
  if (sc) return launch_bwd_t<D, kBF16, false, true>(p, s);
  return launch_bwd_t<D, kBF16, false, false>(p, s);
}

}  // namespace

cudaError_t launch_bwd(const BwdParams& p, int D, bool bf16, bool has_mask, bool has_score, cudaStream_t s) {
  if (D == 128) return bf16 ? launch_bwd_d<128, true>(p, has_mask, has_score, s)
                            : launch_bwd_d<128, false>(p, has_mask, has_score, s);
  if (D == 64) return bf16 ? launch_bwd_d<64, true>(p, has_mask, has_score, s)
                           : launch_bwd_d<64, false>(p, has_mask, has_score, s);
  if (D == 256) return launch_bwd256(p, bf16, has_mask, has_score, s);
  return cudaErrorInvalidValue;
}

// Threads per block for a row of `chunks` 8-column pieces: whole warps, at most 1024.
int row_block(int chunks) { return std::min(1024, (chunks + 31) / 32 * 32); }

cudaError_t launch_bwd_prep(const PrepParams& p, bool bf16, cudaStream_t s) {
  const int64_t blocks = static_cast<int64_t>(p.B) * p.lse_ld;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;  // one block per (b, t) row
  const int threads = row_block(p.Hq * (p.D / 8));
  if (p.D == 128) {
    if (bf16) bwd_prep_kernel<128, true><<<blocks, threads, 0, s>>>(p);
    else bwd_prep_kernel<128, false><<<blocks, threads, 0, s>>>(p);
  } else if (p.D == 64) {
    if (bf16) bwd_prep_kernel<64, true><<<blocks, threads, 0, s>>>(p);
    else bwd_prep_kernel<64, false><<<blocks, threads, 0, s>>>(p);
  } else if (p.D == 256) {
    if (bf16) bwd_prep_kernel<256, true><<<blocks, threads, 0, s>>>(p);
    else bwd_prep_kernel<256, false><<<blocks, threads, 0, s>>>(p);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_dkv_convert(const DkvConvertParams& p, bool bf16, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(p.B) * p.Tk;
  if (rows > 0x7fffffff) return cudaErrorInvalidValue;  // one block per (b, t) row
  const dim3 grid(static_cast<unsigned>(rows), 2);
  const int threads = row_block(p.Hk * (p.d_out / 8));
  if (bf16) dkv_convert_kernel<true><<<grid, threads, 0, s>>>(p);
  else dkv_convert_kernel<false><<<grid, threads, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_dq_convert(const ConvertParams& p, bool bf16, cudaStream_t s) {
  const dim3 grid((p.Tq + 31) / 32, p.Hq, p.B);
  if (bf16) dq_convert_kernel<true><<<grid, 256, 0, s>>>(p);
  else dq_convert_kernel<false><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace fa4d
