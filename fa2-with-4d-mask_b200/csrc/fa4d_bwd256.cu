// fa4d_bwd256.cu — FlashAttention-2 backward at head dim 256 for sm_100a, with an
// optional 4D mask/score: dK and dV (dQ comes from the ordered pass, dq256_kernel in
// fa4d_dq256.cu, in both backward modes).
//
// Same math as the other head dims (python/fa2.py:181-302; dS carried without the
// factor `scale`, applied to dK in its epilogue).  At D = 256 the dK and dV
// accumulators of a 128-key tile would take all 512 TMEM columns of one SM, so each
// (128-key tile, batch, KV head) runs on a cluster of two CTAs that split the work by
// product, each computing every product it needs exactly once:
//   rank 0  S^T = K Q^T, P = exp2(S^T * scale * log2(e) - LSE) with the causal, bound,
//           mask and score rules, dV += P^T dO (all 256 columns)
//   rank 1  dP^T = V dO^T, dS = P (dP - Delta), dK += dS^T Q (all 256 columns)
// P^T crosses from rank 0 to rank 1 through distributed shared memory: rank 0's threads
// stage it (fp16: P is in [0, 1]) in their own shared memory, one thread copies the
// 16 KB tile into one of four rank-1 buffers with a bulk copy whose bytes that buffer's
// mbarrier counts; rank 1's warp 2 reports each landing back at once (so the staging
// buffer turns over without waiting for the dS work), and its row warps hand a buffer
// back with one remote arrival each once they have read it.  (Storing
// the rows directly into rank 1 from the threads held them for about 800 clocks per
// tile on the distributed-shared-memory bandwidth.)  (Computing dQ^T here as well was measured slower than
// the ordered pass: its fp32 reductions at this width are about 17 GB per backward at
// B1 T8192 Hq32, more than the whole ordered pass costs.)
//
// CTA = 128 keys x one (batch, KV head) x one rank; 384 threads:
//   warp 0       TMA producer of the operand this rank needs first (rank 0: Q per
//                64-row query tile; rank 1: dO), 2-stage ring
//   warp 1       tcgen05.mma issuer
//   warp 2       TMEM allocator; then rank 0: copies each staged P^T tile to rank 1;
//                rank 1: counts each tile's bytes in and reports its landing
//   warp 3       TMA producer of the operand needed last, with the row statistic
//                (rank 0: dO and LSE; rank 1: Q and Delta), 2-stage ring, so each
//                stage is released by its last reader and neither ring waits on the other
//   warps 4-7    first K (rank 0) or V (rank 1) columns 0-127 of their key into TMEM,
//                then queries 0-31 of every tile (one thread per key row), then
//                columns 0-127 of dV (rank 0) or dK (rank 1)
//   warps 8-11   the same for columns 128-255 and queries 32-63
// TMEM (512 columns): rank 0  S^T x2 [0,128) (P^T over the first 16 columns of each
//                             warpgroup's 32), K [128,256) (16-bit pairs, the A
//                             operand of S^T: only Q is read from shared memory, which
//                             took 6.3% off the kernel against S^T from shared memory),
//                             dV [256,512)
//                     rank 1  dP^T [0,64), V [64,192) (16-bit pairs, the A operand of
//                             dP^T), dS^T x2 [192,256) (the A operand of dK), dK [256,512)
// Shared memory: rank 0  Q x2, dO x2 (32 KB each), P^T staged x2 (16 KB each), LSE (its
//                        first 64 KB unused)
//                rank 1  P^T received x4 (16 KB each), Q x2, dO x2, Delta
#include <algorithm>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kThreads = 384;
// Register split (launch: 384 threads x 168 = 64512): producer/MMA warpgroup 112,
// the two row warpgroups 192 -> 128*112 + 256*192 = 63488.
constexpr uint32_t kRegsLaunch = 168, kRegsCtl = 112, kRegsRows = 192;
static_assert(128 * kRegsCtl + 256 * kRegsRows <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");

struct Layout {
  static constexpr int kKT = 128 * 256 * 2;  // one 128-key tile x 256 (rank 1's received P^T ring)
  static constexpr int kQT = 64 * 256 * 2;   // Q or dO tile (64 queries x 256)
  static constexpr int kXT = 128 * 64 * 2;   // P^T or dS^T tile (128 keys x 64 queries, 16-bit)
  static constexpr int kPin = 0;             // rank 1: P^T received, kPinBufs buffers
  static constexpr int kPinBufs = 4;
  static constexpr int kQ = kKT;             // 2 stages
  static constexpr int kDO = kQ + 2 * kQT;   // 2 stages
  static constexpr int kDS = kDO + 2 * kQT;  // rank 0: P^T staging (rank 1: unused)
  static constexpr int kStage = kDS;         // rank 0: P^T (fp16) staged for the peer, 2 buffers
  static constexpr int kStat = kDS + 2 * kXT;  // 2 stages x 64 floats: rank 0 LSE, rank 1 Delta
  static constexpr int kBar = kStat + 2 * 256;
  static constexpr int kNumBars = 30;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static_assert(kPin + kPinBufs * kXT <= kQ, "rank 1's received P^T overlaps the Q ring");
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
};

constexpr uint32_t kColS = 0;      // rank 0: S^T, 2 buffers of 64 columns
constexpr uint32_t kColDP = 0;     // rank 1: dP^T
constexpr uint32_t kColV = 64;     // rank 1: V, 128 columns
constexpr uint32_t kColK = 128;    // rank 0: K, 128 columns (the A operand of S^T)
constexpr uint32_t kColDS = 192;   // rank 1: dS^T, 2 buffers of 32 columns (the A operand of dK)
constexpr uint32_t kColAcc = 256;  // rank 0 dV, rank 1 dK: 256 columns
constexpr uint32_t kPBytes = 128 * 64 * 2;  // bytes of one P^T tile sent to rank 1

// Byte offset of 16-byte chunk cc of row r in a tile of 128-byte rows, 128-B swizzled
// (chunk ^ (row % 8)): the layout of the P^T tiles, so that a warp's 32 rows spread over
// all banks.
__device__ __forceinline__ uint32_t sw_chunk(int r, int cc) {
  return static_cast<uint32_t>(r * 128 + ((cc ^ (r & 7)) << 4));
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

// dV += P^T dO: M=128 keys, N=256, K=64 queries.  P^T of queries 0-31 sits in S^T
// columns [0,16) and of queries 32-63 in [32,48); dO MN-major (4 chunks of 64 columns).
template <bool kBF16>
__device__ __forceinline__ void issue_dv(uint32_t tD, uint32_t tS, uint32_t sDO, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, 256, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tD, tS + (kk >> 1) * 32 + (kk & 1) * 8, sw128_desc(sDO + kk * 2048, 8192, 1024), idesc,
           (acc || kk > 0) ? 1u : 0u);
}

// dK += dS^T Q: M=128 keys, N=256, K=64 queries; dS^T from TMEM (queries 0-31 in
// columns [0,16), 32-63 in [16,32)), Q MN-major.
template <bool kBF16>
__device__ __forceinline__ void issue_dk(uint32_t tD, uint32_t tDS, uint32_t sQ, bool acc) {
  constexpr uint32_t idesc = make_idesc(128, 256, kBF16, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_ts(tD, tDS + kk * 8, sw128_desc(sQ + kk * 2048, 8192, 1024), idesc, (acc || kk > 0) ? 1u : 0u);
}

template <bool kBF16, bool kMask, bool kScore>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    bwd256_kernel(const __grid_constant__ BwdParams p) {
  using L = Layout;
  extern __shared__ uint8_t smem_raw[];
  // Both CTAs of the cluster realign by the same amount (same kernel, same base), so
  // a shared-memory offset names the same buffer in either.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* v_full = bars + 1;     // rank 1: V in TMEM; rank 0: K in TMEM (256 arrivals)
  uint64_t* dkv_full = bars + 2;   // every dV / dK product done
  uint64_t* mma_drain = bars + 3;
  uint64_t* q_full = bars + 4;     // [2]
  uint64_t* q_empty = bars + 6;    // [2]
  uint64_t* do_full = bars + 8;    // [2]
  uint64_t* do_empty = bars + 10;  // [2]
  uint64_t* s_full = bars + 12;    // rank 0 [2]: S^T in TMEM
  uint64_t* dp_full = bars + 12;   // rank 1: dP^T in TMEM
  uint64_t* dp_empty = bars + 13;  // rank 1: dP^T read out (256 arrivals)
  uint64_t* p_full = bars + 14;    // rank 0 [2]: P^T written to TMEM (256 arrivals)
  uint64_t* ds_full = bars + 14;   // rank 1 [2]: dS^T written to shared memory (256 arrivals)
  uint64_t* in_full = bars + 16;    // rank 1 [4]: a P^T tile received (1 arrival + kPBytes)
  uint64_t* out_free = bars + 20;   // rank 0 [4]: the peer has read P^T buffer j (8 peer arrivals)
  uint64_t* ds_empty = bars + 24;   // rank 1 [2]: the dK product is done with dS^T
  uint64_t* p_staged = bars + 26;   // rank 0 [2]: P^T (fp16) staged for the copy (256 arrivals)
  uint64_t* copy_done = bars + 28;  // rank 0 [2]: the copy out of staging buffer s landed (1 peer arrival)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const uint32_t peer = rank ^ 1u;
  // Grid as in the other head dims with the cluster rank innermost in x:
  // x = 2 * (key tile or KV head x split) + rank.
  const int maj = static_cast<int>(blockIdx.x >> 1);
  const int kb = p.kb_fastest ? maj : static_cast<int>(blockIdx.y);
  const int hx = p.kb_fastest ? static_cast<int>(blockIdx.y) : maj;
  const int k0 = kb * 128;
  const int hk = hx / p.g_split;
  const int split = hx - hk * p.g_split;
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
    mbar_init(v_full, 256);
    mbar_init(dkv_full, 1);
    mbar_init(mma_drain, 1);
    if (rank == 0) {
      mbar_init(&s_full[0], 1);
      mbar_init(&s_full[1], 1);
      mbar_init(&p_full[0], 256);
      mbar_init(&p_full[1], 256);
      mbar_init(&p_staged[0], 256);
      mbar_init(&p_staged[1], 256);
    } else {
      mbar_init(dp_full, 1);
      mbar_init(dp_empty, 256);
      mbar_init(&ds_full[0], 256);
      mbar_init(&ds_full[1], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&do_full[i], 1);
      mbar_init(&do_empty[i], 1);
      mbar_init(&ds_empty[i], 1);
      mbar_init(&copy_done[i], 1);
    }
    for (int i = 0; i < L::kPinBufs; ++i) {
      mbar_init(&in_full[i], 1);
      mbar_init(&out_free[i], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  // Both CTAs' barriers are initialised before either touches the other's.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    regs_dec<kRegsCtl>();
    if ((warp == 0 || warp == 3) && lane == 0 && any_work) {
      // ---------------------------------------------------------- TMA producers
      // Warp 0: the ring read first (rank 0 Q, rank 1 dO); warp 3: the ring read last,
      // with the 64 row statistics of the tile (rank 0 dO + LSE, rank 1 Q + Delta).
      const bool late = warp == 3;
      const bool is_q = late == (rank == 1);
      const CUtensorMap* tm = is_q ? &p.tm_q : &p.tm_do;
      uint64_t* full = is_q ? q_full : do_full;
      uint64_t* empty = is_q ? q_empty : do_empty;
      uint8_t* ring = smem + (is_q ? L::kQ : L::kDO);
      prefetch_tmap(tm);
      if (kScore && p.score_pf && rank == 0 && late) prefetch_tmap(&p.tm_score);
      int issued = 0;
      QTiles<kMask> cur = first;
      for (int it = 0; cur.valid(); ++it, cur.advance()) {
        const int s = it & 1;
        const int h = h_first + cur.g();
        const int q0 = cur.q0();
        if (!mbar_wait(&empty[s], ((it >> 1) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], L::kQT + (late ? 256 : 0));
#pragma unroll
        for (int c = 0; c < 4; ++c) tma_load_4d(ring + s * L::kQT + c * 8192, tm, &full[s], c * 64, q0, h, b);
        if (late) {
          const int64_t row = (static_cast<int64_t>(b) * p.Hq + h) * p.lse_ld + q0;
          bulk_load(smem + L::kStat + s * 256, (rank == 0 ? p.lse : p.delta) + row, 256, &full[s]);
        }
        if (kScore && p.score_pf && rank == 0 && late) {
          const int hs = p.score_stride[1] ? h : 0, bs = p.score_stride[0] ? b : 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) tma_prefetch_l2_4d(&p.tm_score, k0 + 32 * c, q0, hs, bs);
        }
        issued = it + 1;
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        // Let the copies in flight land before the CTA leaves.
        for (int it = max(0, issued - 2); it < issued; ++it) mbar_wait_short(&full[it & 1], (it >> 1) & 1);
      }
    } else if (warp == 2 && rank == 0 && any_work) {
      // ---------------------------------------------------------- P^T copier (rank 0)
      // Staged tile it goes to the peer's buffer it % kPinBufs once the peer has read
      // the tile kPinBufs earlier out of it.
      const uint32_t peer_pin = peer_addr(smem_u32(smem + L::kPin), peer);
      const uint32_t peer_in_full = peer_addr(smem_u32(in_full), peer);
      QTiles<kMask> cur = first;
      for (int it = 0; cur.valid(); ++it, cur.advance()) {
        const int s = it & 1, j = it % L::kPinBufs;
        if (!__all_sync(0xffffffffu, mbar_wait(&p_staged[s], (it >> 1) & 1, abort_flag) &&
                                         mbar_wait_cl(&out_free[j], ((it / L::kPinBufs) & 1) ^ 1, abort_flag)))
          break;
        if (elect_one())
          bulk_copy_to_peer(peer_pin + j * L::kXT, smem + L::kStage + s * L::kXT, kPBytes, peer_in_full + 8u * j);
        __syncwarp();
      }
    } else if (warp == 2 && rank == 1 && any_work) {
      // ---------------------------------------------------------- P^T receiver (rank 1)
      // Registers the bytes of each incoming tile and, as soon as it has landed, tells
      // the peer that its staging buffer may be refilled.
      const uint32_t peer_copy_done = peer_addr(smem_u32(copy_done), peer);
      QTiles<kMask> cur = first;
      int it = 0, n_expected = 0;
      for (; cur.valid(); ++it, cur.advance()) {
        const int j = it % L::kPinBufs;
        if (elect_one()) mbar_arrive_expect_tx(&in_full[j], kPBytes);
        n_expected = it + 1;
        __syncwarp();
        if (!__all_sync(0xffffffffu, mbar_wait_cl(&in_full[j], (it / L::kPinBufs) & 1, abort_flag))) break;
        if (elect_one()) mbar_arrive_remote(peer_copy_done + 8u * (it & 1));
        __syncwarp();
      }
      if (*reinterpret_cast<volatile int*>(abort_flag) && lane == 0) {
        // The peer copies at most kPinBufs tiles ahead of what was received: let any such
        // copy land before the CTA leaves (registering its bytes if not done yet).
        for (int jt = it; jt < it + L::kPinBufs && cur.valid(); ++jt, cur.advance()) {
          if (jt >= n_expected) {
            mbar_arrive_expect_tx(&in_full[jt % L::kPinBufs], kPBytes);
            n_expected = jt + 1;
          }
          mbar_wait_short_cl(&in_full[jt % L::kPinBufs], (jt / L::kPinBufs) & 1);
        }
      }
      __syncwarp();
    } else if (warp == 1 && any_work) {
      // ---------------------------------------------------------- MMA issuer
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sDO = smem_u32(smem + L::kDO);
      const uint32_t tAcc = tmem + kColAcc;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      bool ok;
      if (rank == 0) {
        // Per tile: dV after its P^T, then S^T of the tile two ahead into the same
        // buffer (MMAs run in issue order, so it overwrites P^T only after dV read it).
        // S^T = K Q^T with K from TMEM (TS form, as dP^T on rank 1): only Q is read from
        // shared memory.
        const uint32_t tK = tmem + kColK;
        const uint32_t tS = tmem + kColS;
        ok = wait(v_full, 0) && wait(&q_full[0], 0);
        if (ok) {
          tc_fence_after();
          if (elect_one()) {
            issue_dp<kBF16>(tS, tK, sQ);
            tc_commit(&s_full[0]);
            tc_commit(&q_empty[0]);
          }
          __syncwarp();
          QTiles<kMask> second = first;
          second.advance();
          if (second.valid()) {
            ok = wait(&q_full[1], 0);
            if (ok) {
              tc_fence_after();
              if (elect_one()) {
                issue_dp<kBF16>(tS + 64, tK, sQ + L::kQT);
                tc_commit(&s_full[1]);
                tc_commit(&q_empty[1]);
              }
              __syncwarp();
            }
          }
        }
        QTiles<kMask> cur = first;
        for (int it = 0; ok && cur.valid(); ++it) {
          QTiles<kMask> nxt = cur;
          nxt.advance();
          QTiles<kMask> nxt2 = nxt;
          if (nxt2.valid()) nxt2.advance();
          const int s = it & 1;
          const uint32_t par = (it >> 1) & 1;
          ok = wait(&p_full[s], par) && wait(&do_full[s], par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_dv<kBF16>(tAcc, tS + 64 * s, sDO + s * L::kQT, it > 0);
            tc_commit(&do_empty[s]);
          }
          __syncwarp();
          if (nxt2.valid()) {
            ok = wait(&q_full[s], par ^ 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_dp<kBF16>(tS + 64 * s, tK, sQ + s * L::kQT);
              tc_commit(&s_full[s]);
              tc_commit(&q_empty[s]);
            }
            __syncwarp();
          }
          cur = nxt;
        }
      } else {
        // Per tile: dP^T of the next tile as soon as this tile's dP^T has been read out
        // (one buffer), then dK of this tile after its dS^T.
        const uint32_t tDP = tmem + kColDP, tV = tmem + kColV;
        ok = wait(v_full, 0) && wait(&do_full[0], 0);
        if (ok) {
          tc_fence_after();
          if (elect_one()) {
            issue_dp<kBF16>(tDP, tV, sDO);
            tc_commit(dp_full);
            tc_commit(&do_empty[0]);
          }
          __syncwarp();
        }
        QTiles<kMask> cur = first;
        for (int it = 0; ok && cur.valid(); ++it) {
          QTiles<kMask> nxt = cur;
          nxt.advance();
          const int s = it & 1;
          const uint32_t par = (it >> 1) & 1;
          if (nxt.valid()) {
            ok = wait(dp_empty, it & 1) && wait(&do_full[s ^ 1], ((it + 1) >> 1) & 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_dp<kBF16>(tDP, tV, sDO + (s ^ 1) * L::kQT);
              tc_commit(dp_full);
              tc_commit(&do_empty[s ^ 1]);
            }
            __syncwarp();
          }
          ok = wait(&ds_full[s], par) && wait(&q_full[s], par);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_dk<kBF16>(tAcc, tmem + kColDS + 32 * s, sQ + s * L::kQT, it > 0);
            tc_commit(&q_empty[s]);
            tc_commit(&ds_empty[s]);
          }
          __syncwarp();
          cur = nxt;
        }
      }
      if (elect_one()) {
        if (ok) tc_commit(dkv_full);
        tc_commit(mma_drain);
      }
      __syncwarp();
      wait(mma_drain, 0);
    }
  } else {
    regs_inc<kRegsRows>();
    // ------------------------------------------------------------ rows: P or dS, epilogue
    const int wg = (warp - 4) >> 2;  // queries 32*wg .. 32*wg+31 of every tile
    const int r = (warp & 3) * 32 + lane;
    const int k = k0 + r;
    const bool k_valid = k < p.Tk;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int kc = min(k, p.Tk - 1);
    const float* sStat = reinterpret_cast<const float*>(smem + L::kStat);
    bool ok = true;

    if (rank == 0) {
      if (any_work) {
        // K columns [128 wg, 128 wg + 128) of this key into TMEM (zeros past Tk).
        const uint4* krow = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.k) +
                                                           b * p.k_stride[0] + static_cast<int64_t>(kc) * p.k_stride[1] +
                                                           hk * p.k_stride[2] + 128 * wg);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t w[16];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 x = k_valid ? __ldg(krow + 4 * j + u) : make_uint4(0u, 0u, 0u, 0u);
            w[4 * u] = x.x;
            w[4 * u + 1] = x.y;
            w[4 * u + 2] = x.z;
            w[4 * u + 3] = x.w;
          }
          tmem_st16(tmem + lane_base + kColK + 64 * wg + 16 * j, w);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(v_full);
      }
      QTiles<kMask> cur = first;
      auto load_bits = [&](const QTiles<kMask>& c) {
        const int hh = h_first + c.g();
        const uint2 v2 = __ldg(reinterpret_cast<const uint2*>(p.mask_bits_t + b * p.mbt_stride[0] +
                                                               hh * p.mbt_stride[1]) +
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
        const int s = it & 1;
        const uint32_t par = (it >> 1) & 1;
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
        // S^T of the tile, and its LSE (loaded beside dO).
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], par, abort_flag) &&
                                         mbar_wait(&do_full[s], par, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint32_t tS = tmem + lane_base + kColS + 64 * s + 32 * wg;
        const bool need_causal = p.causal && (k0 + 127 > q0 + p.causal_off);
        const bool need_bounds = (q0 + 64 > p.Tq) || (k0 + 128 > p.Tk);
        const bool fast = !use_mask && !kScore && !need_causal && !need_bounds;
        const float* lse = sStat + s * 64 + 32 * wg;
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
        uint32_t ph[16];  // P^T for the peer, fp16 pairs
        {
          float pv[32];
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
          // P^T in the input type over the first 16 of this warpgroup's 32 S^T columns
          // (all of which this thread has read), the A operand of dV.
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pk[i] = pack2<kBF16>(pv[2 * i], pv[2 * i + 1]);
            ph[i] = pack2<false>(pv[2 * i], pv[2 * i + 1]);
          }
          tmem_st16(tS, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[s]);
        // P^T row r into staging buffer s once the copy that last read it has landed in
        // the peer (warp 2 then copies the tile across).
        ok = __all_sync(0xffffffffu, mbar_wait_cl(&copy_done[s], par ^ 1, abort_flag));
        if (!ok) break;
        uint8_t* stage = smem + L::kStage + s * L::kXT;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(stage + sw_chunk(r, 4 * wg + u)) =
              make_uint4(ph[4 * u], ph[4 * u + 1], ph[4 * u + 2], ph[4 * u + 3]);
        fence_async_smem();
        mbar_arrive(&p_staged[s]);
        cur = nxt;
      }
    } else {
      if (any_work) {
        // V columns [128 wg, 128 wg + 128) of this key into TMEM (zeros past Tk).
        const uint4* vrow = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.v) +
                                                           b * p.v_stride[0] + static_cast<int64_t>(kc) * p.v_stride[1] +
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
      const uint32_t peer_out_free = peer_addr(smem_u32(out_free), peer);
      QTiles<kMask> cur = first;
      for (int it = 0; cur.valid(); ++it) {
        QTiles<kMask> nxt = cur;
        nxt.advance();
        const int s = it & 1, jp = it % L::kPinBufs;
        const uint32_t par = (it >> 1) & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(dp_full, it & 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        uint32_t dp[32];
        tmem_ld32(tmem + lane_base + kColDP + 32 * wg, dp);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(dp_empty);
        // The peer's P^T of the tile, and Delta (loaded beside Q).
        ok = __all_sync(0xffffffffu, mbar_wait_cl(&in_full[jp], (it / L::kPinBufs) & 1, abort_flag) &&
                                         mbar_wait(&q_full[s], par, abort_flag));
        if (!ok) break;
        uint32_t dsk[16];
        {
          const uint8_t* pin = smem + L::kPin + jp * L::kXT;
          const float4* d4 = reinterpret_cast<const float4*>(sStat + s * 64 + 32 * wg);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 x = *reinterpret_cast<const uint4*>(pin + sw_chunk(r, 4 * wg + u));
            const uint32_t pw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float4 t = d4[2 * u + i];
              const float2 pa = unpack2<false>(pw[2 * i]), pb = unpack2<false>(pw[2 * i + 1]);
              dsk[4 * u + 2 * i] = pack2<kBF16>(pa.x * (__uint_as_float(dp[8 * u + 4 * i]) - t.x),
                                                pa.y * (__uint_as_float(dp[8 * u + 4 * i + 1]) - t.y));
              dsk[4 * u + 2 * i + 1] = pack2<kBF16>(pb.x * (__uint_as_float(dp[8 * u + 4 * i + 2]) - t.z),
                                                    pb.y * (__uint_as_float(dp[8 * u + 4 * i + 3]) - t.w));
            }
          }
        }
        // dS^T row r into TMEM buffer s (A operand of dK) once the last dK has read it.
        ok = __all_sync(0xffffffffu, mbar_wait(&ds_empty[s], par ^ 1, abort_flag));
        if (!ok) break;
        tc_fence_after();
        tmem_st16(tmem + lane_base + kColDS + 32 * s + 16 * wg, dsk);
        tmem_wait_st();
        // The peer may refill P^T buffer jp.  The hand-back is a relaxed arrival, which
        // does not wait for this thread's earlier loads; it comes after the dS^T stores
        // have completed, which cannot happen before the P^T loads they depend on have
        // returned (handing the buffer back straight after the loads let the next copy
        // overwrite the first rows of a tile before they were read).
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(peer_out_free + 8u * jp);
        tc_fence_before();
        mbar_arrive(&ds_full[s]);
        cur = nxt;
      }
    }

    // Epilogue: rank 0 writes dV, rank 1 dK (scaled), warpgroup wg columns
    // [128 wg, 128 wg + 128); zeros when no query interacts with this key tile.
    const int col0 = 128 * wg;
    const float out_scale = rank == 0 ? 1.f : p.scale;  // dK = scale * dS^T Q
    if (p.g_split > 1) {
      float* part = (rank == 0 ? p.dv_part : p.dk_part) + split * p.part_stride +
                    ((static_cast<int64_t>(b) * p.Tk + kc) * p.Hk + hk) * 256 + col0;
      if (any_work && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + kColAcc + col0 + 32 * c, v);
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
    } else {
      uint16_t* dst_row = nullptr;
      if (k_valid) {
        const int64_t* st3 = rank == 0 ? p.dv_stride : p.dk_stride;
        dst_row = reinterpret_cast<uint16_t*>(rank == 0 ? p.dv : p.dk) + b * st3[0] +
                  static_cast<int64_t>(k) * st3[1] + hk * st3[2] + col0;
      }
      if (any_work && ok) {
        ok = __all_sync(0xffffffffu, mbar_wait(dkv_full, 0, abort_flag));
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + kColAcc + col0 + 32 * c, v);
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
    }
    tc_fence_before();
  }

  // Neither CTA leaves while the other may still arrive on its barriers.
  cluster_sync();
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
  const unsigned nkb = (p.Tk + 127) / 128, nh = p.Hk * p.g_split;
  const dim3 grid = p.kb_fastest ? dim3(2 * nkb, nh, p.B) : dim3(2 * nh, nkb, p.B);
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
