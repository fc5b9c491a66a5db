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
//   warp 0      TMA producer (Q once, then K/V tiles into a 1- or 2-stage ring each)
//   warp 1      tcgen05.mma issuer (whole warp, one elected lane issues)
//   warp 2      TMEM allocator, then mask/score staging for query slot 1
//   warp 3      mask/score staging for query slot 0
//   warps 4-7   softmax + epilogue for query slot 0 (one thread per row)
//   warps 8-11  softmax + epilogue for query slot 1
// The key tiles visited are the union of the two slots' tiles: those below the
// causal / key-length limit minus the blocks the mask's block map marks EMPTY
// (block-sparse skipping; the reference visits every tile, python/fa2.py:95).
// Mask tiles (PARTIAL blocks only) and score chunks reach shared memory by TMA
// through a per-slot ring, so the softmax threads read them with 16-B shared loads
// instead of waiting on global memory.
// At D=256 the CTA has one slot whose S has two buffers, [0,128) and [128,256), with
// O0 [256,512): the next key tile's S is computed while the softmax works on the
// current one.  Warp 2 then loads V (warp 0 Q and K) and warps 8-11 stay idle.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [256+D,256+2D).
// P (16-bit) overwrites the first 64 columns of S and feeds the PV MMA from TMEM.
#include <cfloat>

#include "fa4d.h"
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"
#include "fa4d_tiles.cuh"

namespace fa4d {

namespace {

constexpr int kFwdThreads = 384;
// Register split (launch: 384 threads x 168 = 64512): producer/MMA warpgroup 112, the
// two softmax warpgroups 192 -> 128*112 + 256*192 = 63488.  The mask-only variants at
// D = 64 / 128 take 96 / 200 (128*96 + 256*200 = 63488): at 192 their softmax code
// spilled 96-108 bytes per thread, at 200 8-16, and the packed-document forward (config
// 3) ran 2.9% faster; the dense and score variants ran 1-4% slower at 96 / 200, and at
// D = 256 the control warps spilled at 96.
template <int D, bool kMask, bool kScore>
constexpr bool kFwdWideSoftmax = D != 256 && kMask && !kScore;
template <int D, bool kMask, bool kScore>
constexpr uint32_t kFwdRegsCtl = kFwdWideSoftmax<D, kMask, kScore> ? 96 : 112;
template <int D, bool kMask, bool kScore>
constexpr uint32_t kFwdRegsSoftmax = kFwdWideSoftmax<D, kMask, kScore> ? 200 : 192;
constexpr uint32_t kFwdRegsLaunch = 168;
static_assert(128 * 112 + 256 * 192 <= kFwdThreads * kFwdRegsLaunch && 128 * 96 + 256 * 200 <= kFwdThreads * kFwdRegsLaunch,
              "register split exceeds the launch allocation");
constexpr float kNegInf = -INFINITY;
// O is only rescaled when the running max grows by more than this (log2 units);
// in between, P = exp2(s - stale max) stays <= 2^8, exact after the final 1/l.
constexpr float kRescaleThreshold = 8.0f;
// In the unmasked fast path one exponential pair in kPolyEvery is evaluated on the FMA
// pipe (ex2_poly2) instead of the MUFU unit.
#ifndef FA4D_POLY_EVERY
#define FA4D_POLY_EVERY 3
#endif
constexpr int kPolyEvery = FA4D_POLY_EVERY;
// At D = 64 the softmax warps signal P of keys 0-63 on their own barrier and the MMA
// warp issues that half of PV at once, so only the second half of PV sits between the
// end of the softmax and the slot's next S.  Measured (interleaved A/B, medians of 8
// blocks of 10): D = 64 forward at config 2's shape -2.9%, config 5 forward -1.2%; at
// D = 128 the same split made the forward 2% slower, so it is kept to D = 64.
template <int D>
constexpr bool kSplitPVFor = D == 64;
// One staged score chunk (128 rows x 32 keys, fp32): 128 B per row, 128-B swizzled.
constexpr int kRingEntry = 16384;

template <int D, bool kMask, bool kScore>
struct FwdLayout {
  static constexpr int kTile = 128 * D * 2;  // one 128-row tile of 16-bit elements
  // Query slots per CTA.  At D=256 one slot's O takes 256 of the 512 TMEM columns and
  // its Q, K and V tiles 192 KB of shared memory, so the CTA has one slot (with two S
  // buffers) and single-stage K/V (the second slot's warps stay idle).
  static constexpr int kSlots = D == 256 ? 1 : 2;
  // With a score at D=128 the score staging rings take the room of one K/V stage.
  static constexpr int kKVStages = (D == 256 || (kScore && D == 128)) ? 1 : 2;
  static constexpr int kQ = 0;  // kSlots query slots
  static constexpr int kK = kQ + kSlots * kTile;
  static constexpr int kV = kK + kKVStages * kTile;
  static constexpr int kRing = kV + kKVStages * kTile;  // [kSlots][kRingDepth] entries
  static constexpr int kRingRoom = 232448 - 1024 - 512 - kRing;
  static constexpr int kRingFit = kRingRoom / (kSlots * kRingEntry);
  static constexpr int kRingDepth = kScore ? (kRingFit < 4 ? kRingFit : 4) : 0;
  static constexpr int kBar = kRing + kSlots * kRingDepth * kRingEntry;
  static constexpr int kNumBars = 19 + 4 * kRingDepth;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024 B
  static_assert(kAlloc <= 232448, "shared memory beyond the 227 KB per-block limit");
  static_assert(!kScore || kRingDepth >= 1, "no room for the score staging ring");
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

// O[slot] (+)= P[slot] V : M=128, N=D, K=128; P from TMEM, V MN-major.  Covers keys
// [64 * first_half, 64 * last_half + 64) of the tile (K-steps of 16 keys).
template <int D, bool kBF16>
__device__ __forceinline__ void issue_pv(uint32_t tO, uint32_t tP, uint32_t sV, bool accumulate, int first_half = 0,
                                         int last_half = 1) {
  constexpr uint32_t idesc = make_idesc(128, D, kBF16, false, true);
#pragma unroll
  for (int kk = 4 * first_half; kk < 4 * last_half + 4; ++kk) {
    mma_ts(tO, tP + kk * 8, sw128_desc(sV + kk * 2048, 16384, 1024), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
  }
}

// First tile at or after kt that either slot visits (n_max if none).
template <bool kMask>
__device__ __forceinline__ int next_union(const SlotTiles<kMask>& s0, const SlotTiles<kMask>& s1, int kt, int n_max) {
  while (kt < n_max && s0.state(kt) == 0 && s1.state(kt) == 0) ++kt;
  return kt;
}

template <int D, bool kBF16, bool kMask, bool kScore>
__global__ void __launch_bounds__(kFwdThreads, 1) fwd_kernel(const __grid_constant__ FwdParams p) {
  using L = FwdLayout<D, kMask, kScore>;
  constexpr bool kSplitPV = kSplitPVFor<D>;
  // One query slot per CTA (D = 256): the slot's S has two TMEM buffers, [0,128) and
  // [128,256) (O takes [256,512)), so the S of the next key tile is computed while the
  // softmax works on the current one; V comes from its own producer warp (warp 2).
  constexpr bool kDoubleS = L::kSlots == 1;
  constexpr int R = L::kRingDepth > 0 ? L::kRingDepth : 1;  // ring index modulus (ring unused if 0 deep)
  constexpr int KVS = L::kKVStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-B aligned base, derived by pointer arithmetic on the shared array so the
  // compiler keeps the shared address space (LDS/STS rather than generic loads/stores).
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
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
  uint64_t* ring_full = bars + 16;                         // [2 slots][kRingDepth]
  uint64_t* ring_empty = bars + 16 + 2 * L::kRingDepth;   // [2 slots][kRingDepth], 128 arrivals
  uint64_t* p_half = bars + 16 + 4 * L::kRingDepth;       // [2] per slot: P of keys 0-63 written (D = 64)
  uint64_t* pv_done = bars + 18 + 4 * L::kRingDepth;      // one slot (D = 256): PV of a tile completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  int* abort_flag = reinterpret_cast<int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (Hq, query blocks, B): CTAs are dispatched x-fastest, so all heads of one
  // query block go out together; causal runs the longest blocks (last rows) first.
  const int qblk = p.causal ? static_cast<int>(gridDim.y - 1 - blockIdx.y) : static_cast<int>(blockIdx.y);
  const int h = blockIdx.x;
  const int b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qblk * 128 * L::kSlots;

  SlotTiles<kMask> tiles0, tiles1;
  {
    const uint8_t* row = nullptr;
    if (kMask && p.mask_blocks) row = p.mask_blocks + b * p.mb_stride[0] + h * p.mb_stride[1];
    tiles0.n = kv_tile_count(q0, min(q0 + 128, p.Tq), p.Tq, p.Tk, p.causal, p.causal_off);
    tiles1.n = L::kSlots == 2 ? kv_tile_count(q0 + 128, min(q0 + 256, p.Tq), p.Tq, p.Tk, p.causal, p.causal_off) : 0;
    tiles0.map = (row && tiles0.n > 0) ? row + static_cast<int64_t>(q0 / 128) * p.nkb : nullptr;
    tiles1.map = (row && tiles1.n > 0) ? row + static_cast<int64_t>(q0 / 128 + 1) * p.nkb : nullptr;
  }
  const int n_max = max(tiles0.n, tiles1.n);
  const int kt_first = next_union(tiles0, tiles1, 0, n_max);
  const bool any_work = kt_first < n_max;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_half[i], 128);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(mma_drain, 1);
    mbar_init(pv_done, 1);
    for (int i = 0; i < 2 * L::kRingDepth; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 128);
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
    // Each role starts with its register budget so the compiler allocates that
    // role's code under it.
    regs_dec<kFwdRegsCtl<D, kMask, kScore>>();
    if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && any_work) {
      prefetch_tmap(&p.tm_q);
      prefetch_tmap(&p.tm_k);
      prefetch_tmap(&p.tm_v);
      uint8_t* sQ = smem + L::kQ;
      uint8_t* sK = smem + L::kK;
      uint8_t* sV = smem + L::kV;
      mbar_arrive_expect_tx(q_full, L::kSlots * L::kTile);
#pragma unroll
      for (int t = 0; t < L::kSlots; ++t)
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sQ + t * L::kTile + c * 16384, &p.tm_q, q_full, c * 64, q0 + 128 * t, h, b);
      int u = 0;              // union entries whose K and V loads were issued
      bool k_pending = false;  // K of entry u issued, its V not
      for (int kt = kt_first; kt < n_max; kt = next_union(tiles0, tiles1, kt + 1, n_max), ++u) {
        const int s = u % KVS;
        const uint32_t par = ((u / KVS) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], par, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sK + s * L::kTile + c * 16384, &p.tm_k, &k_full[s], c * 64, kt * 128, hk, b);
        if constexpr (!kDoubleS) {
          if (!mbar_wait(&v_empty[s], par, abort_flag)) {
            k_pending = true;
            break;
          }
          mbar_arrive_expect_tx(&v_full[s], L::kTile);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sV + s * L::kTile + c * 16384, &p.tm_v, &v_full[s], c * 64, kt * 128, hk, b);
        }
      }
      // Abort path only: make sure no copy is still writing shared memory.
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        mbar_wait_short(q_full, 0);
        for (int j = max(0, u - KVS); j < u; ++j) {
          mbar_wait_short(&k_full[j % KVS], (j / KVS) & 1);
          if (!kDoubleS) mbar_wait_short(&v_full[j % KVS], (j / KVS) & 1);
        }
        if (k_pending) mbar_wait_short(&k_full[u % KVS], (u / KVS) & 1);
      }
    }
    __syncwarp();
    } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (waits included); each group of MMAs and its
    // commits is issued by one elected lane, keeping the issue state uniform.
    if (any_work) {
      const uint32_t sQ = smem_u32(smem + L::kQ);
      const uint32_t sK = smem_u32(smem + L::kK);
      const uint32_t sV = smem_u32(smem + L::kV);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      if constexpr (kDoubleS) {
        // Tile u's S sits in buffer u & 1.  S of tile u+1 goes out as soon as its K has
        // landed, ahead of PV of tile u; its buffer last held P of tile u-1, whose PV
        // was issued in the previous iteration (the tensor pipe runs them in order).
        bool ok = wait(q_full, 0) && wait(&k_full[0], 0);
        if (ok) {
          tc_fence_after();
          if (elect_one()) {
            issue_qk<D, kBF16>(tmem, sQ, sK);
            tc_commit(&s_full[0]);
            tc_commit(&k_empty[0]);
          }
          __syncwarp();
        }
        int u = 0;
        for (int kt = kt_first; ok && kt < n_max; ++u) {
          const int ktn = next_union(tiles0, tiles1, kt + 1, n_max);
          const bool has_next = ktn < n_max;
          if (has_next) {
            const int sk = (u + 1) % KVS;
            ok = wait(&k_full[sk], ((u + 1) / KVS) & 1);
            if (!ok) break;
            tc_fence_after();
            if (elect_one()) {
              issue_qk<D, kBF16>(tmem + 128 * ((u + 1) & 1), sQ, sK + sk * L::kTile);
              tc_commit(&s_full[(u + 1) & 1]);
              tc_commit(&k_empty[sk]);
            }
            __syncwarp();
          }
          const int sv = u % KVS;
          ok = wait(&v_full[sv], (u / KVS) & 1) && wait(&p_full[u & 1], (u >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            issue_pv<D, kBF16>(tmem + 256, tmem + 128 * (u & 1), sV + sv * L::kTile, u > 0);
            tc_commit(pv_done);
            tc_commit(&v_empty[sv]);
            if (!has_next) tc_commit(&o_full[0]);
          }
          __syncwarp();
          kt = ktn;
        }
        if (elect_one()) tc_commit(mma_drain);
        __syncwarp();
        wait(mma_drain, 0);
      } else {
      const int last0 = tiles0.last(), last1 = tiles1.last();
      bool ok = wait(q_full, 0) && wait(&k_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (elect_one()) {
          if (tiles0.state(kt_first)) {
            issue_qk<D, kBF16>(tmem, sQ, sK);
            tc_commit(&s_full[0]);
          }
          if (tiles1.state(kt_first)) {
            issue_qk<D, kBF16>(tmem + 128, sQ + L::kTile, sK);
            tc_commit(&s_full[1]);
          }
          tc_commit(&k_empty[0]);
        }
        __syncwarp();
      }
      int cnt0 = 0, cnt1 = 0;  // PV MMAs issued per slot
      int u = 0;
      for (int kt = kt_first; ok && kt < n_max; ++u) {
        const int sv = u % KVS;
        ok = wait(&v_full[sv], (u / KVS) & 1);
        if (!ok) break;
        const int ktn = next_union(tiles0, tiles1, kt + 1, n_max);
        const bool has_next = ktn < n_max;
        const int sk = (u + 1) % KVS;
        if (has_next) {
          ok = wait(&k_full[sk], ((u + 1) / KVS) & 1);
          if (!ok) break;
        }
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const SlotTiles<kMask>& tl = t ? tiles1 : tiles0;
          int& cnt = t ? cnt1 : cnt0;
          const bool cur = tl.state(kt) != 0;
          const bool nxt = has_next && tl.state(ktn) != 0;
          if (cur) {
            if constexpr (kSplitPV) {
              // The first half of PV goes out once the softmax warps have written P of
              // keys 0-63, while they still work on the rest of the row.
              ok = wait(&p_half[t], cnt & 1);
              if (!ok) break;
              tc_fence_after();
              if (elect_one()) issue_pv<D, kBF16>(tmem + 256 + D * t, tmem + 128 * t, sV + sv * L::kTile, cnt > 0, 0, 0);
              __syncwarp();
            }
            ok = wait(&p_full[t], cnt & 1);
            if (!ok) break;
            tc_fence_after();
          }
          if (elect_one()) {
            if (cur) {
              if constexpr (kSplitPV)
                issue_pv<D, kBF16>(tmem + 256 + D * t, tmem + 128 * t, sV + sv * L::kTile, true, 1, 1);
              else
                issue_pv<D, kBF16>(tmem + 256 + D * t, tmem + 128 * t, sV + sv * L::kTile, cnt > 0);
            }
            if (nxt) {
              // S of the slot's next tile; the PV above (or an earlier one) has
              // consumed the P that shares these TMEM columns.
              issue_qk<D, kBF16>(tmem + 128 * t, sQ + t * L::kTile, sK + sk * L::kTile);
              tc_commit(&s_full[t]);
            } else if (cur && kt == (t ? last1 : last0)) {
              tc_commit(&o_full[t]);
            }
          }
          __syncwarp();
          if (cur) ++cnt;
        }
        if (!ok) break;
        if (elect_one()) {
          tc_commit(&v_empty[sv]);
          if (has_next) tc_commit(&k_empty[sk]);
        }
        __syncwarp();
        kt = ktn;
      }
      // Every MMA must have completed before TMEM is released.
      if (elect_one()) tc_commit(mma_drain);
      __syncwarp();
      wait(mma_drain, 0);
      }
    }
    __syncwarp();
    } else if (kDoubleS && warp == 2) {
    // ------------------------------------------------------------ V producer (one slot)
    // V of tile u is loaded once PV of tile u-1 has freed the stage; K (warp 0) does not
    // wait behind it.
    if (lane == 0 && any_work) {
      uint8_t* sV = smem + L::kV;
      int u = 0;
      for (int kt = kt_first; kt < n_max; kt = next_union(tiles0, tiles1, kt + 1, n_max), ++u) {
        const int s = u % KVS;
        if (!mbar_wait(&v_empty[s], ((u / KVS) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sV + s * L::kTile + c * 16384, &p.tm_v, &v_full[s], c * 64, kt * 128, hk, b);
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        for (int j = max(0, u - KVS); j < u; ++j) mbar_wait_short(&v_full[j % KVS], (j / KVS) & 1);
      }
    }
    __syncwarp();
    } else if (kScore) {
    // ------------------------------------------------------------ score staging
    // Warp 3 feeds query slot 0, warp 2 (after the TMEM allocation) slot 1: the four
    // 32-key score chunks of every tile the slot visits, in order, into its ring.
    const int t = warp == 3 ? 0 : 1;
    const SlotTiles<kMask> tl = t ? tiles1 : tiles0;
    if (lane == 0 && p.bias_tma && tl.n > 0) {
      prefetch_tmap(&p.tm_score);
      const int qs = q0 + 128 * t;
      const int hs = p.score_stride[1] ? h : 0, bs = p.score_stride[0] ? b : 0;
      uint8_t* ring = smem + L::kRing + t * R * kRingEntry;
      uint64_t* full = ring_full + t * R;
      uint64_t* empty = ring_empty + t * R;
      int g = 0;
      bool ok = true;
      for (int kt = tl.next(0); ok && kt < tl.n; kt = tl.next(kt + 1)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          const int e = g % R;
          ok = mbar_wait(&empty[e], ((g / R) & 1) ^ 1, abort_flag);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[e], kRingEntry);
          tma_load_4d(ring + e * kRingEntry, &p.tm_score, &full[e], kt * 128 + 32 * c, qs, hs, bs);
          ++g;
        }
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) {
        for (int j = max(0, g - R); j < g; ++j) mbar_wait_short(&full[j % R], (j / R) & 1);
      }
    }
    __syncwarp();
    }
  } else if ((warp - 4) >> 2 >= L::kSlots) {
    regs_inc<kFwdRegsSoftmax<D, kMask, kScore>>();  // a slot this CTA does not have (D=256): nothing to do
  } else {
    regs_inc<kFwdRegsSoftmax<D, kMask, kScore>>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int row = (warp & 3) * 32 + lane;
    const int qs = q0 + 128 * t;
    const int q = qs + row;
    const bool q_valid = q < p.Tq;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS_slot = tmem + lane_base + 128 * t;
    const uint32_t tO = tmem + lane_base + 256 + D * t;
    const SlotTiles<kMask> tl = t ? tiles1 : tiles0;

    // Rows past Tq read row Tq-1 of the mask / score (always in bounds) and are never
    // stored, so the loads carry no per-lane branch and the warp stays converged for
    // the TMEM ops.
    const int64_t qc = min(q, p.Tq - 1);
    const float* score_row = nullptr;
    const uint8_t* mask_row = nullptr;
    const uint4* bits_row = nullptr;  // prepared mask bits: one uint4 per key tile
    if (kScore) score_row = p.score + b * p.score_stride[0] + h * p.score_stride[1] + qc * p.score_stride[2];
    if (kMask) {
      mask_row = p.mask + b * p.mask_stride[0] + h * p.mask_stride[1] + qc * p.mask_stride[2];
      if (p.mask_bits)
        bits_row = reinterpret_cast<const uint4*>(p.mask_bits + b * p.mbits_stride[0] + h * p.mbits_stride[1]) + qc;
    }
    // Staged score: this thread's row of each ring entry (128 B, 16-B units swizzled by row % 8).
    const uint32_t ring_row = smem_u32(smem + L::kRing + t * R * kRingEntry + row * 128);
    uint64_t* full = ring_full + t * R;
    uint64_t* empty = ring_empty + t * R;
    const int sw = row & 7;
    int g = 0;
    // Keys this row may see at all: below Tk and, when causal, k <= q + causal_off.
    const int key_lim = p.causal ? min(p.Tk, static_cast<int>(min(static_cast<long long>(q) + p.causal_off + 1,
                                                                     static_cast<long long>(p.Tk))))
                                 : p.Tk;

    float m_run = kNegInf;
    float l_run = 0.f;
    bool ok = true;
    int i = 0;  // tiles processed by this slot
    int kt = tl.next(0);
    // Mask bits of the next PARTIAL tile are loaded one tile ahead.
    uint4 bits_next = make_uint4(0u, 0u, 0u, 0u);
    if (kMask && bits_row && kt < tl.n && tl.state(kt) == 1) bits_next = __ldg(bits_row + static_cast<int64_t>(kt) * p.Tq);
    for (; kt < tl.n; ++i) {
      const int kt_next = tl.next(kt + 1);
      const bool use_mask = kMask && tl.state(kt) == 1;  // warp-uniform
      uint32_t mw[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};  // keep bit per key
      if (kMask && use_mask && bits_row) {
        mw[0] = bits_next.x;
        mw[1] = bits_next.y;
        mw[2] = bits_next.z;
        mw[3] = bits_next.w;
      }
      if (kMask && bits_row && kt_next < tl.n && tl.state(kt_next) == 1)
        bits_next = __ldg(bits_row + static_cast<int64_t>(kt_next) * p.Tq);

      // Warp-uniform outcome: the tcgen05.ld below is warp-collective.
      // S buffer of this tile (one-slot CTAs alternate two) and its completion phase.
      const int sb = kDoubleS ? (i & 1) : t;
      const uint32_t tS = kDoubleS ? tmem + lane_base + 128 * sb : tS_slot;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], kDoubleS ? (i >> 1) & 1 : i & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();

      const int kbase = kt * 128;
      const bool need_bounds = kbase + 128 > p.Tk;
      const bool need_causal = p.causal && (kbase + 127 > qs + p.causal_off);
      // Interior tile with nothing to add or mask (warp-uniform): the row max is taken
      // on raw S and the scale is folded into the exponent's FMA below.
      const bool fast = !kScore && !use_mask && !need_bounds && !need_causal && p.scale_log2 > 0.f;
      // Online softmax with lazy rescaling of O; returns the max the exponents use.
      auto online_update = [&](float m_tile) {
        const float m_new = fmaxf(m_run, m_tile);
        const bool need = m_new > m_run + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = ex2(m_run - m_new);  // m_run == -inf -> 0
          l_run *= alpha;
          m_run = m_new;
        }
        if (i > 0 && __any_sync(0xffffffffu, need)) {
          // The slot's previous PV has completed (this tile's S was issued after it), or,
          // with two S buffers, is waited for here: PV of tile i cannot have completed
          // (it needs this tile's P) and PV of tile i-2 ran before this tile's S, so
          // pv_done is in the phase of PV i-1 or the one after it.
          if (kDoubleS) mbar_wait(pv_done, (i - 1) & 1, abort_flag);
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t o[16];
            tmem_ld16(tO + 16 * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st16(tO + 16 * c, o);
          }
        }
        return (m_run == kNegInf) ? 0.f : m_run;
      };
      float rowsum = 0.f;
      if (fast) {
        uint32_t sr[128];  // the whole row of S
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * c]));
        tmem_wait_ld();
        float m4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int k = 0; k < 128; k += 2)
          m4[(k >> 1) & 3] = fmax3(m4[(k >> 1) & 3], __uint_as_float(sr[k]), __uint_as_float(sr[k + 1]));
        const float m_use = online_update(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2);
        // exp2(s * scale * log2(e) - m) on pairs of packed fp32; every kPolyEvery-th
        // pair on the FMA pipe (ex2_poly2) so the MUFU unit is not the limit.
        const uint64_t sc2 = f2(p.scale_log2, p.scale_log2), nm2 = f2(-m_use, -m_use);
        uint64_t rs2 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 a = f2_split(
                ffma2(f2(__uint_as_float(sr[32 * c + 2 * k]), __uint_as_float(sr[32 * c + 2 * k + 1])), sc2, nm2));
            const float2 pr = (k % kPolyEvery == kPolyEvery - 1) ? ex2_poly2(a.x, a.y)
                                                                 : make_float2(ex2(a.x), ex2(a.y));
            rs2 = fadd2(rs2, f2(pr.x, pr.y));
            pk[k] = pack2<kBF16>(pr.x, pr.y);
          }
          tmem_st16(tS + 16 * c, pk);
          if (kSplitPV && c == 1) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_half[t]);
          }
        }
        const float2 rs = f2_split(rs2);
        rowsum = rs.x + rs.y;
      } else if constexpr (!kScore) {
        // Masked or edge tile without a score: one pass over the whole row in registers.
        // x = s * scale (log2 units), -inf where the keep bit is clear; every exponential
        // on MUFU (ex2_poly clamps its argument and would leave cut keys a tiny weight).
        if (kMask && use_mask && !bits_row) {
          // No prepared bits: read this row's 128 mask bytes from global memory.
          const uint4 v = mask_words_from_bytes(mask_row, kbase, p.Tk, p.mask_vec);
          mw[0] = v.x;
          mw[1] = v.y;
          mw[2] = v.z;
          mw[3] = v.w;
        }
        if (need_bounds || need_causal) {
#pragma unroll
          for (int c = 0; c < 4; ++c) mw[c] &= low_bits(key_lim - (kbase + 32 * c));
        }
        uint32_t xr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&xr[32 * c]));
        tmem_wait_ld();
        float m4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int k = 0; k < 128; k += 2) {
          const float x0 = ((mw[k >> 5] >> (k & 31)) & 1u) ? __uint_as_float(xr[k]) * p.scale_log2 : kNegInf;
          const float x1 = ((mw[k >> 5] >> ((k + 1) & 31)) & 1u) ? __uint_as_float(xr[k + 1]) * p.scale_log2 : kNegInf;
          xr[k] = __float_as_uint(x0);
          xr[k + 1] = __float_as_uint(x1);
          m4[(k >> 1) & 3] = fmax3(m4[(k >> 1) & 3], x0, x1);
        }
        const float m_use = online_update(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
        const uint64_t nm2 = f2(m_use, m_use);
        uint64_t rs2 = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 a = f2_split(fsub2(f2(__uint_as_float(xr[32 * c + 2 * k]), __uint_as_float(xr[32 * c + 2 * k + 1])), nm2));
            const float p0 = ex2(a.x), p1 = ex2(a.y);
            rs2 = fadd2(rs2, f2(p0, p1));
            pk[k] = pack2<kBF16>(p0, p1);
          }
          tmem_st16(tS + 16 * c, pk);
          if (kSplitPV && c == 1) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_half[t]);
          }
        }
        const float2 rs = f2_split(rs2);
        rowsum = rs.x + rs.y;
      } else {
        // Tile with a score (the variants with a score only reach this branch).
        if (kMask && use_mask && !bits_row) {
          // No prepared bits: read this row's 128 mask bytes from global memory.
          const uint4 v = mask_words_from_bytes(mask_row, kbase, p.Tk, p.mask_vec);
          mw[0] = v.x;
          mw[1] = v.y;
          mw[2] = v.z;
          mw[3] = v.w;
        }
        if (need_bounds || need_causal) {
#pragma unroll
          for (int c = 0; c < 4; ++c) mw[c] &= low_bits(key_lim - (kbase + 32 * c));
        }
        float m4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
        // x = (s + score) * scale, -inf where the keep bit is clear, in two halves of
        // 64 keys: each half is read from TMEM, transformed and written back, so only 64
        // values are live beside the mask words and the score state (the whole row in
        // registers spilled).  The score is consumed four values at a time.
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t xr[64];
          tmem_ld32(tS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&xr[0]));
          tmem_ld32(tS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&xr[32]));
          tmem_wait_ld();
          auto apply4 = [&](int e0, float a0, float a1, float a2, float a3, uint32_t w) {
            const float av[4] = {a0, a1, a2, a3};
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
              const int e = e0 + j;
              // (s + score) * scale on a packed fp32 pair (same rounding as scalar).
              const float2 x = f2_split(fmul2(fadd2(f2(__uint_as_float(xr[e]), __uint_as_float(xr[e + 1])),
                                                    f2(av[j], av[j + 1])),
                                              f2(p.scale_log2, p.scale_log2)));
              float x0 = x.x, x1 = x.y;
              x0 = ((w >> (e & 31)) & 1u) ? x0 : kNegInf;
              x1 = ((w >> ((e + 1) & 31)) & 1u) ? x1 : kNegInf;
              xr[e] = __float_as_uint(x0);
              xr[e + 1] = __float_as_uint(x1);
              m4[j] = fmaxf(m4[j], x0);
              m4[j + 1] = fmaxf(m4[j + 1], x1);
            }
          };
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * hh + cc;
            const int kc = kbase + 32 * c;
            const uint32_t w = mw[c];
            if (p.bias_tma) {
              const int e = g % R;
              ok = __all_sync(0xffffffffu, mbar_wait(&full[e], (g / R) & 1, abort_flag));
              if (!ok) break;
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const float4 v = lds_f4(ring_row + e * kRingEntry + ((u ^ sw) << 4));
                apply4(32 * cc + 4 * u, v.x, v.y, v.z, v.w, w);
              }
              mbar_arrive(&empty[e]);
              ++g;
            } else if (p.score_vec && kc + 31 < p.Tk) {
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(score_row + kc) + u);
                apply4(32 * cc + 4 * u, v.x, v.y, v.z, v.w, w);
              }
            } else {
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int k4 = kc + 4 * u;
                apply4(32 * cc + 4 * u, (k4 < p.Tk) ? __ldg(score_row + k4) : 0.f,
                       (k4 + 1 < p.Tk) ? __ldg(score_row + k4 + 1) : 0.f,
                       (k4 + 2 < p.Tk) ? __ldg(score_row + k4 + 2) : 0.f,
                       (k4 + 3 < p.Tk) ? __ldg(score_row + k4 + 3) : 0.f, w);
              }
            }
          }
          if (!ok) break;
          tmem_st32(tS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&xr[0]));
          tmem_st32(tS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&xr[32]));
        }
        if (!ok) break;
        tmem_wait_st();  // the transformed row is read back below
        const float m_use = online_update(fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])));
        // The transformed row comes back in halves; P of keys 64 hh .. 64 hh + 63 goes
        // to columns 32 hh .. 32 hh + 31, whose x values have been read by then.
        const uint64_t nm2 = f2(m_use, m_use);
        uint64_t rs2 = f2(0.f, 0.f);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t xr[64];
          tmem_ld32(tS + 64 * hh, *reinterpret_cast<uint32_t(*)[32]>(&xr[0]));
          tmem_ld32(tS + 64 * hh + 32, *reinterpret_cast<uint32_t(*)[32]>(&xr[32]));
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const float2 a = f2_split(
                  fsub2(f2(__uint_as_float(xr[32 * c + 2 * k]), __uint_as_float(xr[32 * c + 2 * k + 1])), nm2));
              const float p0 = ex2(a.x), p1 = ex2(a.y);
              rs2 = fadd2(rs2, f2(p0, p1));
              pk[k] = pack2<kBF16>(p0, p1);
            }
            tmem_st16(tS + 32 * hh + 16 * c, pk);
          }
          if (kSplitPV && hh == 0) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_half[t]);
          }
        }
        const float2 rs = f2_split(rs2);
        rowsum = rs.x + rs.y;
      }
      l_run += rowsum;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      kt = kt_next;
    }

    // Epilogue: O / l and LSE.  A slot that visits no tile (every block EMPTY) has
    // only fully masked rows: O = NaN and LSE = -inf, as softmax over -inf gives.
    using Elem = uint16_t;
    Elem* o_row = nullptr;
    if (q_valid)
      o_row = reinterpret_cast<Elem*>(p.o) + b * p.o_stride[0] + static_cast<int64_t>(q) * p.o_stride[1] +
              h * p.o_stride[2];
    if (i > 0 && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], 0, abort_flag));
      tc_fence_after();
      // l == 0 (no valid key): O = NaN like the oracle (inv_l = inf, O = 0 * inf), or
      // O = 0 in document mode.
      const float inv_l = (l_run > 0.f || !p.empty_rows_zero) ? 1.f / l_run : 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        if (q_valid && 32 * c < p.d_out) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k)
            pk[k] = pack2<kBF16>(__uint_as_float(o[2 * k]) * inv_l, __uint_as_float(o[2 * k + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(o_row + 32 * c);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
    } else if (q_valid) {
      const uint32_t nan2 = p.empty_rows_zero ? 0u : pack2<kBF16>(NAN, NAN);
      uint4* dst = reinterpret_cast<uint4*>(o_row);
#pragma unroll
      for (int v = 0; v < D / 8; ++v)
        if (8 * v < p.d_out) dst[v] = make_uint4(nan2, nan2, nan2, nan2);
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
  using L = FwdLayout<D, kMask, kScore>;
  auto kern = fwd_kernel<D, kBF16, kMask, kScore>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Hq, (p.Tq + 128 * L::kSlots - 1) / (128 * L::kSlots), p.B);
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
  if (D == 256) return bf16 ? launch_fwd_d<256, true>(p, has_mask, has_score, s)
                            : launch_fwd_d<256, false>(p, has_mask, has_score, s);
  return cudaErrorInvalidValue;
}

}  // namespace fa4d

namespace {

// out[i] = ex2_poly2(x_i) / exp2f(x_i) - 1 on an even grid x_i over [lo, hi].
__global__ void exp2_check_kernel(float* out, int n, float lo, float hi) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = lo + (hi - lo) * (static_cast<float>(i) / static_cast<float>(n - 1));
  out[i] = fa4d::ex2_poly2(x, x).y / exp2f(x) - 1.0f;
}

}  // namespace

namespace {

// A wait on an mbarrier that nothing ever completes: the same bounded wait the
// attention kernels use must give up after `limit` clocks and report it through the
// status word, leaving the context usable.
__global__ void wait_timeout_check_kernel(int* status, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    fa4d::mbar_init(&bar, 1);
    abort_flag = 0;
    fa4d::fence_mbar_init();
  }
  __syncthreads();
  const bool done = fa4d::mbar_wait(&bar, 0, &abort_flag, limit);
  __syncwarp();
  if (threadIdx.x == 0 && !done && *reinterpret_cast<volatile int*>(&abort_flag))
    atomicOr(status, FA4D_DEV_TIMEOUT_CHECK);
}

}  // namespace

namespace fa4d {
cudaError_t launch_wait_timeout_check(int* status, long long limit, cudaStream_t s) {
  wait_timeout_check_kernel<<<1, 32, 0, s>>>(status, limit);
  return cudaGetLastError();
}
cudaError_t launch_exp2_check(float* out, int n, float lo, float hi, cudaStream_t s) {
  exp2_check_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, n, lo, hi);
  return cudaGetLastError();
}
}  // namespace fa4d
