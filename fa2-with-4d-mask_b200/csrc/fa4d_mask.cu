// fa4d_mask.cu — block-occupancy pre-pass over a 4D bool mask.
//
// The reference's kernels visit every 128-key tile of every query block and apply
// the mask element by element (python/fa2.py:95-124 forward, :242-302 backward),
// so a packed-document mask whose tiles are mostly False costs as much as a dense
// one.  This pass reads the mask once and classifies each 128 x 128 block as
// EMPTY (no True element), FULL (every in-bounds element True) or PARTIAL.  The
// forward and backward kernels then skip EMPTY blocks and skip the mask loads of
// FULL ones.  Elements past Tq / Tk do not affect the state of an edge block.
//
// Grid: (ceil(Tk / 512), ceil(Tq / 128), Bm * Hm); 256 threads.  Warp w reads rows
// w, w+8, ... of the CTA's 128-row block; lane l covers 16 consecutive keys, so a
// warp covers 512 keys = 4 blocks and lanes 8j..8j+7 cover block j.
#include "fa4d_kernels.h"
#include "fa4d_ptx.cuh"

namespace fa4d {

namespace {

// True when no byte of w is zero.
__device__ __forceinline__ bool no_zero_byte(uint32_t w) { return ((w - 0x01010101u) & ~w & 0x80808080u) == 0u; }

template <bool kVec>
__global__ void __launch_bounds__(256) mask_blocks_kernel(const MaskBlocksParams p) {
  __shared__ uint32_t s_any[4], s_all[4];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.z;
  const int b = bh / p.Hm;
  const int h = bh - b * p.Hm;
  const int qb = blockIdx.y;
  const int c0 = blockIdx.x * 512 + 16 * lane;
  if (tid < 4) {
    s_any[tid] = 0u;
    s_all[tid] = 1u;
  }
  __syncthreads();

  const uint8_t* base = p.mask + b * p.stride[0] + h * p.stride[1];
  const int r_end = min(qb * 128 + 128, p.Tq);
  bool any = false, all = true;
  if (kVec) {
    // Tk is a multiple of 16 here, so a lane's 16 keys are all in or all out of bounds.
    if (c0 < p.Tk) {
#pragma unroll 4
      for (int r = qb * 128 + warp; r < r_end; r += 8) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(r) * p.stride[2] + c0));
        any = any || ((w.x | w.y | w.z | w.w) != 0u);
        all = all && no_zero_byte(w.x) && no_zero_byte(w.y) && no_zero_byte(w.z) && no_zero_byte(w.w);
      }
    }
  } else {
    for (int r = qb * 128 + warp; r < r_end; r += 8) {
      const uint8_t* row = base + static_cast<int64_t>(r) * p.stride[2];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (c0 + e < p.Tk) {
          const bool keep = __ldg(row + c0 + e) != 0;
          any = any || keep;
          all = all && keep;
        }
      }
    }
  }
  const uint32_t any_b = __ballot_sync(0xffffffffu, any);
  const uint32_t all_b = __ballot_sync(0xffffffffu, all);
  if (lane < 4) {
    if ((any_b >> (8 * lane)) & 0xFFu) atomicOr(&s_any[lane], 1u);
    if (((all_b >> (8 * lane)) & 0xFFu) != 0xFFu) atomicAnd(&s_all[lane], 0u);
  }
  __syncthreads();
  if (tid < 4) {
    const int kb = blockIdx.x * 4 + tid;
    if (kb < p.nkb) {
      const uint8_t state = s_any[tid] ? (s_all[tid] ? 2 : 1) : 0;
      p.blocks[(static_cast<int64_t>(bh) * p.nqb + qb) * p.nkb + kb] = state;
    }
  }
}

// Keep flags of 32 consecutive bytes as one word (bit j = byte j nonzero).
__device__ __forceinline__ uint32_t keep_word(const uint4& a, const uint4& b) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t r = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) r |= keep_bits4(w[i]) << (4 * i);
  return r;
}

// One pass over the mask writes, for every 128 x 128 block, its state, plus the mask
// as packed bits in the two tile layouts the kernels read with one vector load per
// thread and tile:
//   row bits [Bm*Hm][nkb][Tq][4] words: 128 keys of key tile kt for query row q
//     (bit j of word w = key 128*kt + 32*w + j), read by the forward;
//   column bits [Bm*Hm][nqt][Tk][2] words: 64 queries of query tile qt for key k
//     (bit j of word w = query 64*qt + 32*w + j), read by the backward.
// Keys / queries past Tk / Tq read as 0.
//
// One CTA walks kPrepTiles consecutive 128 x 128 blocks of one 128-row block row
// (grid (ceil(nkb / kPrepTiles), nqb, Bm * Hm), 128 threads); per block:
//   1. the block's keep flags as bytes into shared memory: thread t covers the 16-key
//      chunk t % 8 of rows t / 8 + 16 i (i < 8), so each group of 8 threads reads 128
//      contiguous bytes of one row (kSrc 0: 16-byte loads, issued for the next block
//      before the current one is packed, so loads stay in flight); or byte loads (kSrc
//      1: unaligned rows or Tk % 16 != 0); or flags computed from document ids (kSrc 2:
//      keep iff the query's and key's ids are equal and not negative);
//   2. thread r packs row r's 128 flags into 4 words and stores them as one 16-byte
//      vector (the CTA's 128 rows are one contiguous 2 KB run of the row bits);
//   3. warp w (rows 32w..32w+31, lane = row) transposes each 32 x 32 bit block of its
//      words with five shuffle steps, so lane i holds the column word of key 32 j + i;
//      the words go through shared memory and thread t writes key t's two words of each
//      64-row query tile as one 8-byte vector (contiguous over the CTA's keys).
// Rows are padded to 144 bytes in shared memory, so both the chunk stores of step 1 and
// the row reads of step 2 are free of bank conflicts.
constexpr int kPrepTiles = 4;

// 32 x 32 bit transpose across a warp: lane i holds row i (bit j = column j) and gets
// column i (bit j = row j).  Each step swaps the off-diagonal s x s sub-blocks of every
// 2s x 2s block (s = 16, 8, 4, 2, 1), which composes to the full transpose.
__device__ __forceinline__ uint32_t transpose32(uint32_t x, int lane) {
  constexpr uint32_t kMask[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int sh = 16 >> i;
    const uint32_t m = kMask[i];
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x, sh);
    x = (lane & sh) ? ((x & ~m) | ((y & ~m) >> sh)) : ((x & m) | ((y & m) << sh));
  }
  return x;
}

template <int kSrc>
__global__ void __launch_bounds__(128) mask_prepare_kernel(const MaskPrepParams p) {
  constexpr int kPitch = 144;
  __shared__ __align__(16) uint8_t tile[128 * kPitch];
  __shared__ uint32_t cols[4][128];  // [32-row quarter][key]: column word of that quarter
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int bh = blockIdx.z;
  const int b = bh / p.Hm;
  const int h = bh - b * p.Hm;
  const int qb = blockIdx.y;
  const int q0 = qb * 128;
  const int kt0 = blockIdx.x * kPrepTiles;
  const int c = tid & 7, r0 = tid >> 3;
  const uint8_t* mask_base = kSrc == 2 ? nullptr : p.mask + b * p.stride[0] + h * p.stride[1];
  // The key-tile order pass may be scheduled now; it waits for this grid's completion
  // (griddepcontrol.wait) before reading the block map.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // kSrc 0: one block's 16-byte chunks, loaded into registers ahead of their use.
  auto load_block = [&](int kt, uint4 (&v)[8]) {
    const int kk = kt * 128 + 16 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = q0 + r0 + 16 * i;
      // Tk % 16 == 0: a 16-key chunk is entirely inside or outside Tk.
      v[i] = (q < p.Tq && kk < p.Tk)
                 ? __ldg(reinterpret_cast<const uint4*>(mask_base + static_cast<int64_t>(q) * p.stride[2] + kk))
                 : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint4 v[8];
  if constexpr (kSrc == 0) load_block(kt0, v);

  for (int u = 0; u < kPrepTiles; ++u) {
    const int kt = kt0 + u;
    if (kt >= p.nkb) break;
    const int k0 = kt * 128;
    __syncthreads();  // the previous block's shared-memory reads are done
    // ---- 1. keep flags as bytes
    if constexpr (kSrc == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(tile + (r0 + 16 * i) * kPitch + 16 * c) = v[i];
      if (u + 1 < kPrepTiles && kt + 1 < p.nkb) load_block(kt + 1, v);
    } else if constexpr (kSrc == 1) {
      const int kk = k0 + 16 * c;
      for (int i = 0; i < 8; ++i) {
        const int q = q0 + r0 + 16 * i;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (q < p.Tq) {
          const uint8_t* row = mask_base + static_cast<int64_t>(q) * p.stride[2];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (kk + e < p.Tk && __ldg(row + kk + e) != 0) w[e >> 2] |= 1u << (8 * (e & 3));
        }
        *reinterpret_cast<uint4*>(tile + (r0 + 16 * i) * kPitch + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      const int kk = k0 + 16 * c;
      int32_t dk[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) dk[e] = kk + e < p.Tk ? __ldg(p.doc_k + b * p.doc_k_stride + kk + e) : -2;
      for (int i = 0; i < 8; ++i) {
        const int q = q0 + r0 + 16 * i;
        const int32_t dq = q < p.Tq ? __ldg(p.doc_q + b * p.doc_q_stride + q) : -1;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (dq >= 0 && dk[e] == dq) w[e >> 2] |= 1u << (8 * (e & 3));
        *reinterpret_cast<uint4*>(tile + (r0 + 16 * i) * kPitch + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncthreads();

    // ---- 2. row bits (thread = row)
    const int row = q0 + tid;
    const bool row_ok = row < p.Tq;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 x = *reinterpret_cast<const uint4*>(tile + tid * kPitch + 32 * j);
      const uint4 y = *reinterpret_cast<const uint4*>(tile + tid * kPitch + 32 * j + 16);
      w[j] = keep_word(x, y);
    }
    if (row_ok)
      *reinterpret_cast<uint4*>(p.row_bits + ((static_cast<int64_t>(bh) * p.nkb + kt) * p.Tq + row) * 4) =
          make_uint4(w[0], w[1], w[2], w[3]);
    // Block state over the in-bounds elements only.
    bool full = true;
#pragma unroll
    for (int j = 0; j < 4; ++j) full = full && (w[j] == low_bits(p.Tk - k0 - 32 * j));
    const int any = __syncthreads_or(row_ok && (w[0] | w[1] | w[2] | w[3]) != 0u);
    const int all = __syncthreads_and(!row_ok || full);

    // ---- 3. column bits: bit transpose of the warp's 32 rows (lane = row)
#pragma unroll
    for (int j = 0; j < 4; ++j) cols[warp][32 * j + lane] = transpose32(w[j], lane);
    __syncthreads();
    const int k = k0 + tid;
    if (k < p.Tk) {
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int qt = 2 * qb + t;
        if (qt < p.nqt)
          *reinterpret_cast<uint2*>(p.col_bits + ((static_cast<int64_t>(bh) * p.nqt + qt) * p.Tk + k) * 2) =
              make_uint2(cols[2 * t][tid], cols[2 * t + 1][tid]);
      }
    }
    if (tid == 0) p.blocks[(static_cast<int64_t>(bh) * p.nqb + qb) * p.nkb + kt] = any ? (all ? 2 : 1) : 0;
  }
}

}  // namespace

// Key tiles longest first, for the backward grid: one block per (b, h) row of the block
// map counts each key tile's non-EMPTY 128-row query blocks and writes kb_order[rank] =
// key tile, by decreasing count (ties by key tile index, so the order is reproducible).
// With more than kOrderMaxTiles key tiles the order is the identity.
constexpr int kOrderMaxTiles = 1024;

__global__ void __launch_bounds__(256) kb_order_kernel(const MaskPrepParams p) {
  __shared__ int cnt[kOrderMaxTiles];
  // Launched as a programmatic dependent of the prepare kernel: wait until that grid has
  // finished and its block map is visible.  The map is read through L2 only (__ldcg).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nkb = p.nkb;
  const uint8_t* blocks = p.blocks + static_cast<size_t>(blockIdx.x) * p.nqb * nkb;
  int32_t* out = p.kb_order + static_cast<size_t>(blockIdx.x) * nkb;
  if (nkb > kOrderMaxTiles) {
    for (int kb = threadIdx.x; kb < nkb; kb += blockDim.x) out[kb] = kb;
    return;
  }
  for (int kb = threadIdx.x; kb < nkb; kb += blockDim.x) cnt[kb] = 0;
  __syncthreads();
  // The whole CTA reads the map row-major, kUnroll independent byte loads per thread in
  // flight, and adds the non-EMPTY ones into shared counters (a walk down one column
  // per thread would wait out one load latency per query block).
  constexpr int kUnroll = 8;
  const int n = p.nqb * nkb;
  for (int i0 = threadIdx.x; i0 < n; i0 += blockDim.x * kUnroll) {
    uint8_t st[kUnroll];
#pragma unroll
    for (int j = 0; j < kUnroll; ++j) {
      const int i = i0 + j * static_cast<int>(blockDim.x);
      st[j] = i < n ? __ldcg(blocks + i) : 0;
    }
#pragma unroll
    for (int j = 0; j < kUnroll; ++j)
      if (st[j] != 0) atomicAdd(&cnt[(i0 + j * static_cast<int>(blockDim.x)) % nkb], 1);
  }
  __syncthreads();
  for (int kb = threadIdx.x; kb < nkb; kb += blockDim.x) {
    const int c = cnt[kb];
    int rank = 0;
    for (int j = 0; j < nkb; ++j) rank += (cnt[j] > c) || (cnt[j] == c && j < kb);
    out[rank] = kb;
  }
}

cudaError_t launch_mask_prepare(const MaskPrepParams& p, cudaStream_t s) {
  dim3 grid((p.nkb + kPrepTiles - 1) / kPrepTiles, p.nqb, p.Bm * p.Hm);
  if (p.doc_q)
    mask_prepare_kernel<2><<<grid, 128, 0, s>>>(p);
  else if (p.vec)
    mask_prepare_kernel<0><<<grid, 128, 0, s>>>(p);
  else
    mask_prepare_kernel<1><<<grid, 128, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !p.kb_order) return e;
  // Programmatic dependent launch: the order pass's CTAs are scheduled while the
  // prepare kernel's last wave runs, instead of after a launch gap.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.Bm * p.Hm);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kb_order_kernel, p);
}

cudaError_t launch_mask_blocks(const MaskBlocksParams& p, cudaStream_t s) {
  const bool vec = p.vec != 0;
  dim3 grid((p.Tk + 511) / 512, p.nqb, p.Bm * p.Hm);
  if (vec)
    mask_blocks_kernel<true><<<grid, 256, 0, s>>>(p);
  else
    mask_blocks_kernel<false><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace fa4d
